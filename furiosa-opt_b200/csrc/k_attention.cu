// Fused attention: softmax(Q K^T * scale + causal mask) V with an online (running max / sum)
// softmax, the single-kernel form of the reference's per-chunk op chain
// (furiosa-opt-examples/src/transformer/kernel/attention.rs:32-392: qk_scaled, row_max, masked_exp,
// row_sum (+ EPS), weighted_sum, online rescale, norm).
//
// Layout: Q [B, S, Hq, D], K / V [B, S, Hkv, D], O [B, S, Hq, D], bf16, D = 128. GQA: query head h
// reads kv head h / (Hq / Hkv). Scores, max, sum and the output accumulator are f32.
//
// CUDA-core version: a block owns 8 query rows of one head (one warp each) and streams 32-key tiles
// of K (transposed into shared memory, so lanes read consecutive keys) and V through shared memory.
#include <algorithm>

#include "ctx.hpp"

namespace fopt {
namespace {

constexpr int kD = 128;
constexpr int kRows = 8;   // query rows (warps) per block
constexpr int kKeys = 32;  // keys per tile

__device__ __forceinline__ float bf(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }

__global__ void __launch_bounds__(256) attention_rows_kernel(uint16_t* __restrict__ O, const uint16_t* __restrict__ Q,
                                                             const uint16_t* __restrict__ K,
                                                             const uint16_t* __restrict__ V, int S, int Hq, int Hkv,
                                                             float scale, int causal, float eps) {
  __shared__ float kt[kD][kKeys + 1];
  __shared__ float vs[kKeys][kD];
  __shared__ float qs[kRows][kD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row_tiles = (S + kRows - 1) / kRows;
  const int h = blockIdx.x % Hq;
  const int rt = (blockIdx.x / Hq) % row_tiles;
  const int b = blockIdx.x / (Hq * row_tiles);
  const int hk = h / (Hq / Hkv);
  const int i = rt * kRows + warp;  // this warp's query row
  const int64_t qstride = (int64_t)Hq * kD, kstride = (int64_t)Hkv * kD;
  const uint16_t* qrow = Q + ((int64_t)b * S + min(i, S - 1)) * qstride + (int64_t)h * kD;
  for (int d = lane; d < kD; d += 32) qs[warp][d] = bf(qrow[d]) * scale;
  float m = -INFINITY, l = 0.0f, acc[4] = {0, 0, 0, 0};
  const int last_row = min(S - 1, rt * kRows + kRows - 1);
  const int kend = causal ? last_row + 1 : S;
  for (int k0 = 0; k0 < kend; k0 += kKeys) {
    __syncthreads();
    // stage K^T and V tiles (256 threads: 32 keys x 128 dims each)
    for (int e = threadIdx.x; e < kKeys * kD; e += blockDim.x) {
      int j = e / kD, d = e % kD;
      int key = k0 + j;
      float kv = 0.0f, vv = 0.0f;
      if (key < S) {
        int64_t off = ((int64_t)b * S + key) * kstride + (int64_t)hk * kD + d;
        kv = bf(K[off]);
        vv = bf(V[off]);
      }
      kt[d][j] = kv;
      vs[j][d] = vv;
    }
    __syncthreads();
    if (i >= S) continue;
    int key = k0 + lane;
    float s = 0.0f;
#pragma unroll 8
    for (int d = 0; d < kD; ++d) s = fmaf(qs[warp][d], kt[d][lane], s);
    bool valid = key < S && (!causal || key <= i);
    s = valid ? s : -INFINITY;
    float tmax = s;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
    float mnew = fmaxf(m, tmax);
    if (mnew == -INFINITY) continue;  // fully masked tile (cannot happen for causal row >= k0)
    float alpha = expf(m - mnew);
    float p = valid ? expf(s - mnew) : 0.0f;
    float psum = p;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
    l = l * alpha + psum;
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[c] *= alpha;
#pragma unroll 4
    for (int j = 0; j < kKeys; ++j) {
      float pj = __shfl_sync(0xffffffffu, p, j);
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[c] = fmaf(pj, vs[j][lane * 4 + c], acc[c]);
    }
    m = mnew;
  }
  if (i >= S) return;
  float inv = 1.0f / (l + eps);
  uint16_t* orow = O + ((int64_t)b * S + i) * qstride + (int64_t)h * kD;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t w = f32_to_bf16w(__float_as_uint(acc[c] * inv));
    orow[lane * 4 + c] = (uint16_t)(w >> 16);
  }
}

}  // namespace

void launch_attention(fopt_ctx* ctx, void* o, const void* q, const void* k, const void* v, int B, int S, int Hq,
                      int Hkv, int D, float scale, int causal, float eps) {
  if (launch_attention_tc(ctx, o, q, k, v, B, S, Hq, Hkv, D, scale, causal, eps)) return;
  int row_tiles = (S + kRows - 1) / kRows;
  int64_t blocks = (int64_t)B * Hq * row_tiles;
  attention_rows_kernel<<<(unsigned)blocks, 256, 0, ctx->stream>>>((uint16_t*)o, (const uint16_t*)q,
                                                                   (const uint16_t*)k, (const uint16_t*)v, S, Hq, Hkv,
                                                                   scale, causal, eps);
  launched(ctx, "attention");
}

}  // namespace fopt
