// Fold kernels: BufStorage::reduce (furiosa-opt-std/src/storage/buf.rs:331-376) and the generic
// per-output-cell contraction (buf.rs:401-447) for operands whose layout is not a plain GEMM.
//
// Both follow the reference's ReadPlan (buf.rs:680-753): each output cell has a base read offset
// (the output walk) plus a shared list of live residue deltas (the residue walk, in the
// reference's wire order). The delta lists live in device scratch.
//   * exact mode / order-sensitive folds: one thread per output cell folds its deltas in order
//     (bit-identical to the reference for every dtype; coalesced when the output's innermost
//     wheel is unit-stride in the source, e.g. [R, C] -> [C]);
//   * fast mode for order-insensitive folds over a unit-stride residue: one warp per output cell,
//     lanes read consecutive elements and combine with warp shuffles.
#include <algorithm>

#include "ctx.hpp"
#include "ew_ops.cuh"

namespace fopt {
namespace {

__device__ __forceinline__ float F(uint32_t w) { return __uint_as_float(w); }
__device__ __forceinline__ uint32_t W(float f) { return __float_as_uint(f); }

// The combine step in dtype's arithmetic. bf16 adds round back to bf16 after each step (the
// `half` crate's `bf16 + bf16`).
__device__ __forceinline__ uint32_t combine(int op, int dt, uint32_t a, uint32_t b) {
  if (dt == FOPT_I32) {
    int32_t x = (int32_t)a, y = (int32_t)b;
    switch (op) {
      case FOPT_RED_ADD: return a + b;
      case FOPT_RED_ADD_SAT: {
        int64_t s = (int64_t)x + y;
        return (uint32_t)(int32_t)max((int64_t)INT32_MIN, min((int64_t)INT32_MAX, s));
      }
      case FOPT_RED_MAX: return (uint32_t)max(x, y);
      case FOPT_RED_MIN: return (uint32_t)min(x, y);
      default: return a * b;
    }
  }
  float x = F(a), y = F(b), r;
  switch (op) {
    case FOPT_RED_ADD: case FOPT_RED_ADD_SAT: r = __fadd_rn(x, y); break;
    case FOPT_RED_MAX: r = fmaxf(x, y); break;
    case FOPT_RED_MIN: r = fminf(x, y); break;
    default: r = __fmul_rn(x, y); break;
  }
  uint32_t w = W(r);
  if (dt == FOPT_BF16) {
    // plain IEEE RNE narrowing, as `half::bf16::from_f32`
    uint32_t hi = w >> 16;
    if ((w & 0x7fffffffu) > 0x7f800000u) hi |= 0x40;
    else if ((w & 0x8000u) && (w & 0x17fffu)) hi += 1;
    w = hi << 16;
  }
  return w;
}

__device__ __forceinline__ uint32_t load_acc(const void* p, int dt, int64_t i) {
  // I32 / F32 raw; BF16 widened exactly (bits << 16).
  return load_word(p, dt, i);
}

__global__ void reduce_cell_kernel(void* __restrict__ out, const void* __restrict__ src, int dt, int op, uint32_t ident,
                                   KWalk ow, int64_t out_positions, const int64_t* __restrict__ delta, int64_t nd,
                                   int64_t src_elems) {
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < out_positions;
       o += (int64_t)gridDim.x * blockDim.x) {
    int64_t base = 0;
    uint32_t acc = ident;
    if (walk_offsets<1>(ow, o, &base)) {
      for (int64_t r = 0; r < nd; ++r) {
        int64_t p = base + delta[r];
        if (p >= 0 && p < src_elems) acc = combine(op, dt, acc, load_acc(src, dt, p));
      }
    }
    store_word(out, dt, o, acc);
  }
}

// One warp per output cell; the residue is one unit-stride run of `nd` elements. 32-bit rows whose
// base is 16-byte aligned are read as uint4 (4 elements per lane per step) into 4 independent
// partial folds, combined at the end (order-insensitive folds only).
__global__ void reduce_warp_kernel(void* __restrict__ out, const void* __restrict__ src, int dt, int op, uint32_t ident,
                                   KWalk ow, int64_t out_positions, int64_t nd, int64_t src_elems) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t o = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); o < out_positions; o += warps) {
    int64_t base = 0;
    uint32_t acc = ident;
    bool live = walk_offsets<1>(ow, o, &base);
    if (live) {
      const bool vec = dtype_bits(dt) == 32 && (base & 3) == 0 && ((uintptr_t)src & 15) == 0 &&
                       base + nd <= src_elems;
      if (vec) {
        uint32_t a0 = ident, a1 = ident, a2 = ident, a3 = ident;
        const uint4* row = (const uint4*)((const uint32_t*)src + base);
        const int64_t nv = nd >> 2;
        for (int64_t r = lane; r < nv; r += 32) {
          uint4 v = row[r];
          a0 = combine(op, dt, a0, v.x);
          a1 = combine(op, dt, a1, v.y);
          a2 = combine(op, dt, a2, v.z);
          a3 = combine(op, dt, a3, v.w);
        }
        for (int64_t r = (nv << 2) + lane; r < nd; r += 32) a0 = combine(op, dt, a0, load_acc(src, dt, base + r));
        acc = combine(op, dt, combine(op, dt, a0, a1), combine(op, dt, a2, a3));
      } else {
        for (int64_t r = lane; r < nd; r += 32) {
          int64_t p = base + r;
          if (p < src_elems) acc = combine(op, dt, acc, load_acc(src, dt, p));
        }
      }
#pragma unroll
      for (int s = 16; s > 0; s >>= 1) acc = combine(op, dt, acc, __shfl_xor_sync(0xffffffffu, acc, s));
    }
    if (lane == 0) store_word(out, dt, o, acc);
  }
}

// ---- generic contraction ----
__device__ __forceinline__ bool is_int_in(int dt) {
  return dt == FOPT_I8 || dt == FOPT_I4 || dt == FOPT_I5 || dt == FOPT_I9 || dt == FOPT_I16 || dt == FOPT_I32;
}

__device__ __forceinline__ float widen_f(const void* p, int dt, int64_t i) {
  uint32_t w = load_word(p, dt, i);
  if (dt == FOPT_BF16) return F(bf16w_to_f32_bits(w));
  if (dt == FOPT_F8E4M3) return F(ew::f8e4_to_f32w(w));  // Cast<f32> for f8e4m3 (cast.rs:193-198)
  if (dt == FOPT_F8E5M2) return F(ew::f8e5_to_f32w(w));  // Cast<f32> for f8e5m2 (cast.rs:207-212)
  return F(w);  // F32 prewidened
}

struct CArgs {
  void* out;
  int out_dt;
  const void* lhs;
  const void* rhs;
  int in_dt;
  int64_t lhs_elems, rhs_elems;
  const int64_t* dl;
  const int64_t* dr;
  int64_t nd;
  int ep_kind;
  int int_width;
  int clip_lo, clip_hi;
  const float* scale;
};

__device__ __forceinline__ uint32_t int_finish(const CArgs& a, int32_t acc, int64_t sidx);

__device__ __forceinline__ uint32_t contract_cell(const CArgs& a, int64_t bl, int64_t br, int64_t sidx) {
  uint32_t res;
  if (is_int_in(a.in_dt)) {
    uint32_t acc = 0;  // wrapping i32 sum
    for (int64_t r = 0; r < a.nd; ++r) {
      int64_t pl = bl + a.dl[r], pr = br + a.dr[r];
      if (pl < a.lhs_elems && pr < a.rhs_elems)
        acc += (uint32_t)((int32_t)load_word(a.lhs, a.in_dt, pl) * (int32_t)load_word(a.rhs, a.in_dt, pr));
    }
    return int_finish(a, (int32_t)acc, sidx);
  } else {
    float acc = 0.0f;
    for (int64_t r = 0; r < a.nd; ++r) {
      int64_t pl = bl + a.dl[r], pr = br + a.dr[r];
      if (pl < a.lhs_elems && pr < a.rhs_elems)
        acc = __fadd_rn(acc, __fmul_rn(widen_f(a.lhs, a.in_dt, pl), widen_f(a.rhs, a.in_dt, pr)));
    }
    res = W(acc);
    if (a.out_dt == FOPT_BF16) {
      if (a.ep_kind == 2) {
        bool nan = (res & 0x7fffffffu) > 0x7f800000u;
        res = (!nan && (res >> 31)) ? 0u : f32_to_bf16w(res);
      } else {
        res = f32_to_bf16w(res);
      }
    } else if (a.out_dt == FOPT_F8E4M3 || a.out_dt == FOPT_F8E5M2) {
      // narrow once per cell through the f8 encoder (cast.rs:200-217), after the commit ReLU if any
      if (a.ep_kind == 2 && (res & 0x7fffffffu) <= 0x7f800000u && (res >> 31)) res = 0u;
      res = a.out_dt == FOPT_F8E4M3 ? ew::f32w_to_f8e4(res) : ew::f32w_to_f8e5(res);
    } else if (a.ep_kind == 2) {
      res = W(fmaxf(acc, 0.0f));
    }
  }
  return res;
}

// The epilogue of an integer cell: requant (1), ReLU (2) or the raw i32 sum.
__device__ __forceinline__ uint32_t int_finish(const CArgs& a, int32_t acc, int64_t sidx) {
  uint32_t res;
  {
    if (a.ep_kind == 1) {
      float y = F(fxp_to_fp_bits(acc, (uint32_t)a.int_width));
      const float sv = a.scale[sidx];
      // x86 products (the reference's host) return a NaN operand unchanged and make 0 * inf the
      // negative default NaN; the GPU would return a positive canonical NaN for both
      y = __fmul_rn(y, sv);
      if (y != y) y = sv != sv ? sv : __uint_as_float(0xffc00000u);
      int32_t q = fp_to_fxp(y, (uint32_t)a.int_width);
      q = max(a.clip_lo, min(a.clip_hi, q));
      return (uint32_t)q;
    }
    if (a.ep_kind == 2) acc = max(acc, 0);
    res = (uint32_t)acc;
  }
  return res;
}

__global__ void contract_cell_kernel(CArgs a, KWalk ow, int64_t out_positions) {
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < out_positions;
       o += (int64_t)gridDim.x * blockDim.x) {
    int64_t off[3] = {0, 0, 0};
    uint32_t v = 0;
    if (walk_offsets<3>(ow, o, off)) v = contract_cell(a, off[0], off[1], off[2]);
    store_word(a.out, a.out_dt, o, v);
  }
}

// Integer contractions with long residue lists: a warp per output cell, its lanes taking every
// 32nd residue; the wrapping i32 sum does not depend on the order, so the cell is the same.
__global__ void contract_cell_warp_kernel(CArgs a, KWalk ow, int64_t out_positions) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t o = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; o < out_positions; o += nw) {
    int64_t off[3] = {0, 0, 0};
    const bool live = walk_offsets<3>(ow, o, off);
    uint32_t acc = 0;
    if (live)
      for (int64_t r = lane; r < a.nd; r += 32) {
        const int64_t pl = off[0] + a.dl[r], pr = off[1] + a.dr[r];
        if (pl < a.lhs_elems && pr < a.rhs_elems)
          acc += (uint32_t)((int32_t)load_word(a.lhs, a.in_dt, pl) * (int32_t)load_word(a.rhs, a.in_dt, pr));
      }
#pragma unroll
    for (int m = 16; m; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
    if (lane == 0) store_word(a.out, a.out_dt, o, live ? int_finish(a, (int32_t)acc, off[2]) : 0u);
  }
}

// i8 x i8 contractions whose residue is one fully live run of unit stride in both operands (a
// dense dot product per cell, e.g. [B, I] x [H, I]): a warp per cell reads both rows as 16-byte
// vectors and multiplies four byte pairs per instruction (dp4a). The i32 sum wraps like the fold's,
// and integer sums do not depend on their order. Cells whose rows are not 16-byte aligned, or
// reach past either operand, take the per-element loop.
__global__ void contract_dense_i8_warp_kernel(CArgs a, KWalk ow, int64_t out_positions, int64_t K) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int8_t* lhs = (const int8_t*)a.lhs;
  const int8_t* rhs = (const int8_t*)a.rhs;
  for (int64_t o = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; o < out_positions; o += nw) {
    int64_t off[3] = {0, 0, 0};
    const bool live = walk_offsets<3>(ow, o, off);
    uint32_t acc = 0;  // wraps, as the fold's sum does
    if (live) {
      const int64_t pl = off[0], pr = off[1];
      const bool inside = pl >= 0 && pr >= 0 && pl + K <= a.lhs_elems && pr + K <= a.rhs_elems;
      const bool vec = inside && ((((uintptr_t)(lhs + pl)) | ((uintptr_t)(rhs + pr))) & 15) == 0;
      int64_t r0 = 0;
      if (vec) {
        const int4* x = (const int4*)(lhs + pl);
        const int4* w = (const int4*)(rhs + pr);
        const int64_t nv = K >> 4;
        for (int64_t v = lane; v < nv; v += 32) {
          const int4 xa = x[v], wa = w[v];
          acc = (uint32_t)__dp4a(xa.x, wa.x, (int)acc);
          acc = (uint32_t)__dp4a(xa.y, wa.y, (int)acc);
          acc = (uint32_t)__dp4a(xa.z, wa.z, (int)acc);
          acc = (uint32_t)__dp4a(xa.w, wa.w, (int)acc);
        }
        r0 = nv << 4;
      }
      for (int64_t r = r0 + lane; r < K; r += 32) {
        const int64_t il = pl + r, ir = pr + r;
        if (il < a.lhs_elems && ir < a.rhs_elems) acc += (uint32_t)((int32_t)lhs[il] * (int32_t)rhs[ir]);
      }
    }
#pragma unroll
    for (int m = 16; m; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
    if (lane == 0) store_word(a.out, a.out_dt, o, live ? int_finish(a, (int32_t)acc, off[2]) : 0u);
  }
}

__global__ void contract_cell_nibble_kernel(CArgs a, KWalk ow, int64_t out_positions) {
  for (int64_t by = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; by * 2 < out_positions;
       by += (int64_t)gridDim.x * blockDim.x) {
    uint32_t b = 0;
    for (int h = 0; h < 2; ++h) {
      int64_t o = by * 2 + h;
      if (o >= out_positions) break;
      int64_t off[3] = {0, 0, 0};
      uint32_t v = 0;
      if (walk_offsets<3>(ow, o, off)) v = contract_cell(a, off[0], off[1], off[2]);
      b |= (v & 15u) << (4 * h);
    }
    ((uint8_t*)a.out)[by] = (uint8_t)b;
  }
}

bool int_in_host(int dt) {
  return dt == FOPT_I8 || dt == FOPT_I4 || dt == FOPT_I5 || dt == FOPT_I9 || dt == FOPT_I16 || dt == FOPT_I32;
}

int grid_for(int64_t work) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, 148 * 32));
}

}  // namespace

// Live residue deltas in walk order, for `m` memories, in device memory owned by the plan: uploaded
// on first use and kept, so a launch captured into a CUDA graph reads a table that outlives it.
static const int64_t* upload_deltas(fopt_ctx* ctx, const FoldKPlan& p, int nmem, int64_t* count) {
  std::lock_guard<std::mutex> g(p.dev_mu);
  if (p.dev_deltas[nmem - 1]) {
    *count = p.dev_count[nmem - 1];
    return p.dev_deltas[nmem - 1];
  }
  if (ctx->capture) throw Fail{FOPT_ERR_INVALID, "a reduce / contraction plan first used inside a capture: run the step once before capturing"};
  const KWalk& rw = p.residue;
  std::vector<int64_t> d[3];
  int64_t n = 1;
  for (int i = 0; i < rw.n; ++i) n *= rw.extent[i];
  std::vector<int64_t> digit(rw.n, 0);
  for (int64_t r = 0; r < n; ++r) {
    int64_t q = r;
    bool live = true;
    int64_t off[3] = {0, 0, 0};
    for (int i = 0; i < rw.n; ++i) {
      int64_t dd = q % rw.extent[i];
      q /= rw.extent[i];
      live &= dd < rw.live[i];
      for (int m = 0; m < nmem; ++m) off[m] += dd * rw.stride[m][i];
    }
    if (!live) continue;
    for (int m = 0; m < nmem; ++m) d[m].push_back(off[m]);
  }
  *count = (int64_t)d[0].size();
  size_t bytes = sizeof(int64_t) * d[0].size() * nmem;
  int64_t* dev = nullptr;
  cuda_check(cudaMalloc(&dev, std::max<size_t>(bytes, 16)), "delta table alloc");
  for (int m = 0; m < nmem; ++m)
    cuda_check(cudaMemcpy(dev + m * d[0].size(), d[m].data(), sizeof(int64_t) * d[m].size(), cudaMemcpyHostToDevice),
               "upload deltas");
  p.dev_deltas[nmem - 1] = dev;
  p.dev_count[nmem - 1] = *count;
  return dev;
}

void launch_reduce(fopt_ctx* ctx, const FoldKPlan& p, void* out, const void* src, int dtype, int op, uint32_t ident,
                   int64_t src_elems) {
  // Unit-stride single-run residue and an order-insensitive fold -> warp per cell.
  bool order_free = (dtype == FOPT_I32 && op != FOPT_RED_ADD_SAT) || (dtype == FOPT_F32 && !ctx->exact_fold) ||
                    (dtype != FOPT_BF16 && (op == FOPT_RED_MAX || op == FOPT_RED_MIN));
  bool unit_run = p.residue.n == 1 && p.residue.live[0] == p.residue.extent[0] && p.residue.stride[0][0] == 1;
  if (order_free && unit_run && p.residue_live >= 32) {
    int64_t warps_per_block = 8;
    int grid = (int)std::max<int64_t>(1, std::min<int64_t>((p.out_positions + 7) / warps_per_block, 148 * 64));
    reduce_warp_kernel<<<grid, 256, 0, ctx->stream>>>(out, src, dtype, op, ident, p.out, p.out_positions,
                                                      p.residue_live, src_elems);
    launched(ctx, "reduce_warp");
    return;
  }
  int64_t nd;
  const int64_t* delta = upload_deltas(ctx, p, 1, &nd);
  reduce_cell_kernel<<<grid_for(p.out_positions), 256, 0, ctx->stream>>>(out, src, dtype, op, ident, p.out,
                                                                          p.out_positions, delta, nd, src_elems);
  launched(ctx, "reduce_cell");
}

void launch_contraction_generic(fopt_ctx* ctx, const FoldKPlan& p, void* out, int out_dt, const void* lhs,
                                const void* rhs, int in_dt, int64_t lhs_elems, int64_t rhs_elems,
                                const fopt_epilogue* ep, const int64_t*, const float* scale) {
  int64_t nd;
  const int64_t* d = upload_deltas(ctx, p, 2, &nd);
  CArgs a{};
  a.out = out;
  a.out_dt = out_dt;
  a.lhs = lhs;
  a.rhs = rhs;
  a.in_dt = in_dt;
  a.lhs_elems = lhs_elems;
  a.rhs_elems = rhs_elems;
  a.dl = d;
  a.dr = d + nd;
  a.nd = nd;
  a.ep_kind = ep ? ep->kind : 0;
  a.int_width = ep ? ep->int_width : 31;
  a.clip_lo = ep ? ep->clip_lo : INT32_MIN;
  a.clip_hi = ep ? ep->clip_hi : INT32_MAX;
  a.scale = scale;
  if (dtype_bits(out_dt) == 4) {
    contract_cell_nibble_kernel<<<grid_for((p.out_positions + 1) / 2), 256, 0, ctx->stream>>>(a, p.out,
                                                                                               p.out_positions);
  } else if (in_dt == FOPT_I8 && p.residue.n == 1 && p.residue.live[0] == p.residue.extent[0] &&
             p.residue.stride[0][0] == 1 && p.residue.stride[1][0] == 1 && nd >= 32 &&
             !getenv("FOPT_FOLD_NO_DENSE")) {
    contract_dense_i8_warp_kernel<<<grid_for(p.out_positions * 32), 256, 0, ctx->stream>>>(a, p.out, p.out_positions,
                                                                                         p.residue.extent[0]);
  } else if (int_in_host(in_dt) && nd >= 32) {
    contract_cell_warp_kernel<<<grid_for(p.out_positions * 32), 256, 0, ctx->stream>>>(a, p.out, p.out_positions);
  } else {
    contract_cell_kernel<<<grid_for(p.out_positions), 256, 0, ctx->stream>>>(a, p.out, p.out_positions);
  }
  launched(ctx, "contract_cell");
}

// Live residue deltas of memory 0 computed on the host (walk order), without touching device memory.
std::vector<int64_t> host_deltas(const KWalk& rw) {
  std::vector<int64_t> d;
  int64_t n = 1;
  for (int i = 0; i < rw.n; ++i) n *= rw.extent[i];
  for (int64_t r = 0; r < n; ++r) {
    int64_t q = r, off = 0;
    bool live = true;
    for (int i = 0; i < rw.n; ++i) {
      int64_t dd = q % rw.extent[i];
      q /= rw.extent[i];
      live &= dd < rw.live[i];
      off += dd * rw.stride[0][i];
    }
    if (live) d.push_back(off);
  }
  return d;
}

// The per-cell reduce over a delta list the caller has already placed in device memory.
void launch_reduce_cells(fopt_ctx* ctx, const FoldKPlan& p, void* out, const void* src, int dtype, int op,
                         uint32_t ident, int64_t src_elems, const int64_t* d_delta, int64_t nd) {
  reduce_cell_kernel<<<grid_for(p.out_positions), 256, 0, ctx->stream>>>(out, src, dtype, op, ident, p.out,
                                                                          p.out_positions, d_delta, nd, src_elems);
  launched(ctx, "reduce_cell");
}

}  // namespace fopt
