// Tensor-core contraction for GEMM-shaped BufStorage::contraction_in calls
// (furiosa-opt-std/src/storage/buf.rs:401-447): D[M, N] = sum_k A[M, k] * B[N, k], both operands
// K-major in HBM, on the 5th-generation tensor cores.
//
//   * int8 x int8 -> s32 (tcgen05.mma kind::i8) and bf16 x bf16 -> f32 (kind::f16) accumulate in
//     TMEM (Tensor Memory); the accumulator is exact for int8 (s32, K <= 2^17 at |x| <= 128), so the
//     result is bit-identical to the reference's per-cell i32 fold.
//   * Operands stream HBM -> shared memory through TMA (cp.async.bulk.tensor, 128-byte swizzle) into
//     a 4-stage ring; one elected thread issues the MMAs; a tcgen05.commit per stage frees the slot.
//   * Persistent CTAs (one per SM, 320 threads): warp 0 = TMA producer, warp 1 = MMA issuer (and
//     TMEM owner), warps 2-9 = epilogue. Two TMEM accumulators (2 x BN columns) let the epilogue
//     of tile i overlap the MMAs of tile i+1.
//   * The epilogue fuses the narrow that follows the fold: i32 -> i8 wrap, f32 -> bf16 (RNE, flush,
//     NaN canonical), or the vector-engine requant chain FxpToFp -> MulF(scale[n]) -> FpToFxp ->
//     Clip -> i8, each in the reference's exact arithmetic.
//   * Every wait is bounded (about 2 s of %globaltimer); on expiry the CTA records an error code
//     in the context's device error word and leaves its loops, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <mutex>
#include <vector>

#include "ctx.hpp"
#include "ew_ops.cuh"

namespace fopt {
namespace gemm {

constexpr int BM = 128;
constexpr int BKB = 128;  // bytes of K per stage row (one 128-byte swizzle atom row)
constexpr int STAGES = 4;
constexpr int EPI_WARPS = 8;  // two per TMEM lane quarter, splitting the columns
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr uint64_t kWaitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// The same test, but a thread whose phase has not completed sleeps until it does (or for at most
// the hint, 20 us) instead of returning at once: waiting warps then leave the issue slots to the
// warps doing work.
__device__ __forceinline__ bool mbar_try_sleep(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(20000)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and raises the shared abort flag) after ~kWaitNs.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int code) {
  if (mbar_try(bar, parity)) return true;
  uint64_t t0 = globaltimer();
  for (;;) {
    if (mbar_try_sleep(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > kWaitNs) {
      *abort_flag = 1;
      atomicExch(err, code);
      return false;
    }
  }
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          dst),
      "l"((uint64_t)map), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row core-matrix groups 1024 B apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFF) >> 4);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset
  d |= (uint64_t)1 << 46;             // descriptor version (sm100)
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void mma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

#define R32(i) "=r"(r[i])
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : R32(0), R32(1), R32(2), R32(3), R32(4), R32(5), R32(6), R32(7), R32(8), R32(9), R32(10), R32(11), R32(12),
        R32(13), R32(14), R32(15), R32(16), R32(17), R32(18), R32(19), R32(20), R32(21), R32(22), R32(23), R32(24),
        R32(25), R32(26), R32(27), R32(28), R32(29), R32(30), R32(31)
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// The load alone, and a wait that takes the loaded registers as operands, so that no use of them
// can be scheduled before it: a chunk's load stays in flight while the previous chunk is processed.
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : R32(0), R32(1), R32(2), R32(3), R32(4), R32(5), R32(6), R32(7), R32(8), R32(9), R32(10), R32(11), R32(12),
        R32(13), R32(14), R32(15), R32(16), R32(17), R32(18), R32(19), R32(20), R32(21), R32(22), R32(23), R32(24),
        R32(25), R32(26), R32(27), R32(28), R32(29), R32(30), R32(31)
      : "r"(taddr));
}
#define RW32(i) "+r"(r[i])
__device__ __forceinline__ void tmem_wait32(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : RW32(0), RW32(1), RW32(2), RW32(3), RW32(4), RW32(5), RW32(6), RW32(7), RW32(8), RW32(9), RW32(10),
                 RW32(11), RW32(12), RW32(13), RW32(14), RW32(15), RW32(16), RW32(17), RW32(18), RW32(19), RW32(20),
                 RW32(21), RW32(22), RW32(23), RW32(24), RW32(25), RW32(26), RW32(27), RW32(28), RW32(29), RW32(30),
                 RW32(31)
               :
               : "memory");
}
#undef RW32
#define W32(i) "r"(r[i])
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      W32(0), W32(1), W32(2), W32(3), W32(4), W32(5), W32(6), W32(7), W32(8), W32(9), W32(10), W32(11), W32(12),
      W32(13), W32(14), W32(15), W32(16), W32(17), W32(18), W32(19), W32(20), W32(21), W32(22), W32(23), W32(24),
      W32(25), W32(26), W32(27), W32(28), W32(29), W32(30), W32(31)
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
#undef W32
#undef R32

struct Params {
  void* D;
  int M, N, K;  // K in elements
  int64_t ldd;  // elements
  int out_dt;   // FOPT_I8 / FOPT_I32 / FOPT_BF16 / FOPT_F32
  int ep_kind;  // 0 none, 1 requant, 2 relu
  const float* scale;
  int int_width, clip_lo, clip_hi;
  const float* row_scale;
  const uint16_t* residual;  // EP_DQ: optional bf16 [M, N] added after the cast (same ldd as D)
  int* err;
  // split of the last wave (paired kernel): tiles [n_whole, ntiles) each run as `split` K-ranges;
  // every range leaves its partial accumulator in ws, and the last range to finish adds them up
  // and runs the epilogue (cnt: one arrival counter per split tile, CTA and epilogue warp)
  int n_whole, split;
  // or (halves = 1) the last wave's tiles [n_whole, ntiles) each run as two half-width tiles (BN / 2
  // columns), which fill up to twice as many pairs in half the time; no partials are involved
  int halves;
  uint32_t* ws;
  uint32_t* cnt;
  int trace_units;
  uint64_t* trace;  // diagnostics (FOPT_GEMM_TRACE): per unit {mma start, mma end, epilogue start, end,
                    // first chunk loaded from TMEM (whole tiles) or SM id (split ranges)}
};

// One unit of the paired kernel's persistent loop: a whole tile, or one K-range of a split tile.
struct Unit {
  int tile, kb0, kb1, part, sp;  // sp: index among the split tiles (-1 for a whole tile)
  int nh;                        // half-width unit: which half of the tile's columns (-1: all of them)
};
__device__ __forceinline__ Unit unit_of(const Params& p, int u, int kblocks) {
  Unit w;
  w.nh = -1;
  if (u < p.n_whole) {
    w.tile = u; w.kb0 = 0; w.kb1 = kblocks; w.part = 0; w.sp = -1;
  } else if (p.halves) {
    const int v = u - p.n_whole;
    w.tile = p.n_whole + (v >> 1); w.nh = v & 1; w.kb0 = 0; w.kb1 = kblocks; w.part = 0; w.sp = -1;
  } else {
    const int v = u - p.n_whole;
    w.sp = v / p.split;
    w.part = v - w.sp * p.split;
    w.tile = p.n_whole + w.sp;
    // K-range boundaries at (q * (S + q) ) / (2 S^2 ... ) are skewed so that range q ends before q + 1:
    // the share of range q is proportional to (7 + 2 q), e.g. 7/16 : 9/16 for two ranges.
    auto edge = [&](int q) {
      const int64_t num = (int64_t)q * 7 + (int64_t)q * (q - 1);  // sum_{i<q} (7 + 2 i)
      const int64_t den = (int64_t)p.split * 7 + (int64_t)p.split * (p.split - 1);
      return (int)((int64_t)kblocks * num / den);
    };
    w.kb0 = edge(w.part);
    w.kb1 = edge(w.part + 1);
  }
  return w;
}

// Epilogue modes, one specialised kernel each so the epilogue code stays small:
//   EP_I8    i32 accumulator -> i8 (the `as i8` wrap), optional relu
//   EP_WIDE  raw accumulator (i32 / f32), optional relu
//   EP_RQ31  requant at int_width 31 with clip bounds exact in f32 (the fast exact form below)
//   EP_RQ    requant at any int_width (bit-level fixed-point restatement)
//   EP_BF16  f32 accumulator -> bf16 (RNE, flush, canonical NaN), optional relu (cast_relu)
//   EP_DQ    dequant: f32(acc) * row_scale[m] * scale[n] -> bf16 (FxpToFp, two MulF, cast)
//   EP_SWIGLU  the gate / up projections of a SwiGLU in one GEMM: the B rows interleave 128 gate
//            rows and 128 up rows, so a 256-wide tile holds matching gate and up columns; each pair
//            is dequantised and cast to bf16 as EP_DQ does, then act = (g * sigmoid(g)) * u in f32
//            (the elementwise program's operations) is written to the [M, N / 2] f32 output
enum { EP_I8 = 0, EP_WIDE = 1, EP_RQ31 = 2, EP_RQ = 3, EP_BF16 = 4, EP_DQ = 5, EP_SWIGLU = 6 };

// The requant chain FxpToFp -> MulF(s) -> FpToFxp -> Clip at int_width 31, for clip bounds exact in
// f32 (float/mod.rs:22-34 for float_to_fixedpoint):
//   * FxpToFp(31) is IEEE round-to-nearest int -> f32, and the product is one f32 multiply;
//   * a NaN saturates by its sign, then clips. A NaN scale is the x86 product itself (the operand
//     comes back unchanged) and is handled per column by the caller; the only other NaN is 0 * inf,
//     whose x86 result is the negative default NaN, i.e. the low bound. fmaxf(NaN, lo) = lo gives
//     exactly that, so clipping in f32 first also covers the saturation;
//   * round half away from zero of the clipped value y is trunc(RZ(y + copysign(0.5, y))): adding
//     with round-toward-zero never crosses an integer, and all integers in range are floats.
__device__ __forceinline__ int32_t requant31(int32_t acc, float s, float lo, float hi) {
  float y = fminf(fmaxf(__fmul_rn(__int2float_rn(acc), s), lo), hi);
  const float h = __uint_as_float((__float_as_uint(y) & 0x80000000u) | 0x3f000000u);
  return __float2int_rz(__fadd_rz(y, h));
}
// The same chain for a NaN scale: the product is that NaN, which saturates by its sign.
__device__ __forceinline__ int32_t requant31_nan_scale(float s, int32_t lo, int32_t hi) {
  return (__float_as_uint(s) >> 31) ? lo : hi;
}

// Epilogue for 32 consecutive columns of one row.
// csc: the 32 column scales of this chunk (global or shared memory); rs: the row's scale (EP_DQ).
// nanmask: bit j set when column j's scale is a NaN (requant modes).
template <bool IS_F16, int MODE>
__device__ __forceinline__ void epilogue_store(const Params& p, int row, int col, const uint32_t* r,
                                               const float* csc, float rs, uint32_t nanmask) {
  uint8_t* base = (uint8_t*)p.D;
  const bool relu = p.ep_kind == 2;
  if constexpr (MODE == EP_I8 || MODE == EP_RQ31 || MODE == EP_RQ) {
    float sc[32];
    if constexpr (MODE != EP_I8) {
      const float4* s4 = (const float4*)csc;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 v = s4[q];
        sc[4 * q] = v.x; sc[4 * q + 1] = v.y; sc[4 * q + 2] = v.z; sc[4 * q + 3] = v.w;
      }
    }
    const float flo = (float)p.clip_lo, fhi = (float)p.clip_hi;
    uint32_t packed[8];
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      uint32_t w = 0;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        int32_t acc = (int32_t)r[j + t];
        int32_t q;
        if constexpr (MODE == EP_RQ31) {
          q = requant31(acc, sc[j + t], flo, fhi);
          if (nanmask & (1u << (j + t))) q = requant31_nan_scale(sc[j + t], p.clip_lo, p.clip_hi);
        } else if constexpr (MODE == EP_RQ) {
          // x86 products return a NaN operand unchanged and make 0 * inf the negative default NaN
          float sv = sc[j + t];
          float y = __fmul_rn(__uint_as_float(fxp_to_fp_bits(acc, (uint32_t)p.int_width)), sv);
          if (y != y) y = sv != sv ? sv : __uint_as_float(0xffc00000u);
          q = max(p.clip_lo, min(p.clip_hi, fp_to_fxp(y, (uint32_t)p.int_width)));
        } else {
          q = relu ? max(acc, 0) : acc;
        }
        w |= ((uint32_t)q & 0xffu) << (8 * t);
      }
      packed[j / 4] = w;
    }
    uint4* dst = (uint4*)(base + (int64_t)row * p.ldd + col);
    dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  } else if constexpr (MODE == EP_WIDE) {
    uint4* dst = (uint4*)(base + ((int64_t)row * p.ldd + col) * 4);
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      uint32_t v[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        if (!relu) v[t] = r[j + t];
        else if (IS_F16) v[t] = __float_as_uint(fmaxf(__uint_as_float(r[j + t]), 0.0f));
        else v[t] = (uint32_t)max((int32_t)r[j + t], 0);
      }
      dst[j / 4] = make_uint4(v[0], v[1], v[2], v[3]);
    }
  } else {  // EP_BF16, EP_DQ
    uint32_t rr[32];
    if constexpr (MODE == EP_DQ) {
      const float4* s4 = (const float4*)csc;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 v = s4[q];
        const float sv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          float y = __fmul_rn(__int2float_rn((int32_t)r[4 * q + t]), rs);
          rr[4 * q + t] = __float_as_uint(__fmul_rn(y, sv[t]));
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) rr[j] = r[j];
    }
    uint32_t packed[16];
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      uint32_t a = rr[j], b = rr[j + 1];
      if (relu) {  // commit_cast_relu: negative non-NaN values become +0
        if ((a & 0x7fffffffu) <= 0x7f800000u && (a >> 31)) a = 0u;
        if ((b & 0x7fffffffu) <= 0x7f800000u && (b >> 31)) b = 0u;
      }
      packed[j / 2] = bf16x2_rule(__uint_as_float(a), __uint_as_float(b));
    }
    if (MODE == EP_DQ && p.residual) {
      // the residual add that follows the projection: bf16(f32(x) + f32(o)), o the bf16 just formed
      const uint4* xr = (const uint4*)(p.residual + (int64_t)row * p.ldd + col);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 xv = xr[q];
        const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const uint32_t o = packed[4 * q + t], x = xs[t];
          packed[4 * q + t] = bf16x2_rule(__fadd_rn(__uint_as_float(x << 16), __uint_as_float(o << 16)),
                                          __fadd_rn(__uint_as_float(x & 0xffff0000u), __uint_as_float(o & 0xffff0000u)));
        }
      }
    }
    uint4* dst = (uint4*)(base + ((int64_t)row * p.ldd + col) * 2);
#pragma unroll
    for (int q = 0; q < 4; ++q)
      dst[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
  }
}

template <bool IS_F16, int BN, int MODE>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
  constexpr int A_BYTES = BM * BKB;
  constexpr int B_BYTES = BN * BKB;
  constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr int KSTEP_BYTES = 32;  // K bytes per MMA (int8: 32 elements; bf16: 16 elements)
  constexpr uint32_t TMEM_COLS = 2 * BN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = (uint64_t*)(smem + STAGES * STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = bars + 2 * STAGES + 2;
  uint32_t* tmem_slot = (uint32_t*)(bars + 2 * STAGES + 4);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_m = p.M / BM, tiles_n = p.N / BN;
  const int ntiles = tiles_m * tiles_n;
  const int kblocks = p.K * (IS_F16 ? 2 : 1) / BKB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&acc_full[a]), 1);
      mbar_init(smem_u32(&acc_empty[a]), 32 * EPI_WARPS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int m0 = (tile % tiles_m) * BM, n0 = (tile / tiles_m) * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag, p.err, 101)) goto done_producer;
          const uint32_t fb = smem_u32(&full[stage]);
          mbar_expect_tx(fb, STAGE_BYTES);
          const int kx = kb * (IS_F16 ? BKB / 2 : BKB);
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          tma_load_2d(sa, &tmA, fb, kx, m0);
          tma_load_2d(sa + A_BYTES, &tmB, fb, kx, n0);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: wait until the MMAs released every slot we filled, so no TMA write is in flight at exit.
      for (int s = 0; s < STAGES; ++s) {
        if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag, p.err, 102)) break;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  done_producer:;
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t idesc;
      if (IS_F16)
        idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
      else
        idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        if (!mbar_wait(smem_u32(&acc_empty[acc]), acc_phase ^ 1, abort_flag, p.err, 103)) break;
        fence_after();
        const uint32_t dcol = tmem_base + (uint32_t)(acc * BN);
        bool aborted = false;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, p.err, 104)) {
            aborted = true;
            break;
          }
          fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint64_t da = smem_desc(sa), db = smem_desc(sa + A_BYTES);
#pragma unroll
          for (int k = 0; k < BKB / KSTEP_BYTES; ++k) {
            const uint64_t adv = (uint64_t)((k * KSTEP_BYTES) >> 4);
            if (IS_F16)
              mma_f16(dcol, da + adv, db + adv, idesc, (kb | k) != 0);
            else
              mma_i8(dcol, da + adv, db + adv, idesc, (kb | k) != 0);
          }
          mma_commit(smem_u32(&empty[stage]));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (aborted) break;
        mma_commit(smem_u32(&acc_full[acc]));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..2+EPI_WARPS) ----------------
    const int sub = warp & 3;  // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;  // which interleaved half of the 32-column chunks
    const int row_in_tile = sub * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      const int m0 = (tile % tiles_m) * BM, n0 = (tile / tiles_m) * BN;
      bool ok = mbar_wait(smem_u32(&acc_full[acc]), acc_phase, abort_flag, p.err, 105);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      fence_after();
      const uint32_t tbase = tmem_base + (uint32_t)(acc * BN) + ((uint32_t)(sub * 32) << 16);
#pragma unroll 1
      for (int c = half; c < BN / 32; c += EPI_WARPS / 4) {
        uint32_t r[32];
        tmem_ld32(tbase + (uint32_t)(c * 32), r);
        const float* csc = p.scale ? p.scale + n0 + c * 32 : nullptr;
        const uint32_t nanmask = MODE == EP_RQ31 ? __ballot_sync(0xffffffffu, __ldg(csc + lane) != __ldg(csc + lane)) : 0u;
        epilogue_store<IS_F16, MODE>(p, m0 + row_in_tile, n0 + c * 32, r, csc,
                                     MODE == EP_DQ ? __ldg(p.row_scale + m0 + row_in_tile) : 0.0f, nanmask);
      }
      fence_before();
      mbar_arrive(smem_u32(&acc_empty[acc]));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
  }
}

// ---------------------------------------------------------------------------------------------
// Paired-SM variant (cta_group::2): a cluster of two CTAs computes a 256 x 256 tile. Each CTA streams
// its own 128 rows of A and its own 128 rows of B (half of N) into a 6-stage ring of 32 KiB slices;
// the even CTA issues tcgen05.mma.cta_group::2 (M = 256), which reads both CTAs' shared memory and
// leaves rows [128 r, 128 r + 128) of the accumulator in CTA r's TMEM. Per SM this halves the B
// bytes streamed per MMA compared with the single-CTA kernel.
//   full[s]      (even CTA): both CTAs' TMA bytes land here (cta_group::2 TMA signals the pair's barrier)
//   empty[s]     (each CTA): arrival from the MMA commit, delivered to both CTAs of the pair
//   acc_full[a]  (each CTA): MMA commit after the tile's last k-block, delivered to both
//   acc_empty[a] (even CTA): one arrival per epilogue warp of both CTAs (16)
// ---------------------------------------------------------------------------------------------
// EP_SWIGLU for one 32-column chunk: rg / ru the gate and up accumulators of the same 32 output
// columns, cg / cu their channel scales, rs the row's scale; writes 32 f32 activations at col.
__device__ __forceinline__ void swiglu_store(const Params& p, int row, int col, const uint32_t* rg, const uint32_t* ru,
                                             const float* cg, const float* cu, float rs) {
  float4* dst = (float4*)((float*)p.D + (int64_t)row * p.ldd + col);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 g4 = ((const float4*)cg)[q], u4 = ((const float4*)cu)[q];
    const float gs[4] = {g4.x, g4.y, g4.z, g4.w}, us[4] = {u4.x, u4.y, u4.z, u4.w};
    float yg[4], yu[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      yg[t] = __fmul_rn(__fmul_rn(__int2float_rn((int32_t)rg[4 * q + t]), rs), gs[t]);
      yu[t] = __fmul_rn(__fmul_rn(__int2float_rn((int32_t)ru[4 * q + t]), rs), us[t]);
    }
    // the bf16 projections, read back as f32 (a bf16 is its bits << 16)
    const uint32_t g01 = bf16x2_rule(yg[0], yg[1]), g23 = bf16x2_rule(yg[2], yg[3]);
    const uint32_t u01 = bf16x2_rule(yu[0], yu[1]), u23 = bf16x2_rule(yu[2], yu[3]);
    const float g[4] = {__uint_as_float(g01 << 16), __uint_as_float(g01 & 0xffff0000u), __uint_as_float(g23 << 16),
                        __uint_as_float(g23 & 0xffff0000u)};
    const float u[4] = {__uint_as_float(u01 << 16), __uint_as_float(u01 & 0xffff0000u), __uint_as_float(u23 << 16),
                        __uint_as_float(u23 & 0xffff0000u)};
    float a[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) a[t] = __fmul_rn(__fmul_rn(g[t], fopt::ew::sigmoid_f(g[t])), u[t]);
    dst[q] = make_float4(a[0], a[1], a[2], a[3]);
  }
}

// The operand ring: the mainloop is bound by the bytes in flight from L2 (a half-width tile's
// k-blocks take as long as a whole one's), so the ring takes all the shared memory it can: 7 stages
// at BN = 256 (the column scales are then read from L1 instead of staged), 9 at BN = 128.
constexpr int RING2_BYTES = 224 * 1024;
constexpr int SMEM_LIMIT = 232448;  // dynamic shared memory a CTA may opt in to on sm_100
template <int BN>
constexpr int stages2() {
  return RING2_BYTES / (128 * BKB + (BN / 2) * BKB);
}
template <int BN>
constexpr int scale_stage_bytes2() {  // the epilogue's staged column scales, when they still fit
  return stages2<BN>() * (128 * BKB + (BN / 2) * BKB) + 1024 + 256 + 2 * EPI_WARPS * (BN / 2) * 4 <= SMEM_LIMIT
             ? 2 * EPI_WARPS * (BN / 2) * 4
             : 0;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster, int c0,
                                                 int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void mma2_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma2_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// Commit the issuing thread's MMAs to the barrier at `bar` in both CTAs of the pair (CTA mask 0b11).
__device__ __forceinline__ void mma2_commit_both(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          bar)
      : "memory");
}

// r += one parked K-range partial (32 accumulators; f32 adds in range order for the bf16 kernel).
// Parked K-range partials: each epilogue warp's share of a tile (its 32 rows x BN / 2 columns) is
// one contiguous slice, chunk-major then column then row, so parking is 128-byte coalesced stores
// and fetching is one bulk copy.
template <int BN>
__device__ __forceinline__ uint32_t* partial_slice(const Params& p, int slot, uint32_t rank, int ew) {
  return p.ws + ((int64_t)(slot * 2 + (int)rank) * EPI_WARPS + ew) * (BN / 2) * 32;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
// r (chunk i of this warp) += the staged partial in shared memory.
template <bool IS_F16>
__device__ __forceinline__ void add_staged(uint32_t* r, const uint32_t* stage, int i, int lane) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const uint32_t x = stage[(i * 32 + j) * 32 + lane];
    if (IS_F16) r[j] = __float_as_uint(__fadd_rn(__uint_as_float(r[j]), __uint_as_float(x)));
    else r[j] += x;
  }
}

template <bool IS_F16, int BN, int MODE>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmBh, Params p) {
  constexpr int STAGES2 = stages2<BN>();
  constexpr int A_BYTES = 128 * BKB;
  constexpr int B_BYTES = (BN / 2) * BKB;
  constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr int KSTEP_BYTES = 32;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = (uint64_t*)(smem + STAGES2 * STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES2;
  uint64_t* acc_full = bars + 2 * STAGES2;
  uint64_t* acc_empty = bars + 2 * STAGES2 + 2;
  uint64_t* xbar = bars + 2 * STAGES2 + 4;  // one per epilogue warp: partial fetches
  uint32_t* tmem_slot = (uint32_t*)(bars + 2 * STAGES2 + 4 + EPI_WARPS);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  float* sscale = (float*)(smem + STAGES2 * STAGE_BYTES + 256);  // 2 x EPI_WARPS x BN / 2 column scales

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  if (p.trace && threadIdx.x == 0) p.trace[p.trace_units * 5 + blockIdx.x * 3] = globaltimer();
  const int tiles_m = p.M / 256, tiles_n = p.N / BN;
  const int ntiles = tiles_m * tiles_n;
  const int kblocks = p.K * (IS_F16 ? 2 : 1) / BKB;
  const int nunits = p.n_whole + (ntiles - p.n_whole) * (p.halves ? 2 : p.split);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES2; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&acc_full[a]), 1);
      mbar_init(smem_u32(&acc_empty[a]), 2 * EPI_WARPS);
    }
    for (int e = 0; e < EPI_WARPS; ++e) mbar_init(smem_u32(&xbar[e]), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised before any TMA or remote arrive
  fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int u = pair; u < nunits; u += npairs) {
        const Unit w = unit_of(p, u, kblocks);
        const int m0 = (w.tile % tiles_m) * 256 + (int)rank * 128;
        // each CTA holds half the unit's columns of B: BN / 2 of a whole tile, BN / 4 of a half
        // (through the narrower box of tmBh)
        const int n0 = (w.tile / tiles_m) * BN + (w.nh < 0 ? (int)rank * (BN / 2) : w.nh * (BN / 2) + (int)rank * (BN / 4));
        const CUtensorMap* mB = w.nh < 0 ? &tmB : &tmBh;
        const uint32_t tx = w.nh < 0 ? 2 * STAGE_BYTES : 2 * (A_BYTES + B_BYTES / 2);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag, p.err, 201)) goto done_producer2;
          const uint32_t fb_local = smem_u32(&full[stage]);
          const uint32_t fb_pair = map_to_rank(fb_local, 0);
          if (rank == 0) mbar_expect_tx(fb_local, tx);
          const int kx = kb * (IS_F16 ? BKB / 2 : BKB);
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          tma_load_2d_pair(sa, &tmA, fb_pair, kx, m0);
          tma_load_2d_pair(sa + A_BYTES, mB, fb_pair, kx, n0);
          if (++stage == STAGES2) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      for (int s = 0; s < STAGES2; ++s) {
        if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag, p.err, 202)) break;
        if (++stage == STAGES2) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  done_producer2:;
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      uint32_t idesc;
      if (IS_F16)
        idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
      else
        idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
      const uint32_t idesc_half = (idesc & ~(0x3fu << 17)) | ((uint32_t)(BN >> 4) << 17);  // N = BN / 2
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int u = pair; u < nunits; u += npairs) {
        const Unit w = unit_of(p, u, kblocks);
        const uint32_t id = w.nh < 0 ? idesc : idesc_half;
        if (!mbar_wait(smem_u32(&acc_empty[acc]), acc_phase ^ 1, abort_flag, p.err, 203)) break;
        fence_after();
        if (p.trace) p.trace[u * 5] = globaltimer();
        const uint32_t dcol = tmem_base + (uint32_t)(acc * BN);
        bool aborted = false;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, p.err, 204)) {
            aborted = true;
            break;
          }
          fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint64_t da = smem_desc(sa), db = smem_desc(sa + A_BYTES);
#pragma unroll
          for (int k = 0; k < BKB / KSTEP_BYTES; ++k) {
            const uint64_t adv = (uint64_t)((k * KSTEP_BYTES) >> 4);
            if (IS_F16)
              mma2_f16(dcol, da + adv, db + adv, id, (kb != w.kb0) | (k != 0));
            else
              mma2_i8(dcol, da + adv, db + adv, id, (kb != w.kb0) | (k != 0));
          }
          mma2_commit_both(smem_u32(&empty[stage]));
          if (++stage == STAGES2) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (aborted) break;
        mma2_commit_both(smem_u32(&acc_full[acc]));
        if (p.trace) p.trace[u * 5 + 1] = globaltimer();
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
    __syncwarp();
  } else {
    const int sub = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = (int)rank * 128 + sub * 32 + lane;
    const bool tracer = p.trace && rank == 0 && warp == 2 && lane == 0;
    const uint32_t acc_empty_pair = map_to_rank(smem_u32(&acc_empty[0]), 0);
    constexpr bool kColScale = MODE == EP_RQ31 || MODE == EP_RQ || MODE == EP_DQ || MODE == EP_SWIGLU;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = pair; u < nunits; u += npairs) {
      const Unit w = unit_of(p, u, kblocks);
      const int m0 = (w.tile % tiles_m) * 256, n0 = (w.tile / tiles_m) * BN + (w.nh < 0 ? 0 : w.nh * (BN / 2));
      const int ncols = w.nh < 0 ? BN : BN / 2;
      // Stage this warp's column scales in shared memory while the MMAs run: its own copy, so
      // only the warp synchronises (double-buffered by accumulator). Chunk c = half + 2 i has its
      // 32 scales at wsc + 32 i.
      float* wsc = sscale + (acc * EPI_WARPS + (warp - 2)) * (BN / 2);
      float rs = 0.0f;
      constexpr bool kStaged = scale_stage_bytes2<BN>() > 0;
      if constexpr (kColScale && kStaged) {
#pragma unroll
        for (int i = 0; i < BN / 64; ++i)
          if (i < ncols / 64) wsc[i * 32 + lane] = __ldg(p.scale + n0 + (half + 2 * i) * 32 + lane);
        __syncwarp();
      }
      if constexpr (MODE == EP_DQ || MODE == EP_SWIGLU) rs = __ldg(p.row_scale + m0 + row_in_tile);
      bool ok = mbar_wait(smem_u32(&acc_full[acc]), acc_phase, abort_flag, p.err, 205);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      fence_after();
      if (tracer) p.trace[u * 5 + 2] = globaltimer();
      const uint32_t tbase = tmem_base + (uint32_t)(acc * BN) + ((uint32_t)(sub * 32) << 16);
      uint32_t* ctr = nullptr;
      bool finish = w.sp < 0;  // this unit runs the epilogue straight from TMEM
      if (!finish) {
        // Have all other K-ranges of this tile already parked their partials? Then this range adds
        // them to its own accumulator and runs the epilogue without parking its own.
        ctr = p.cnt + ((int64_t)w.sp * 2 + rank) * EPI_WARPS + (warp - 2);
        uint32_t seen = 0;
        if (lane == 0) asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(seen) : "l"(ctr) : "memory");
        finish = __shfl_sync(0xffffffffu, seen, 0) == (uint32_t)(p.split - 1);
        if (finish) __threadfence();
      }
      // A split unit is always its pair's last unit (the split ranges fill the last wave), so by
      // now the operand ring is idle: each warp stages fetched partials in its own 16 KiB of it.
      const int ew = warp - 2;
      const uint32_t xb = smem_u32(&xbar[ew]);
      const uint32_t* stage = (const uint32_t*)(smem + ew * (BN / 2) * 32 * 4);
      uint32_t xphase = 0;
      // Fetch the partial of range q into this warp's staging slice; false if the wait expired.
      auto fetch = [&](int q) {
        constexpr uint32_t bytes = (BN / 2) * 32 * 4;
        if (lane == 0) {
          asm volatile("fence.proxy.async;" ::: "memory");
          mbar_expect_tx(xb, bytes);
          bulk_g2s(smem_u32(stage), partial_slice<BN>(p, w.sp * p.split + q, rank, ew), bytes, xb);
        }
        __syncwarp();
        const bool got = __all_sync(0xffffffffu, mbar_wait(xb, xphase, abort_flag, p.err, 206));
        xphase ^= 1;
        return got;
      };
      // After reading a staged slice: order those reads before the next bulk write into it.
      auto release_stage = [&]() {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
      };
      if (w.sp >= 0 && !finish) {
        // park this range's partial, then count this warp's arrival: every lane's partial is
        // visible device-wide before the count, so the range that counts last sees all of them
        uint32_t* mine = partial_slice<BN>(p, w.sp * p.split + w.part, rank, ew);
#pragma unroll 1
        for (int i = 0; i < BN / 64; ++i) {
          uint32_t r[32];
          tmem_ld32(tbase + (uint32_t)((half + 2 * i) * 32), r);
#pragma unroll
          for (int j = 0; j < 32; ++j) __stcg(mine + (i * 32 + j) * 32 + lane, r[j]);
        }
        __threadfence();
        __syncwarp();
        uint32_t last = 0;
        if (lane == 0) last = atomicAdd(ctr, 1u) == (uint32_t)(p.split - 1);
        finish = __shfl_sync(0xffffffffu, last, 0) != 0;
        if (finish) __threadfence();
      }
      if (finish) {
        bool good = true;
        int q_last = p.split - 1;
        if (w.sp >= 0 && q_last == w.part) --q_last;
        // Split unit: add the other ranges' partials (ascending range order) to this range's
        // accumulator, through TMEM for all but the last one.
        for (int q = 0; w.sp >= 0 && q < q_last && good; ++q) {
          if (q == w.part) continue;
          good = fetch(q);
#pragma unroll 1
          for (int i = 0; i < BN / 64 && good; ++i) {
            uint32_t r[32];
            const uint32_t ta = tbase + (uint32_t)((half + 2 * i) * 32);
            tmem_ld32(ta, r);
            add_staged<IS_F16>(r, stage, i, lane);
            tmem_st32(ta, r);
          }
          release_stage();
        }
        if (w.sp >= 0 && good) good = fetch(q_last);
        if constexpr (MODE == EP_SWIGLU) {
          // gate chunk c (c < BN / 64) pairs with up chunk c + BN / 64: same warp, same parity
#pragma unroll 1
          for (int c = half; good && c < BN / 64; c += EPI_WARPS / 4) {
            uint32_t rg[32], ru[32];
            tmem_ld32(tbase + (uint32_t)(c * 32), rg);
            tmem_ld32(tbase + (uint32_t)((c + BN / 64) * 32), ru);
            if (w.sp >= 0) {
              add_staged<IS_F16>(rg, stage, (c - half) >> 1, lane);
              add_staged<IS_F16>(ru, stage, (c + BN / 64 - half) >> 1, lane);
            }
            const float* cg = kStaged ? wsc + (c - half) * 16 : p.scale + n0 + c * 32;
            const float* cu = kStaged ? wsc + (c + BN / 64 - half) * 16 : p.scale + n0 + (c + BN / 64) * 32;
            swiglu_store(p, m0 + row_in_tile, n0 / 2 + c * 32, rg, ru, cg, cu, rs);
          }
        } else if (good) {
          // This warp's chunks are c = half + 2 i (i < nch); chunk i + 1's TMEM load is in flight
          // while chunk i is converted and stored.
          const int nch = ncols / 64;
          auto chunk = [&](int i, uint32_t* r) {
            const int c = half + 2 * i;
            if (tracer && w.sp < 0 && i == 0) p.trace[u * 5 + 4] = globaltimer();
            if (w.sp >= 0) add_staged<IS_F16>(r, stage, i, lane);
            const float* csc = kStaged ? wsc + (c - half) * 16 : p.scale + n0 + c * 32;
            const uint32_t nanmask = MODE == EP_RQ31 ? __ballot_sync(0xffffffffu, csc[lane] != csc[lane]) : 0u;
            epilogue_store<IS_F16, MODE>(p, m0 + row_in_tile, n0 + c * 32, r, csc, rs, nanmask);
          };
          auto taddr = [&](int i) { return tbase + (uint32_t)((half + 2 * i) * 32); };
          uint32_t ra[32], rb[32];
          tmem_ld32_nowait(taddr(0), ra);
          tmem_wait32(ra);
#pragma unroll 1
          for (int i = 0; i < nch; i += 2) {
            const bool n1 = i + 1 < nch, n2 = i + 2 < nch;
            if (n1) tmem_ld32_nowait(taddr(i + 1), rb);
            chunk(i, ra);
            if (n1) {
              tmem_wait32(rb);
              if (n2) tmem_ld32_nowait(taddr(i + 2), ra);
              chunk(i + 1, rb);
              if (n2) tmem_wait32(ra);
            }
          }
        }
        if (w.sp >= 0) {
          release_stage();
          if (lane == 0) atomicExch(ctr, 0u);  // every other range has counted: reset for the next launch
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_pair + (uint32_t)(acc * sizeof(uint64_t)));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
      if (tracer) {
        uint32_t smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        p.trace[u * 5 + 3] = globaltimer();
        if (w.sp >= 0) p.trace[u * 5 + 4] = smid;
      }
    }
  }

  fence_before();
  cluster_sync_all();  // no CTA leaves while its pair may still read its smem or signal its barriers
  fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
    if (p.trace && lane == 0) p.trace[p.trace_units * 5 + blockIdx.x * 3 + 2] = globaltimer();
  }
  if (p.trace && threadIdx.x == 0) p.trace[p.trace_units * 5 + blockIdx.x * 3 + 1] = globaltimer();
}

// ---- host side ----
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  });
  if (!fn) throw Fail{FOPT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable"};
  return fn;
}

CUtensorMap make_map(const void* base, bool f16, int64_t inner, int64_t outer, int64_t ld_elems, int box_outer) {
  CUtensorMap m;
  const int esz = f16 ? 2 : 1;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(ld_elems * esz)};
  cuuint32_t box[2] = {(cuuint32_t)(BKB / esz), (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, f16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                           const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Fail{FOPT_ERR_CUDA, "cuTensorMapEncodeTiled failed"};
  return m;
}

template <bool IS_F16, int BN, int MODE>
void launch(fopt_ctx* ctx, const CUtensorMap& a, const CUtensorMap& b, const Params& p) {
  constexpr int smem = STAGES * (BM * BKB + BN * BKB) + 1024 + 256;
  static bool attr = false;
  if (!attr) {
    cuda_check(cudaFuncSetAttribute(gemm_tc_kernel<IS_F16, BN, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
               "gemm smem attribute");
    attr = true;
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device);
  int tiles = (p.M / BM) * (p.N / BN);
  int grid = std::min(tiles, sms);
  gemm_tc_kernel<IS_F16, BN, MODE><<<grid, THREADS, smem, ctx->stream>>>(a, b, p);
  launched(ctx, "gemm_tc");
}

// Split of the last wave: when the tiles leave the last round over the SM pairs less than half
// full, its tiles run as `split` K-ranges each on the idle pairs. Returns the number of ranges
// (1 = no split) and sizes the workspace and counters.
int plan_split(fopt_ctx* ctx, Params& p, int ntiles, int pairs, int kblocks, int bn, bool f32_acc) {
  p.n_whole = ntiles;
  p.split = 1;
  p.halves = 0;
  p.ws = nullptr;
  p.cnt = nullptr;
  const int rem = ntiles % pairs;
  if (rem == 0) return 1;
  // Without a K split, a last wave that fills at most half the pairs runs as half-width tiles: the
  // same columns on twice the pairs, in about half the time.
  auto halves = [&]() {
    if (ntiles > pairs && 2 * rem <= pairs && !getenv("FOPT_GEMM_NO_HALVES")) {
      p.n_whole = ntiles - rem;
      p.halves = 1;
    }
    return 1;
  };
  if (getenv("FOPT_GEMM_NO_SPLIT")) return halves();
  // Parking and fetching a partial costs about one epilogue (a few microseconds), so the split pays
  // when the ranges it shortens are long: a single part-filled wave, or a long K.
  // (at 4096^3 a 2-way split of the last wave measured 62.5 us against 59.7 us for half-width tiles)
  const int min_kb = getenv("FOPT_GEMM_SPLIT_MIN_KB") ? atoi(getenv("FOPT_GEMM_SPLIT_MIN_KB")) : 96;
  if (!(ntiles < pairs ? kblocks >= 16 : kblocks >= min_kb)) return halves();
  // f32 partials: two ranges only, whose sum is the same whichever range finishes last
  const int split = std::min({pairs / rem, kblocks / 4, f32_acc ? 2 : 4});
  if (split < 2) return halves();
  const size_t ws_bytes = (size_t)rem * split * 256 * bn * 4;
  const size_t n_cnt = (size_t)rem * 2 * EPI_WARPS;
  if (ws_bytes > ctx->gemm_ws_bytes) {
    release_ctx_buffer(ctx, ctx->gemm_ws);
    cuda_check(cudaMalloc(&ctx->gemm_ws, ws_bytes), "gemm workspace alloc");
    ctx->gemm_ws_bytes = ws_bytes;
  }
  if (n_cnt > ctx->gemm_cnt_n) {
    release_ctx_buffer(ctx, ctx->gemm_cnt);
    cuda_check(cudaMalloc(&ctx->gemm_cnt, n_cnt * 4), "gemm counters alloc");
    ctx->gemm_cnt_n = n_cnt;
    ctx->gemm_cnt_dirty = true;
  }
  if (ctx->gemm_cnt_dirty) {  // fresh, or a launch may have left mid-count after a timeout
    cuda_check(cudaMemsetAsync(ctx->gemm_cnt, 0, ctx->gemm_cnt_n * 4, ctx->stream), "gemm counters clear");
    ctx->gemm_cnt_dirty = false;
  }
  p.n_whole = ntiles - rem;
  p.split = split;
  p.ws = (uint32_t*)ctx->gemm_ws;
  p.cnt = ctx->gemm_cnt;
  return split;
}

template <bool IS_F16, int BN, int MODE>
void launch2(fopt_ctx* ctx, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& bh, Params p) {
  constexpr int smem = stages2<BN>() * (128 * BKB + (BN / 2) * BKB) + 1024 + 256 + scale_stage_bytes2<BN>();
  static_assert(smem <= SMEM_LIMIT, "paired GEMM shared memory");
  static bool attr = false;
  if (!attr) {
    cuda_check(cudaFuncSetAttribute(gemm_tc2_kernel<IS_F16, BN, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
               "gemm2 smem attribute");
    attr = true;
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device);
  const int tiles = (p.M / 256) * (p.N / BN);
  const int split = plan_split(ctx, p, tiles, sms / 2, p.K * (IS_F16 ? 2 : 1) / BKB, BN, IS_F16);
  if (MODE == EP_SWIGLU && p.halves) {  // a half-width unit would hold gate or up columns only
    p.halves = 0;
    p.n_whole = tiles;
  }
  const int units = p.n_whole + (tiles - p.n_whole) * (p.halves ? 2 : split);
  const int pairs = std::min(units, sms / 2);
  const char* trace_path = getenv("FOPT_GEMM_TRACE");
  p.trace = nullptr;
  p.trace_units = units;
  if (trace_path) cuda_check(cudaMallocAsync((void**)&p.trace, units * 40 + 2 * pairs * 24, ctx->stream), "trace alloc");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = 2;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 1;
  cuda_check(cudaLaunchKernelEx(&cfg, gemm_tc2_kernel<IS_F16, BN, MODE>, a, b, bh, p), "gemm_tc2 launch");
  launched(ctx, "gemm_tc2");
  if (trace_path) {  // diagnostics only: append "unit mma0 mma1 epi0 epi1 sm" lines (ns from the first start)
    std::vector<uint64_t> t((size_t)units * 5 + 2 * pairs * 3);
    cuda_check(cudaMemcpyAsync(t.data(), p.trace, t.size() * 8, cudaMemcpyDeviceToHost, ctx->stream), "trace copy");
    cuda_check(cudaStreamSynchronize(ctx->stream), "trace sync");
    cudaFreeAsync(p.trace, ctx->stream);
    uint64_t t0 = ~0ull;
    for (int u = 0; u < units; ++u) t0 = std::min(t0, t[u * 5]);
    if (FILE* f = fopen(trace_path, "a")) {
      uint64_t e0 = ~0ull, e1 = 0, x1 = 0;
      for (int b = 0; b < 2 * pairs; ++b) {
        e0 = std::min(e0, t[units * 5 + b * 3]);
        e1 = std::max(e1, t[units * 5 + b * 3]);
        x1 = std::max(x1, t[units * 5 + b * 3 + 1]);
      }
      fprintf(f, "# M=%d N=%d K=%d units=%d whole=%d split=%d entry_first=%lld entry_last=%lld exit_last=%lld\n", p.M,
              p.N, p.K, units, p.n_whole, p.split, (long long)(e0 - t0), (long long)(e1 - t0), (long long)(x1 - t0));
      for (int u = 0; u < units; ++u)
        fprintf(f, "%d %llu %llu %llu %llu %llu\n", u, (unsigned long long)(t[u * 5] - t0),
                (unsigned long long)(t[u * 5 + 1] - t0), (unsigned long long)(t[u * 5 + 2] - t0),
                (unsigned long long)(t[u * 5 + 3] - t0),
                (unsigned long long)(t[u * 5 + 4] > t0 ? t[u * 5 + 4] - t0 : t[u * 5 + 4]));
      fclose(f);
    }
  }
}

// Tile width of the paired kernel: 256 whenever N allows. The narrower tile streams 1.5x the
// L2 -> shared-memory bytes per MMA (96 vs 64 bytes per SM-cycle at the full int8 rate), which on
// B200 costs more than its fuller last wave gains; the last wave is evened out by the K split.
int pair_tile_n(int max_bn) {
  if (const char* e = getenv("FOPT_GEMM_BN")) {
    int v = atoi(e);
    if ((v == 128 || v == 256) && v <= max_bn) return v;
  }
  return max_bn;
}

}  // namespace gemm

bool launch_gemm_tc(fopt_ctx* ctx, void* out, int out_dt, const void* a, const void* b, int in_dt, int64_t M,
                    int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldd, const fopt_epilogue* ep,
                    const float* scale, int scale_along_n) {
  using namespace gemm;
  const bool f16 = in_dt == FOPT_BF16;
  if (!(in_dt == FOPT_I8 || f16)) return false;
  if (getenv("FOPT_DISABLE_TC")) return false;
  const int esz = f16 ? 2 : 1;
  if (M % BM || K * esz % BKB || M > (1 << 30) || N > (1 << 30) || K > (1 << 30)) return false;
  int bn = N % 256 == 0 ? 256 : (N % 128 == 0 ? 128 : 0);
  if (!bn) return false;
  if ((uintptr_t)a % 16 || (uintptr_t)b % 16 || (uintptr_t)out % 16) return false;
  if ((lda * esz) % 16 || (ldb * esz) % 16) return false;
  int ep_kind = ep ? ep->kind : 0;
  if (ep_kind == 1 && !scale_along_n) return false;
  int odt = out_dt;
  int osz = dtype_bits(odt) / 8;
  if ((ldd * osz) % 16) return false;
  Params p{};
  p.D = out;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.ldd = ldd;
  p.out_dt = odt;
  p.ep_kind = ep_kind;
  p.scale = scale;
  p.int_width = ep ? ep->int_width : 31;
  p.clip_lo = ep ? ep->clip_lo : INT32_MIN;
  p.clip_hi = ep ? ep->clip_hi : INT32_MAX;
  p.err = ctx->dev_err;
  p.row_scale = ep ? ep->row_scale : nullptr;
  int mode;
  if (f16) {
    if (odt == FOPT_BF16) mode = EP_BF16;
    else if (odt == FOPT_F32) mode = EP_WIDE;
    else return false;
  } else if (ep_kind == 4) {
    if ((uintptr_t)scale % 16 || !p.row_scale || odt != FOPT_F32 || N % 256 || M % 256 ||
        getenv("FOPT_GEMM_1SM"))
      return false;
    mode = EP_SWIGLU;
  } else if (ep_kind == 3 || ep_kind == 5) {
    if ((uintptr_t)scale % 16 || !p.row_scale || odt != FOPT_BF16) return false;
    if (ep_kind == 5) {
      if (!ep->residual || (uintptr_t)ep->residual % 16) return false;
      p.residual = (const uint16_t*)ep->residual;
    }
    mode = EP_DQ;
  } else if (ep_kind == 1) {
    if ((uintptr_t)scale % 16) return false;
    const int64_t lim = 1 << 24;
    bool fast = p.int_width == 31 && p.clip_lo >= -lim && p.clip_hi <= lim && p.clip_lo <= p.clip_hi;
    mode = fast ? EP_RQ31 : EP_RQ;
  } else if (odt == FOPT_I8) {
    mode = EP_I8;
  } else if (odt == FOPT_I32) {
    mode = EP_WIDE;
  } else {
    return false;
  }
  const bool pair = M % 256 == 0 && bn && !getenv("FOPT_GEMM_1SM");
  if (pair) bn = pair_tile_n(bn);
  CUtensorMap ma = make_map(a, f16, K, M, lda, pair ? 128 : BM);
  CUtensorMap mb = make_map(b, f16, K, N, ldb, pair ? bn / 2 : bn);
  CUtensorMap mbh = pair ? make_map(b, f16, K, N, ldb, bn / 4) : mb;  // half-width tail tiles
  if (mode == EP_SWIGLU) {
    if (!pair || bn != 256) return false;
    launch2<false, 256, EP_SWIGLU>(ctx, ma, mb, mbh, p);
    return true;
  }
#define FOPT_GEMM_DISPATCH(F16, MODE)                                     \
  if (pair && bn == 256) launch2<F16, 256, MODE>(ctx, ma, mb, mbh, p);    \
  else if (pair) launch2<F16, 128, MODE>(ctx, ma, mb, mbh, p);            \
  else if (bn == 256) launch<F16, 256, MODE>(ctx, ma, mb, p);        \
  else launch<F16, 128, MODE>(ctx, ma, mb, p);
  if (f16) {
    if (mode == EP_BF16) { FOPT_GEMM_DISPATCH(true, EP_BF16) }
    else { FOPT_GEMM_DISPATCH(true, EP_WIDE) }
  } else {
    switch (mode) {
      case EP_RQ31: { FOPT_GEMM_DISPATCH(false, EP_RQ31) } break;
      case EP_RQ: { FOPT_GEMM_DISPATCH(false, EP_RQ) } break;
      case EP_I8: { FOPT_GEMM_DISPATCH(false, EP_I8) } break;
      case EP_DQ: { FOPT_GEMM_DISPATCH(false, EP_DQ) } break;
      default: { FOPT_GEMM_DISPATCH(false, EP_WIDE) } break;
    }
  }
#undef FOPT_GEMM_DISPATCH
  return true;
}

}  // namespace fopt
