// Tensor-core fused attention (tcgen05 + TMEM + TMA), the sm_100a path of fopt_attention:
// softmax(Q K^T * scale + causal mask) V with the online softmax of the reference's chunked op chain
// (furiosa-opt-examples/src/transformer/kernel/attention.rs:32-392: qk_scaled, row_max, masked_exp,
// row_sum + EPS, weighted_sum, online rescale, norm).
//
// One CTA per (batch, query head, 128-row query block); 192 threads:
//   warp 0   TMA producer: Q once, then K and V tiles (128 keys) into a 2-stage ring;
//   warp 1   TMEM owner and single-thread MMA issuer: S_j = Q K_j^T (M=N=K=128, bf16 -> f32) into one of
//            two TMEM S buffers, then O += P_j V_j into the TMEM O accumulator;
//   warps 2-5 softmax: one thread per query row reads its 128 scores from TMEM (no cross-thread
//            reduction), keeps the running max / sum in registers, rescales its O row in TMEM when the
//            max grows, and writes P_j (bf16) into shared memory in the UMMA K-major 128B-swizzle layout.
// S_{j+1} is issued before waiting for P_j, so the QK^T of the next block overlaps this block's
// softmax. V is read in its own [B, S, Hkv, D] layout: the PV product takes it as an MN-major B
// operand (D contiguous), so no transposed copy is made.
// Every wait is bounded (~2 s of %globaltimer) and reports through the context's device error word.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <mutex>
#include <vector>

#include "ctx.hpp"

namespace fopt {
namespace attn {

constexpr int BQ = 128, BK = 128, D = 128;
constexpr int STAGES = 2;
constexpr int THREADS = 192;
constexpr int TILE = BQ * D * 2;    // one 128 x 128 bf16 tile = 32 KiB (two 128-byte-row chunks)
constexpr int CHUNK = TILE / 2;     // 128 rows x 128 B
constexpr uint64_t kWaitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
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

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int code) {
  if (mbar_try(bar, parity)) return true;
  uint64_t t0 = gtimer();
  for (;;) {
    if (mbar_try_sleep(bar, parity)) return true;
    if (*abort_flag) return false;
    if (gtimer() - t0 > kWaitNs) {
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
__device__ __forceinline__ void tma3(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(dst),
      "l"((uint64_t)map), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// Tiled TMA store shared -> global (bulk async group of the issuing thread).
__device__ __forceinline__ void tma3_store(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"((uint64_t)map),
               "r"(src), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ uint64_t sdesc(uint32_t addr) {
  uint64_t d = (uint64_t)((addr & 0x3FFFF) >> 4);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// V [keys, D] as the PV product's B operand read MN-major (D contiguous) straight from its natural
// layout: each 64-wide half of D is one TMA box of 128 keys x 128 bytes, 128-byte swizzled in 8-key
// atoms. Leading byte offset = the distance between the two D halves (one box), stride byte offset =
// the distance between 8-key atoms (1024 bytes); a 16-key MMA step starts 16 x 128 bytes further on.
__device__ __forceinline__ uint64_t vdesc(uint32_t addr) {
  uint64_t d = (uint64_t)((addr & 0x3FFFF) >> 4);
  d |= (uint64_t)(16384 >> 4) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
constexpr uint32_t kIdescBMajorMN = 1u << 16;  // instruction descriptor: B operand MN-major
__device__ __forceinline__ void mma_bf16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

#define R32(i) "=r"(r[i])
__device__ __forceinline__ void tld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : R32(0), R32(1), R32(2), R32(3), R32(4), R32(5), R32(6), R32(7), R32(8), R32(9), R32(10), R32(11), R32(12),
        R32(13), R32(14), R32(15), R32(16), R32(17), R32(18), R32(19), R32(20), R32(21), R32(22), R32(23), R32(24),
        R32(25), R32(26), R32(27), R32(28), R32(29), R32(30), R32(31)
      : "r"(taddr));
}
#undef R32
#define S32(i) "r"(r[i])
__device__ __forceinline__ void tst32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      S32(0), S32(1), S32(2), S32(3), S32(4), S32(5), S32(6), S32(7), S32(8), S32(9), S32(10), S32(11), S32(12),
      S32(13), S32(14), S32(15), S32(16), S32(17), S32(18), S32(19), S32(20), S32(21), S32(22), S32(23), S32(24),
      S32(25), S32(26), S32(27), S32(28), S32(29), S32(30), S32(31)
      : "memory");
}
#undef S32
#define S16(i) "r"(r[i])
__device__ __forceinline__ void tst16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      S16(0), S16(1), S16(2), S16(3), S16(4), S16(5), S16(6), S16(7), S16(8), S16(9), S16(10), S16(11), S16(12),
      S16(13), S16(14), S16(15)
      : "memory");
}
#undef S16
// tcgen05.wait::ld that also ties the 32 destination registers of the loads it completes, so the
// compiler cannot move their uses above it.
#define T32(i) "+r"(r[i])
__device__ __forceinline__ void tld_wait_regs(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : T32(0), T32(1), T32(2), T32(3), T32(4), T32(5), T32(6), T32(7), T32(8), T32(9), T32(10), T32(11),
                 T32(12), T32(13), T32(14), T32(15), T32(16), T32(17), T32(18), T32(19), T32(20), T32(21), T32(22),
                 T32(23), T32(24), T32(25), T32(26), T32(27), T32(28), T32(29), T32(30), T32(31)
               :
               : "memory");
}
#undef T32
__device__ __forceinline__ void tld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tst_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

struct Params {
  uint16_t* O;
  int B, S, Hq, Hkv;
  int causal;
  float scale_log2;  // scale * log2(e)
  float eps;
  int* err;
  int pv_wait;      // 1: issue S_t(j+1) only after PV_t(j) has completed (FOPT_ATTN_PV_WAIT, for comparison)
  uint64_t* trace;  // diagnostics (FOPT_ATTN_TRACE): per CTA 128 stamps, see attention_tc2_kernel
};

// 2^x on the special-function unit (relative error ~2^-22; the scores' bf16 rounding dominates).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Blackwell's three-input max and packed f32 pair arithmetic (two independent IEEE operations).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float m;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
  return m;
}
__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack_f32x2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// Two f32 -> packed bf16x2 with one round-to-nearest-even conversion instruction.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// Packs two f32 into bf16x2 under the reference's conversion rule.
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) { return bf16x2_rule(lo, hi); }

__global__ void __launch_bounds__(THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = smem;                       // 32 KiB
  uint8_t* sP = smem + TILE;                // 32 KiB
  uint8_t* sKV = smem + 2 * TILE;           // STAGES x (K tile + V tile)
  uint64_t* bars = (uint64_t*)(smem + 2 * TILE + STAGES * 2 * TILE);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = bars + 1 + STAGES;
  uint64_t* s_full = bars + 1 + 2 * STAGES;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_ready = s_free + 2;
  uint64_t* o_done = p_ready + 1;
  uint32_t* tmem_slot = (uint32_t*)(o_done + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = p.S / BQ;
  // longest work first across the grid (the last query blocks under causal masking)
  const int bh = (int)(blockIdx.x % (p.B * p.Hq));
  const int qb = nqb - 1 - (int)(blockIdx.x / (p.B * p.Hq));
  const int h = bh % p.Hq;
  const int b = bh / p.Hq;
  const int hk = h / (p.Hq / p.Hkv);
  const int nkb = p.causal ? qb + 1 : p.S / BK;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&kv_full[s]), 1);
      mbar_init(smem_u32(&kv_empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&s_full[s]), 1);
      mbar_init(smem_u32(&s_free[s]), 128);
    }
    mbar_init(smem_u32(p_ready), 128);
    mbar_init(smem_u32(o_done), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS[2] = {tmem, tmem + 128};
  const uint32_t tO = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      const int row0 = b * p.S;  // flattened (batch, seq) row of the tensor maps
      const uint32_t qb_ = smem_u32(q_full);
      mbar_expect_tx(qb_, TILE);
      tma3(smem_u32(sQ), &tmQ, qb_, 0, h, row0 + qb * BQ);
      tma3(smem_u32(sQ + CHUNK), &tmQ, qb_, 64, h, row0 + qb * BQ);
      for (int j = 0; j < nkb; ++j) {
        const int st = j % STAGES;
        if (!mbar_wait(smem_u32(&kv_empty[st]), ((j / STAGES) & 1) ^ 1, abort_flag, p.err, 301)) break;
        const uint32_t fb = smem_u32(&kv_full[st]);
        mbar_expect_tx(fb, 2 * TILE);
        uint8_t* sK = sKV + st * 2 * TILE;
        uint8_t* sV = sK + TILE;
        tma3(smem_u32(sK), &tmK, fb, 0, hk, row0 + j * BK);
        tma3(smem_u32(sK + CHUNK), &tmK, fb, 64, hk, row0 + j * BK);
        tma3(smem_u32(sV), &tmV, fb, 0, hk, row0 + j * BK);
        tma3(smem_u32(sV + CHUNK), &tmV, fb, 64, hk, row0 + j * BK);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(128 >> 3) << 17) |
                             ((uint32_t)(128 >> 4) << 24);
      bool ok = mbar_wait(smem_u32(q_full), 0, abort_flag, p.err, 302);
      auto issue_s = [&](int j) -> bool {
        const int st = j % STAGES, buf = j & 1;
        if (!mbar_wait(smem_u32(&kv_full[st]), (j / STAGES) & 1, abort_flag, p.err, 303)) return false;
        if (j >= 2 && !mbar_wait(smem_u32(&s_free[buf]), ((j - 2) >> 1) & 1, abort_flag, p.err, 304)) return false;
        fence_after();
        const uint32_t sK = smem_u32(sKV + st * 2 * TILE);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (uint32_t)((k >> 2) * CHUNK + (k & 3) * 32);
          mma_bf16(tS[buf], sdesc(smem_u32(sQ) + off), sdesc(sK + off), idesc, k != 0);
        }
        commit(smem_u32(&s_full[buf]));
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < nkb; ++j) {
        if (j + 1 < nkb && !issue_s(j + 1)) break;
        if (!mbar_wait(smem_u32(p_ready), j & 1, abort_flag, p.err, 305)) break;
        fence_after();
        const int st = j % STAGES;
        const uint32_t sV = smem_u32(sKV + st * 2 * TILE + TILE);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (uint32_t)((k >> 2) * CHUNK + (k & 3) * 32);
          mma_bf16(tO, sdesc(smem_u32(sP) + off), vdesc(sV + 2048 * k), idesc | kIdescBMajorMN, (j | k) != 0);
        }
        commit(smem_u32(&kv_empty[st]));
        commit(smem_u32(o_done));
      }
    }
    __syncwarp();
  } else {
    // ---------------- softmax: one thread per query row ----------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // row within the block = TMEM lane
    const int qrow = qb * BQ + r;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      const int buf = j & 1;
      ok = mbar_wait(smem_u32(&s_full[buf]), (j >> 1) & 1, abort_flag, p.err, 306);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      fence_after();
      uint32_t s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tld32(tS[buf] + lane_base + c * 32, s + 32 * c);
      tld_wait();
      fence_before();
      mbar_arrive(smem_u32(&s_free[buf]));
      // row max of the raw scores; the causal mask only touches the diagonal block (a CTA-uniform branch)
      const bool diag = p.causal && j == qb;
      float mx = -INFINITY;
      if (diag) {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          if (c > r) s[c] = __float_as_uint(-INFINITY);
          mx = fmaxf(mx, __uint_as_float(s[c]));
        }
      } else {
#pragma unroll
        for (int c = 0; c < 128; ++c) mx = fmaxf(mx, __uint_as_float(s[c]));
      }
      // p = 2^(s * scale*log2(e) - m), the running max m kept in scaled log2 units
      const float mnew = fmaxf(m, mx * p.scale_log2);
      const float alpha = ex2(m - mnew);  // m = -inf on the first block -> alpha = 0
      float sum = 0.0f;
      uint32_t* pk = s;  // packed bf16 pairs overwrite the scores in place (index c / 2 <= c)
#pragma unroll
      for (int c = 0; c < 128; c += 2) {
        const float p0 = ex2(fmaf(__uint_as_float(s[c]), p.scale_log2, -mnew));
        const float p1 = ex2(fmaf(__uint_as_float(s[c + 1]), p.scale_log2, -mnew));
        sum += p0 + p1;
        pk[c / 2] = pack_bf16x2(p0, p1);
      }
      l = l * alpha + sum;
      m = mnew;
      // PV_{j-1} must be complete: P smem is free and the O row is stable
      if (j > 0) {
        ok = mbar_wait(smem_u32(o_done), (j - 1) & 1, abort_flag, p.err, 307);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        fence_after();
        // tcgen05.ld / st are warp-collective (.sync.aligned): the whole warp rescales when any row
        // of it needs to, rows whose max did not move multiply by 1.
        if (__any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tld32(tO + lane_base + c * 32, o);
            tld_wait();
#pragma unroll
            for (int t = 0; t < 32; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * alpha);
            tst32(tO + lane_base + c * 32, o);
          }
          tst_wait();
        }
      }
      // P row -> shared memory, K-major 128B swizzle: chunk = key / 64, 16-byte unit u ^ (row % 8)
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int chunk = u >> 3, unit = u & 7;
        uint4* dst = (uint4*)(sP + chunk * CHUNK + r * 128 + ((unit ^ (r & 7)) << 4));
        *dst = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      fence_before();
      mbar_arrive(smem_u32(p_ready));
    }
    if (ok && nkb > 0) {
      ok = mbar_wait(smem_u32(o_done), (nkb - 1) & 1, abort_flag, p.err, 308);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok && qrow < p.S) {
      fence_after();
      const float inv = 1.0f / (l + p.eps);
      uint16_t* orow = p.O + (((int64_t)b * p.S + qrow) * p.Hq + h) * D;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tld32(tO + lane_base + c * 32, o);
        tld_wait();
        uint4* dst = (uint4*)(orow + c * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(pack_bf16(__uint_as_float(o[8 * q]) * inv, __uint_as_float(o[8 * q + 1]) * inv),
                              pack_bf16(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv),
                              pack_bf16(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv),
                              pack_bf16(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv));
      }
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}

// ---------------------------------------------------------------------------------------------
// Two query tiles per CTA (ping-pong), P kept in tensor memory.
//
// One CTA per (batch, query head, pair of adjacent 128-row query blocks); 320 threads:
//   warp 0     TMA producer: both Q tiles once, then K and V tiles into a 2-stage ring that both
//              query tiles read;
//   warp 1     TMEM owner and MMA issuer, in the order S0(0) S1(0) | PV0(j) S0(j+1) PV1(j) S1(j+1) ...:
//              S_t = Q_t K^T into TMEM, and O_t += P_t V with P_t read from TMEM (the A operand);
//   warps 2-5  softmax of query tile 0, warps 6-9 of tile 1: one thread per row reads its scores from
//              TMEM, keeps the running max / sum, rescales its O row when the max grows, and writes
//              the bf16 probabilities back over the first 64 columns of its S row (tcgen05.st).
// While one tile's softmax runs, the tensor cores work on the other tile. P_t shares S_t's columns;
// S_t(j+1) is issued right behind PV_t(j), which the tensor pipe runs first (MMAs of one issuing
// thread execute in order).
// TMEM columns: S0 [0, 128), S1 [128, 256), O0 [256, 384), O1 [384, 512).
// ---------------------------------------------------------------------------------------------
constexpr int THREADS2 = 320;

__device__ __forceinline__ void mma_bf16_ta(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}

__global__ void __launch_bounds__(THREADS2, 1)
    attention_tc2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = smem;               // 2 x 32 KiB (tile t at sQ + t * TILE)
  uint8_t* sKV = smem + 2 * TILE;   // STAGES x (K tile + V tile)
  uint64_t* bars = (uint64_t*)(smem + 2 * TILE + STAGES * 2 * TILE);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;  // K and V of a stage are released separately: K after both S MMAs
  uint64_t* k_empty = k_full + STAGES;
  uint64_t* v_full = k_empty + STAGES;
  uint64_t* v_empty = v_full + STAGES;
  uint64_t* s_full = v_empty + STAGES;  // [2] per tile
  uint64_t* p_ready = s_full + 2;        // [2]
  uint64_t* pv_done = p_ready + 2;       // [2]
  uint32_t* tmem_slot = (uint32_t*)(pv_done + 2);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int npair = p.S / (2 * BQ);
  // Longest work first across the whole grid: the B * Hq heaviest pairs (the last query blocks under
  // causal masking) take the lowest block indices, then the next heaviest, and so on, so the blocks
  // the hardware schedules last, as SMs free up, are the shortest.
  const int bh = (int)(blockIdx.x % (p.B * p.Hq));
  const int qp = npair - 1 - (int)(blockIdx.x / (p.B * p.Hq));
  const int h = bh % p.Hq;
  const int b = bh / p.Hq;
  const int hk = h / (p.Hq / p.Hkv);
  const int qb0 = 2 * qp;  // tile t covers query block qb0 + t
  uint64_t* tr = p.trace ? p.trace + (int64_t)blockIdx.x * 128 : nullptr;
  if (tr && threadIdx.x == 0) tr[0] = gtimer();
  // last key block of each tile (inclusive)
  const int last0 = p.causal ? qb0 : p.S / BK - 1;
  const int last1 = p.causal ? qb0 + 1 : p.S / BK - 1;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&k_full[s]), 1);
      mbar_init(smem_u32(&k_empty[s]), 2);
      mbar_init(smem_u32(&v_full[s]), 1);
      mbar_init(smem_u32(&v_empty[s]), 2);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(smem_u32(&s_full[t]), 1);
      mbar_init(smem_u32(&p_ready[t]), 128);
      mbar_init(smem_u32(&pv_done[t]), 1);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const int row0 = b * p.S;  // flattened (batch, seq) row of the tensor maps
      const uint32_t qf = smem_u32(q_full);
      mbar_expect_tx(qf, 2 * TILE);
      for (int t = 0; t < 2; ++t) {
        tma3(smem_u32(sQ + t * TILE), &tmQ, qf, 0, h, row0 + (qb0 + t) * BQ);
        tma3(smem_u32(sQ + t * TILE + CHUNK), &tmQ, qf, 64, h, row0 + (qb0 + t) * BQ);
      }
      for (int j = 0; j <= last1; ++j) {
        const int st = j % STAGES;
        const uint32_t ph = ((j / STAGES) & 1) ^ 1;
        uint8_t* sK = sKV + st * 2 * TILE;
        uint8_t* sV = sK + TILE;
        if (!mbar_wait(smem_u32(&k_empty[st]), ph, abort_flag, p.err, 311)) break;
        const uint32_t kb = smem_u32(&k_full[st]);
        mbar_expect_tx(kb, TILE);
        tma3(smem_u32(sK), &tmK, kb, 0, hk, row0 + j * BK);
        tma3(smem_u32(sK + CHUNK), &tmK, kb, 64, hk, row0 + j * BK);
        if (!mbar_wait(smem_u32(&v_empty[st]), ph, abort_flag, p.err, 319)) break;
        const uint32_t vb = smem_u32(&v_full[st]);
        mbar_expect_tx(vb, TILE);
        tma3(smem_u32(sV), &tmV, vb, 0, hk, row0 + j * BK);
        tma3(smem_u32(sV + CHUNK), &tmV, vb, 64, hk, row0 + j * BK);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(128 >> 3) << 17) |
                             ((uint32_t)(128 >> 4) << 24);
      const uint32_t sQ0 = smem_u32(sQ);
      auto issue_s = [&](int t, int j) {  // S_t = Q_t K_j^T
        const uint32_t sK = smem_u32(sKV + (j % STAGES) * 2 * TILE);
        const uint32_t sq = sQ0 + t * TILE;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (uint32_t)((k >> 2) * CHUNK + (k & 3) * 32);
          mma_bf16(tmem + t * 128, sdesc(sq + off), sdesc(sK + off), idesc, k != 0);
        }
        commit(smem_u32(&s_full[t]));
      };
      auto issue_pv = [&](int t, int j) {  // O_t += P_t V_j, P_t in TMEM columns [128 t, 128 t + 64)
        const uint32_t sV = smem_u32(sKV + (j % STAGES) * 2 * TILE + TILE);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          mma_bf16_ta(tmem + 256 + t * 128, tmem + t * 128 + 8 * k, vdesc(sV + 2048 * k), idesc | kIdescBMajorMN,
                      (j | k) != 0);
        }
        commit(smem_u32(&pv_done[t]));
      };
      bool ok = mbar_wait(smem_u32(q_full), 0, abort_flag, p.err, 312) &&
                mbar_wait(smem_u32(&k_full[0]), 0, abort_flag, p.err, 313);
      if (ok) {
        fence_after();
        issue_s(0, 0);
        commit(smem_u32(&k_empty[0]));
        issue_s(1, 0);
        commit(smem_u32(&k_empty[0]));
      }
      for (int j = 0; ok && j <= last1; ++j) {
        for (int t = 0; t < 2 && ok; ++t) {
          const int last = t ? last1 : last0;
          if (j > last) continue;
          const bool solo = t == 1 && j > last0;  // tile 0 does not use this block
          ok = mbar_wait(smem_u32(&p_ready[t]), j & 1, abort_flag, p.err, 314) &&
               mbar_wait(smem_u32(&v_full[j % STAGES]), (j / STAGES) & 1, abort_flag, p.err, 320);
          if (!ok) break;
          fence_after();
          if (tr && t == 0 && j < 14) tr[80 + 3 * j] = gtimer();
          issue_pv(t, j);
          if (tr && t == 0 && j < 14) tr[81 + 3 * j] = gtimer();
          // the K and V "empty" barriers take one commit per tile per block (two from tile 1 for the
          // block tile 0 does not use)
          commit(smem_u32(&v_empty[j % STAGES]));
          if (solo) commit(smem_u32(&v_empty[j % STAGES]));
          if (j + 1 <= last) {
            // S_t(j+1) overwrites the columns PV_t(j) reads P_t from. MMAs issued by one thread run
            // in issue order (tcgen05.mma -> tcgen05.mma is implicitly pipelined), so PV_t(j) has
            // read P_t before S_t(j+1) writes there, and the issuer goes on to the other tile's PV
            // instead of waiting for PV_t(j) to finish.
            ok = (!p.pv_wait || mbar_wait(smem_u32(&pv_done[t]), j & 1, abort_flag, p.err, 315)) &&
                 mbar_wait(smem_u32(&k_full[(j + 1) % STAGES]), ((j + 1) / STAGES) & 1, abort_flag, p.err, 316);
            if (!ok) break;
            fence_after();
            issue_s(t, j + 1);
            if (tr && t == 0 && j < 14) tr[82 + 3 * j] = gtimer();
            commit(smem_u32(&k_empty[(j + 1) % STAGES]));
            if (t == 1 && j + 1 > last0) commit(smem_u32(&k_empty[(j + 1) % STAGES]));
          }
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- softmax: one thread per query row of tile t ----------------
    const int t = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // row within the tile = TMEM lane
    const int qb = qb0 + t;
    const int qrow = qb * BQ + r;
    const int last = t ? last1 : last0;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + t * 128 + lane_base, tO = tmem + 256 + t * 128 + lane_base;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j <= last; ++j) {
      ok = mbar_wait(smem_u32(&s_full[t]), j & 1, abort_flag, p.err, 317);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      fence_after();
      const bool tracer = tr && r == 0 && j < 17;
      if (tracer) tr[40 * t + 1 + 2 * j] = gtimer();
      uint32_t s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tld32(tS + c * 32, s + 32 * c);
      tld_wait();
      const bool diag = p.causal && j == qb;
      if (diag) {
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (c > r) s[c] = __float_as_uint(-INFINITY);
      }
      // Row max with the three-input max (two new scores per instruction, 8 independent chains);
      // scale-and-subtract and the running sums on packed f32 pairs (two independent
      // round-to-nearest operations each, the same results as scalar fmaf / add).
      float mx8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx8[k] = fmaxf(__uint_as_float(s[2 * k]), __uint_as_float(s[2 * k + 1]));
#pragma unroll
      for (int c = 16; c < 128; c += 16)
#pragma unroll
        for (int k = 0; k < 8; ++k) mx8[k] = max3f(mx8[k], __uint_as_float(s[c + 2 * k]), __uint_as_float(s[c + 2 * k + 1]));
      const float mx = max3f(max3f(mx8[0], mx8[1], mx8[2]), max3f(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])) *
                       p.scale_log2;
      // Lazy rescaling: the exponent base m moves only when the block max exceeds it by more than
      // 8 (log2 units), so probabilities stay below 2^8 and O and l share one base; the normalised
      // result is unchanged and the O rescale below becomes rare.
      const float mnew = mx > m + 8.0f ? mx : m;
      const float alpha = ex2(m - mnew);
      const uint64_t scale2 = pack_f32x2(p.scale_log2, p.scale_log2), neg2 = pack_f32x2(-mnew, -mnew);
      uint64_t sum2[4] = {0, 0, 0, 0};
      uint32_t* pk = s;  // packed bf16 pairs overwrite the scores in place (index c / 2 <= c)
#pragma unroll
      for (int c = 0; c < 128; c += 2) {
        float x0, x1;
        unpack_f32x2(fma_f32x2(pack_f32x2(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), scale2, neg2), x0, x1);
        const float p0 = ex2(x0), p1 = ex2(x1);
        const uint64_t pp = pack_f32x2(p0, p1);
        sum2[(c >> 1) & 3] = add_f32x2(sum2[(c >> 1) & 3], pp);
        pk[c / 2] = pack_bf16x2(p0, p1);
      }
      float sa[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) unpack_f32x2(sum2[k], sa[2 * k], sa[2 * k + 1]);
      const float sum = ((sa[0] + sa[1]) + (sa[2] + sa[3])) + ((sa[4] + sa[5]) + (sa[6] + sa[7]));
      l = l * alpha + sum;
      m = mnew;
      // S_t(j) was issued after PV_t(j - 1), and s_full's commit tracks every earlier MMA of the
      // issuer, so PV_t(j - 1) has completed and the O row is stable here
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tld32(tO + c * 32, o);
          tld_wait_regs(o);
#pragma unroll
          for (int q = 0; q < 32; ++q) o[q] = __float_as_uint(__uint_as_float(o[q]) * alpha);
          tst32(tO + c * 32, o);
        }
      }
      tst32(tS, pk);
      tst32(tS + 32, pk + 32);
      tst_wait();
      fence_before();
      mbar_arrive(smem_u32(&p_ready[t]));
      if (tracer) tr[40 * t + 2 + 2 * j] = gtimer();
    }
    if (tr && t == 0 && r == 0) tr[35] = gtimer();
    if (ok) {
      ok = mbar_wait(smem_u32(&pv_done[t]), last & 1, abort_flag, p.err, 318);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (tr && t == 0 && r == 0) tr[37] = gtimer();
    if (ok) {
      fence_after();
      // O row -> this tile's (now idle) Q buffer in the 128-byte-swizzled TMA layout, then each warp
      // stores its 32 rows with two tensor stores: whole 128-byte lines instead of one 16-byte piece
      // per row per lane.
      const float inv = 1.0f / (l + p.eps);
      uint8_t* stage = sQ + t * TILE;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tld32(tO + c * 32, o);
        tld_wait();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int u = c * 4 + q;  // 16-byte unit of the row: columns 8 u .. 8 u + 7
          uint4* dst = (uint4*)(stage + (u >> 3) * CHUNK + r * 128 + (((u & 7) ^ (r & 7)) << 4));
          *dst = make_uint4(pack_bf16(__uint_as_float(o[8 * q]) * inv, __uint_as_float(o[8 * q + 1]) * inv),
                            pack_bf16(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv),
                            pack_bf16(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv),
                            pack_bf16(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv));
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        const int grow = b * p.S + qb * BQ + quarter * 32;
        tma3_store(&tmO, smem_u32(stage + quarter * 32 * 128), 0, h, grow);
        tma3_store(&tmO, smem_u32(stage + CHUNK + quarter * 32 * 128), 64, h, grow);
        bulk_commit();
        bulk_wait_read0();
      }
      __syncwarp();
      if (tr && t == 0 && r == 0) tr[36] = gtimer();
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}


// ---------------------------------------------------------------------------------------------
// Persistent kernel: one query tile at a time per CTA, three S buffers in tensor memory, each row's
// softmax split over two threads.
//
// One CTA per SM. CTA c takes the query tiles c, 2G - 1 - c, 2G + c, ... of the longest-first
// order (G CTAs, the tile list walked back and forth so that every CTA gets about the same number
// of key blocks). The key blocks of all of a CTA's tiles form one sequence g = 0, 1, 2, ...: S(g)
// goes to S buffer g % 3, and the K / V rings, the S buffers and their barriers run on g across
// tile boundaries, so the next tile's first QK^T runs while this tile finishes. 352 threads:
//   warp 0     TMA producer of Q (per tile, once the previous tile's last S has read the Q buffer)
//              and of K tiles into a 3-stage ring; warp 10 produces V tiles into a 2-stage ring;
//   warp 1     TMEM owner and MMA issuer, in the order S(0) S(1) S(2) | PV(g) S(g + 3) ...; the
//              first PV of a tile overwrites O once the previous tile's epilogue has read it;
//   warps 2-9  softmax: warp w reads TMEM lanes 32 (w % 4) .. + 31 (rows), warps 2-5 columns 0-63
//              and warps 6-9 columns 64-127 of each score row. The two threads of a row exchange
//              their partial maxima through shared memory (a 64-thread named barrier per lane
//              quarter), keep their own running sums, and write their 32 packed bf16 probability
//              words over the first 64 columns of the row's S buffer; PV reads P from there. At the
//              end of a tile they normalise the O row and store it (128 bytes per thread).
// TMEM columns: O [0, 128), S buffers [128, 256), [256, 384) and [384, 512). With three S buffers
// S(g + 3) is issued right behind PV(g), so the S a softmax needs next has been computed one softmax
// period earlier; with two, it waited behind PV(g - 1) on every block.
// ---------------------------------------------------------------------------------------------
constexpr int THREADS3 = 352;
constexpr int KST3 = 3, VST3 = 2;  // K and V ring depths
constexpr int NSB = 3;             // S buffers in tensor memory


__device__ __forceinline__ void bar_pair(int id) { asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory"); }

// The k-th query tile of CTA c among `total` (longest first), or -1.
__device__ __forceinline__ int tile_of(int k, int c, int G, int total) {
  const int i = k * G + ((k & 1) ? G - 1 - c : c);
  return i < total ? i : -1;
}

__global__ void __launch_bounds__(THREADS3, 1)
    attention_tc3_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = smem;                   // 32 KiB
  uint8_t* sKr = smem + TILE;           // KST3 K tiles
  uint8_t* sVr = sKr + KST3 * TILE;     // VST3 V tiles
  float* xch = (float*)(sVr + VST3 * TILE);  // [2 parities][2 halves][128 rows]
  float* xl = xch + 2 * 2 * BQ;                                // [2 halves][128 rows] row sums
  uint64_t* bars = (uint64_t*)(xl + 2 * BQ);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;
  uint64_t* k_empty = k_full + KST3;
  uint64_t* v_full = k_empty + KST3;
  uint64_t* v_empty = v_full + VST3;
  uint64_t* s_full = v_empty + VST3;    // [NSB] per S buffer
  uint64_t* p_ready = s_full + NSB;      // [NSB] per S buffer
  uint64_t* pv_done = p_ready + NSB;     // [NSB] PV(g) completes pv_done[g % NSB]
  uint64_t* o_free = pv_done + NSB;      // the epilogue has read O
  uint32_t* tmem_slot = (uint32_t*)(o_free + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = p.S / BQ, BH = p.B * p.Hq, total = BH * nq, G = (int)gridDim.x, c = (int)blockIdx.x;
  auto tile_geo = [&](int idx, int& b, int& h, int& qb, int& last) {
    const int bh = idx % BH;
    qb = nq - 1 - idx / BH;
    h = bh % p.Hq;
    b = bh / p.Hq;
    last = p.causal ? qb : p.S / BK - 1;
  };
  uint64_t* tr = p.trace ? p.trace + (int64_t)blockIdx.x * 128 : nullptr;  // diagnostics (FOPT_ATTN_TRACE)
  if (tr && threadIdx.x == 0) tr[0] = gtimer();

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    mbar_init(smem_u32(q_empty), 1);
    mbar_init(smem_u32(o_free), 256);
    for (int s = 0; s < KST3; ++s) {
      mbar_init(smem_u32(&k_full[s]), 1);
      mbar_init(smem_u32(&k_empty[s]), 1);
    }
    for (int s = 0; s < VST3; ++s) {
      mbar_init(smem_u32(&v_full[s]), 1);
      mbar_init(smem_u32(&v_empty[s]), 1);
    }
    for (int t = 0; t < NSB; ++t) {
      mbar_init(smem_u32(&s_full[t]), 1);
      mbar_init(smem_u32(&p_ready[t]), 256);
      mbar_init(smem_u32(&pv_done[t]), 1);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int k = 0, idx; ok && (idx = tile_of(k, c, G, total)) >= 0; ++k) {
        int b, h, qb, last;
        tile_geo(idx, b, h, qb, last);
        const int hk = h / (p.Hq / p.Hkv), row0 = b * p.S;
        // the previous tile's last S has read the Q buffer
        if (k > 0 && !(ok = mbar_wait(smem_u32(q_empty), (k - 1) & 1, abort_flag, p.err, 341))) break;
        const uint32_t qf = smem_u32(q_full);
        mbar_expect_tx(qf, TILE);
        tma3(smem_u32(sQ), &tmQ, qf, 0, h, row0 + qb * BQ);
        tma3(smem_u32(sQ + CHUNK), &tmQ, qf, 64, h, row0 + qb * BQ);
        for (int j = 0; j <= last; ++j, ++g) {
          const int st = g % KST3;
          const uint32_t ph = ((g / KST3) & 1) ^ 1;
          uint8_t* sK = sKr + st * TILE;
          if (!(ok = mbar_wait(smem_u32(&k_empty[st]), ph, abort_flag, p.err, 331))) break;
          const uint32_t kb = smem_u32(&k_full[st]);
          mbar_expect_tx(kb, TILE);
          tma3(smem_u32(sK), &tmK, kb, 0, hk, row0 + j * BK);
          tma3(smem_u32(sK + CHUNK), &tmK, kb, 64, hk, row0 + j * BK);
        }
      }
    }
  } else if (warp == 10) {
    // V producer: V tiles free up only after their PV, so they run on their own thread and the K
    // loads above are never held behind them
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int k = 0, idx; ok && (idx = tile_of(k, c, G, total)) >= 0; ++k) {
        int b, h, qb, last;
        tile_geo(idx, b, h, qb, last);
        const int hk = h / (p.Hq / p.Hkv), row0 = b * p.S;
        for (int j = 0; j <= last; ++j, ++g) {
          const int st = g % VST3;
          const uint32_t ph = ((g / VST3) & 1) ^ 1;
          uint8_t* sV = sVr + st * TILE;
          if (!(ok = mbar_wait(smem_u32(&v_empty[st]), ph, abort_flag, p.err, 332))) break;
          const uint32_t vb = smem_u32(&v_full[st]);
          mbar_expect_tx(vb, TILE);
          tma3(smem_u32(sV), &tmV, vb, 0, hk, row0 + j * BK);
          tma3(smem_u32(sV + CHUNK), &tmV, vb, 64, hk, row0 + j * BK);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(128 >> 3) << 17) |
                             ((uint32_t)(128 >> 4) << 24);
      // The global block sequence over this CTA's tiles; the issuer walks it with two cursors (the
      // next S to issue runs NSB blocks ahead of the PV).
      struct Cursor {
        int k = 0, idx = -1, j = 0, last = -1, g = 0;
      };
      const int G_ = G, c_ = c, total_ = total;
      auto first = [&](Cursor& u) {
        u.k = 0;
        u.g = 0;
        u.j = 0;
        u.idx = tile_of(0, c_, G_, total_);
        if (u.idx >= 0) {
          int b, h, qb;
          tile_geo(u.idx, b, h, qb, u.last);
        }
      };
      auto next = [&](Cursor& u) {
        ++u.g;
        if (++u.j > u.last) {
          u.j = 0;
          ++u.k;
          u.idx = tile_of(u.k, c_, G_, total_);
          if (u.idx >= 0) {
            int b, h, qb;
            tile_geo(u.idx, b, h, qb, u.last);
          }
        }
      };
      bool ok = true;
      const uint32_t sq = smem_u32(sQ);
      // S(g) = Q K^T into buffer g % NSB; the first S of a tile waits for its Q, the last releases Q
      auto issue_s = [&](const Cursor& u) -> bool {
        if (u.j == 0 && !mbar_wait(smem_u32(q_full), u.k & 1, abort_flag, p.err, 333)) return false;
        if (!mbar_wait(smem_u32(&k_full[u.g % KST3]), (u.g / KST3) & 1, abort_flag, p.err, 334)) return false;
        fence_after();
        // descriptors of the tile bases; a k-step adds its offset (in 16-byte units) to the start
        // address field, which stays below 2^14 units for any shared-memory address
        const uint64_t qd = sdesc(sq), kd = sdesc(smem_u32(sKr + (u.g % KST3) * TILE));
        const uint32_t dS = tmem + 128 + (u.g % NSB) * 128;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (uint32_t)((k >> 2) * CHUNK + (k & 3) * 32) >> 4;
          mma_bf16(dS, qd + off, kd + off, idesc, k != 0);
        }
        commit(smem_u32(&s_full[u.g % NSB]));
        commit(smem_u32(&k_empty[u.g % KST3]));
        if (u.j == u.last) commit(smem_u32(q_empty));
        return true;
      };
      Cursor sc, pc;
      first(sc);
      first(pc);
      for (int i = 0; ok && i < NSB && sc.idx >= 0; ++i) {
        ok = issue_s(sc);
        next(sc);
      }
      for (; ok && pc.idx >= 0; next(pc)) {
        const int g = pc.g;
        // PV of a tile's first block overwrites O: the previous tile's epilogue has read it
        if (pc.j == 0 && pc.k >= 1 && !(ok = mbar_wait(smem_u32(o_free), (pc.k - 1) & 1, abort_flag, p.err, 342)))
          break;
        ok = mbar_wait(smem_u32(&p_ready[g % NSB]), (g / NSB) & 1, abort_flag, p.err, 335) &&
             mbar_wait(smem_u32(&v_full[g % VST3]), (g / VST3) & 1, abort_flag, p.err, 336);
        if (!ok) break;
        fence_after();
        const bool mtr = tr && pc.k == 0 && pc.j < 16;
        if (mtr) tr[50 + 3 * pc.j] = gtimer();
        const uint64_t vd = vdesc(smem_u32(sVr + (g % VST3) * TILE));
        const uint32_t pa = tmem + 128 + (g % NSB) * 128, dO = tmem;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ta(dO, pa + 8 * k, vd + (uint64_t)(128 * k), idesc | kIdescBMajorMN, (pc.j | k) != 0);
        commit(smem_u32(&pv_done[g % NSB]));
        commit(smem_u32(&v_empty[g % VST3]));
        if (mtr) tr[51 + 3 * pc.j] = gtimer();
        // S(g + NSB) overwrites the buffer PV(g) reads P(g) from; MMAs of one issuing thread run in
        // issue order, so PV(g) has read it first
        if (sc.idx >= 0) {
          ok = issue_s(sc);
          next(sc);
          if (mtr) tr[52 + 3 * pc.j] = gtimer();
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- softmax: two threads per query row ----------------
    const int quarter = warp & 3;
    const int hf = (warp - 2) >> 2;      // column half
    const int r = quarter * 32 + lane;   // row within the tile = TMEM lane
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    int g = 0;
    for (int k = 0, idx; ok && (idx = tile_of(k, c, G, total)) >= 0; ++k) {
      int b, h, qb, last;
      tile_geo(idx, b, h, qb, last);
      const uint32_t tO = tmem + lane_base + hf * 64;
      float m = -INFINITY, l = 0.0f;
      for (int j = 0; j <= last; ++j, ++g) {
        const uint32_t tS = tmem + 128 + (g % NSB) * 128 + lane_base;
        ok = mbar_wait(smem_u32(&s_full[g % NSB]), (g / NSB) & 1, abort_flag, p.err, 338);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        fence_after();
        const bool tracer = tr && r == 0 && hf == 0 && k == 0 && j < 16;
        if (tracer) tr[1 + 2 * j] = gtimer();
        uint32_t s[64];
        tld32(tS + hf * 64, s);
        tld32(tS + hf * 64 + 32, s + 32);
        tld_wait();
        if (p.causal && j == qb) {
#pragma unroll
          for (int cc = 0; cc < 64; ++cc)
            if (hf * 64 + cc > r) s[cc] = __float_as_uint(-INFINITY);
        }
        float mx8[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) mx8[q] = fmaxf(__uint_as_float(s[2 * q]), __uint_as_float(s[2 * q + 1]));
#pragma unroll
        for (int cc = 16; cc < 64; cc += 16)
#pragma unroll
          for (int q = 0; q < 8; ++q)
            mx8[q] = max3f(mx8[q], __uint_as_float(s[cc + 2 * q]), __uint_as_float(s[cc + 2 * q + 1]));
        const float mxh = max3f(max3f(mx8[0], mx8[1], mx8[2]), max3f(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
        // the partner thread's partial maximum; the barrier also orders both threads' S reads before
        // either writes P over the buffer's first 64 columns
        xch[((g & 1) * 2 + hf) * BQ + r] = mxh;
        bar_pair(1 + quarter);
        const float mx = fmaxf(mxh, xch[((g & 1) * 2 + (hf ^ 1)) * BQ + r]) * p.scale_log2;
        // lazy rescaling, as in the two-tile kernel: both threads of a row take the same decisions
        const float mnew = mx > m + 8.0f ? mx : m;
        const float alpha = ex2(m - mnew);
        const uint64_t scale2 = pack_f32x2(p.scale_log2, p.scale_log2), neg2 = pack_f32x2(-mnew, -mnew);
        uint64_t sum2[4] = {0, 0, 0, 0};
        uint32_t* pk = s;
#pragma unroll
        for (int cc = 0; cc < 64; cc += 2) {
          float x0, x1;
          unpack_f32x2(fma_f32x2(pack_f32x2(__uint_as_float(s[cc]), __uint_as_float(s[cc + 1])), scale2, neg2), x0,
                       x1);
          const float p0 = ex2(x0), p1 = ex2(x1);
          sum2[(cc >> 1) & 3] = add_f32x2(sum2[(cc >> 1) & 3], pack_f32x2(p0, p1));
          pk[cc / 2] = pack_bf16x2(p0, p1);
        }
        float sa[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) unpack_f32x2(sum2[q], sa[2 * q], sa[2 * q + 1]);
        l = l * alpha + (((sa[0] + sa[1]) + (sa[2] + sa[3])) + ((sa[4] + sa[5]) + (sa[6] + sa[7])));
        m = mnew;
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
          // S(g) was issued before PV(g - 1): wait for PV(g - 1) before touching O
          ok = mbar_wait(smem_u32(&pv_done[(g - 1) % NSB]), ((g - 1) / NSB) & 1, abort_flag, p.err, 339);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          fence_after();
#pragma unroll 1
          for (int cc = 0; cc < 2; ++cc) {
            uint32_t o[32];
            tld32(tO + cc * 32, o);
            tld_wait_regs(o);
#pragma unroll
            for (int q = 0; q < 32; ++q) o[q] = __float_as_uint(__uint_as_float(o[q]) * alpha);
            tst32(tO + cc * 32, o);
          }
        }
        tst32(tS + hf * 32, pk);
        tst_wait();
        fence_before();
        mbar_arrive(smem_u32(&p_ready[g % NSB]));
        if (tracer) tr[2 + 2 * j] = gtimer();
      }
      if (!ok) break;
      // the tile's last PV (its commit tracks every earlier MMA); the previous completion of its
      // barrier, PV(g - 1 - NSB), is done: S(g - 1) was issued after it
      ok = mbar_wait(smem_u32(&pv_done[(g - 1) % NSB]), ((g - 1) / NSB) & 1, abort_flag, p.err, 340);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      fence_after();
      xl[hf * BQ + r] = l;
      bar_pair(1 + quarter);
      const float inv = 1.0f / ((l + xl[(hf ^ 1) * BQ + r]) + p.eps);
      uint32_t o[64];
      tld32(tO, o);
      tld32(tO + 32, o + 32);
      tld_wait();
      // O buffer k % 2 is free for tile k + 2; the row sums may be rewritten after this barrier
      fence_before();
      mbar_arrive(smem_u32(o_free));
      bar_pair(1 + quarter);
      // each thread stores its 64 columns (128 contiguous bytes of its output row)
      uint4* dst = (uint4*)(p.O + (((int64_t)b * p.S + qb * BQ + r) * p.Hq + h) * D + hf * 64);
#pragma unroll
      for (int u = 0; u < 8; ++u)  // columns 8 u .. 8 u + 7
        dst[u] = make_uint4(pack_bf16(__uint_as_float(o[8 * u]) * inv, __uint_as_float(o[8 * u + 1]) * inv),
                            pack_bf16(__uint_as_float(o[8 * u + 2]) * inv, __uint_as_float(o[8 * u + 3]) * inv),
                            pack_bf16(__uint_as_float(o[8 * u + 4]) * inv, __uint_as_float(o[8 * u + 5]) * inv),
                            pack_bf16(__uint_as_float(o[8 * u + 6]) * inv, __uint_as_float(o[8 * u + 7]) * inv));
      if (tr && r == 0 && hf == 0 && k == 0) tr[36] = gtimer();
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (tr && threadIdx.x == 64) tr[42] = gtimer();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)ptr;
  });
  if (!fn) throw Fail{FOPT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable"};
  return fn;
}

// A 3-d bf16 tensor map with a 64-element (128-byte) inner box and 128-byte swizzle.
CUtensorMap map3(const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_bytes,
                 uint64_t stride2_bytes, uint32_t box1, uint32_t box2) {
  CUtensorMap m;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {64, box1, box2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Fail{FOPT_ERR_CUDA, "cuTensorMapEncodeTiled (attention) failed"};
  return m;
}

// Diagnostics only (FOPT_ATTN_TRACE): one line per CTA, its 128 stamps in ns from the earliest entry.
void dump_trace(fopt_ctx* ctx, uint64_t* trace, int64_t blocks, int S, const char* path) {
  std::vector<uint64_t> t((size_t)blocks * 128);
  cuda_check(cudaMemcpyAsync(t.data(), trace, t.size() * 8, cudaMemcpyDeviceToHost, ctx->stream), "trace copy");
  cuda_check(cudaStreamSynchronize(ctx->stream), "trace sync");
  cudaFreeAsync(trace, ctx->stream);
  uint64_t t0 = ~0ull;
  for (int64_t c = 0; c < blocks; ++c) t0 = std::min(t0, t[c * 128]);
  if (FILE* f = fopen(path, "a")) {
    fprintf(f, "# blocks=%lld S=%d\n", (long long)blocks, S);
    for (int64_t c = 0; c < blocks; ++c) {
      fprintf(f, "%lld", (long long)c);
      for (int k = 0; k < 128; ++k) fprintf(f, " %lld", t[c * 128 + k] ? (long long)(t[c * 128 + k] - t0) : -1LL);
      fprintf(f, "\n");
    }
    fclose(f);
  }
}

}  // namespace attn

bool launch_attention_tc(fopt_ctx* ctx, void* o, const void* q, const void* k, const void* v, int B, int S, int Hq,
                         int Hkv, int Dh, float scale, int causal, float eps) {
  using namespace attn;
  if (Dh != 128 || S % 128 || getenv("FOPT_ATTN_NO_TC")) return false;
  if ((uintptr_t)q % 16 || (uintptr_t)k % 16 || (uintptr_t)v % 16 || (uintptr_t)o % 16) return false;
  const uint64_t rows = (uint64_t)B * S;
  CUtensorMap mq = map3(q, D, Hq, rows, (uint64_t)D * 2, (uint64_t)Hq * D * 2, 1, 128);
  CUtensorMap mk = map3(k, D, Hkv, rows, (uint64_t)D * 2, (uint64_t)Hkv * D * 2, 1, 128);
  CUtensorMap mv = map3(v, D, Hkv, rows, (uint64_t)D * 2, (uint64_t)Hkv * D * 2, 1, 128);
  Params p{};
  p.O = (uint16_t*)o;
  p.B = B;
  p.S = S;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.causal = causal;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.eps = eps;
  p.err = ctx->dev_err;
  p.pv_wait = getenv("FOPT_ATTN_PV_WAIT") != nullptr;
  constexpr int smem = 2 * TILE + STAGES * 2 * TILE + 1024 + 256;
  static bool attr = false;
  if (!attr) {
    cuda_check(cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
               "attention smem attribute");
    cuda_check(cudaFuncSetAttribute(attention_tc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
               "attention smem attribute");
    attr = true;
  }
  // The persistent kernel for sequences up to 1024 (B = 8, S = 512: 57.3 against 63.5 us for the
  // paired kernel; B = 4, S = 1024: 73.7 against 77.8), where the paired kernel's per-CTA start and
  // finish weigh most; the paired kernel beyond (S = 2048: 59.4 against 61.4). FOPT_ATTN_SPLIT_ROWS /
  // FOPT_ATTN_PAIRED force one or the other.
  const bool split_rows = getenv("FOPT_ATTN_SPLIT_ROWS") || (S <= 1024 && !getenv("FOPT_ATTN_PAIRED") &&
                                                             !getenv("FOPT_ATTN_ONE_TILE"));
  if (split_rows) {
    constexpr int smem3 = (1 + KST3 + VST3) * TILE + 1024 + 3 * 2 * BQ * 4 + 256;
    static bool attr3 = false;
    if (!attr3) {
      cuda_check(cudaFuncSetAttribute(attention_tc3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem3),
                 "attention smem attribute");
      attr3 = true;
    }
    static int sms = 0;
    if (!sms) cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device), "SM count");
    const int64_t blocks = std::min<int64_t>((int64_t)B * Hq * (S / 128), sms);  // persistent: one CTA per SM
    const char* trace_path = getenv("FOPT_ATTN_TRACE");
    if (trace_path) {
      cuda_check(cudaMallocAsync((void**)&p.trace, blocks * 128 * 8, ctx->stream), "trace alloc");
      cuda_check(cudaMemsetAsync(p.trace, 0, blocks * 128 * 8, ctx->stream), "trace clear");
    }
    CUtensorMap mo = map3(o, D, Hq, rows, (uint64_t)D * 2, (uint64_t)Hq * D * 2, 1, 32);
    attention_tc3_kernel<<<(unsigned)blocks, THREADS3, smem3, ctx->stream>>>(mq, mk, mv, mo, p);
    launched(ctx, "attention_tc3");
    if (trace_path) dump_trace(ctx, p.trace, blocks, S, trace_path);
    return true;
  }
  if ((S / 128) % 2 == 0 && !getenv("FOPT_ATTN_ONE_TILE")) {
    const int64_t blocks = (int64_t)B * Hq * (S / 256);
    const char* trace_path = getenv("FOPT_ATTN_TRACE");
    if (trace_path) {
      cuda_check(cudaMallocAsync((void**)&p.trace, blocks * 128 * 8, ctx->stream), "trace alloc");
      cuda_check(cudaMemsetAsync(p.trace, 0, blocks * 128 * 8, ctx->stream), "trace clear");
    }
    CUtensorMap mo = map3(o, D, Hq, rows, (uint64_t)D * 2, (uint64_t)Hq * D * 2, 1, 32);
    attention_tc2_kernel<<<(unsigned)blocks, THREADS2, smem, ctx->stream>>>(mq, mk, mv, mo, p);
    launched(ctx, "attention_tc2");
    if (trace_path) dump_trace(ctx, p.trace, blocks, S, trace_path);
    return true;
  }
  const int64_t blocks = (int64_t)B * Hq * (S / 128);
  attention_tc_kernel<<<(unsigned)blocks, THREADS, smem, ctx->stream>>>(mq, mk, mv, p);
  launched(ctx, "attention_tc");
  return true;
}

}  // namespace fopt
