// Elementwise kernels: BufStorage::map / zip_with / zip3_with (furiosa-opt-std/src/storage/buf.rs:203-250)
// with the vector-engine opcode semantics (furiosa-opt-std/src/engine/vector/op/semantics.rs) and the
// cast rules (furiosa-opt-std/src/cast.rs, float/bf16.rs, float/mod.rs).
//
// One launch runs a short register program per element, so a chain of engine stages that the
// reference materialises one by one (e.g. FxpToFp -> MulF -> FpToFxp -> Clip -> cast) costs one
// read of each input and one write of the output. Memory-bound: each thread handles 4 elements
// per iteration for memory-level parallelism; every opcode is uniform across the warp.
#include <algorithm>

#include "ctx.hpp"

namespace fopt {
namespace {

__device__ __forceinline__ float F(uint32_t w) { return __uint_as_float(w); }
__device__ __forceinline__ uint32_t W(float f) { return __float_as_uint(f); }

__device__ __forceinline__ int32_t sat_add(int32_t a, int32_t b) {
  int64_t s = (int64_t)a + b;
  return (int32_t)max((int64_t)INT32_MIN, min((int64_t)INT32_MAX, s));
}
__device__ __forceinline__ int32_t sat_sub(int32_t a, int32_t b) {
  int64_t s = (int64_t)a - b;
  return (int32_t)max((int64_t)INT32_MIN, min((int64_t)INT32_MAX, s));
}

// f32 -> i32 `as` cast: truncation toward zero, saturating, NaN -> 0.
__device__ __forceinline__ int32_t f2i_as(float x) {
  if (x != x) return 0;
  if (x >= 2147483648.0f) return INT32_MAX;
  if (x <= -2147483904.0f) return INT32_MIN;
  return (int32_t)x;
}

// f8 conversions are restated from the OCP 8-bit float definitions (E4M3: bias 7, no infinities,
// 0x7f/0xff NaN, max 448; E5M2: bias 15, IEEE-like) with round-to-nearest-even on narrowing.
__device__ __forceinline__ float f8_to_f32(uint32_t code, int ebits) {
  int mbits = 7 - ebits, bias = (1 << (ebits - 1)) - 1;
  uint32_t s = code >> 7, e = (code >> mbits) & ((1 << ebits) - 1), m = code & ((1 << mbits) - 1);
  float v;
  if (ebits == 4 && e == 15 && m == 7) return __uint_as_float(0x7fc00000u);
  if (ebits == 5 && e == 31) return m ? __uint_as_float(0x7fc00000u) : (s ? -INFINITY : INFINITY);
  if (e == 0) v = ldexpf((float)m, 1 - bias - mbits);
  else v = ldexpf((float)((1 << mbits) | m), (int)e - bias - mbits);
  return s ? -v : v;
}
__device__ __forceinline__ uint32_t f32_to_f8(float x, int ebits) {
  int mbits = 7 - ebits, bias = (1 << (ebits - 1)) - 1;
  uint32_t bits = __float_as_uint(x);
  uint32_t s = (bits >> 31) << 7;
  if (x != x) return ebits == 4 ? 0x7f : 0x7e;
  float a = fabsf(x);
  float maxv = ebits == 4 ? 448.0f : 57344.0f;
  if (ebits == 5 && isinf(a)) return s | 0x7c;
  // quantum at this magnitude
  int e;
  frexpf(a, &e);  // a = f * 2^e, f in [0.5, 1)
  int ee = max(e - 1, 1 - bias);
  float q = ldexpf(1.0f, ee - mbits);
  float r = rintf(a / q) * q;  // RNE (division by a power of two is exact)
  if (r > maxv) return ebits == 4 ? (s | 0x7e) /* saturate finite */ : (s | 0x7c);
  if (r == 0.0f) return s;
  int re;
  frexpf(r, &re);
  int be = re - 1 + bias;
  uint32_t code;
  if (be <= 0) code = (uint32_t)(r / ldexpf(1.0f, 1 - bias - mbits));
  else code = ((uint32_t)be << mbits) | ((uint32_t)(r / ldexpf(1.0f, re - 1 - mbits)) & ((1u << mbits) - 1));
  return s | code;
}

// The opcode table: X(code, expression over the operand words a, b, c and the immediate imm).
// ia / ib are the signed views, fa / fb / fc the f32 views.
#define FOPT_EW_OPS(X)                                                                                    \
  X(FOPT_OP_MOV, a)                                                                                       \
  X(FOPT_OP_BF16_TO_F32, bf16w_to_f32_bits(a & 0xffff0000u))                                              \
  X(FOPT_OP_F32_TO_BF16, f32_to_bf16w(a))                                                                 \
  X(FOPT_OP_F32_TO_BF16_RELU, (((a & 0x7fffffffu) <= 0x7f800000u) && (a >> 31)) ? 0u : f32_to_bf16w(a))   \
  X(FOPT_OP_I32_TO_F32, W(__int2float_rn(ia)))                                                            \
  X(FOPT_OP_F32_TO_I32, (uint32_t)f2i_as(fa))                                                             \
  X(FOPT_OP_FXP_TO_FP, fxp_to_fp_bits(ia, (uint32_t)imm))                                                 \
  X(FOPT_OP_FP_TO_FXP, (uint32_t)fp_to_fxp(fa, (uint32_t)imm))                                            \
  X(FOPT_OP_F8E4M3_TO_F32, W(f8_to_f32(a & 0xff, 4)))                                                     \
  X(FOPT_OP_F32_TO_F8E4M3, f32_to_f8(fa, 4))                                                              \
  X(FOPT_OP_F8E5M2_TO_F32, W(f8_to_f32(a & 0xff, 5)))                                                     \
  X(FOPT_OP_F32_TO_F8E5M2, f32_to_f8(fa, 5))                                                              \
  X(FOPT_OP_I4_SEXT, (uint32_t)(((int32_t)(a << 28)) >> 28))                                              \
  X(FOPT_OP_I5_SEXT, (uint32_t)(((int32_t)(a << 27)) >> 27))                                              \
  X(FOPT_OP_I9_SEXT, (uint32_t)(((int32_t)(a << 23)) >> 23))                                              \
  X(FOPT_OP_EXP, W(expf(fa)))                                                                             \
  X(FOPT_OP_NEGEXP, W(expf(-fa)))                                                                         \
  X(FOPT_OP_SQRT, W(__fsqrt_rn(fa)))                                                                      \
  X(FOPT_OP_TANH, W(tanhf(fa)))                                                                           \
  X(FOPT_OP_SIGMOID, W(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-fa)))))                                      \
  X(FOPT_OP_LOG, W(logf(fa)))                                                                             \
  X(FOPT_OP_SIN, W(sinf(fa)))                                                                             \
  X(FOPT_OP_COS, W(cosf(fa)))                                                                             \
  X(FOPT_OP_ADDF, W(__fadd_rn(fa, fb)))                                                                   \
  X(FOPT_OP_SUBF, W(__fsub_rn(fa, fb)))                                                                   \
  X(FOPT_OP_MULF, W(__fmul_rn(fa, fb)))                                                                   \
  X(FOPT_OP_DIVF, W(__fdiv_rn(fa, fb)))                                                                   \
  X(FOPT_OP_FMAF, W(__fmaf_rn(fa, fb, fc)))                                                               \
  X(FOPT_OP_MINF, W(fminf(fa, fb)))                                                                       \
  X(FOPT_OP_MAXF, W(fmaxf(fa, fb)))                                                                       \
  X(FOPT_OP_ABSMINF, fabsf(fa) < fabsf(fb) ? a : b)                                                       \
  X(FOPT_OP_ABSMAXF, fabsf(fa) > fabsf(fb) ? a : b)                                                       \
  X(FOPT_OP_ADD_FXP, a + b)                                                                               \
  X(FOPT_OP_ADD_FXP_SAT, (uint32_t)sat_add(ia, ib))                                                       \
  X(FOPT_OP_SUB_FXP, a - b)                                                                               \
  X(FOPT_OP_SUB_FXP_SAT, (uint32_t)sat_sub(ia, ib))                                                       \
  X(FOPT_OP_SHL, a << (b & 31))                                                                           \
  X(FOPT_OP_SHL_SAT, shl_sat(ia, b))                                                                      \
  X(FOPT_OP_MUL_FXP, mul_fxp(ia, ib))                                                                     \
  X(FOPT_OP_MUL_INT, a * b)                                                                               \
  X(FOPT_OP_SHR_LOGIC, a >> (b & 31))                                                                     \
  X(FOPT_OP_SHR_ARITH, (uint32_t)(ia >> (b & 31)))                                                        \
  X(FOPT_OP_MINI, (uint32_t)min(ia, ib))                                                                  \
  X(FOPT_OP_MAXI, (uint32_t)max(ia, ib))                                                                  \
  X(FOPT_OP_ABSMINI, (abs(ia) < abs(ib)) ? a : b)                                                         \
  X(FOPT_OP_ABSMAXI, (abs(ia) > abs(ib)) ? a : b)                                                         \
  X(FOPT_OP_AND, a & b)                                                                                   \
  X(FOPT_OP_OR, a | b)                                                                                    \
  X(FOPT_OP_XOR, a ^ b)                                                                                   \
  X(FOPT_OP_SELECT, a ? b : c)                                                                            \
  X(FOPT_OP_CONST, (uint32_t)imm)

__device__ __forceinline__ uint32_t shl_sat(int32_t ia, uint32_t b) {
  int64_t m = (int64_t)(int32_t)(1u << (b & 31));
  int64_t pr = (int64_t)ia * m;
  return (uint32_t)(int32_t)max((int64_t)INT32_MIN, min((int64_t)INT32_MAX, pr));
}
__device__ __forceinline__ uint32_t mul_fxp(int32_t ia, int32_t ib) {
  if (ia == INT32_MIN && ib == INT32_MIN) return (uint32_t)INT32_MAX;
  return (uint32_t)(int32_t)((((int64_t)ia * ib) >> 30) + 1 >> 1);
}

// One opcode applied to EPT independent elements (the switch is uniform across the warp and is
// taken once per EPT elements).
template <int EPT>
__device__ __forceinline__ void apply(int op, int32_t imm, const uint32_t* A, const uint32_t* B, const uint32_t* Cc,
                                      uint32_t* O) {
  switch (op) {
#define FOPT_EW_CASE(code, expr)                                                                   \
  case code:                                                                                       \
    _Pragma("unroll") for (int e = 0; e < EPT; ++e) {                                              \
      const uint32_t a = A[e], b = B[e], c = Cc[e];                                                \
      const int32_t ia = (int32_t)a, ib = (int32_t)b;                                              \
      const float fa = F(a), fb = F(b), fc = F(c);                                                 \
      (void)ia; (void)ib; (void)fa; (void)fb; (void)fc; (void)c; (void)imm;                        \
      O[e] = (expr);                                                                               \
    }                                                                                              \
    break;
    FOPT_EW_OPS(FOPT_EW_CASE)
#undef FOPT_EW_CASE
    default:
#pragma unroll
      for (int e = 0; e < EPT; ++e) O[e] = 0;
  }
}

// The register file lives in real registers: a dynamic register index becomes a uniform switch.
constexpr int NR = 8;   // physical registers after host-side allocation
constexpr int EPT = 4;  // elements per thread per iteration

__device__ __forceinline__ void reg_read(const uint32_t (&R)[NR][EPT], int idx, uint32_t* out) {
  switch (idx) {
#define RD(i) \
  case i: _Pragma("unroll") for (int e = 0; e < EPT; ++e) out[e] = R[i][e]; break;
    RD(0) RD(1) RD(2) RD(3) RD(4) RD(5) RD(6) RD(7)
#undef RD
  }
}
__device__ __forceinline__ void reg_write(uint32_t (&R)[NR][EPT], int idx, const uint32_t* in) {
  switch (idx) {
#define WR(i) \
  case i: _Pragma("unroll") for (int e = 0; e < EPT; ++e) R[i][e] = in[e]; break;
    WR(0) WR(1) WR(2) WR(3) WR(4) WR(5) WR(6) WR(7)
#undef WR
  }
}

struct EwArgs {
  const void* in[3];
  int dt[3];
  int n_in;
  void* out;
  int out_dt;
  int64_t n;
  int vec;  // every pointer aligned for the EPT-element vector loads / stores
};

// EPT consecutive elements of one operand as 32-bit words (one vector load when aligned).
__device__ __forceinline__ void load_ept(const void* p, int dt, int64_t base, int64_t n, bool vec, uint32_t* w) {
  if (vec && base + EPT <= n) {
    const int bits = dtype_bits(dt);
    if (bits == 32) {
      uint4 x = *(const uint4*)((const uint32_t*)p + base);
      w[0] = x.x; w[1] = x.y; w[2] = x.z; w[3] = x.w;
      return;
    }
    if (bits == 16) {
      uint2 x = *(const uint2*)((const uint16_t*)p + base);
      const uint32_t h[2] = {x.x, x.y};
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        uint32_t lo = h[k] & 0xffffu, hi = h[k] >> 16;
        if (dt == FOPT_BF16) { w[2 * k] = lo << 16; w[2 * k + 1] = hi << 16; }
        else { w[2 * k] = (uint32_t)(int32_t)(int16_t)lo; w[2 * k + 1] = (uint32_t)(int32_t)(int16_t)hi; }
      }
      return;
    }
    if (bits == 8) {
      uint32_t x = *(const uint32_t*)((const uint8_t*)p + base);
      const bool sgn = dt == FOPT_I8 || dt == FOPT_I5;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t b = (x >> (8 * k)) & 0xffu;
        w[k] = sgn ? (uint32_t)(int32_t)(int8_t)b : b;
      }
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < EPT; ++e) w[e] = base + e < n ? load_word(p, dt, base + e) : 0u;
}

__device__ __forceinline__ void store_ept(void* p, int dt, int64_t base, int64_t n, bool vec, const uint32_t* w) {
  if (vec && base + EPT <= n) {
    const int bits = dtype_bits(dt);
    if (bits == 32) {
      *(uint4*)((uint32_t*)p + base) = make_uint4(w[0], w[1], w[2], w[3]);
      return;
    }
    if (bits == 16) {
      uint32_t h[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        uint32_t lo = dt == FOPT_BF16 ? (w[2 * k] >> 16) : (w[2 * k] & 0xffffu);
        uint32_t hi = dt == FOPT_BF16 ? (w[2 * k + 1] >> 16) : (w[2 * k + 1] & 0xffffu);
        h[k] = lo | (hi << 16);
      }
      *(uint2*)((uint16_t*)p + base) = make_uint2(h[0], h[1]);
      return;
    }
    if (bits == 8) {
      uint32_t h = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) h |= (w[k] & 0xffu) << (8 * k);
      *(uint32_t*)((uint8_t*)p + base) = h;
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < EPT; ++e)
    if (base + e < n) store_word(p, dt, base + e, w[e]);
}

// prog: registers already renamed into [0, NR), inputs in registers 0..n_in-1.
__global__ void __launch_bounds__(256) ew_kernel(fopt_program prog, EwArgs a) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * EPT;
  for (int64_t base = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * EPT; base < a.n; base += stride) {
    uint32_t R[NR][EPT];
#pragma unroll
    for (int k = 0; k < 3; ++k)
      if (k < a.n_in) load_ept(a.in[k], a.dt[k], base, a.n, a.vec, R[k]);
#pragma unroll 1
    for (int i = 0; i < prog.n_insn; ++i) {
      const fopt_insn in = prog.insn[i];
      uint32_t A[EPT], B[EPT], Cc[EPT], O[EPT];
      reg_read(R, in.a, A);
      reg_read(R, in.b, B);
      reg_read(R, in.c, Cc);
      apply<EPT>(in.op, in.imm_i, A, B, Cc, O);
      reg_write(R, in.dst, O);
    }
    uint32_t res[EPT];
    reg_read(R, prog.ret, res);
    store_ept(a.out, a.out_dt, base, a.n, a.vec, res);
  }
}

// 4-bit outputs: one thread owns one output byte (two elements).
__global__ void ew_kernel_nibble_out(fopt_program prog, EwArgs a) {
  int64_t bytes = (a.n + 1) / 2;
  for (int64_t by = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; by < bytes;
       by += (int64_t)gridDim.x * blockDim.x) {
    uint32_t outb = ((const uint8_t*)a.out)[by];
    for (int h = 0; h < 2; ++h) {
      int64_t i = by * 2 + h;
      if (i >= a.n) break;
      uint32_t R[NR][1] = {};
      for (int k = 0; k < a.n_in; ++k) R[k][0] = load_word(a.in[k], a.dt[k], i);
      for (int q = 0; q < prog.n_insn; ++q) {
        const fopt_insn in = prog.insn[q];
        uint32_t A[1] = {R[in.a][0]}, B[1] = {R[in.b][0]}, Cc[1] = {R[in.c][0]}, O[1];
        apply<1>(in.op, in.imm_i, A, B, Cc, O);
        R[in.dst][0] = O[0];
      }
      uint32_t v = R[prog.ret][0] & 15u;
      outb = h ? ((outb & 0x0f) | (v << 4)) : ((outb & 0xf0) | v);
    }
    ((uint8_t*)a.out)[by] = (uint8_t)outb;
  }
}

// Which of a, b, c an opcode reads.
int arity(int op) {
  switch (op) {
    case FOPT_OP_CONST: return 0;
    case FOPT_OP_FMAF: case FOPT_OP_SELECT: return 3;
    case FOPT_OP_ADDF: case FOPT_OP_SUBF: case FOPT_OP_MULF: case FOPT_OP_DIVF: case FOPT_OP_MINF:
    case FOPT_OP_MAXF: case FOPT_OP_ABSMINF: case FOPT_OP_ABSMAXF: case FOPT_OP_ADD_FXP: case FOPT_OP_ADD_FXP_SAT:
    case FOPT_OP_SUB_FXP: case FOPT_OP_SUB_FXP_SAT: case FOPT_OP_SHL: case FOPT_OP_SHL_SAT: case FOPT_OP_MUL_FXP:
    case FOPT_OP_MUL_INT: case FOPT_OP_SHR_LOGIC: case FOPT_OP_SHR_ARITH: case FOPT_OP_MINI: case FOPT_OP_MAXI:
    case FOPT_OP_ABSMINI: case FOPT_OP_ABSMAXI: case FOPT_OP_AND: case FOPT_OP_OR: case FOPT_OP_XOR: return 2;
    default: return 1;
  }
}

// Renames the program's registers (0..15) onto NR physical registers by last use. Inputs keep
// registers 0..n_in-1. Registers never written read as 0, as in the unrenamed program.
fopt_program rename_registers(const fopt_program& p, int n_in) {
  const int n = p.n_insn;
  int last[16];
  for (int r = 0; r < 16; ++r) last[r] = -1;
  for (int i = 0; i < n; ++i) {
    const fopt_insn& in = p.insn[i];
    const int src[3] = {in.a, in.b, in.c};
    for (int k = 0; k < arity(in.op); ++k) last[src[k] & 15] = i;
  }
  last[p.ret & 15] = n;
  int phys[16];
  bool written[16] = {};
  for (int r = 0; r < 16; ++r) phys[r] = -1;
  bool used[NR] = {};
  for (int r = 0; r < n_in; ++r) {
    phys[r] = r;
    used[r] = true;
    written[r] = true;
  }
  // A read of a never-written register yields 0: give such registers one shared zero register.
  int zero_reg = -1;
  fopt_program q = p;
  for (int i = 0; i < n; ++i) {
    fopt_insn in = p.insn[i];
    int* src[3] = {&in.a, &in.b, &in.c};
    for (int k = 0; k < 3; ++k) {
      int v = *src[k] & 15;
      if (k >= arity(in.op)) { *src[k] = 0; continue; }
      if (!written[v]) {
        if (zero_reg < 0) {
          for (int r = 0; r < NR; ++r)
            if (!used[r]) { zero_reg = r; used[r] = true; break; }
          if (zero_reg < 0) throw Fail{FOPT_ERR_UNSUPPORTED, "elementwise program needs more than 8 registers"};
          // materialise the zero with a CONST at the front
          fopt_insn z{FOPT_OP_CONST, zero_reg, 0, 0, 0, 0};
          if (q.n_insn >= 32) throw Fail{FOPT_ERR_UNSUPPORTED, "elementwise program too long"};
          for (int j = q.n_insn; j > 0; --j) q.insn[j] = q.insn[j - 1];
          q.insn[0] = z;
          q.n_insn++;
        }
        *src[k] = zero_reg;
      } else {
        *src[k] = phys[v];
      }
    }
    // free registers whose last read is this instruction (inputs included)
    for (int v = 0; v < 16; ++v)
      if (phys[v] >= 0 && last[v] <= i && written[v] && phys[v] != zero_reg) {
        used[phys[v]] = false;
        phys[v] = -1;
      }
    int d = in.dst & 15;
    int pd = -1;
    for (int r = 0; r < NR; ++r)
      if (!used[r]) { pd = r; break; }
    if (pd < 0) throw Fail{FOPT_ERR_UNSUPPORTED, "elementwise program needs more than 8 registers"};
    used[pd] = true;
    if (phys[d] >= 0) used[phys[d]] = false;  // overwritten register
    phys[d] = pd;
    written[d] = true;
    in.dst = pd;
    q.insn[q.n_insn - n + i] = in;
  }
  int rv = p.ret & 15;
  q.ret = written[rv] ? phys[rv] : (zero_reg >= 0 ? zero_reg : 0);
  if (!written[rv]) {
    // returning a never-written register: the result is 0
    if (q.n_insn >= 32) throw Fail{FOPT_ERR_UNSUPPORTED, "elementwise program too long"};
    int r = 0;
    q.insn[q.n_insn++] = fopt_insn{FOPT_OP_CONST, r, 0, 0, 0, 0};
    q.ret = r;
  }
  return q;
}

}  // namespace

void launch_elementwise(fopt_ctx* ctx, const fopt_program* prog, int n_in, const void* const* in,
                        const fopt_dtype* in_dt, void* out, fopt_dtype out_dt, int64_t n) {
  if (n <= 0) return;
  EwArgs a{};
  a.n_in = n_in;
  bool vec = (uintptr_t)out % 16 == 0;
  for (int k = 0; k < n_in; ++k) {
    a.in[k] = in[k];
    a.dt[k] = in_dt[k];
    vec &= (uintptr_t)in[k] % 16 == 0 && dtype_bits(in_dt[k]) >= 8;
  }
  a.out = out;
  a.out_dt = out_dt;
  a.n = n;
  a.vec = vec;
  fopt_program q = rename_registers(*prog, n_in);
  if (dtype_bits(out_dt) == 4) {
    int64_t bytes = (n + 1) / 2;
    int grid = (int)std::max<int64_t>(1, std::min<int64_t>((bytes + 255) / 256, 148 * 32));
    ew_kernel_nibble_out<<<grid, 256, 0, ctx->stream>>>(q, a);
  } else {
    int64_t threads = (n + EPT - 1) / EPT;
    int grid = (int)std::max<int64_t>(1, std::min<int64_t>((threads + 255) / 256, 148 * 16));
    ew_kernel<<<grid, 256, 0, ctx->stream>>>(q, a);
  }
  launched(ctx, "elementwise");
}

}  // namespace fopt
