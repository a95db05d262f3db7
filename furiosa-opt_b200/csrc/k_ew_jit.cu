// Elementwise programs compiled to their own kernels at run time (NVRTC -> sm_100a cubin).
//
// The interpreter in k_elementwise.cu dispatches every opcode through switches; a generated kernel
// instead has the program's expressions inlined with every value in a real register, dtype-specific
// 16-byte loads and stores, and 8 elements per thread, so a map / zip / zip3 runs at memory speed.
// The expressions come from the same FOPT_EW_OPS table (stringified) that the interpreter expands,
// and the same device helpers (ew_ops.cuh, handed to NVRTC verbatim), so both paths compute the
// identical bit patterns. Kernels are cached per (program, dtypes, device). When NVRTC or the driver
// entry points are unavailable, or FOPT_EW_NO_JIT is set, the interpreter runs instead.
#include <cuda.h>
#include <dlfcn.h>
#include <nvrtc.h>

#include <atomic>
#include <map>
#include <mutex>
#include <sstream>
#include <cstring>
#include <string>
#include <vector>

#include "ctx.hpp"
#include "ew_ops.cuh"

namespace fopt {
namespace {

const char* kPrelude =
#include "ew_ops_src.inc"
    ;

struct OpText {
  int code;
  const char* expr;
};
const OpText kOps[] = {
#define FOPT_EW_TEXT(code, expr) {code, #expr},
    FOPT_EW_OPS(FOPT_EW_TEXT)
#undef FOPT_EW_TEXT
};

const char* op_expr(int op) {
  for (const auto& o : kOps)
    if (o.code == op) return o.expr;
  return nullptr;
}

struct Jit {
  bool ok = false;
  nvrtcResult (*create)(nvrtcProgram*, const char*, const char*, int, const char* const*, const char* const*) = nullptr;
  nvrtcResult (*compile)(nvrtcProgram, int, const char* const*) = nullptr;
  nvrtcResult (*cubin_size)(nvrtcProgram, size_t*) = nullptr;
  nvrtcResult (*cubin)(nvrtcProgram, char*) = nullptr;
  nvrtcResult (*log_size)(nvrtcProgram, size_t*) = nullptr;
  nvrtcResult (*log)(nvrtcProgram, char*) = nullptr;
  nvrtcResult (*destroy)(nvrtcProgram*) = nullptr;
  CUresult (*load)(CUmodule*, const void*) = nullptr;
  CUresult (*get_fn)(CUfunction*, CUmodule, const char*) = nullptr;
  CUresult (*launch)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, CUstream,
                     void**, void**) = nullptr;
  CUresult (*set_attr)(CUfunction, int, int) = nullptr;
};

template <typename T>
bool driver_sym(const char* name, T* out) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return false;
  *out = (T)p;
  return true;
}

Jit& jit() {
  static Jit j;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = nullptr;
    for (const char* n : {"libnvrtc.so.12", "libnvrtc.so"})
      if ((h = dlopen(n, RTLD_NOW | RTLD_LOCAL))) break;
    if (!h) return;
#define SYM(f, s) j.f = (decltype(j.f))dlsym(h, s)
    SYM(create, "nvrtcCreateProgram");
    SYM(compile, "nvrtcCompileProgram");
    SYM(cubin_size, "nvrtcGetCUBINSize");
    SYM(cubin, "nvrtcGetCUBIN");
    SYM(log_size, "nvrtcGetProgramLogSize");
    SYM(log, "nvrtcGetProgramLog");
    SYM(destroy, "nvrtcDestroyProgram");
#undef SYM
    bool drv = driver_sym("cuModuleLoadData", &j.load) && driver_sym("cuModuleGetFunction", &j.get_fn) &&
               driver_sym("cuLaunchKernel", &j.launch) && driver_sym("cuFuncSetAttribute", &j.set_attr);
    j.ok = drv && j.create && j.compile && j.cubin_size && j.cubin && j.destroy;
  });
  return j;
}

// ---- code generation ----
std::string load_vec(int k, int dt, const std::string& idx = "base") {
  std::ostringstream o;
  const std::string in = "in" + std::to_string(k), x = "x" + std::to_string(k);
  switch (dtype_bits(dt)) {
    case 32:
      o << "{ const uint4* q = (const uint4*)" << in << " + ((" << idx << ") >> 2); uint4 u0 = q[0], u1 = q[1]; " << x
        << "[0]=u0.x; " << x << "[1]=u0.y; " << x << "[2]=u0.z; " << x << "[3]=u0.w; " << x << "[4]=u1.x; " << x
        << "[5]=u1.y; " << x << "[6]=u1.z; " << x << "[7]=u1.w; }\n";
      break;
    case 16:
      o << "{ uint4 u = *((const uint4*)" << in << " + ((" << idx << ") >> 3)); const unsigned h[4] = {u.x, u.y, u.z, u.w};\n"
        << "  for (int j = 0; j < 4; ++j) { ";
      if (dt == FOPT_BF16)
        o << x << "[2*j] = h[j] << 16; " << x << "[2*j+1] = h[j] & 0xffff0000u; }";
      else
        o << x << "[2*j] = (unsigned)(int)(short)(h[j] & 0xffffu); " << x << "[2*j+1] = (unsigned)((int)h[j] >> 16); }";
      o << " }\n";
      break;
    default: {
      const bool sgn = dt == FOPT_I8 || dt == FOPT_I5;
      o << "{ uint2 u = *((const uint2*)" << in << " + ((" << idx << ") >> 3)); const unsigned h[2] = {u.x, u.y};\n"
        << "  for (int j = 0; j < 8; ++j) { unsigned b = (h[j >> 2] >> (8 * (j & 3))) & 0xffu; " << x << "[j] = "
        << (sgn ? "(unsigned)(int)(signed char)b" : "b") << "; } }\n";
    }
  }
  return o.str();
}

std::string load_one(int k, int dt, const std::string& i) {
  const std::string in = "in" + std::to_string(k);
  switch (dt) {
    case FOPT_I32: case FOPT_F32: return "((const unsigned*)" + in + ")[" + i + "]";
    case FOPT_BF16: return "(((unsigned)((const unsigned short*)" + in + ")[" + i + "]) << 16)";
    case FOPT_I16: case FOPT_I9: return "((unsigned)(int)((const short*)" + in + ")[" + i + "])";
    case FOPT_I8: case FOPT_I5: return "((unsigned)(int)((const signed char*)" + in + ")[" + i + "])";
    default: return "((unsigned)((const unsigned char*)" + in + ")[" + i + "])";
  }
}

std::string store_vec(int dt) {
  switch (dtype_bits(dt)) {
    case 32:
      return "{ uint4* q = (uint4*)out + (base >> 2); q[0] = make_uint4(r[0], r[1], r[2], r[3]); "
             "q[1] = make_uint4(r[4], r[5], r[6], r[7]); }\n";
    case 16:  // one byte permute per pair: the bf16's high halves, or the 16-bit integers' low halves
      if (dt == FOPT_BF16)
        return "{ *((uint4*)out + (base >> 3)) = make_uint4(__byte_perm(r[0], r[1], 0x7632), __byte_perm(r[2], r[3], "
               "0x7632), __byte_perm(r[4], r[5], 0x7632), __byte_perm(r[6], r[7], 0x7632)); }\n";
      return "{ *((uint4*)out + (base >> 3)) = make_uint4(__byte_perm(r[0], r[1], 0x5410), __byte_perm(r[2], r[3], "
             "0x5410), __byte_perm(r[4], r[5], 0x5410), __byte_perm(r[6], r[7], 0x5410)); }\n";
    default:  // low bytes of four words into one: two permutes to byte pairs, one to join them
      return "{ const unsigned h0 = __byte_perm(__byte_perm(r[0], r[1], 0x0040), __byte_perm(r[2], r[3], 0x0040), "
             "0x5410), h1 = __byte_perm(__byte_perm(r[4], r[5], 0x0040), __byte_perm(r[6], r[7], 0x0040), 0x5410); "
             "*((uint2*)out + (base >> 3)) = make_uint2(h0, h1); }\n";
  }
}

std::string store_one(int dt, const std::string& i, const std::string& v) {
  switch (dtype_bits(dt)) {
    case 32: return "((unsigned*)out)[" + i + "] = " + v + ";";
    case 16:
      return "((unsigned short*)out)[" + i + "] = (unsigned short)(" + (dt == FOPT_BF16 ? v + " >> 16" : v) + ");";
    default: return "((unsigned char*)out)[" + i + "] = (unsigned char)(" + v + ");";
  }
}

int arity_of(int op) {
  switch (op) {
    case FOPT_OP_CONST: return 0;
    case FOPT_OP_FMAF: case FOPT_OP_SELECT: return 3;
    default: break;
  }
  switch (op) {
    case FOPT_OP_ADDF: case FOPT_OP_SUBF: case FOPT_OP_MULF: case FOPT_OP_DIVF: case FOPT_OP_MINF: case FOPT_OP_MAXF:
    case FOPT_OP_ABSMINF: case FOPT_OP_ABSMAXF: case FOPT_OP_ADD_FXP: case FOPT_OP_ADD_FXP_SAT: case FOPT_OP_SUB_FXP:
    case FOPT_OP_SUB_FXP_SAT: case FOPT_OP_SHL: case FOPT_OP_SHL_SAT: case FOPT_OP_MUL_FXP: case FOPT_OP_MUL_INT:
    case FOPT_OP_SHR_LOGIC: case FOPT_OP_SHR_ARITH: case FOPT_OP_MINI: case FOPT_OP_MAXI: case FOPT_OP_ABSMINI:
    case FOPT_OP_ABSMAXI: case FOPT_OP_AND: case FOPT_OP_OR: case FOPT_OP_XOR: return 2;
    default: return 1;
  }
}

// Emits the program's instructions for element e of inputs x0..x2 (one scoped block per
// instruction, every value in a named register); *ret names the result. False for an opcode the
// table lacks.
// A DivF by a row-uniform input whose quotient only feeds one FpToFxp: run as qdiv_fxp.
struct QuantFuse {
  int div_i = -1, fxp_i = -1, slot_reg = -1;
  unsigned iw = 31;
};

std::vector<QuantFuse> find_quant_fuses(const fopt_program& p, int uniform_lo, int uniform_hi) {
  std::vector<QuantFuse> out;
  unsigned written = 0;
  for (int i = 0; i < p.n_insn; ++i) {
    const fopt_insn& in = p.insn[i];
    if (in.op == FOPT_OP_DIVF) {
      const int b = in.b & 15, d = in.dst & 15;
      if (b >= uniform_lo && b < uniform_hi && !(written >> b & 1)) {
        int uses = 0, fxp = -1;
        bool overwritten = false;
        for (int j = i + 1; j < p.n_insn && !overwritten; ++j) {
          const fopt_insn& q = p.insn[j];
          const int ar = arity_of(q.op), rs[3] = {q.a & 15, q.b & 15, q.c & 15};
          for (int k = 0; k < ar; ++k)
            if (rs[k] == d) {
              ++uses;
              if (q.op == FOPT_OP_FP_TO_FXP && k == 0) fxp = j;
            }
          if ((q.dst & 15) == d) overwritten = true;
        }
        if (uses == 1 && fxp >= 0 && (overwritten || (p.ret & 15) != d) && p.insn[fxp].imm_i >= 0 &&
            p.insn[fxp].imm_i <= 31)
          out.push_back(QuantFuse{i, fxp, b, (unsigned)p.insn[fxp].imm_i});
      }
    }
    written |= 1u << (in.dst & 15);
  }
  return out;
}

bool emit_program_named(std::ostringstream& o, const fopt_program& p, const std::string* inputs, int n_in,
                        std::string* ret, const std::string& tag = "t",
                        const std::vector<QuantFuse>* fuses = nullptr) {
  std::string name[16];
  for (int v = 0; v < 16; ++v) name[v] = "0u";
  for (int k = 0; k < n_in && k < 16; ++k) name[k] = inputs[k];
  std::map<int, std::string> fused_dividend;  // fxp instruction -> dividend name
  for (int i = 0; i < p.n_insn; ++i) {
    const fopt_insn& in = p.insn[i];
    const QuantFuse* qf = nullptr;
    if (fuses)
      for (const auto& f : *fuses)
        if (f.div_i == i || f.fxp_i == i) qf = &f;
    if (qf && qf->div_i == i) {  // the quotient is formed inside the FpToFxp below
      fused_dividend[qf->fxp_i] = name[in.a & 15];
      name[in.dst & 15] = "0u";
      continue;
    }
    const std::string t = tag + std::to_string(i);
    if (qf && qf->fxp_i == i) {
      o << "      const unsigned " << t << " = qdiv_fxp(" << fused_dividend[i] << ", " << inputs[qf->slot_reg] << ", rq"
        << qf->slot_reg << "_" << qf->iw << ", " << qf->iw << "u);\n";
      name[in.dst & 15] = t;
      continue;
    }
    const char* expr = op_expr(in.op);
    if (!expr) return false;
    const int ar = arity_of(in.op);
    const std::string A = ar > 0 ? name[in.a & 15] : "0u", B = ar > 1 ? name[in.b & 15] : "0u",
                      C = ar > 2 ? name[in.c & 15] : "0u";
    o << "      unsigned " << t << "; { const unsigned a = " << A << ", b = " << B << ", c = " << C
      << "; const int ia = (int)a, ib = (int)b; const float fa = F(a), fb = F(b), fc = F(c); const int imm = "
      << in.imm_i << "; (void)ia; (void)ib; (void)fa; (void)fb; (void)fc; (void)c; (void)imm; " << t << " = ("
      << expr << "); }\n";
    name[in.dst & 15] = t;
  }
  *ret = name[p.ret & 15];
  return true;
}

// The same program emitted instruction by instruction over a group of 8 elements: each instruction
// is an unrolled loop over e writing an 8-entry array, so the 8 independent chains interleave.
// Inputs are expressions in e ("x0[e]") or uniform names. A fused quantising division computes
// every element's fast result and a flag without branching, then one rarely taken loop redoes the
// flagged elements exactly. *ret names the result as an expression in e.
bool emit_program_vec(std::ostringstream& o, const fopt_program& p, const std::string* inputs, int n_in,
                      std::string* ret, const std::string& tag, const std::vector<QuantFuse>* fuses = nullptr) {
  std::string name[16];
  for (int v = 0; v < 16; ++v) name[v] = "0u";
  for (int k = 0; k < n_in && k < 16; ++k) name[k] = inputs[k];
  std::map<int, std::string> fused_dividend;
  for (int i = 0; i < p.n_insn; ++i) {
    const fopt_insn& in = p.insn[i];
    const QuantFuse* qf = nullptr;
    if (fuses)
      for (const auto& f : *fuses)
        if (f.div_i == i || f.fxp_i == i) qf = &f;
    if (qf && qf->div_i == i) {
      fused_dividend[qf->fxp_i] = name[in.a & 15];
      name[in.dst & 15] = "0u";
      continue;
    }
    const std::string t = tag + std::to_string(i);
    if (qf && qf->fxp_i == i) {
      const std::string a = fused_dividend[i], sv = inputs[qf->slot_reg],
                        rq = "rq" + std::to_string(qf->slot_reg) + "_" + std::to_string(qf->iw);
      o << "      unsigned " << t << "[8]; bool " << t << "_slow = false;\n#pragma unroll\n"
        << "      for (int e = 0; e < 8; ++e) { bool ok; " << t << "[e] = qdiv_fxp_fast(" << a << ", " << rq
        << ", &ok); " << t << "_slow |= !ok; }\n"
        << "      if (" << t << "_slow) {\n#pragma unroll\n      for (int e = 0; e < 8; ++e) { bool ok; "
        << "(void)qdiv_fxp_fast(" << a << ", " << rq << ", &ok); if (!ok) " << t << "[e] = qdiv_fxp(" << a << ", "
        << sv << ", " << rq << ", " << qf->iw << "u); }\n      }\n";
      name[in.dst & 15] = t + "[e]";
      continue;
    }
    const char* expr = op_expr(in.op);
    if (!expr) return false;
    const int ar = arity_of(in.op);
    const std::string A = ar > 0 ? name[in.a & 15] : "0u", B = ar > 1 ? name[in.b & 15] : "0u",
                      C = ar > 2 ? name[in.c & 15] : "0u";
    o << "      unsigned " << t << "[8];\n#pragma unroll\n      for (int e = 0; e < 8; ++e) { const unsigned a = " << A
      << ", b = " << B << ", c = " << C
      << "; const int ia = (int)a, ib = (int)b; const float fa = F(a), fb = F(b), fc = F(c); const int imm = "
      << in.imm_i << "; (void)ia; (void)ib; (void)fa; (void)fb; (void)fc; (void)c; (void)imm; " << t << "[e] = ("
      << expr << "); }\n";
    name[in.dst & 15] = t + "[e]";
  }
  *ret = name[p.ret & 15];
  return true;
}

bool emit_program(std::ostringstream& o, const fopt_program& p, int n_in, std::string* ret) {
  std::string names[16];
  for (int k = 0; k < n_in && k < 16; ++k) names[k] = "x" + std::to_string(k) + "[e]";
  return emit_program_named(o, p, names, n_in, ret);
}

// Loads the 8 elements at `base` of every input into x0..x2 (modes as for generate below).
void emit_loads(std::ostringstream& o, int n_in, const fopt_dtype* in_dt, const int* modes) {
  for (int k = 0; k < n_in; ++k) {
    const std::string bk = "b" + std::to_string(k), xk = "x" + std::to_string(k);
    if (modes[k] == 1)
      o << "      { const unsigned v = " << load_one(k, in_dt[k], "base / " + bk) << "; for (int e = 0; e < 8; ++e) " << xk
        << "[e] = v; }\n";
    else
      o << "      " << load_vec(k, in_dt[k], modes[k] == 2 ? "base % " + bk : "base");
  }
}

}  // namespace
// Returns "" when the program uses an opcode the table lacks (the interpreter then runs it).
// modes[k]: 0 input k is read at the element index i, 1 at i / b_k (a per-row value broadcast along
// rows of b_k elements), 2 at i % b_k (a row of b_k values repeated); b_k is a multiple of 8, so an
// 8-element group never straddles a row.
std::string generate(const fopt_program& p, int n_in, const fopt_dtype* in_dt, int out_dt, const int* modes) {
  std::ostringstream o;
  o << kPrelude << "\nusing namespace fopt::ew;\n"
    << "extern \"C\" __global__ void __launch_bounds__(256) fopt_ew_gen(const void* __restrict__ in0, "
       "const void* __restrict__ in1, const void* __restrict__ in2, void* __restrict__ out, long long n, "
       "long long b0, long long b1, long long b2) {\n"
    << "  const long long stride = (long long)gridDim.x * blockDim.x * 8;\n"
    << "  for (long long base = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 8; base < n; base += stride) {\n"
    << "    unsigned x0[8], x1[8], x2[8], r[8];\n"
    << "    const bool full = base + 8 <= n;\n"
    << "    if (full) {\n";
  emit_loads(o, n_in, in_dt, modes);
  o << "    } else {\n";
  for (int k = 0; k < n_in; ++k) {
    const std::string bk = "b" + std::to_string(k);
    const std::string idx = modes[k] == 1 ? "(base + e) / " + bk : modes[k] == 2 ? "(base + e) % " + bk : "base + e";
    o << "      for (int e = 0; e < 8; ++e) x" << k << "[e] = base + e < n ? " << load_one(k, in_dt[k], idx)
      << " : 0u;\n";
  }
  o << "    }\n#pragma unroll\n    for (int e = 0; e < 8; ++e) {\n";
  std::string ret;
  if (!emit_program(o, p, n_in, &ret)) return "";
  o << "      r[e] = " << ret << ";\n    }\n"
    << "    if (full) " << store_vec(out_dt) << "    else for (int e = 0; e < 8; ++e) if (base + e < n) "
    << store_one(out_dt, "base + e", "r[e]") << "\n  }\n}\n";
  return o.str();
}

namespace {
struct Entry {
  CUfunction fn = nullptr;
  bool failed = false;
};
std::mutex g_mu;
std::map<std::string, Entry> g_cache;

// Compiles (once per key) the source that make_src returns and fetches its kernel `entry`.
template <typename MakeSrc>
CUfunction compiled(const std::string& key, MakeSrc make_src, const char* entry) {
  Jit& j = jit();
  if (!j.ok) return nullptr;
  std::lock_guard<std::mutex> g(g_mu);
  auto it = g_cache.find(key);
  if (it != g_cache.end()) return it->second.failed ? nullptr : it->second.fn;
  Entry& e = g_cache[key];
  e.failed = true;
  std::string src = make_src();
  if (src.empty()) return nullptr;
  nvrtcProgram prog;
  if (j.create(&prog, src.c_str(), "fopt_gen.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS) return nullptr;
  const char* opts[] = {"--gpu-architecture=sm_100a", "--std=c++17", "--fmad=false"};
  nvrtcResult rc = j.compile(prog, 3, opts);
  if (rc != NVRTC_SUCCESS) {
    if (getenv("FOPT_EW_JIT_LOG") && j.log_size && j.log) {
      size_t n = 0;
      j.log_size(prog, &n);
      std::string logs(n, '\0');
      j.log(prog, &logs[0]);
      fprintf(stderr, "fopt JIT failed:\n%s\n", logs.c_str());
    }
    j.destroy(&prog);
    return nullptr;
  }
  size_t n = 0;
  j.cubin_size(prog, &n);
  std::string bin(n, '\0');
  j.cubin(prog, &bin[0]);
  j.destroy(&prog);
  CUmodule mod;
  if (j.load(&mod, bin.data()) != CUDA_SUCCESS) return nullptr;
  CUfunction fn;
  if (j.get_fn(&fn, mod, entry) != CUDA_SUCCESS) return nullptr;
  e.fn = fn;
  e.failed = false;
  return fn;
}

std::string program_key(const fopt_program& p, int n_in, const fopt_dtype* in_dt, const int* modes) {
  std::string key((const char*)&p, sizeof(int32_t) * 2 + sizeof(fopt_insn) * p.n_insn);
  for (int k = 0; k < n_in; ++k) key += "," + std::to_string(in_dt[k]) + "/" + std::to_string(modes[k]);
  return key;
}

CUfunction kernel_for(fopt_ctx* ctx, const fopt_program& p, int n_in, const fopt_dtype* in_dt, int out_dt,
                      const int* modes) {
  const std::string key = "ew|" + program_key(p, n_in, in_dt, modes) + "|" + std::to_string(ctx->device) + ":" +
                          std::to_string(out_dt);
  return compiled(key, [&] { return generate(p, n_in, in_dt, out_dt, modes); }, "fopt_ew_gen");
}

// A row reduction of the program's values: one warp per row of W elements (W a multiple of 8), in
// a fixed order that does not depend on the launch: 8-element group g of the row goes to slot
// g % 256 and each slot folds its groups in order (lane L keeps slots L + 32 j, j < 8, in acc[j]);
// a butterfly folds each set of 32 slots, then the 8 results fold in order j = 0 .. 7. The row
// programs (generate_row) fold in the same order with one thread per slot. fold: 0 f32 add, 2 max, 3 min, 4 f32 mul (f32 values), 10 i32 wrapping add, 12 / 13 i32
// max / min.
std::string generate_reduce(const fopt_program& p, int n_in, const fopt_dtype* in_dt, const int* modes, int fold) {
  std::ostringstream o;
  const char* f = nullptr;
  switch (fold) {
    case 0: f = "W(__fadd_rn(F(u), F(v)))"; break;
    case 2: f = "W(fmaxf(F(u), F(v)))"; break;
    case 3: f = "W(fminf(F(u), F(v)))"; break;
    case 4: f = "W(__fmul_rn(F(u), F(v)))"; break;
    case 10: f = "(u + v)"; break;
    case 12: f = "(unsigned)max((int)u, (int)v)"; break;
    case 13: f = "(unsigned)min((int)u, (int)v)"; break;
    default: return "";
  }
  o << kPrelude << "\nusing namespace fopt::ew;\n"
    << "__device__ __forceinline__ unsigned fold(unsigned u, unsigned v) { return " << f << "; }\n"
    << "extern \"C\" __global__ void __launch_bounds__(256) fopt_red_gen(const void* __restrict__ in0, "
       "const void* __restrict__ in1, const void* __restrict__ in2, unsigned* __restrict__ out, long long rows, "
       "long long row_len, long long b0, long long b1, long long b2, unsigned ident) {\n"
    << "  const int lane = threadIdx.x & 31;\n"
    << "  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;\n"
    << "  for (long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows; row += nw) {\n"
    << "    unsigned acc[8];\n"
    << "#pragma unroll\n    for (int j = 0; j < 8; ++j) acc[j] = ident;\n"
    << "    for (long long c0 = 8 * lane; c0 < row_len; c0 += 2048) {\n"
    << "#pragma unroll\n    for (int j = 0; j < 8; ++j) {\n"
    << "      const long long c = c0 + 256 * j;\n"
    << "      if (c >= row_len) break;\n"
    << "      const long long base = row * row_len + c;\n"
    << "      unsigned x0[8], x1[8], x2[8];\n";
  emit_loads(o, n_in, in_dt, modes);
  o << "#pragma unroll\n      for (int e = 0; e < 8; ++e) {\n";
  std::string ret;
  if (!emit_program(o, p, n_in, &ret)) return "";
  o << "        acc[j] = fold(acc[j], " << ret << ");\n      }\n    }\n    }\n"
    << "#pragma unroll\n    for (int j = 0; j < 8; ++j)\n"
    << "#pragma unroll\n      for (int m = 16; m; m >>= 1) acc[j] = fold(acc[j], __shfl_xor_sync(0xffffffffu, acc[j], m));\n"
    << "    unsigned r = acc[0];\n"
    << "#pragma unroll\n    for (int j = 1; j < 8; ++j) r = fold(r, acc[j]);\n"
    << "    if (lane == 0) out[row] = r;\n  }\n}\n";
  return o.str();
}


// ---- row programs ----
const char* fold_expr(int fold) {
  switch (fold) {
    case 0: return "W(__fadd_rn(F(u), F(v)))";
    case 2: return "W(fmaxf(F(u), F(v)))";
    case 3: return "W(fminf(F(u), F(v)))";
    case 4: return "W(__fmul_rn(F(u), F(v)))";
    case 10: return "(u + v)";
    case 12: return "(unsigned)max((int)u, (int)v)";
    case 13: return "(unsigned)min((int)u, (int)v)";
    default: return nullptr;
  }
}

// Which of the first n registers the program reads before writing them (its inputs in use).
unsigned inputs_read(const fopt_program& p, int n) {
  unsigned used = 0, written = 0;
  for (int i = 0; i < p.n_insn; ++i) {
    const fopt_insn& in = p.insn[i];
    const int ar = arity_of(in.op), rs[3] = {in.a & 15, in.b & 15, in.c & 15};
    for (int q = 0; q < ar; ++q)
      if (rs[q] < n && !(written >> rs[q] & 1)) used |= 1u << rs[q];
    written |= 1u << (in.dst & 15);
  }
  if ((p.ret & 15) < n && !(written >> (p.ret & 15) & 1)) used |= 1u << (p.ret & 15);
  return used;
}

// words (32-bit) of one 8-element group of a leaf held raw
int raw_words(int dt) { return dtype_bits(dt) / 4; }

std::string raw_load(int k, int dt, const std::string& dst) {
  const std::string in = "in" + std::to_string(k);
  std::ostringstream o;
  switch (dtype_bits(dt)) {
    case 32:
      o << "{ const uint4* q = (const uint4*)" << in << " + (base >> 2); const uint4 u0 = q[0], u1 = q[1]; " << dst
        << "[0]=u0.x; " << dst << "[1]=u0.y; " << dst << "[2]=u0.z; " << dst << "[3]=u0.w; " << dst << "[4]=u1.x; "
        << dst << "[5]=u1.y; " << dst << "[6]=u1.z; " << dst << "[7]=u1.w; }\n";
      break;
    case 16:
      o << "{ const uint4 u = *((const uint4*)" << in << " + (base >> 3)); " << dst << "[0]=u.x; " << dst << "[1]=u.y; "
        << dst << "[2]=u.z; " << dst << "[3]=u.w; }\n";
      break;
    default:
      o << "{ const uint2 u = *((const uint2*)" << in << " + (base >> 3)); " << dst << "[0]=u.x; " << dst
        << "[1]=u.y; }\n";
  }
  return o.str();
}

// x[0..7] from the raw words of one group (the element forms load_vec gives)
std::string raw_unpack(int dt, const std::string& raw, const std::string& x) {
  std::ostringstream o;
  switch (dtype_bits(dt)) {
    case 32: o << "for (int j = 0; j < 8; ++j) " << x << "[j] = " << raw << "[j];\n"; break;
    case 16:
      if (dt == FOPT_BF16)
        o << "for (int j = 0; j < 4; ++j) { " << x << "[2*j] = " << raw << "[j] << 16; " << x << "[2*j+1] = " << raw
          << "[j] & 0xffff0000u; }\n";
      else
        o << "for (int j = 0; j < 4; ++j) { " << x << "[2*j] = (unsigned)(int)(short)(" << raw << "[j] & 0xffffu); "
          << x << "[2*j+1] = (unsigned)((int)" << raw << "[j] >> 16); }\n";
      break;
    default: {
      const bool sgn = dt == FOPT_I8 || dt == FOPT_I5;
      o << "for (int j = 0; j < 8; ++j) { const unsigned b = (" << raw << "[j >> 2] >> (8 * (j & 3))) & 0xffu; " << x
        << "[j] = " << (sgn ? "(unsigned)(int)(signed char)b" : "b") << "; }\n";
    }
  }
  return o.str();
}

std::string load_at(int dt, const std::string& ptr, const std::string& i) {
  switch (dt) {
    case FOPT_I32: case FOPT_F32: return "((const unsigned*)" + ptr + ")[" + i + "]";
    case FOPT_BF16: return "(((unsigned)((const unsigned short*)" + ptr + ")[" + i + "]) << 16)";
    case FOPT_I16: case FOPT_I9: return "((unsigned)(int)((const short*)" + ptr + ")[" + i + "])";
    case FOPT_I8: case FOPT_I5: return "((unsigned)(int)((const signed char*)" + ptr + ")[" + i + "])";
    default: return "((unsigned)((const unsigned char*)" + ptr + ")[" + i + "])";
  }
}

// How a row program is laid out on threads: tpr threads per row (32, 64, 128 or 256; 256 / tpr rows
// per CTA of 256), each keeping spt = 256 / tpr fold slots; the row's data a later pass needs stays in
// registers (held values, and mode-0 leaves kept raw) within about 64 registers a thread.
struct RowLayout {
  int KC = 1, tpr = 256, spt = 1;
  unsigned keep_raw = 0, later_leaves = 0, held_leaves = 0;
  std::vector<int> pass_slot;  // FOLD slot index per pass, -1 for the final program
  bool unrolled = false;       // slots and groups unrolled (held values in registers)
  int held_reg_groups = 0;     // groups g = i * KC + kc < this hold their values in registers, the rest in shared memory
  size_t held_smem = 0;        // dynamic shared memory bytes of the held values kept there
  bool ok = false;
};

// Registers a thread gives to held values before the rest go to shared memory (FOPT_ROW_HELD_REGS
// overrides). SwiGLU + quantise over 14336-wide rows: all 56 in registers holds 2 rows per SM
// (161 us at 4096 rows); 8 registers and 48 KB of shared memory per row hold 4 (112 us).
constexpr int kHeldRegWords = 8;

RowLayout row_layout(const fopt_row_plan& P) {
  RowLayout L;
  const int nL = P.n_leaves, nH = P.n_held, nS = P.n_slots, nE = nL + nH + nS;
  L.KC = (int)((P.row_len + 2047) / 2048);
  for (int j = 0; j < nS; ++j)
    if (P.slot[j].kind == FOPT_ROW_FOLD) L.pass_slot.push_back(j);
  L.pass_slot.push_back(-1);
  auto pass_prog = [&](int j) -> const fopt_program& { return j < 0 ? *P.final_prog : *P.slot[j].prog; };
  for (size_t q = 1; q < L.pass_slot.size(); ++q)
    L.later_leaves |= inputs_read(pass_prog(L.pass_slot[q]), nE) & ((1u << nL) - 1);
  for (int h = 0; h < nH; ++h) L.held_leaves |= inputs_read(*P.held[h], nL);
  if (nH * 8 * L.KC > 64) return L;  // held values must fit in registers
  int words = nH * 8;                // registers per slot and group of 8 elements
  // Without held values the passes loop over the row (small code, few registers, many rows per
  // SM) and read their leaves again from cache. With held values every slot and group is unrolled
  // to keep them in registers; leaves a later pass reads are then kept raw when they fit too.
  L.unrolled = nH > 0;
  for (int k = 0; L.unrolled && k < nL; ++k)
    if ((L.later_leaves >> k & 1) && P.leaf_bcast[k] == 0 && (words + raw_words(P.leaf_dtype[k])) * L.KC <= 64) {
      L.keep_raw |= 1u << k;
      words += raw_words(P.leaf_dtype[k]);
    }
  L.tpr = 256;
  for (int tpr = 32; tpr <= 256; tpr *= 2)
    if ((256 / tpr) * L.KC * words <= 64) {
      L.tpr = tpr;
      break;
    }
  // enough warps to hide latency: about 192 per SM over the 148 SMs, counted over the whole grid
  // (RMSNorm + quantise over 4096 x 4096: 32 / 64 / 128 / 256 threads a row took 44.3 / 42.2 / 40.2
  // / 38.2 us; more threads a row shorten each row's chain of passes)
  while (L.tpr < 256 && P.rows * (L.tpr / 32) < 148 * 192) L.tpr *= 2;
  L.spt = 256 / L.tpr;
  // Held values beyond a register budget go to shared memory ([group][element][thread], one bank
  // per lane): a row's activation then takes fewer registers and more rows stay resident per SM.
  const int groups = L.spt * L.KC;
  L.held_reg_groups = groups;
  if (L.unrolled && nH > 0) {
    static const int budget = [] {
      const char* e = getenv("FOPT_ROW_HELD_REGS");
      return e ? atoi(e) : kHeldRegWords;
    }();
    L.held_reg_groups = std::min(groups, budget / (nH * 8));
    L.held_smem = (size_t)(groups - L.held_reg_groups) * nH * 8 * 256 * sizeof(unsigned);
  }
  L.ok = true;
  return L;
}

// Thread t of a row (lane = t % 32, warp w = t / 32 of nw = tpr / 32) keeps slots 32 j + lane for
// j = w + nw i (i < spt): the 8-element groups g = 32 j + lane + 256 kc of the row, folded in kc
// order, which is the order generate_reduce documents. Passes: one per FOLD slot, then the final
// program.
std::string generate_row(const fopt_row_plan& P, const int* folds) {
  const int nL = P.n_leaves, nH = P.n_held, nS = P.n_slots, nE = nL + nH + nS;
  const int64_t W = P.row_len;
  const RowLayout L = row_layout(P);
  if (!L.ok) return "";
  const int KC = L.KC, TPR = L.tpr, SPT = L.spt, NW = TPR / 32, RPC = 256 / TPR;
  std::ostringstream o;
  int modes[FOPT_ROW_MAX_LEAVES];
  for (int k = 0; k < nL; ++k) modes[k] = P.leaf_bcast[k] == 0 ? 0 : P.leaf_bcast[k] > 0 ? 1 : 2;
  auto pass_prog = [&](int j) -> const fopt_program& { return j < 0 ? *P.final_prog : *P.slot[j].prog; };
  o << kPrelude << "\nusing namespace fopt::ew;\n";
  for (int j = 0; j < nS; ++j)
    if (P.slot[j].kind == FOPT_ROW_FOLD)
      o << "__device__ __forceinline__ unsigned fold" << j << "(unsigned u, unsigned v) { return " << fold_expr(folds[j])
        << "; }\n";
  o << "struct RowArgs { const void* in[8]; long long b[8]; const void* ld[8]; void* so[8]; void* out; long long rows; };\n"
    << "extern \"C\" __global__ void __launch_bounds__(256) fopt_row_gen(const RowArgs a) {\n"
    << "  constexpr long long RL = " << W << "LL;\n  constexpr int KC = " << KC << ", SPT = " << SPT
    << ", NW = " << NW << ", RPC = " << RPC << ", NR = " << L.held_reg_groups << ";\n  (void)NR;\n"
    << "  __shared__ unsigned part[" << std::max<size_t>(1, L.pass_slot.size() - 1) << "][RPC][8];\n"
    << "  const int t = threadIdx.x % " << TPR << ", rr = threadIdx.x / " << TPR
    << ", lane = t & 31, w = t >> 5;\n  (void)lane; (void)w; (void)rr;\n"
    << "  void* const out = a.out;\n  (void)out;\n";
  for (int k = 0; k < nL; ++k)
    // the broadcast divisor is part of the kernel's key, so it is a constant here (a power of two
    // becomes a shift or a mask instead of a 64-bit division per group)
    o << "  const void* const in" << k << " = a.in[" << k << "]; constexpr long long b" << k << " = "
      << (P.leaf_bcast[k] < 0 ? -P.leaf_bcast[k] : P.leaf_bcast[k]) << "LL; (void)b" << k << ";\n";
  o << "  for (long long row0 = (long long)blockIdx.x * RPC; row0 < a.rows; row0 += (long long)gridDim.x * RPC) {\n"
    << "    const long long row = row0 + rr;\n    const bool live = row < a.rows;\n";
  for (int k = 0; k < nL; ++k)
    if (L.keep_raw >> k & 1) o << "    unsigned raw" << k << "[SPT][KC][" << raw_words(P.leaf_dtype[k]) << "];\n";
  for (int h = 0; h < nH; ++h) o << "    unsigned hv" << h << "[SPT][KC][8];\n";
  if (L.held_smem) {
    o << "    extern __shared__ unsigned held_smem[];\n";
    for (int h = 0; h < nH; ++h)
      o << "    unsigned* const hs" << h << " = held_smem + " << h << " * (SPT * KC - NR) * 2048 + threadIdx.x;\n";
  }
  for (int j = 0; j < nS; ++j) o << "    unsigned s" << j << " = 0u;\n";
  std::string names[16];
  for (int k = 0; k < nL; ++k) names[k] = "x" + std::to_string(k) + "[e]";
  // group g = i * KC + kc is a compile-time constant once the loops unroll, so each read and write
  // below resolves to a register or to a shared-memory word
  auto held_at = [&](int h) {
    const std::string hs = std::to_string(h);
    if (!L.held_smem) return "hv" + hs + "[i][kc][e]";
    return "(i * KC + kc < NR ? hv" + hs + "[i][kc][e] : hs" + hs + "[((i * KC + kc < NR) ? 0 : i * KC + kc - NR) * 2048 + e * 256])";
  };
  for (int h = 0; h < nH; ++h) names[nL + h] = held_at(h);
  for (int j = 0; j < nS; ++j) names[nL + nH + j] = "s" + std::to_string(j);
  std::string snames[16];
  for (int j = 0; j < nS; ++j) snames[j] = "s" + std::to_string(j);
  size_t pass = 0;
  int nfold = 0;
  auto emit_pass = [&](int j) -> bool {
    const bool first = pass == 0;
    const fopt_program& prog = pass_prog(j);
    unsigned need = inputs_read(prog, nE) & ((1u << nL) - 1);
    if (first) need |= L.held_leaves;
    const std::vector<QuantFuse> fuses =
        getenv("FOPT_ROW_NO_QDIV") ? std::vector<QuantFuse>{} : find_quant_fuses(prog, nL + nH, nE);
    o << "    {\n";
    for (const auto& f : fuses)
      o << "    const float rq" << f.slot_reg << "_" << f.iw << " = qdiv_factor(" << names[f.slot_reg] << ", " << f.iw
        << "u);\n";
    if (L.unrolled) {
      if (j >= 0)
        o << "    unsigned acc[SPT];\n#pragma unroll\n    for (int i = 0; i < SPT; ++i) acc[i] = "
          << P.slot[j].identity_bits << "u;\n";
      o << "#pragma unroll\n    for (int i = 0; i < SPT; ++i)\n#pragma unroll\n    for (int kc = 0; kc < KC; ++kc) {\n";
    } else {
      o << "#pragma unroll 1\n    for (int i = 0; i < SPT; ++i) {\n";
      if (j >= 0) o << "    unsigned acc = " << P.slot[j].identity_bits << "u;\n";
      o << "#pragma unroll " << (KC <= 4 ? KC : 2) << "\n    for (int kc = 0; kc < KC; ++kc) {\n";
    }
    o << "      const long long c = 256 * (w + NW * i) + 8 * lane + 2048 * kc;\n      if (live && c < RL) {\n"
      << "      const long long base = row * RL + c;\n";
    for (int k = 0; k < nL; ++k) {
      if (!(need >> k & 1) && !(first && (L.keep_raw >> k & 1))) continue;
      const std::string xk = "x" + std::to_string(k), bk = "b" + std::to_string(k);
      o << "      unsigned " << xk << "[8];\n";
      if (L.keep_raw >> k & 1) {
        const std::string raw = "raw" + std::to_string(k) + "[i][kc]";
        if (first) o << "      " << raw_load(k, P.leaf_dtype[k], raw);
        o << "#pragma unroll\n      " << raw_unpack(P.leaf_dtype[k], raw, xk);
      } else if (modes[k] == 1) {
        o << "      { const unsigned v = " << load_one(k, P.leaf_dtype[k], "base / " + bk) << "; for (int e = 0; e < 8; ++e) "
          << xk << "[e] = v; }\n";
      } else {
        o << "      " << load_vec(k, P.leaf_dtype[k], modes[k] == 2 ? "base % " + bk : "base");
      }
    }
    if (j < 0) o << "      unsigned r[8];\n";
    if (first) {
      for (int h = 0; h < nH; ++h) {
        std::string ret;
        if (!emit_program_vec(o, *P.held[h], names, nL, &ret, "h" + std::to_string(h) + "_")) return false;
        if (!L.held_smem)
          o << "#pragma unroll\n      for (int e = 0; e < 8; ++e) hv" << h << "[i][kc][e] = " << ret << ";\n";
        else
          o << "      if (i * KC + kc < NR) {\n#pragma unroll\n      for (int e = 0; e < 8; ++e) hv" << h << "[i][kc][e] = "
            << ret << ";\n      } else {\n#pragma unroll\n      for (int e = 0; e < 8; ++e) hs" << h
            << "[(i * KC + kc - NR) * 2048 + e * 256] = " << ret << ";\n      }\n";
      }
    }
    std::string ret;
    if (!emit_program_vec(o, prog, names, nE, &ret, "t", &fuses)) return false;
    const std::string acc = L.unrolled ? "acc[i]" : "acc";
    o << "#pragma unroll\n      for (int e = 0; e < 8; ++e) {\n";
    if (j >= 0)
      o << "        " << acc << " = fold" << j << "(" << acc << ", " << ret << ");\n      }\n";
    else
      o << "        r[e] = " << ret << ";\n      }\n      " << store_vec(P.out_dtype);
    o << "      }\n    }\n";
    if (!L.unrolled) {
      // slot set w + NW i is complete: butterfly it and fold it in (NW = 1: sets come in order
      // j = i), or park it for the in-order fold across the row's warps
      if (j >= 0) {
        o << "#pragma unroll\n    for (int m = 16; m; m >>= 1) acc = fold" << j
          << "(acc, __shfl_xor_sync(0xffffffffu, acc, m));\n";
        if (NW == 1)
          o << "    s" << j << " = i == 0 ? acc : fold" << j << "(s" << j << ", acc);\n";
        else
          o << "    if (lane == 0) part[" << nfold << "][rr][w + NW * i] = acc;\n";
      }
      o << "    }\n";
      if (j >= 0 && NW > 1)
        o << "    __syncthreads();\n    s" << j << " = part[" << nfold << "][rr][0];\n#pragma unroll\n"
          << "    for (int q = 1; q < 8; ++q) s" << j << " = fold" << j << "(s" << j << ", part[" << nfold << "][rr][q]);\n";
      if (j >= 0) ++nfold;
      o << "    }\n";
      ++pass;
      return true;
    }
    if (j >= 0) {
      // butterfly per slot set, then the 8 sets in order j = 0 .. 7 (set w + NW i of this thread)
      o << "#pragma unroll\n    for (int i = 0; i < SPT; ++i)\n#pragma unroll\n"
        << "      for (int m = 16; m; m >>= 1) acc[i] = fold" << j << "(acc[i], __shfl_xor_sync(0xffffffffu, acc[i], m));\n";
      if (NW == 1) {
        o << "    s" << j << " = acc[0];\n#pragma unroll\n    for (int i = 1; i < 8; ++i) s" << j << " = fold" << j
          << "(s" << j << ", acc[i]);\n";
      } else {
        o << "    if (lane == 0)\n#pragma unroll\n      for (int i = 0; i < SPT; ++i) part[" << nfold
          << "][rr][w + NW * i] = acc[i];\n    __syncthreads();\n"
          << "    s" << j << " = part[" << nfold << "][rr][0];\n#pragma unroll\n    for (int q = 1; q < 8; ++q) s" << j
          << " = fold" << j << "(s" << j << ", part[" << nfold << "][rr][q]);\n";
      }
      ++nfold;
    }
    o << "    }\n";
    ++pass;
    return true;
  };
  for (int j = 0; j < nS; ++j) {
    const fopt_row_slot& sl = P.slot[j];
    if (sl.kind == FOPT_ROW_FOLD) {
      if (!emit_pass(j)) return "";
    } else if (sl.kind == FOPT_ROW_SCALAR) {
      o << "    {\n";
      std::string ret;
      if (!emit_program_named(o, *sl.prog, snames, j, &ret, "q" + std::to_string(j) + "_")) return "";
      o << "    s" << j << " = " << ret << ";\n    }\n";
    } else {
      o << "    if (live) s" << j << " = " << load_at(sl.dtype, "a.ld[" + std::to_string(j) + "]", "row") << ";\n";
    }
    if (sl.kind != FOPT_ROW_LOAD)
      o << "    if (t == 0 && live && a.so[" << j << "]) ((unsigned*)a.so[" << j << "])[row] = s" << j << ";\n";
  }
  if (!emit_pass(-1)) return "";
  if (NW > 1) o << "    __syncthreads();\n";
  o << "  }\n}\n";
  return o.str();
}

std::string row_key(const fopt_row_plan& P, const int* folds) {
  auto prog_bytes = [](const fopt_program* p) {
    return p ? std::string((const char*)p, sizeof(int32_t) * 2 + sizeof(fopt_insn) * p->n_insn) : std::string("-");
  };
  std::string key = "row|" + std::to_string(P.row_len) + "|" + std::to_string(P.out_dtype) + "|";
  for (int k = 0; k < P.n_leaves; ++k)
    key += std::to_string(P.leaf_dtype[k]) + "/" + std::to_string(P.leaf_bcast[k]) + ",";
  key += "|";
  for (int h = 0; h < P.n_held; ++h) key += prog_bytes(P.held[h]) + "#";
  key += "|";
  for (int j = 0; j < P.n_slots; ++j) {
    const fopt_row_slot& sl = P.slot[j];
    key += std::to_string(sl.kind) + ":" + std::to_string(folds[j]) + ":" + std::to_string(sl.identity_bits) + ":" +
           std::to_string(sl.dtype) + ":" + (sl.kind == FOPT_ROW_LOAD ? std::string("-") : prog_bytes(sl.prog)) + "#";
  }
  return key + "|" + prog_bytes(P.final_prog);
}
}  // namespace

std::atomic<int64_t> g_jit_launches{0};

// Runs the program as a generated kernel; false when that path does not apply. bcast (optional):
// per input 0 (read at i), > 0 (read at i / bcast[k]) or < 0 (read at i % -bcast[k]).
bool launch_elementwise_jit_ex(fopt_ctx* ctx, const fopt_program* prog, int n_in, const void* const* in,
                               const fopt_dtype* in_dt, const int64_t* bcast, void* out, fopt_dtype out_dt, int64_t n) {
  if (getenv("FOPT_EW_NO_JIT")) return false;
  if (dtype_bits(out_dt) < 8 || (uintptr_t)out % 16) return false;
  int modes[3] = {0, 0, 0};
  long long inner[3] = {1, 1, 1};
  for (int k = 0; k < n_in; ++k) {
    if (dtype_bits(in_dt[k]) < 8 || (uintptr_t)in[k] % 16) return false;
    if (bcast && bcast[k]) {
      const int64_t b = bcast[k] > 0 ? bcast[k] : -bcast[k];
      if (b % 8 || n % b) return false;
      modes[k] = bcast[k] > 0 ? 1 : 2;
      inner[k] = b;
    }
  }
  CUfunction fn = kernel_for(ctx, *prog, n_in, in_dt, out_dt, modes);
  if (!fn) return false;
  const void* a0 = n_in > 0 ? in[0] : out;
  const void* a1 = n_in > 1 ? in[1] : a0;
  const void* a2 = n_in > 2 ? in[2] : a0;
  long long nn = n;
  void* args[] = {(void*)&a0, (void*)&a1, (void*)&a2, (void*)&out, (void*)&nn, (void*)&inner[0], (void*)&inner[1],
                  (void*)&inner[2]};
  const int64_t threads = (n + 7) / 8;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((threads + 255) / 256, 148 * 16));
  CUresult r = jit().launch(fn, grid, 1, 1, 256, 1, 1, 0, (CUstream)ctx->stream, args, nullptr);
  if (r != CUDA_SUCCESS) throw Fail{FOPT_ERR_CUDA, "elementwise kernel launch failed"};
  ctx->launches++;
  g_jit_launches.fetch_add(1, std::memory_order_relaxed);
  return true;
}

bool launch_elementwise_jit(fopt_ctx* ctx, const fopt_program* prog, int n_in, const void* const* in,
                            const fopt_dtype* in_dt, void* out, fopt_dtype out_dt, int64_t n) {
  return launch_elementwise_jit_ex(ctx, prog, n_in, in, in_dt, nullptr, out, out_dt, n);
}

// Row reduction of a program's values (see generate_reduce); false when the generated kernel does
// not apply (no NVRTC, 4-bit types, misalignment, W not a multiple of 8).
bool launch_reduce_map_jit(fopt_ctx* ctx, const fopt_program* prog, int n_in, const void* const* in,
                           const fopt_dtype* in_dt, const int64_t* bcast, int fold, uint32_t ident, void* out,
                           int64_t rows, int64_t W) {
  if (getenv("FOPT_EW_NO_JIT")) return false;
  if (W % 8 || (uintptr_t)out % 4) return false;
  int modes[3] = {0, 0, 0};
  long long inner[3] = {1, 1, 1};
  for (int k = 0; k < n_in; ++k) {
    if (dtype_bits(in_dt[k]) < 8 || (uintptr_t)in[k] % 16) return false;
    if (bcast && bcast[k]) {
      const int64_t b = bcast[k] > 0 ? bcast[k] : -bcast[k];
      if (b % 8 || (rows * W) % b) return false;
      modes[k] = bcast[k] > 0 ? 1 : 2;
      inner[k] = b;
    }
  }
  const std::string key = "red|" + std::to_string(fold) + "|" + program_key(*prog, n_in, in_dt, modes) + "|" +
                          std::to_string(ctx->device);
  CUfunction fn = compiled(key, [&] { return generate_reduce(*prog, n_in, in_dt, modes, fold); }, "fopt_red_gen");
  if (!fn) return false;
  const void* a0 = n_in > 0 ? in[0] : out;
  const void* a1 = n_in > 1 ? in[1] : a0;
  const void* a2 = n_in > 2 ? in[2] : a0;
  long long rr = rows, ww = W;
  unsigned id = ident;
  void* args[] = {(void*)&a0, (void*)&a1, (void*)&a2, (void*)&out, (void*)&rr, (void*)&ww,
                  (void*)&inner[0], (void*)&inner[1], (void*)&inner[2], (void*)&id};
  const int64_t warps = rows;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((warps * 32 + 255) / 256, 148 * 16));
  CUresult r = jit().launch(fn, grid, 1, 1, 256, 1, 1, 0, (CUstream)ctx->stream, args, nullptr);
  if (r != CUDA_SUCCESS) throw Fail{FOPT_ERR_CUDA, "reduce kernel launch failed"};
  ctx->launches++;
  g_jit_launches.fetch_add(1, std::memory_order_relaxed);
  return true;
}


// The fold code (generate_reduce's numbering) of a reduce op on a 32-bit value type, -1 if none.
int row_fold_code(int dtype, int op, bool exact) {
  if (dtype == FOPT_F32) {
    if (op == FOPT_RED_MAX) return 2;
    if (op == FOPT_RED_MIN) return 3;
    if (!exact && op == FOPT_RED_ADD) return 0;
    if (!exact && op == FOPT_RED_MUL) return 4;
  } else if (dtype == FOPT_I32) {
    if (op == FOPT_RED_ADD) return 10;
    if (op == FOPT_RED_MAX) return 12;
    if (op == FOPT_RED_MIN) return 13;
  }
  return -1;
}

// Validates a row plan's shape and fills the fold codes; false when the generated kernel does not
// apply to it (pointers are not looked at).
bool row_plan_supported(const fopt_row_plan& P, bool exact, int* folds) {
  if (P.n_leaves < 0 || P.n_leaves > FOPT_ROW_MAX_LEAVES || P.n_held < 0 || P.n_held > FOPT_ROW_MAX_HELD ||
      P.n_slots < 0 || P.n_slots > FOPT_ROW_MAX_SLOTS || P.n_leaves + P.n_held + P.n_slots > 16)
    return false;
  if (P.row_len <= 0 || P.row_len % 8 || P.row_len > 32768 || P.rows <= 0 || !P.final_prog) return false;
  if (dtype_bits(P.out_dtype) < 8) return false;
  for (int k = 0; k < P.n_leaves; ++k) {
    if (dtype_bits(P.leaf_dtype[k]) < 8) return false;
    const int64_t b = P.leaf_bcast[k] < 0 ? -P.leaf_bcast[k] : P.leaf_bcast[k];
    if (b && b % 8) return false;
  }
  for (int h = 0; h < P.n_held; ++h)
    if (!P.held[h] || P.held[h]->n_insn > 32) return false;
  for (int j = 0; j < P.n_slots; ++j) {
    const fopt_row_slot& sl = P.slot[j];
    folds[j] = -1;
    if (sl.kind == FOPT_ROW_FOLD) {
      if (!sl.prog || sl.prog->n_insn > 32 || (folds[j] = row_fold_code(sl.dtype, sl.op, exact)) < 0) return false;
    } else if (sl.kind == FOPT_ROW_SCALAR) {
      if (!sl.prog || sl.prog->n_insn > 32 || (sl.dtype != FOPT_F32 && sl.dtype != FOPT_I32)) return false;
    } else if (sl.kind == FOPT_ROW_LOAD) {
      if (dtype_bits(sl.dtype) < 8) return false;
    } else {
      return false;
    }
  }
  return P.final_prog->n_insn <= 32;
}

bool launch_row_jit(fopt_ctx* ctx, const fopt_row_plan& P) {
  if (getenv("FOPT_EW_NO_JIT")) return false;
  int folds[FOPT_ROW_MAX_SLOTS];
  if (!row_plan_supported(P, ctx->exact_fold, folds)) return false;
  if ((uintptr_t)P.out % 16) return false;
  for (int k = 0; k < P.n_leaves; ++k)
    if (!P.leaf[k] || (uintptr_t)P.leaf[k] % 16) return false;
  for (int j = 0; j < P.n_slots; ++j) {
    if (P.slot[j].kind == FOPT_ROW_LOAD && !P.slot[j].src) return false;
    if (P.slot[j].out && (uintptr_t)P.slot[j].out % 4) return false;
  }
  const std::string key = row_key(P, folds) + "|" + std::to_string(ctx->device);
  CUfunction fn = compiled(key, [&] { return generate_row(P, folds); }, "fopt_row_gen");
  if (!fn) return false;
  struct RowArgs {
    const void* in[8];
    long long b[8];
    const void* ld[8];
    void* so[8];
    void* out;
    long long rows;
  } args{};
  for (int k = 0; k < P.n_leaves; ++k) {
    args.in[k] = P.leaf[k];
    args.b[k] = P.leaf_bcast[k] < 0 ? -P.leaf_bcast[k] : P.leaf_bcast[k];
  }
  for (int j = 0; j < P.n_slots; ++j) {
    args.ld[j] = P.slot[j].kind == FOPT_ROW_LOAD ? P.slot[j].src : nullptr;
    args.so[j] = P.slot[j].kind == FOPT_ROW_LOAD ? nullptr : P.slot[j].out;
  }
  args.out = P.out;
  args.rows = P.rows;
  void* params[] = {(void*)&args};
  const RowLayout L = row_layout(P);
  const int rpc = 256 / L.tpr;
  const unsigned grid = (unsigned)std::min<int64_t>((P.rows + rpc - 1) / rpc, 1 << 30);
  if (L.held_smem &&
      jit().set_attr(fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, (int)L.held_smem) != CUDA_SUCCESS)
    throw Fail{FOPT_ERR_CUDA, "row program shared memory attribute refused"};
  CUresult r = jit().launch(fn, grid, 1, 1, 256, 1, 1, (unsigned)L.held_smem, (CUstream)ctx->stream, params, nullptr);
  if (r != CUDA_SUCCESS) throw Fail{FOPT_ERR_CUDA, "row program launch failed"};
  ctx->launches++;
  g_jit_launches.fetch_add(1, std::memory_order_relaxed);
  return true;
}
}  // namespace fopt

extern "C" fopt_status fopt_reduce_map_source(const fopt_program* prog, int32_t n_in, const fopt_dtype* in_dtypes,
                                              int32_t fold, char* buf, size_t len, size_t* needed) {
  if (!prog || n_in < 0 || n_in > 3) return FOPT_ERR_INVALID;
  const int modes[3] = {0, 0, 0};
  std::string src = fopt::generate_reduce(*prog, n_in, in_dtypes, modes, fold);
  if (src.empty()) return FOPT_ERR_UNSUPPORTED;
  if (needed) *needed = src.size() + 1;
  if (buf && len) {
    size_t n = std::min(len - 1, src.size());
    memcpy(buf, src.data(), n);
    buf[n] = 0;
  }
  return FOPT_OK;
}

extern "C" int64_t fopt_elementwise_jit_launches(void) { return fopt::g_jit_launches.load(); }

extern "C" fopt_status fopt_elementwise_source(const fopt_program* prog, int32_t n_in, const fopt_dtype* in_dtypes,
                                               fopt_dtype out_dtype, char* buf, size_t len, size_t* needed) {
  if (!prog || n_in < 0 || n_in > 3) return FOPT_ERR_INVALID;
  const int modes[3] = {0, 0, 0};
  std::string src = fopt::generate(*prog, n_in, in_dtypes, out_dtype, modes);
  if (src.empty()) return FOPT_ERR_UNSUPPORTED;
  if (needed) *needed = src.size() + 1;
  if (buf && len) {
    size_t n = std::min(len - 1, src.size());
    memcpy(buf, src.data(), n);
    buf[n] = 0;
  }
  return FOPT_OK;
}

extern "C" fopt_status fopt_row_program_source(const fopt_row_plan* plan, char* buf, size_t len, size_t* needed) {
  int folds[FOPT_ROW_MAX_SLOTS];
  if (!plan) return FOPT_ERR_INVALID;
  if (!fopt::row_plan_supported(*plan, false, folds)) return FOPT_ERR_UNSUPPORTED;
  std::string src = fopt::generate_row(*plan, folds);
  if (src.empty()) return FOPT_ERR_UNSUPPORTED;
  if (needed) *needed = src.size() + 1;
  if (buf && len) {
    size_t n = std::min(len - 1, src.size());
    memcpy(buf, src.data(), n);
    buf[n] = 0;
  }
  return FOPT_OK;
}
