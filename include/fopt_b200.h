/* fopt_b200.h -- C ABI of the furiosa-opt B200 execution backend.
 *
 * The reference crate `furiosa-opt-std` runs every tensor value-op of its CPU emulator through the
 * `Backend` trait (furiosa-opt-std/src/backend/mod.rs:41-248), which `Cpu` forwards to
 * `BufStorage` (furiosa-opt-std/src/storage/buf.rs). This header is the seam a `B200` backend binds
 * instead: every `BufStorage` value-op below runs as sm_100a CUDA kernels on the packed device byte
 * image (element i at position i, padding included, 4-bit types two per byte low nibble first --
 * furiosa-opt-std/src/scalar.rs:45-94,657-680).
 *
 * Conventions follow the NPU runtime header the reference already binds
 * (furiosa-opt-std/vendor/x86_64-unknown-linux-gnu/device_runtime.h:86-233): opaque handles, an
 * int32 status (0 = OK), caller-owned buffers, no exceptions across the boundary. A non-zero status
 * leaves a message in fopt_last_error(); the Rust binding panics with it, as the reference panics on
 * an ill-formed mapping (buf.rs:279,718).
 *
 * Mappings cross the boundary as text in the `m!` grammar
 * (furiosa-mapping-macro/src/parser/parser.lalrpop) with the axis sizes declared beside them
 * ("A=8, B=512"), which is what `furiosa_mapping::Mapping`'s Display plus its symbol sizes print.
 *
 * All ops are asynchronous on the context's stream; fopt_sync() waits. Device pointers are plain
 * `void*` from fopt_alloc() (or any cudaMalloc'd memory on the context's device).
 */
#ifndef FOPT_B200_H
#define FOPT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t fopt_status;
typedef struct fopt_ctx fopt_ctx;
typedef struct fopt_mapping fopt_mapping;

enum {
  FOPT_OK = 0,
  FOPT_ERR_INVALID = 1,   /* ill-formed argument or mapping */
  FOPT_ERR_CUDA = 2,      /* a CUDA runtime call failed */
  FOPT_ERR_UNSUPPORTED = 3,
  FOPT_ERR_NCCL = 4,
  FOPT_ERR_TIMEOUT = 5    /* a bounded device-side wait gave up */
};

/* Element types (furiosa-opt-std/src/scalar.rs:10-19). Storage width in bits: I4/F4E2M1 4 (packed),
 * I8/I5/F8* 8, I16/I9/BF16 16, I32/F32 32. I5/I9 are the zero-point staging types, held in the
 * i8/i16 that back them (scalar.rs:777-781,884-888). */
typedef enum {
  FOPT_I8 = 0, FOPT_I16 = 1, FOPT_I32 = 2, FOPT_BF16 = 3, FOPT_F32 = 4,
  FOPT_I4 = 5, FOPT_F8E4M3 = 6, FOPT_F8E5M2 = 7, FOPT_F4E2M1 = 8, FOPT_I5 = 9, FOPT_I9 = 10
} fopt_dtype;

/* ---- context (replaces furiosa_runtime_init / Context::acquire, backend/npu/ffi.rs:79-175) ---- */
fopt_status fopt_init(int device, fopt_ctx** out);
fopt_status fopt_destroy(fopt_ctx* ctx);
const char* fopt_last_error(const fopt_ctx* ctx);
fopt_status fopt_sync(fopt_ctx* ctx);
/* Use an external cudaStream_t (NULL = the context's own stream). */
fopt_status fopt_set_stream(fopt_ctx* ctx, void* stream);
void* fopt_get_stream(fopt_ctx* ctx);
/* Reduce/contraction fold order: 0 = fastest (float sums may reassociate), 1 = the reference's
 * per-cell wire order (bit-exact with BufStorage for every dtype). */
fopt_status fopt_set_exact_fold(fopt_ctx* ctx, int exact);
/* Number of kernels this library launched on the context since creation. */
int64_t fopt_launch_count(const fopt_ctx* ctx);

/* ---- memory (BufStorage::zeroed / from_buf / into_buf, buf.rs:83-109,627-629) ---- */
/* Allocations are stream-ordered (the device's memory pool, on the context's stream): they do not
 * synchronise the device, and released blocks are reused. */
fopt_status fopt_alloc(fopt_ctx* ctx, size_t bytes, void** dptr); /* zero-filled */
/* For outputs an op fully overwrites (map / zip / reduce / contraction results): no zero fill. */
fopt_status fopt_alloc_uninit(fopt_ctx* ctx, size_t bytes, void** dptr);
fopt_status fopt_free(fopt_ctx* ctx, void* dptr);
fopt_status fopt_h2d(fopt_ctx* ctx, void* dst, const void* host, size_t bytes);
fopt_status fopt_d2h(fopt_ctx* ctx, void* host, const void* src, size_t bytes);
fopt_status fopt_d2d(fopt_ctx* ctx, void* dst, const void* src, size_t bytes);
fopt_status fopt_memset(fopt_ctx* ctx, void* dst, int value, size_t bytes);
/* PartialEq for BufStorage is byte equality (buf.rs:38-41): *equal = 1 iff the images match. */
fopt_status fopt_equal(fopt_ctx* ctx, const void* a, const void* b, size_t bytes, int* equal);

/* ---- mappings (furiosa-mapping-types/src/lib.rs:144-232, dsl.rs:23-277) ---- */
fopt_status fopt_mapping_parse(const char* axes, const char* expr, fopt_mapping** out);
fopt_status fopt_mapping_free(fopt_mapping* m);
int64_t fopt_mapping_size(const fopt_mapping* m);
/* M::map(pos) (dsl.rs:31): returns 0 live (coords[i] = coordinate of the i-th declared axis),
 * 1 + PaddingKind (Bottom=0, Zero=1, Top=2) for padding, -1 out of bounds. */
int32_t fopt_mapping_eval(const fopt_mapping* m, int64_t pos, int64_t* coords, int32_t ncoords);
/* window_base (buf.rs:760-781): wire position of a partial-view offset given as "A:2, B:0". */
fopt_status fopt_window_base(const fopt_mapping* base, const char* offset, int64_t* out);
/* Human-readable walk the planner derived for transpose(src -> dst), for diagnostics. */
fopt_status fopt_describe_relayout(const fopt_mapping* src, const fopt_mapping* dst, int allow_broadcast,
                                   char* buf, size_t len);

/* ---- layout moves ---- */
/* BufStorage::transpose (buf.rs:257-313; Backend::transpose, backend/mod.rs:118-126): every live
 * position q of the `dst_map` stream writes dst[dst_base + q] = src[src_base + s(q)], where s(q) is
 * the src wire position holding the same logical index (axes absent from src broadcast). Dead
 * (padding / write-hole) positions are left untouched. src_map is the `Src` type, dst_map the
 * `Mapping` type of the reference signature; bases come from fopt_window_base. */
fopt_status fopt_transpose(fopt_ctx* ctx, void* dst, const void* src, fopt_dtype dtype,
                           const fopt_mapping* src_map, const fopt_mapping* dst_map,
                           int64_t src_base, int64_t dst_base, int allow_broadcast);
/* BufStorage::transmute (buf.rs:592-613, 785-795): dst (fresh, dst_map-sized) receives src's live
 * elements in wire order at its own live positions; padding becomes zero. */
fopt_status fopt_transmute(fopt_ctx* ctx, void* dst, const void* src, fopt_dtype dtype,
                           const fopt_mapping* src_map, const fopt_mapping* dst_map);
/* BufStorage::gather (buf.rs:524-576) and scatter (buf.rs:485-520). `payload` is the payload
 * mapping (the axes shared by table and output), `axis_map` the indexed axis, `idx_map` the index
 * tensor's mapping; indices are i32 (byte offsets when `scaled`). Scatter is last-write-wins in key
 * order, as in the reference's serial loop. */
fopt_status fopt_gather(fopt_ctx* ctx, void* dst, const void* table, const int32_t* index, fopt_dtype dtype,
                        const fopt_mapping* src_map, const fopt_mapping* dst_map, const fopt_mapping* payload,
                        const fopt_mapping* axis_map, const fopt_mapping* idx_map, int scaled);
fopt_status fopt_scatter(fopt_ctx* ctx, void* dst, const void* src, const int32_t* index, fopt_dtype dtype,
                         const fopt_mapping* src_map, const fopt_mapping* dst_map, const fopt_mapping* payload,
                         const fopt_mapping* key_map, const fopt_mapping* axis_map, int scaled);

/* ---- elementwise (BufStorage::map / zip_with / zip3_with, buf.rs:203-250) ----
 * The reference passes Rust closures; the B200 seam passes the vector-engine opcode the engine
 * already holds (furiosa-opt-std/src/engine/vector/op/semantics.rs:14-360) as a small register
 * program. Registers 0..n_in-1 hold the loaded inputs as 32-bit words: signed integers sign-extend
 * to i32, bf16 widens exactly to f32 (bits << 16), f32 is its bits. The result is register `ret`;
 * the store narrows it to out_dtype by truncation (i32 -> i8/i16/i4 wrap as Rust `as` does; an f32
 * -> bf16 store keeps the top half, so round first with FOPT_OP_F32_TO_BF16). */
typedef enum {
  /* casts (furiosa-opt-std/src/cast.rs:160-290, float/bf16.rs:16-40, float/mod.rs:99-159) */
  FOPT_OP_MOV = 0,            /* dst = a */
  FOPT_OP_BF16_TO_F32 = 1,    /* flush subnormal to signed zero, canonical NaN 0x7fc00000 */
  FOPT_OP_F32_TO_BF16 = 2,    /* RNE, subnormal flush, NaN -> 0x7fc0 (result is f32 with low half 0) */
  FOPT_OP_F32_TO_BF16_RELU = 3, /* CommitCast::cast_relu (cast.rs:147-152) */
  FOPT_OP_I32_TO_F32 = 4,     /* `as f32` (round to nearest even) */
  FOPT_OP_F32_TO_I32 = 5,     /* `as i32` (truncate, saturate, NaN -> 0) */
  FOPT_OP_FXP_TO_FP = 6,      /* fixedpoint_to_float(a, imm_i = int_width) */
  FOPT_OP_FP_TO_FXP = 7,      /* float_to_fixedpoint(a, imm_i = int_width) */
  FOPT_OP_F8E4M3_TO_F32 = 8, FOPT_OP_F32_TO_F8E4M3 = 9,   /* float/f8e4.rs:10-59 */
  FOPT_OP_F8E5M2_TO_F32 = 10, FOPT_OP_F32_TO_F8E5M2 = 11, /* float/f8e5.rs:10-67 */
  FOPT_OP_I4_SEXT = 12,       /* sign-extend low 4 bits */
  FOPT_OP_I5_SEXT = 13, FOPT_OP_I9_SEXT = 14,
  FOPT_OP_F4E2M1_TO_F8E4M3 = 15, /* fetch table lookup of an e2m1 nibble (scalar.rs:933-959, cast.rs:48-52) */
  /* Fp unary (semantics.rs:77-92) */
  FOPT_OP_EXP = 20, FOPT_OP_NEGEXP = 21, FOPT_OP_SQRT = 22, FOPT_OP_TANH = 23, FOPT_OP_SIGMOID = 24,
  FOPT_OP_LOG = 25, FOPT_OP_SIN = 26, FOPT_OP_COS = 27,
  /* Fp binary / ternary (semantics.rs:94-113, 288-295) */
  FOPT_OP_ADDF = 30, FOPT_OP_SUBF = 31, FOPT_OP_MULF = 32, FOPT_OP_DIVF = 33, FOPT_OP_FMAF = 34,
  /* Clip f32 (semantics.rs:133-144) */
  FOPT_OP_MINF = 35, FOPT_OP_MAXF = 36, FOPT_OP_ABSMINF = 37, FOPT_OP_ABSMAXF = 38,
  /* Fxp / Clip i32 (semantics.rs:43-71,119-131) */
  FOPT_OP_ADD_FXP = 40, FOPT_OP_ADD_FXP_SAT = 41, FOPT_OP_SUB_FXP = 42, FOPT_OP_SUB_FXP_SAT = 43,
  FOPT_OP_SHL = 44, FOPT_OP_SHL_SAT = 45, FOPT_OP_MUL_FXP = 46, FOPT_OP_MUL_INT = 47,
  FOPT_OP_SHR_LOGIC = 48, FOPT_OP_SHR_ARITH = 49,
  FOPT_OP_MINI = 50, FOPT_OP_MAXI = 51, FOPT_OP_ABSMINI = 52, FOPT_OP_ABSMAXI = 53,
  /* Logic (semantics.rs:14-37): bitwise on the 32-bit word (f32 bit ops included) */
  FOPT_OP_AND = 60, FOPT_OP_OR = 61, FOPT_OP_XOR = 62,
  /* select: dst = (a != 0) ? b : c  (branch-tag zip3) */
  FOPT_OP_SELECT = 70,
  /* load an immediate into dst: imm_i (as i32 bits) -- f32 constants pass their bit pattern */
  FOPT_OP_CONST = 71
} fopt_opcode;

typedef struct {
  int32_t op;       /* fopt_opcode */
  int32_t dst;      /* register written (0..15) */
  int32_t a, b, c;  /* source registers (argument modes are expressed by choosing registers) */
  int32_t imm_i;    /* int width for FXP conversions; bit pattern for CONST */
} fopt_insn;

typedef struct {
  int32_t n_insn;   /* <= 32 */
  int32_t ret;      /* register stored */
  fopt_insn insn[32];
} fopt_program;

fopt_status fopt_elementwise(fopt_ctx* ctx, const fopt_program* prog, int32_t n_in, const void* const* inputs,
                             const fopt_dtype* in_dtypes, void* out, fopt_dtype out_dtype, int64_t n);
/* fopt_elementwise where an input is a broadcast that was never written out: bcast[k] = 0 reads
 * input k at the element index i, bcast[k] > 0 at i / bcast[k] (one value per row of bcast[k]
 * elements), bcast[k] < 0 at i % -bcast[k] (one row of -bcast[k] values repeated). Row lengths must be
 * multiples of 8 and divide n. Returns FOPT_ERR_UNSUPPORTED when no generated kernel applies (NVRTC
 * absent, 4-bit types, misalignment); the caller then materialises the broadcast and calls
 * fopt_elementwise. Same results as materialising first. */
fopt_status fopt_elementwise_bcast(fopt_ctx* ctx, const fopt_program* prog, int32_t n_in, const void* const* inputs,
                                   const fopt_dtype* in_dtypes, const int64_t* bcast, void* out, fopt_dtype out_dtype,
                                   int64_t n);
/* Whether relayouting src into dst with broadcasting is a plain row broadcast (*kind = 1: dst[i] =
 * src[i / *inner]) or a repeated row (*kind = 2: dst[i] = src[i % *inner]); *kind = 0 otherwise. */
fopt_status fopt_broadcast_kind(const fopt_mapping* src, const fopt_mapping* dst, int32_t* kind, int64_t* inner);
/* Diagnostic: the CUDA source of the kernel fopt_elementwise generates (NVRTC, sm_100a) for this
 * program and these dtypes (byte-multiple types). *needed = bytes including the terminator. */
fopt_status fopt_elementwise_source(const fopt_program* prog, int32_t n_in, const fopt_dtype* in_dtypes,
                                    fopt_dtype out_dtype, char* buf, size_t len, size_t* needed);
/* Diagnostic: the CUDA source of the fused row reduction fopt_reduce_map generates (fold: 0 f32 add,
 * 2 / 3 f32 max / min, 4 f32 mul, 10 i32 add, 12 / 13 i32 max / min). */
fopt_status fopt_reduce_map_source(const fopt_program* prog, int32_t n_in, const fopt_dtype* in_dtypes, int32_t fold,
                                   char* buf, size_t len, size_t* needed);
/* Diagnostic: how many fopt_elementwise calls (process-wide) ran as a generated kernel. */
int64_t fopt_elementwise_jit_launches(void);

/* ---- reduce (BufStorage::reduce, buf.rs:331-376; Backend::reduce, backend/mod.rs:128-133) ----
 * Per output cell of dst_map, fold the src cells sharing its kept coordinates, starting from
 * `identity_bits` (the 32-bit pattern of the identity in dtype's arithmetic type), in the
 * reference's wire order under exact fold. dtype I32/F32/BF16 (bf16 folds round each step). */
typedef enum {
  FOPT_RED_ADD = 0,      /* f32/bf16 `+`; i32 wrapping_add (InterSliceReduceOpI32::Add) */
  FOPT_RED_ADD_SAT = 1,  /* i32 saturating_add */
  FOPT_RED_MAX = 2, FOPT_RED_MIN = 3,
  FOPT_RED_MUL = 4       /* f32 `*` */
} fopt_reduce_op;
fopt_status fopt_reduce(fopt_ctx* ctx, void* out, const void* src, fopt_dtype dtype, fopt_reduce_op op,
                        uint32_t identity_bits, const fopt_mapping* src_map, const fopt_mapping* dst_map,
                        int allow_broadcast);

/* Engine-chain fusion of a map (or zip / zip3) followed by a reduce: reduces prog(inputs) -- the values
 * fopt_elementwise (with fopt_elementwise_bcast's broadcast codes, bcast may be NULL) would write as
 * `dtype` -- without writing them. Covers a plain row reduction (dst cell t folds src cells
 * t W .. t W + W - 1, W a multiple of 8) with a fold whose result does not depend on the order:
 * i32 Add / Max / Min, f32 Max / Min, and f32 Add / Mul outside exact-fold mode (which reassociate,
 * as fopt_reduce does there). Returns FOPT_ERR_UNSUPPORTED otherwise; the caller then writes the
 * values with fopt_elementwise and calls fopt_reduce. */
fopt_status fopt_reduce_map(fopt_ctx* ctx, void* out, const fopt_program* prog, int32_t n_in, const void* const* inputs,
                            const fopt_dtype* in_dtypes, const int64_t* bcast, fopt_dtype dtype, fopt_reduce_op op,
                            uint32_t identity_bits, const fopt_mapping* src_map, const fopt_mapping* dst_map);
/* CUDA graphs of whole steps (no counterpart in the reference, whose host drives every op). Work
 * issued on ctx between fopt_capture_begin and fopt_capture_end is recorded into a graph, not run
 * (no call in between may synchronise: fopt_sync, fopt_d2h, fopt_equal); fopt_graph_launch
 * replays it on ctx's stream. Storages allocated during the capture and not freed in it keep their
 * addresses across launches (the step's outputs) and must not be freed by the caller; they are
 * released when the graph is launched again or destroyed. Frees of older memory requested during
 * the capture happen when it ends. */
typedef struct fopt_graph fopt_graph;
fopt_status fopt_capture_begin(fopt_ctx* ctx);
fopt_status fopt_capture_end(fopt_ctx* ctx, fopt_graph** out);
fopt_status fopt_graph_launch(fopt_ctx* ctx, fopt_graph* graph);
fopt_status fopt_graph_destroy(fopt_ctx* ctx, fopt_graph* graph);

/* Diagnostic for bindings: sizes[0..3] = sizeof fopt_program, fopt_epilogue, fopt_row_slot,
 * fopt_row_plan (n >= 4), so a hand-written binding can check its struct layouts. */
fopt_status fopt_struct_sizes(size_t* sizes, int32_t n);

/* Whether reducing src_map into dst_map is a plain row reduction (dst cell t folds src cells
 * t W .. t W + W - 1): FOPT_OK with *rows and *row_len filled, FOPT_ERR_UNSUPPORTED otherwise.
 * Host-only: ctx may be NULL. */
fopt_status fopt_row_reduce_shape(fopt_ctx* ctx, const fopt_mapping* src_map, const fopt_mapping* dst_map,
                                  int64_t* rows, int64_t* row_len);

/* Engine-chain fusion across a row reduction (no single counterpart in the reference: it runs, in one
 * pass per row, what the reference does as a chain of BufStorage::reduce, broadcast transpose and
 * map / zip / zip3 calls, buf.rs:203-250, 257-313, 331-376). Each row of row_len elements is read
 * once; per-row scalars (a fold of an element program over the row, a program over earlier scalars,
 * or a load of a per-row value) are computed in order, and the final element program writes the
 * row. Element programs read registers: leaves 0 .. n_leaves-1, then held values, then slots.
 * Held values are programs over the leaves, evaluated in the first pass and kept in registers for
 * the later passes. The f32 folds use the fixed order of fopt_reduce_map (256 slots of 8-element
 * groups, each folded in order, a butterfly within each 32 slots, then the 8 partial results in
 * order), so a fused row computes the bits of the unfused chain. FOPT_ERR_UNSUPPORTED when the
 * generated kernel does not apply (no NVRTC, sub-byte types, misalignment, row_len not a multiple of
 * 8 or above 32768, exact-fold mode with an f32 Add / Mul fold); nothing is written then. */
typedef enum { FOPT_ROW_FOLD = 0, FOPT_ROW_SCALAR = 1, FOPT_ROW_LOAD = 2 } fopt_row_slot_kind;
typedef struct fopt_row_slot {
  int32_t kind;                /* fopt_row_slot_kind */
  int32_t op;                  /* FOLD: fopt_reduce_op */
  uint32_t identity_bits;      /* FOLD: the fold's start value */
  int32_t dtype;               /* FOLD / SCALAR: f32 or i32 (the value's type); LOAD: the stored type */
  const fopt_program* prog;    /* FOLD: element program; SCALAR: program over slots 0 .. this - 1 */
  const void* src;             /* LOAD: [rows] values */
  void* out;                   /* optional: [rows] 32-bit values of this slot written out */
} fopt_row_slot;
#define FOPT_ROW_MAX_LEAVES 8
#define FOPT_ROW_MAX_HELD 8
#define FOPT_ROW_MAX_SLOTS 8
typedef struct fopt_row_plan {
  int32_t n_leaves, n_held, n_slots;
  const void* leaf[FOPT_ROW_MAX_LEAVES];
  int32_t leaf_dtype[FOPT_ROW_MAX_LEAVES];
  int64_t leaf_bcast[FOPT_ROW_MAX_LEAVES]; /* 0: element i; > 0: i / b; < 0: i % -b (fopt_elementwise_bcast) */
  const fopt_program* held[FOPT_ROW_MAX_HELD];
  fopt_row_slot slot[FOPT_ROW_MAX_SLOTS];
  const fopt_program* final_prog;
  void* out;
  int32_t out_dtype;
  int64_t rows, row_len;
} fopt_row_plan;
fopt_status fopt_row_program(fopt_ctx* ctx, const fopt_row_plan* plan);
/* Diagnostic: the CUDA source fopt_row_program generates for the plan (pointers may be NULL). */
fopt_status fopt_row_program_source(const fopt_row_plan* plan, char* buf, size_t len, size_t* needed);
/* Allocation-free reduce. No counterpart in the reference: it exists for callers that cannot let the
 * library call cudaMalloc / cudaFree (a host runtime that owns the whole device-memory budget through
 * its own allocator, or a latency-critical loop that cannot absorb the device synchronisation a
 * cudaFree implies). Same arguments as fopt_reduce; the fold always runs per output cell in wire
 * order, so i32 results equal fopt_reduce's and f32 / bf16 Add / Mul equal fopt_reduce's with exact
 * fold on (f32 Max / Min may differ from fopt_reduce in the sign of a zero or which NaN is kept). Its
 * residue table lives in a fixed 256 KiB device array (at most 32768 folded cells per output, larger
 * reduces are rejected with FOPT_ERR_INVALID) that every GPU loading the library keeps until exit.
 * The first call on a device looks the array up. A call while a capture is open is refused with
 * FOPT_ERR_INVALID. All calls share the array: calls whose kernels may overlap on the GPU race. */
fopt_status fopt_reduce_noalloc(fopt_ctx* ctx, void* out, const void* src, fopt_dtype dtype, fopt_reduce_op op,
                                uint32_t identity_bits, const fopt_mapping* src_map, const fopt_mapping* dst_map,
                                int allow_broadcast);

/* ---- contraction (BufStorage::contraction_in, buf.rs:401-481; Backend::contraction /
 * contraction_prewidened, backend/mod.rs:135-157) ----
 * out[o] = narrow( sum_r widen(lhs[.]) * widen(rhs[.]) ) over the axes of pre_reduce absent from
 * out. in_dtype I8/I4/I5/I9 accumulate in i32, BF16/F8 in f32, I32/F32 are prewidened.
 * out_dtype == in_dtype narrows once per cell (contraction); out_dtype == the accumulator type
 * keeps the wide sum (the engine's contract_lane output). An optional epilogue fuses the
 * vector-engine requant chain that follows (FxpToFp -> MulF scale -> FpToFxp -> Clip -> commit). */
typedef struct {
  int32_t kind;           /* 0 none; 1 requant i32 -> i8 with per-channel scale; 2 relu;
                             3 dequant i32 -> bf16: FxpToFp -> MulF row_scale[m] -> MulF scale[n] -> cast
                             (per-token x per-channel W8A8; GEMM-shaped contractions only);
                             4 SwiGLU of interleaved gate / up projections: rhs rows (and scale) alternate
                             128 gate and 128 up channels; each is dequantised to bf16 as kind 3, then
                             act = (g * sigmoid(g)) * u in f32 (the MulF / Sigmoid chain) is written to an
                             [M, N / 2] f32 output (out_map still names the [M, N] product;
                             M % 256 and N % 256);
                             5 dequant as kind 3, then the residual add that follows it:
                             out = bf16(f32(residual) + f32(dequant)) (ResidualAdd of two bf16 values) */
  const float* scale;     /* kind 1, 3: one f32 per coordinate of `scale_axis` */
  const char* scale_axis; /* kind 1, 3: axis name the scale vector runs along (e.g. "N") */
  int32_t int_width;      /* FxpToFp / FpToFxp integer width (31 = plain integers) */
  int32_t clip_lo, clip_hi; /* kind 1: Clip bounds before the i8 commit */
  const float* row_scale; /* kind 3, 4, 5: one f32 per output row (the outer output axis, e.g. the token) */
  const void* residual;   /* kind 5: bf16 values laid out as the output */
} fopt_epilogue;
fopt_status fopt_contraction(fopt_ctx* ctx, void* out, fopt_dtype out_dtype, const void* lhs, const void* rhs,
                             fopt_dtype in_dtype, const fopt_mapping* lhs_map, const fopt_mapping* rhs_map,
                             const fopt_mapping* pre_reduce, const fopt_mapping* out_map,
                             const fopt_epilogue* epilogue);

/* ---- host I/O: safetensors straight to device (HostTensor::from_safetensors + to_hbm,
 * furiosa-opt-std/src/tensor/memory.rs:197-222) ----
 * A safetensors file: an 8-byte little-endian header length, a JSON header of
 * {name: {"dtype", "shape", "data_offsets": [begin, end]}}, then the data. fopt_st_read streams one
 * tensor's bytes (its packed image for byte-multiple dtypes) through pinned staging into device
 * memory on the context's stream. fopt_mapping_flat_shape gives the dimensions the reference
 * checks a tensor's shape against: a mapping's pair-split sizes. */
typedef struct fopt_safetensors fopt_safetensors;
fopt_status fopt_st_open(const char* path, fopt_safetensors** out);
fopt_status fopt_st_close(fopt_safetensors* st);
int32_t fopt_st_count(const fopt_safetensors* st);
fopt_status fopt_st_info(const fopt_safetensors* st, int32_t index, const char** name, const char** dtype,
                         int32_t* ndim, int64_t* shape, int32_t max_dims, int64_t* bytes);
fopt_status fopt_st_find(const fopt_safetensors* st, const char* name, int32_t* index);
fopt_status fopt_st_read(fopt_ctx* ctx, const fopt_safetensors* st, int32_t index, void* dst, size_t bytes);
fopt_status fopt_mapping_flat_shape(const fopt_mapping* m, int64_t* dims, int32_t max_dims, int32_t* n);

/* The same contraction on HOST buffers (the operands' and the result's packed images in host memory):
 * one call copies in, contracts and copies out. GEMM-shaped contractions with dense rows pipeline
 * the lhs rows, the GEMM and the result rows across two copy streams and the compute stream; use
 * pinned host memory for the copies to overlap. Returns when the work is queued on the context's
 * stream (fopt_sync to wait); the result equals fopt_contraction's. Scale vectors stay device
 * pointers. */
fopt_status fopt_contraction_host(fopt_ctx* ctx, void* host_out, fopt_dtype out_dtype, const void* host_lhs,
                                  const void* host_rhs, fopt_dtype in_dtype, const fopt_mapping* lhs_map,
                                  const fopt_mapping* rhs_map, const fopt_mapping* pre_reduce,
                                  const fopt_mapping* out_map, const fopt_epilogue* epilogue);

/* ---- fused attention (furiosa-opt-examples/src/transformer/kernel/attention.rs:32-392) ----
 * softmax(Q K^T * scale + causal mask) V for bf16 Q [B, S, Hq, D], K/V [B, S, Hkv, D] (row-major,
 * GQA: query head h reads kv head h / (Hq/Hkv)), fp32 softmax with the reference's running max /
 * sum (sum + eps), O bf16 [B, S, Hq, D]. D = 128. */
fopt_status fopt_attention(fopt_ctx* ctx, void* o, const void* q, const void* k, const void* v, int32_t batch,
                           int32_t seq, int32_t hq, int32_t hkv, int32_t head_dim, float scale, int32_t causal,
                           float eps);

/* ---- collectives over the Chip axis (memory.rs:657-679, 1186-1233; context.rs:164-235) ---- */
/* NCCL unique id (128 bytes) for rank 0 to broadcast through the host plumbing. */
fopt_status fopt_comm_unique_id(void* id128);
fopt_status fopt_comm_init(fopt_ctx* ctx, int32_t nranks, int32_t rank, const void* id128);
fopt_status fopt_comm_destroy(fopt_ctx* ctx);
/* Sum over the Chip axis then broadcast (reduce::<m![Chip,E], m![E]> + transpose back), in place. */
fopt_status fopt_allreduce(fopt_ctx* ctx, void* buf, int64_t count, fopt_dtype dtype);
/* The same with the fold of an inter-slice reduce (Add, Max, Min, Mul; AddSat has no collective). */
fopt_status fopt_allreduce_op(fopt_ctx* ctx, void* buf, int64_t count, fopt_dtype dtype, fopt_reduce_op op);
/* dm_chip_shuffle / hbm_chip_shuffle: pattern[target] = source; this rank sends its slab to every
 * target whose source it is and receives the slab of pattern[rank]. */
fopt_status fopt_chip_shuffle(fopt_ctx* ctx, void* dst, const void* src, size_t bytes, const int32_t* pattern,
                              int32_t nranks);
/* The peer plan fopt_chip_shuffle runs for `rank` (host only, no communicator): the targets it sends
 * its slab to (sends[0 .. *n_sends), capacity nranks) and the rank it receives from. FOPT_ERR_INVALID
 * unless pattern is a permutation of 0 .. nranks - 1. */
fopt_status fopt_chip_shuffle_plan(const int32_t* pattern, int32_t nranks, int32_t rank, int32_t* sends,
                                   int32_t* n_sends, int32_t* recv_from);

#ifdef __cplusplus
}
#endif
#endif /* FOPT_B200_H */
