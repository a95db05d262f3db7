// fopt_reduce_noalloc: the reduce entry point for callers that must not allocate device memory.
//
// fopt_reduce keeps its per-cell residue delta table in a context scratch buffer that grows with
// cudaMalloc (and frees the old one with cudaFree, which synchronises the device). Some callers cannot
// allow either:
//   * a host runtime that has handed the whole device memory budget to its own allocator up front,
//     so any allocation made behind its back can fail or break its accounting;
//   * a latency-critical loop where the implicit device synchronisation of cudaFree, or a
//     cudaMalloc that has to wait for the driver, is not acceptable.
// This variant never allocates: its delta table lives in the fixed-size device array below, and
// everything else it needs (plans, host vectors) is host memory.
//
// Contract:
//   * the delta table holds at most kNoAllocMaxDeltas (32768) entries, 256 KiB of int64, which every
//     GPU that loads this library reserves until the process exits; a reduce whose live residue is
//     larger is rejected with FOPT_ERR_INVALID and a message;
//   * the first call on each device looks up the array's device address (cudaGetSymbolAddress with
//     that device current); make that first call before any stream capture;
//   * all calls share the one array, and each call overwrites the part it uses: two calls whose
//     kernels can overlap on the GPU (different streams, no ordering between them) race on it;
//   * the fold always runs per output cell in the reference's wire order. i32 results match
//     fopt_reduce in either mode, f32 / bf16 Add and Mul match it with exact fold on; for f32 Max / Min
//     fopt_reduce may fold a long unit-stride row in another order, so the two can differ in the sign
//     of a zero or in which NaN comes back;
//   * it cannot be called while a capture is open: the delta upload reads a host vector that a
//     captured copy would keep pointing at after the call returns.
#include <mutex>

#include "ctx.hpp"

namespace fopt {
namespace {

constexpr int64_t kNoAllocMaxDeltas = 32768;
constexpr int kMaxDevices = 64;

// File-scope device scratch. In host code `g_noalloc_deltas` names a host-side stand-in, not a
// device address: only the pointer obtained from cudaGetSymbolAddress may be given to a kernel.
static __device__ __align__(256) int64_t g_noalloc_deltas[kNoAllocMaxDeltas];

std::mutex g_mu;
int64_t* g_dev_ptr[kMaxDevices] = {};

// Device address of g_noalloc_deltas on ctx's device, looked up once per device.
int64_t* delta_array(fopt_ctx* ctx) {
  if (ctx->device < 0 || ctx->device >= kMaxDevices) throw Fail{FOPT_ERR_INVALID, "reduce_noalloc: device index"};
  std::lock_guard<std::mutex> g(g_mu);
  if (!g_dev_ptr[ctx->device]) {
    int prev = -1;
    cuda_check(cudaGetDevice(&prev), "reduce_noalloc: cudaGetDevice");
    if (prev != ctx->device) cuda_check(cudaSetDevice(ctx->device), "reduce_noalloc: cudaSetDevice");
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_deltas);
    if (prev != ctx->device) cudaSetDevice(prev);
    cuda_check(e, "reduce_noalloc: cudaGetSymbolAddress");
    g_dev_ptr[ctx->device] = (int64_t*)p;
  }
  return g_dev_ptr[ctx->device];
}

}  // namespace
}  // namespace fopt

using namespace fopt;

extern "C" fopt_status fopt_reduce_noalloc(fopt_ctx* ctx, void* out, const void* src, fopt_dtype dtype,
                                           fopt_reduce_op op, uint32_t identity_bits, const fopt_mapping* src_map,
                                           const fopt_mapping* dst_map, int allow_broadcast) {
  if (!ctx) return FOPT_ERR_INVALID;
  return guarded(ctx, [&] {
    require(out && src && src_map && dst_map, "fopt_reduce_noalloc: null argument");
    require(dtype == FOPT_I32 || dtype == FOPT_F32 || dtype == FOPT_BF16,
            "fopt_reduce_noalloc: dtype must be i32, f32 or bf16");
    // The delta upload below reads a host vector; a captured copy node would keep pointing at it.
    require(!ctx->capture, "fopt_reduce_noalloc: cannot be called while a capture is open (call fopt_reduce)");
    auto kp = reduce_plan(ctx, src_map, dst_map, allow_broadcast);  // host-side plan, cached per context
    if (kp->residue_live > kNoAllocMaxDeltas)
      throw Fail{FOPT_ERR_INVALID, "fopt_reduce_noalloc: the reduce folds " + std::to_string(kp->residue_live) +
                                       " cells per output, above the fixed maximum of " +
                                       std::to_string(kNoAllocMaxDeltas) + "; use fopt_reduce"};
    const std::vector<int64_t>& d = kp->host_residue_deltas();
    int64_t* dev = delta_array(ctx);
    if (!d.empty())
      cuda_check(cudaMemcpyAsync(dev, d.data(), sizeof(int64_t) * d.size(), cudaMemcpyHostToDevice, ctx->stream),
                 "reduce_noalloc: delta upload");
    launch_reduce_cells(ctx, *kp, out, src, dtype, op, identity_bits, src_map->m.size(), dev, (int64_t)d.size());
  });
}
