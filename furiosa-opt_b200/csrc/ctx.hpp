// The opaque context behind `fopt_ctx*`: one CUDA device, one stream, the last error, and the
// caches of walk plans derived from mapping pairs.
#pragma once

#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/fopt_b200.h"
#include "common.cuh"
#include "mapping.hpp"

struct fopt_mapping {
  fopt::Mapping m;
  std::string key;  // canonical text + axis sizes, for plan caching
};

namespace fopt {

// A relayout plan ready for launch: either a walk (fast) or an explicit offset table on device.
struct RelayoutPlan {
  bool has_walk = false;
  KWalk walk{};
  int64_t positions = 0;
  int64_t* table = nullptr;  // device, one src offset per dst position (-1 dead)
  std::string desc;
};

std::vector<int64_t> host_deltas(const KWalk& rw);

struct FoldKPlan {
  KWalk out{}, residue{};
  int64_t out_positions = 0, residue_positions = 0, residue_live = 0;
  // the live residue deltas of 1 or 2 memories, uploaded once (freed with the context)
  mutable int64_t* dev_deltas[2] = {nullptr, nullptr};
  mutable int64_t dev_count[2] = {0, 0};
  mutable std::mutex dev_mu;
  // the live residue deltas of memory 0 in host memory, built once on first request
  mutable std::vector<int64_t> host_delta;
  mutable bool host_delta_ready = false;
  const std::vector<int64_t>& host_residue_deltas() const {
    std::lock_guard<std::mutex> g(dev_mu);
    if (!host_delta_ready) {
      host_delta = host_deltas(residue);
      host_delta_ready = true;
    }
    return host_delta;
  }
  FoldKPlan() = default;
  FoldKPlan(const FoldKPlan& o)
      : out(o.out), residue(o.residue), out_positions(o.out_positions), residue_positions(o.residue_positions),
        residue_live(o.residue_live) {}
  ~FoldKPlan() {
    for (auto* d : dev_deltas)
      if (d) cudaFree(d);
  }
};

}  // namespace fopt

struct fopt_graph;

struct fopt_ctx {
  int device = 0;
  fopt_graph* capture = nullptr;        // the step being captured into a CUDA graph, if any
  std::vector<void*> deferred_free;     // frees of pre-capture memory requested during a capture
  std::map<void*, fopt_graph*> graph_mem;  // allocations that belong to a captured graph
  int graphs_alive = 0;                 // captured graphs not yet destroyed
  std::vector<void*> retired;           // outgrown context buffers a live graph may still use
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  int exact_fold = 0;
  int64_t launches = 0;
  std::string err;
  std::mutex mu;
  std::map<std::tuple<std::string, std::string, int>, std::shared_ptr<fopt::RelayoutPlan>> relayouts;
  std::map<std::string, std::shared_ptr<fopt::FoldKPlan>> folds;
  void* nccl_comm = nullptr;
  int nranks = 1, rank = 0;
  int32_t* dev_err = nullptr;  // device error word: bounded waits that expire write a code here
  void* scratch = nullptr;  // grow-only device scratch for kernels that need it
  size_t scratch_bytes = 0;
  void* gemm_ws = nullptr;  // split-K partial accumulators of the paired GEMM's last wave
  size_t gemm_ws_bytes = 0;
  uint32_t* gemm_cnt = nullptr;  // arrival counters of the split tiles (zero between launches)
  size_t gemm_cnt_n = 0;
  bool gemm_cnt_dirty = false;
  cudaStream_t copy_in = nullptr, copy_out = nullptr;  // host <-> device pipelines of the host-buffer calls
  void* pinned[2] = {nullptr, nullptr};  // host staging for file -> device streaming
  cudaEvent_t pinned_ev[2] = {nullptr, nullptr};
};

namespace fopt {

// Status helpers: every C entry point catches everything and returns a status.
struct Fail {
  fopt_status code;
  std::string msg;
};

// The last error of calls made without a context (mapping parsing, file headers).
extern thread_local std::string g_noctx_err;

inline void require(bool ok, const std::string& msg) {
  if (!ok) throw Fail{FOPT_ERR_INVALID, msg};
}

// Runs fn, turning any exception into a status (the message goes to the context's last error).
template <typename Fn>
fopt_status guarded(fopt_ctx* ctx, Fn&& fn) {
  try {
    fn();
    return FOPT_OK;
  } catch (const Fail& f) {
    if (ctx) ctx->err = f.msg;
    return f.code;
  } catch (const MappingError& e) {
    if (ctx) ctx->err = e.what();
    return FOPT_ERR_INVALID;
  } catch (const std::exception& e) {
    if (ctx) ctx->err = e.what();
    return FOPT_ERR_INVALID;
  }
}

inline void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Fail{FOPT_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e)};
}

// After a launch: count it and surface launch-configuration errors immediately.
inline void launched(fopt_ctx* ctx, const char* what) {
  ctx->launches++;
  cuda_check(cudaGetLastError(), what);
}

void* scratch(fopt_ctx* ctx, size_t bytes);

KWalk to_kwalk(const Walk& w);
bool to_kwalk32(const KWalk& w, KWalk32& out);

// Kernel launchers (defined in the .cu files).
void launch_relayout(fopt_ctx* ctx, const RelayoutPlan& p, void* dst, const void* src, int dtype, int64_t src_base,
                     int64_t dst_base, int64_t src_elems, int64_t dst_elems);
void launch_transmute(fopt_ctx* ctx, const RankWalk& src, const RankWalk& dst, void* out, const void* in, int dtype);
bool launch_elementwise_jit_ex(fopt_ctx* ctx, const fopt_program* prog, int n_in, const void* const* in,
                               const fopt_dtype* in_dt, const int64_t* bcast, void* out, fopt_dtype out_dt, int64_t n);
void release_ctx_buffer(fopt_ctx* ctx, void* p);
bool launch_row_jit(fopt_ctx* ctx, const fopt_row_plan& plan);
bool launch_reduce_map_jit(fopt_ctx* ctx, const fopt_program* prog, int n_in, const void* const* in,
                           const fopt_dtype* in_dt, const int64_t* bcast, int fold, uint32_t ident, void* out,
                           int64_t rows, int64_t W);
bool launch_elementwise_jit(fopt_ctx* ctx, const fopt_program* prog, int n_in, const void* const* in,
                            const fopt_dtype* in_dt, void* out, fopt_dtype out_dt, int64_t n);
void launch_elementwise(fopt_ctx* ctx, const fopt_program* prog, int n_in, const void* const* in, const fopt_dtype* in_dt,
                        void* out, fopt_dtype out_dt, int64_t n);
void launch_reduce(fopt_ctx* ctx, const FoldKPlan& p, void* out, const void* src, int dtype, int op, uint32_t ident,
                   int64_t src_elems);
// The cached reduce plan for a (src, dst) mapping pair (host memory only; nothing is uploaded).
std::shared_ptr<FoldKPlan> reduce_plan(fopt_ctx* ctx, const fopt_mapping* src_map, const fopt_mapping* dst_map,
                                       int allow_broadcast);
void launch_reduce_cells(fopt_ctx* ctx, const FoldKPlan& p, void* out, const void* src, int dtype, int op,
                         uint32_t ident, int64_t src_elems, const int64_t* d_delta, int64_t nd);
void launch_contraction_generic(fopt_ctx* ctx, const FoldKPlan& p, void* out, int out_dt, const void* lhs,
                                const void* rhs, int in_dt, int64_t lhs_elems, int64_t rhs_elems,
                                const fopt_epilogue* ep, const int64_t* scale_stride_out, const float* scale);
// GEMM fast path: D[M,N] = A[M,K] . B[N,K]^T, both operands K-major. Returns false if the shape
// does not fit the tensor-core kernel.
bool launch_gemm_tc(fopt_ctx* ctx, void* out, int out_dt, const void* a, const void* b, int in_dt, int64_t M,
                    int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldd, const fopt_epilogue* ep,
                    const float* scale, int scale_along_n);
bool launch_attention_tc(fopt_ctx* ctx, void* o, const void* q, const void* k, const void* v, int B, int S, int Hq,
                         int Hkv, int D, float scale, int causal, float eps);
void launch_attention(fopt_ctx* ctx, void* o, const void* q, const void* k, const void* v, int B, int S, int Hq,
                      int Hkv, int D, float scale, int causal, float eps);
void launch_gather_rows(fopt_ctx* ctx, void* dst, const void* table, const int32_t* idx, int64_t n_idx,
                        int64_t row_bytes, int64_t stride_div, int64_t table_rows, int64_t table_row_stride_bytes,
                        int64_t dst_row_stride_bytes);

}  // namespace fopt
