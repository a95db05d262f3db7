// Collectives over the Chip axis through NCCL (NVLink 5 / NVSwitch on a B200 node).
//
// The reference's multi-chip movers (furiosa-opt-std/src/tensor/memory.rs:657-679 hbm_chip_shuffle,
// 1186-1233 dm_cluster_shuffle / dm_chip_shuffle) permute whole chip slabs; the all-reduce config
// is `reduce` over the Chip axis followed by a broadcast. One process drives one GPU; NCCL is
// loaded with dlopen at communicator creation so the library itself loads on hosts without NCCL.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "ctx.hpp"

using namespace fopt;

namespace {

struct NcclApi {
  void* h = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* names[] = {getenv("FOPT_NCCL_LIB"), "libnccl.so.2", "libnccl.so"};
    for (const char* n : names) {
      if (!n) continue;
      api.h = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
      if (api.h) break;
    }
    if (!api.h) return;
#define LOAD(field, sym) api.field = (decltype(api.field))dlsym(api.h, sym)
    LOAD(GetUniqueId, "ncclGetUniqueId");
    LOAD(CommInitRank, "ncclCommInitRank");
    LOAD(CommDestroy, "ncclCommDestroy");
    LOAD(AllReduce, "ncclAllReduce");
    LOAD(Send, "ncclSend");
    LOAD(Recv, "ncclRecv");
    LOAD(GroupStart, "ncclGroupStart");
    LOAD(GroupEnd, "ncclGroupEnd");
    LOAD(GetErrorString, "ncclGetErrorString");
#undef LOAD
  });
  if (!api.h || !api.AllReduce) throw Fail{FOPT_ERR_NCCL, "NCCL library not found (set FOPT_NCCL_LIB)"};
  return api;
}

void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) {
    auto& a = nccl();
    throw Fail{FOPT_ERR_NCCL, std::string(what) + ": " + (a.GetErrorString ? a.GetErrorString(r) : "nccl error")};
  }
}

bool nccl_type(int dt, ncclDataType_t* t) {
  switch (dt) {
    case FOPT_BF16: *t = ncclBfloat16; return true;
    case FOPT_F32: *t = ncclFloat32; return true;
    case FOPT_I32: *t = ncclInt32; return true;
    case FOPT_I8: *t = ncclInt8; return true;
    default: return false;
  }
}

template <typename Fn>
fopt_status guard(fopt_ctx* ctx, Fn&& fn) {
  try {
    fn();
    return FOPT_OK;
  } catch (const Fail& f) {
    if (ctx) ctx->err = f.msg;
    return f.code;
  } catch (const std::exception& e) {
    if (ctx) ctx->err = e.what();
    return FOPT_ERR_INVALID;
  }
}

}  // namespace

extern "C" {

fopt_status fopt_comm_unique_id(void* id128) {
  try {
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
    ncclUniqueId id;
    nccl_check(nccl().GetUniqueId(&id), "ncclGetUniqueId");
    memcpy(id128, &id, sizeof(id));
    return FOPT_OK;
  } catch (...) {
    return FOPT_ERR_NCCL;
  }
}

fopt_status fopt_comm_init(fopt_ctx* ctx, int32_t nranks, int32_t rank, const void* id128) {
  return guard(ctx, [&] {
    if (nranks < 1 || rank < 0 || rank >= nranks) throw Fail{FOPT_ERR_INVALID, "fopt_comm_init: bad rank"};
    ncclUniqueId id;
    memcpy(&id, id128, sizeof(id));
    ncclComm_t c;
    cuda_check(cudaSetDevice(ctx->device), "cudaSetDevice");
    nccl_check(nccl().CommInitRank(&c, nranks, id, rank), "ncclCommInitRank");
    ctx->nccl_comm = c;
    ctx->nranks = nranks;
    ctx->rank = rank;
  });
}

fopt_status fopt_comm_destroy(fopt_ctx* ctx) {
  if (!ctx || !ctx->nccl_comm) return FOPT_OK;
  return guard(ctx, [&] {
    nccl_check(nccl().CommDestroy((ncclComm_t)ctx->nccl_comm), "ncclCommDestroy");
    ctx->nccl_comm = nullptr;
  });
}

fopt_status fopt_allreduce_op(fopt_ctx* ctx, void* buf, int64_t count, fopt_dtype dtype, fopt_reduce_op op) {
  return guard(ctx, [&] {
    if (!ctx->nccl_comm) throw Fail{FOPT_ERR_INVALID, "fopt_allreduce: no communicator (fopt_comm_init)"};
    ncclDataType_t t;
    if (!nccl_type(dtype, &t)) throw Fail{FOPT_ERR_UNSUPPORTED, "fopt_allreduce: dtype"};
    ncclRedOp_t r;
    switch (op) {
      case FOPT_RED_ADD: r = ncclSum; break;
      case FOPT_RED_MAX: r = ncclMax; break;
      case FOPT_RED_MIN: r = ncclMin; break;
      case FOPT_RED_MUL: r = ncclProd; break;
      default: throw Fail{FOPT_ERR_UNSUPPORTED, "fopt_allreduce: saturating add has no collective"};
    }
    nccl_check(nccl().AllReduce(buf, buf, (size_t)count, t, r, (ncclComm_t)ctx->nccl_comm, ctx->stream),
               "ncclAllReduce");
  });
}

fopt_status fopt_allreduce(fopt_ctx* ctx, void* buf, int64_t count, fopt_dtype dtype) {
  return fopt_allreduce_op(ctx, buf, count, dtype, FOPT_RED_ADD);
}

fopt_status fopt_chip_shuffle_plan(const int32_t* pattern, int32_t nranks, int32_t rank, int32_t* sends,
                                   int32_t* n_sends, int32_t* recv_from) {
  if (!pattern || !sends || !n_sends || !recv_from || nranks <= 0 || rank < 0 || rank >= nranks) return FOPT_ERR_INVALID;
  std::vector<int> seen(nranks, 0);
  for (int t = 0; t < nranks; ++t) {
    if (pattern[t] < 0 || pattern[t] >= nranks || seen[pattern[t]]++) return FOPT_ERR_INVALID;  // a permutation
  }
  int k = 0;
  for (int t = 0; t < nranks; ++t)
    if (pattern[t] == rank && t != rank) sends[k++] = t;
  *n_sends = k;
  *recv_from = pattern[rank];
  return FOPT_OK;
}

fopt_status fopt_chip_shuffle(fopt_ctx* ctx, void* dst, const void* src, size_t bytes, const int32_t* pattern,
                              int32_t nranks) {
  return guard(ctx, [&] {
    if (!ctx->nccl_comm || nranks != ctx->nranks) throw Fail{FOPT_ERR_INVALID, "fopt_chip_shuffle: communicator size"};
    std::vector<int32_t> sends(nranks);
    int32_t n_sends = 0, from = 0;
    if (fopt_chip_shuffle_plan(pattern, nranks, ctx->rank, sends.data(), &n_sends, &from) != FOPT_OK)
      throw Fail{FOPT_ERR_INVALID, "fopt_chip_shuffle: pattern must be a permutation of the ranks"};
    auto& a = nccl();
    nccl_check(a.GroupStart(), "ncclGroupStart");
    for (int i = 0; i < n_sends; ++i)
      nccl_check(a.Send(src, bytes, ncclInt8, sends[i], (ncclComm_t)ctx->nccl_comm, ctx->stream), "ncclSend");
    if (from != ctx->rank)
      nccl_check(a.Recv(dst, bytes, ncclInt8, from, (ncclComm_t)ctx->nccl_comm, ctx->stream), "ncclRecv");
    nccl_check(a.GroupEnd(), "ncclGroupEnd");
    if (from == ctx->rank && dst != src)
      cuda_check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, ctx->stream), "self copy");
  });
}

}  // extern "C"
