// The extern "C" entry points of libfopt_b200.so (declared in include/fopt_b200.h).
//
// Each entry point validates its arguments, derives (and caches) the walk plan for its mappings on
// the host -- the work the reference does with `sequence()` / `carve()` before its rayon loop -- and
// launches the CUDA kernels on the context's stream. Errors never cross the boundary as exceptions:
// they become an fopt_status and a message in fopt_last_error().
#include <algorithm>
#include <cstring>
#include <sstream>

#include <unordered_set>

#include "ctx.hpp"

using namespace fopt;

namespace fopt {

// Frees an outgrown context buffer, or keeps it until the context goes away while a captured graph
// (which may have recorded its address) exists.
void release_ctx_buffer(fopt_ctx* ctx, void* p) {
  if (!p) return;
  if (ctx->graphs_alive > 0 || ctx->capture)
    ctx->retired.push_back(p);
  else
    cuda_check(cudaFree(p), "buffer free");
}

void* scratch(fopt_ctx* ctx, size_t bytes) {
  if (bytes > ctx->scratch_bytes) {
    release_ctx_buffer(ctx, ctx->scratch);
    size_t want = std::max(bytes, ctx->scratch_bytes * 2);
    cuda_check(cudaMalloc(&ctx->scratch, want), "scratch alloc");
    ctx->scratch_bytes = want;
  }
  return ctx->scratch;
}

}  // namespace fopt

thread_local std::string fopt::g_noctx_err;

namespace {

// Mappings parsed by separate fopt_mapping_parse calls carry separate axis tables; re-parse them
// against one merged table so axis identities agree (axes match by name, as Ident does).
std::vector<Mapping> unify(std::initializer_list<const Mapping*> ms) {
  auto table = std::make_shared<AxisTable>();
  for (auto* m : ms)
    for (size_t i = 0; i < m->axes->names.size(); ++i) table->intern(m->axes->names[i], m->axes->sizes[i]);
  std::vector<Mapping> out;
  for (auto* m : ms) out.push_back(parse_mapping(m->to_string(), table));
  return out;
}

std::shared_ptr<RelayoutPlan> relayout_plan(fopt_ctx* ctx, const fopt_mapping* src, const fopt_mapping* dst,
                                            bool allow_broadcast) {
  auto key = std::make_tuple(src->key, dst->key, (int)allow_broadcast);
  {
    std::lock_guard<std::mutex> g(ctx->mu);
    auto it = ctx->relayouts.find(key);
    if (it != ctx->relayouts.end()) return it->second;
  }
  auto p = std::make_shared<RelayoutPlan>();
  Walk w;
  p->positions = dst->m.size();
  auto u = unify({&src->m, &dst->m});
  if (plan_relayout(u[0], u[1], allow_broadcast, w)) {
    p->has_walk = true;
    p->walk = to_kwalk(w);
    p->desc = w.to_string();
  } else {
    auto t = relayout_table(u[0], u[1], allow_broadcast);
    cuda_check(cudaMalloc(&p->table, sizeof(int64_t) * std::max<size_t>(t.size(), 1)), "plan table alloc");
    cuda_check(cudaMemcpy(p->table, t.data(), sizeof(int64_t) * t.size(), cudaMemcpyHostToDevice), "plan table");
    p->desc = "table[" + std::to_string(t.size()) + "]";
  }
  std::lock_guard<std::mutex> g(ctx->mu);
  ctx->relayouts[key] = p;
  return p;
}

FoldKPlan to_kfold(const FoldPlan& fp) {
  FoldKPlan k;
  if ((int)fp.out.wheels.size() > kKWheels || (int)fp.residue.wheels.size() > kKWheels)
    throw Fail{FOPT_ERR_UNSUPPORTED, "fold plan has too many wheels"};
  k.out = to_kwalk(fp.out);
  k.residue = to_kwalk(fp.residue);
  k.out_positions = fp.out.positions();
  k.residue_positions = fp.residue.positions();
  k.residue_live = fp.residue.live_positions();
  return k;
}

std::vector<std::pair<std::string, int64_t>> parse_offset(const std::string& s) {
  std::vector<std::pair<std::string, int64_t>> out;
  std::stringstream ss(s);
  std::string item;
  while (std::getline(ss, item, ',')) {
    auto c = item.find_first_of(":=");
    if (c == std::string::npos) continue;
    std::string n = item.substr(0, c), v = item.substr(c + 1);
    n.erase(std::remove_if(n.begin(), n.end(), ::isspace), n.end());
    out.push_back({n, std::stoll(v)});
  }
  return out;
}

}  // namespace

struct fopt_graph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  std::unordered_set<void*> owned;  // allocations of the capture that it did not free
  bool launched = false;
  int64_t kernels = 0;              // kernels the captured step launches (counted per replay)
  int64_t launches_before = 0;
};

extern "C" {

fopt_status fopt_init(int device, fopt_ctx** out) {
  if (!out) return FOPT_ERR_INVALID;
  auto* ctx = new fopt_ctx();
  fopt_status st = guarded(ctx, [&] {
    cuda_check(cudaSetDevice(device), "cudaSetDevice");
    ctx->device = device;
    cuda_check(cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking), "stream create");
    ctx->stream = ctx->own_stream;
    cuda_check(cudaMalloc(&ctx->dev_err, sizeof(int32_t)), "error word");
    cudaMemPool_t pool;
    cuda_check(cudaDeviceGetDefaultMemPool(&pool, device), "default mem pool");
    uint64_t keep = UINT64_MAX;
    cuda_check(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep), "mem pool threshold");
    cuda_check(cudaMemset(ctx->dev_err, 0, sizeof(int32_t)), "error word");
  });
  if (st != FOPT_OK) {
    g_noctx_err = ctx->err;
    delete ctx;
    *out = nullptr;
    return st;
  }
  *out = ctx;
  return FOPT_OK;
}

fopt_status fopt_destroy(fopt_ctx* ctx) {
  if (!ctx) return FOPT_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  for (auto& kv : ctx->relayouts)
    if (kv.second->table) cudaFree(kv.second->table);
  if (ctx->scratch) cudaFree(ctx->scratch);
  if (ctx->gemm_ws) cudaFree(ctx->gemm_ws);
  if (ctx->gemm_cnt) cudaFree(ctx->gemm_cnt);
  for (void* p : ctx->retired) cudaFree(p);
  if (ctx->copy_in) cudaStreamDestroy(ctx->copy_in);
  if (ctx->copy_out) cudaStreamDestroy(ctx->copy_out);
  for (int k = 0; k < 2; ++k) {
    if (ctx->pinned[k]) cudaFreeHost(ctx->pinned[k]);
    if (ctx->pinned_ev[k]) cudaEventDestroy(ctx->pinned_ev[k]);
  }
  if (ctx->dev_err) cudaFree(ctx->dev_err);
  extern fopt_status fopt_comm_destroy(fopt_ctx*);
  fopt_comm_destroy(ctx);
  if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  delete ctx;
  return FOPT_OK;
}

const char* fopt_last_error(const fopt_ctx* ctx) { return ctx ? ctx->err.c_str() : g_noctx_err.c_str(); }

// After a stream sync: surface (and clear) a device-side bounded-wait expiry.
static void check_device_error(fopt_ctx* ctx) {
  int32_t code = 0;
  cuda_check(cudaMemcpy(&code, ctx->dev_err, sizeof(code), cudaMemcpyDeviceToHost), "error word read");
  if (code) {
    cuda_check(cudaMemset(ctx->dev_err, 0, sizeof(code)), "error word clear");
    ctx->gemm_cnt_dirty = true;
    throw Fail{FOPT_ERR_TIMEOUT, "a kernel's bounded wait expired (code " + std::to_string(code) + ")"};
  }
}

fopt_status fopt_sync(fopt_ctx* ctx) {
  return guarded(ctx, [&] {
    cuda_check(cudaStreamSynchronize(ctx->stream), "sync");
    check_device_error(ctx);
  });
}

fopt_status fopt_set_stream(fopt_ctx* ctx, void* stream) {
  if (!ctx) return FOPT_ERR_INVALID;
  ctx->stream = stream ? (cudaStream_t)stream : ctx->own_stream;
  return FOPT_OK;
}

void* fopt_get_stream(fopt_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

fopt_status fopt_set_exact_fold(fopt_ctx* ctx, int exact) {
  if (!ctx) return FOPT_ERR_INVALID;
  ctx->exact_fold = exact;
  return FOPT_OK;
}

int64_t fopt_launch_count(const fopt_ctx* ctx) { return ctx ? ctx->launches : 0; }

// Storages come from the device's stream-ordered memory pool: allocation and release are ordered on
// the context's stream and never synchronise the device (a plain cudaFree would), and freed blocks
// stay cached in the pool for the next allocation (the release threshold is raised at fopt_init).
fopt_status fopt_alloc(fopt_ctx* ctx, size_t bytes, void** dptr) {
  return guarded(ctx, [&] {
    require(dptr != nullptr, "fopt_alloc: null out pointer");
    cuda_check(cudaMallocAsync(dptr, std::max<size_t>(bytes, 1), ctx->stream), "cudaMallocAsync");
    if (ctx->capture) ctx->capture->owned.insert(*dptr);
    cuda_check(cudaMemsetAsync(*dptr, 0, std::max<size_t>(bytes, 1), ctx->stream), "zero fill");
  });
}

fopt_status fopt_alloc_uninit(fopt_ctx* ctx, size_t bytes, void** dptr) {
  return guarded(ctx, [&] {
    require(dptr != nullptr, "fopt_alloc_uninit: null out pointer");
    cuda_check(cudaMallocAsync(dptr, std::max<size_t>(bytes, 1), ctx->stream), "cudaMallocAsync");
    if (ctx->capture) ctx->capture->owned.insert(*dptr);
  });
}

// Frees device memory outside a capture. A captured graph's allocation is no longer the graph's
// to release afterwards; one from a graph never launched was never mapped and needs no free.
static void release_now(fopt_ctx* ctx, void* dptr) {
  auto it = ctx->graph_mem.find(dptr);
  if (it != ctx->graph_mem.end()) {
    fopt_graph* g = it->second;
    ctx->graph_mem.erase(it);
    g->owned.erase(dptr);
    if (!g->launched) return;
  }
  cuda_check(cudaFreeAsync(dptr, ctx->stream), "cudaFreeAsync");
}

fopt_status fopt_free(fopt_ctx* ctx, void* dptr) {
  if (!ctx) return FOPT_ERR_INVALID;
  return guarded(ctx, [&] {
    if (!dptr) return;
    if (ctx->capture) {
      if (ctx->capture->owned.erase(dptr))
        cuda_check(cudaFreeAsync(dptr, ctx->stream), "cudaFreeAsync");  // a free node of the graph
      else
        ctx->deferred_free.push_back(dptr);  // memory from before the capture: released after it
      return;
    }
    release_now(ctx, dptr);
  });
}

// ---- CUDA graphs of whole steps ----
// A step (for example a decoder block's forward) issued between fopt_capture_begin and
// fopt_capture_end is recorded from the context's stream into a CUDA graph instead of run; each
// fopt_graph_launch then replays every kernel, copy and stream-ordered allocation of the step in
// one call, without the host work that issued them. Allocations made during the capture become the
// graph's own: those freed during it are released inside the graph, the others (the step's
// outputs) keep their addresses across launches and are released when the graph is launched again
// or destroyed.
fopt_status fopt_capture_begin(fopt_ctx* ctx) {
  return guarded(ctx, [&] {
    require(!ctx->capture, "fopt_capture_begin: a capture is already open");
    require(ctx->stream != nullptr, "fopt_capture_begin: the legacy default stream cannot be captured");
    auto* g = new fopt_graph;
    cudaError_t e = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeRelaxed);
    if (e != cudaSuccess) {
      delete g;
      cuda_check(e, "cudaStreamBeginCapture");
    }
    g->launches_before = ctx->launches;
    ctx->capture = g;
  });
}

fopt_status fopt_capture_end(fopt_ctx* ctx, fopt_graph** out) {
  return guarded(ctx, [&] {
    require(ctx->capture && out, "fopt_capture_end: no capture is open");
    fopt_graph* g = ctx->capture;
    ctx->capture = nullptr;
    *out = nullptr;
    g->kernels = ctx->launches - g->launches_before;  // recorded, not run
    ctx->launches = g->launches_before;
    cudaError_t e = cudaStreamEndCapture(ctx->stream, &g->graph);
    if (e == cudaSuccess)
      e = cudaGraphInstantiateWithFlags(&g->exec, g->graph, cudaGraphInstantiateFlagAutoFreeOnLaunch);
    for (void* p : ctx->deferred_free) {
      try {
        release_now(ctx, p);
      } catch (const Fail&) {
      }
    }
    ctx->deferred_free.clear();
    if (e != cudaSuccess) {
      if (g->graph) cudaGraphDestroy(g->graph);
      delete g;
      cuda_check(e, "graph capture");
    }
    for (void* p : g->owned) ctx->graph_mem[p] = g;
    ctx->graphs_alive++;
    *out = g;
  });
}

fopt_status fopt_graph_launch(fopt_ctx* ctx, fopt_graph* g) {
  return guarded(ctx, [&] {
    require(g && g->exec, "fopt_graph_launch: no graph");
    require(!ctx->capture, "fopt_graph_launch: a capture is open");
    cuda_check(cudaGraphLaunch(g->exec, ctx->stream), "cudaGraphLaunch");
    g->launched = true;
    ctx->launches += g->kernels;
  });
}

fopt_status fopt_graph_destroy(fopt_ctx* ctx, fopt_graph* g) {
  if (!g) return FOPT_OK;
  return guarded(ctx, [&] {
    cuda_check(cudaStreamSynchronize(ctx->stream), "sync");
    for (void* p : g->owned) {
      ctx->graph_mem.erase(p);
      if (g->launched) cudaFreeAsync(p, ctx->stream);  // the last launch's allocations still live
    }
    cudaGetLastError();  // a release the runtime had already done reports here, not at the next launch
    cuda_check(cudaStreamSynchronize(ctx->stream), "sync");
    if (g->exec) cudaGraphExecDestroy(g->exec);
    if (g->graph) cudaGraphDestroy(g->graph);
    delete g;
    if (--ctx->graphs_alive == 0) {
      for (void* p : ctx->retired) cudaFree(p);
      ctx->retired.clear();
    }
  });
}

fopt_status fopt_h2d(fopt_ctx* ctx, void* dst, const void* host, size_t bytes) {
  return guarded(ctx, [&] { cuda_check(cudaMemcpyAsync(dst, host, bytes, cudaMemcpyHostToDevice, ctx->stream), "h2d"); });
}

fopt_status fopt_d2h(fopt_ctx* ctx, void* host, const void* src, size_t bytes) {
  return guarded(ctx, [&] {
    cuda_check(cudaMemcpyAsync(host, src, bytes, cudaMemcpyDeviceToHost, ctx->stream), "d2h");
    cuda_check(cudaStreamSynchronize(ctx->stream), "d2h sync");
    check_device_error(ctx);
  });
}

fopt_status fopt_d2d(fopt_ctx* ctx, void* dst, const void* src, size_t bytes) {
  return guarded(ctx, [&] { cuda_check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, ctx->stream), "d2d"); });
}

fopt_status fopt_memset(fopt_ctx* ctx, void* dst, int value, size_t bytes) {
  return guarded(ctx, [&] { cuda_check(cudaMemsetAsync(dst, value, bytes, ctx->stream), "memset"); });
}

// ---- mappings ----
fopt_status fopt_mapping_parse(const char* axes, const char* expr, fopt_mapping** out) {
  try {
    if (!out || !expr) throw MappingError("fopt_mapping_parse: null argument");
    auto table = parse_axes(axes ? axes : "");
    auto m = parse_mapping(expr, table);
    auto* h = new fopt_mapping{m, ""};
    std::ostringstream k;
    k << m.to_string() << "|";
    for (size_t i = 0; i < table->names.size(); ++i) k << table->names[i] << "=" << table->sizes[i] << ",";
    h->key = k.str();
    *out = h;
    return FOPT_OK;
  } catch (const std::exception& e) {
    g_noctx_err = e.what();
    if (out) *out = nullptr;
    return FOPT_ERR_INVALID;
  }
}

fopt_status fopt_mapping_free(fopt_mapping* m) {
  delete m;
  return FOPT_OK;
}

int64_t fopt_mapping_size(const fopt_mapping* m) { return m ? m->m.size() : -1; }

int32_t fopt_mapping_eval(const fopt_mapping* m, int64_t pos, int64_t* coords, int32_t ncoords) {
  if (!m) return -1;
  std::vector<int64_t> c;
  int r = m->m.eval(pos, c);
  for (int i = 0; i < ncoords && i < (int)c.size(); ++i) coords[i] = c[i];
  return r;
}

fopt_status fopt_window_base(const fopt_mapping* base, const char* offset, int64_t* out) {
  try {
    auto kv = parse_offset(offset ? offset : "");
    std::vector<std::string> names;
    std::vector<int64_t> vals;
    for (auto& p : kv) {
      names.push_back(p.first);
      vals.push_back(p.second);
    }
    *out = window_base(base->m, names, vals);
    return FOPT_OK;
  } catch (const std::exception& e) {
    g_noctx_err = e.what();
    return FOPT_ERR_INVALID;
  }
}

fopt_status fopt_describe_relayout(const fopt_mapping* src, const fopt_mapping* dst, int allow_broadcast, char* buf,
                                   size_t len) {
  try {
    Walk w;
    auto u = unify({&src->m, &dst->m});
    std::string s = plan_relayout(u[0], u[1], allow_broadcast != 0, w) ? w.to_string() : std::string("table");
    if (buf && len) {
      strncpy(buf, s.c_str(), len - 1);
      buf[len - 1] = 0;
    }
    return FOPT_OK;
  } catch (const std::exception& e) {
    g_noctx_err = e.what();
    return FOPT_ERR_INVALID;
  }
}

// ---- layout moves ----
fopt_status fopt_transpose(fopt_ctx* ctx, void* dst, const void* src, fopt_dtype dtype, const fopt_mapping* src_map,
                           const fopt_mapping* dst_map, int64_t src_base, int64_t dst_base, int allow_broadcast) {
  return guarded(ctx, [&] {
    require(src_map && dst_map && dst && src, "fopt_transpose: null argument");
    auto p = relayout_plan(ctx, src_map, dst_map, allow_broadcast != 0);
    // The storages are sized by their base mappings; windows only shift the bases. We do not know
    // the allocations' lengths here, so bound reads / writes by the stream itself.
    int64_t src_elems = src_base + src_map->m.size();
    int64_t dst_elems = dst_base + dst_map->m.size();
    launch_relayout(ctx, *p, dst, src, dtype, src_base, dst_base, src_elems, dst_elems);
  });
}

fopt_status fopt_transmute(fopt_ctx* ctx, void* dst, const void* src, fopt_dtype dtype, const fopt_mapping* src_map,
                           const fopt_mapping* dst_map) {
  return guarded(ctx, [&] {
    require(src_map && dst_map && dst && src, "fopt_transmute: null argument");
    std::vector<Factor> fs, fd;
    if (src_map->m.flatten(fs) && dst_map->m.flatten(fd) && fs.size() <= (size_t)kKWheels &&
        fd.size() <= (size_t)kKWheels) {
      RankWalk s = rank_walk(src_map->m), d = rank_walk(dst_map->m);
      int64_t sl = 1, dl = 1;
      for (auto v : s.live) sl *= v;
      for (auto v : d.live) dl *= v;
      require(dl <= sl, "transmute: dst_map has more live elements than src_map");
      launch_transmute(ctx, s, d, dst, src, dtype);
      return;
    }
    // Not affine-factorisable: pair the k-th live src position with the k-th live dst position by
    // brute-force evaluation once, then move the elements on the GPU.
    std::vector<int64_t> live_src, c;
    for (int64_t p = 0; p < src_map->m.size(); ++p)
      if (src_map->m.eval(p, c) == 0) live_src.push_back(p);
    RelayoutPlan plan;
    plan.positions = dst_map->m.size();
    std::vector<int64_t> t(plan.positions, -1);
    size_t k = 0;
    for (int64_t q = 0; q < plan.positions; ++q)
      if (dst_map->m.eval(q, c) == 0) {
        require(k < live_src.size(), "transmute: dst_map has more live elements than src_map");
        t[q] = live_src[k++];
      }
    require(!ctx->capture, "transmute: a non-affine transmute uploads a table per call and cannot be captured");
    int64_t* dt = (int64_t*)scratch(ctx, sizeof(int64_t) * std::max<size_t>(t.size(), 1));
    cuda_check(cudaMemcpyAsync(dt, t.data(), sizeof(int64_t) * t.size(), cudaMemcpyHostToDevice, ctx->stream),
               "transmute table");
    cuda_check(cudaMemsetAsync(dst, 0, (size_t)(plan.positions * dtype_bits(dtype) + 7) / 8, ctx->stream),
               "transmute zero");
    plan.table = dt;
    launch_relayout(ctx, plan, dst, src, dtype, 0, 0, src_map->m.size(), plan.positions);
  });
}

// ---- elementwise ----
fopt_status fopt_elementwise(fopt_ctx* ctx, const fopt_program* prog, int32_t n_in, const void* const* inputs,
                             const fopt_dtype* in_dtypes, void* out, fopt_dtype out_dtype, int64_t n) {
  return guarded(ctx, [&] {
    require(prog && out && n_in >= 0 && n_in <= 3, "fopt_elementwise: bad arguments");
    require(prog->n_insn >= 0 && prog->n_insn <= 32, "fopt_elementwise: program too long");
    for (int i = 0; i < n_in; ++i) require(inputs[i] != nullptr, "fopt_elementwise: null input");
    launch_elementwise(ctx, prog, n_in, inputs, in_dtypes, out, out_dtype, n);
  });
}

fopt_status fopt_elementwise_bcast(fopt_ctx* ctx, const fopt_program* prog, int32_t n_in, const void* const* inputs,
                                   const fopt_dtype* in_dtypes, const int64_t* bcast, void* out, fopt_dtype out_dtype,
                                   int64_t n) {
  fopt_status st = FOPT_OK;
  bool ran = false;
  st = guarded(ctx, [&] {
    require(prog && out && bcast && n_in >= 0 && n_in <= 3, "fopt_elementwise_bcast: bad arguments");
    require(prog->n_insn >= 0 && prog->n_insn <= 32, "fopt_elementwise_bcast: program too long");
    for (int i = 0; i < n_in; ++i) require(inputs[i] != nullptr, "fopt_elementwise_bcast: null input");
    ran = launch_elementwise_jit_ex(ctx, prog, n_in, inputs, in_dtypes, bcast, out, out_dtype, n);
  });
  if (st == FOPT_OK && !ran) {
    ctx->err = "fopt_elementwise_bcast: no generated kernel for these operands";
    return FOPT_ERR_UNSUPPORTED;
  }
  return st;
}

fopt_status fopt_broadcast_kind(const fopt_mapping* src, const fopt_mapping* dst, int32_t* kind, int64_t* inner) {
  try {
    require(src && dst && kind && inner, "fopt_broadcast_kind: null argument");
    *kind = 0;
    *inner = 0;
    Walk w;
    auto u = unify({&src->m, &dst->m});
    if (!plan_relayout(u[0], u[1], true, w) || w.wheels.size() != 2) return FOPT_OK;
    const Wheel &a = w.wheels[0], &b = w.wheels[1];
    if (a.live != a.extent || b.live != b.extent) return FOPT_OK;
    if (a.stride[0] == 0 && b.stride[0] == 1 && src->m.size() == b.extent) {
      *kind = 1;  // dst[i] = src[i / inner]
      *inner = a.extent;
    } else if (a.stride[0] == 1 && b.stride[0] == 0 && src->m.size() == a.extent) {
      *kind = 2;  // dst[i] = src[i % inner]
      *inner = a.extent;
    }
    return FOPT_OK;
  } catch (const Fail& f) {
    g_noctx_err = f.msg;
    return f.code;
  } catch (const std::exception& e) {
    g_noctx_err = e.what();
    return FOPT_ERR_INVALID;
  }
}

// ---- reduce ----
static std::shared_ptr<FoldKPlan> reduce_plan_cached(fopt_ctx* ctx, const fopt_mapping* src_map,
                                                     const fopt_mapping* dst_map, int allow_broadcast) {
  std::string key = "r|" + src_map->key + "|" + dst_map->key + "|" + std::to_string(allow_broadcast);
  if (ctx) {
    std::lock_guard<std::mutex> g(ctx->mu);
    auto it = ctx->folds.find(key);
    if (it != ctx->folds.end()) return it->second;
  }
  FoldPlan fp;
  auto u = unify({&src_map->m, &dst_map->m});
  if (!plan_reduce(u[0], u[1], allow_broadcast != 0, fp))
    throw Fail{FOPT_ERR_UNSUPPORTED, "reduce: mappings are not affine-factorisable"};
  auto kp = std::make_shared<FoldKPlan>(to_kfold(fp));
  if (!ctx) return kp;  // host-only query (fopt_row_reduce_shape without a context)
  std::lock_guard<std::mutex> g(ctx->mu);
  ctx->folds[key] = kp;
  return kp;
}

fopt_status fopt_reduce(fopt_ctx* ctx, void* out, const void* src, fopt_dtype dtype, fopt_reduce_op op,
                        uint32_t identity_bits, const fopt_mapping* src_map, const fopt_mapping* dst_map,
                        int allow_broadcast) {
  return guarded(ctx, [&] {
    require(out && src && src_map && dst_map, "fopt_reduce: null argument");
    require(dtype == FOPT_I32 || dtype == FOPT_F32 || dtype == FOPT_BF16, "fopt_reduce: dtype must be i32, f32 or bf16");
    auto kp = reduce_plan_cached(ctx, src_map, dst_map, allow_broadcast);
    launch_reduce(ctx, *kp, out, src, dtype, op, identity_bits, src_map->m.size());
  });
}

// A plain row reduction: dst cell t folds src cells t * W .. t * W + W - 1.
static bool plain_row_reduce(fopt_ctx* ctx, const fopt_mapping* src_map, const fopt_mapping* dst_map, int64_t* rows,
                             int64_t* W) {
  auto kp = reduce_plan_cached(ctx, src_map, dst_map, 0);
  const KWalk &o = kp->out, &r = kp->residue;
  if (o.n != 1 || r.n != 1 || o.live[0] != o.extent[0] || r.live[0] != r.extent[0] || r.stride[0][0] != 1 ||
      o.stride[0][0] != r.extent[0] || kp->out_positions != o.extent[0] ||
      src_map->m.size() != o.extent[0] * r.extent[0])
    return false;
  *rows = o.extent[0];
  *W = r.extent[0];
  return true;
}

fopt_status fopt_struct_sizes(size_t* sizes, int32_t n) {
  if (!sizes || n < 4) return FOPT_ERR_INVALID;
  sizes[0] = sizeof(fopt_program);
  sizes[1] = sizeof(fopt_epilogue);
  sizes[2] = sizeof(fopt_row_slot);
  sizes[3] = sizeof(fopt_row_plan);
  return FOPT_OK;
}

fopt_status fopt_row_reduce_shape(fopt_ctx* ctx, const fopt_mapping* src_map, const fopt_mapping* dst_map,
                                  int64_t* rows, int64_t* row_len) {
  bool ok = false;
  fopt_status st = guarded(ctx, [&] {
    require(src_map && dst_map && rows && row_len, "fopt_row_reduce_shape: bad arguments");
    ok = plain_row_reduce(ctx, src_map, dst_map, rows, row_len);
  });
  if (st == FOPT_OK && !ok) {
    if (ctx) ctx->err = "fopt_row_reduce_shape: not a plain row reduction";
    return FOPT_ERR_UNSUPPORTED;
  }
  return st;
}

fopt_status fopt_row_program(fopt_ctx* ctx, const fopt_row_plan* plan) {
  bool ran = false;
  fopt_status st = guarded(ctx, [&] {
    require(plan && plan->out, "fopt_row_program: bad arguments");
    ran = launch_row_jit(ctx, *plan);
  });
  if (st == FOPT_OK && !ran) {
    ctx->err = "fopt_row_program: no generated kernel for this plan";
    return FOPT_ERR_UNSUPPORTED;
  }
  return st;
}

fopt_status fopt_reduce_map(fopt_ctx* ctx, void* out, const fopt_program* prog, int32_t n_in, const void* const* inputs,
                            const fopt_dtype* in_dtypes, const int64_t* bcast, fopt_dtype dtype, fopt_reduce_op op,
                            uint32_t identity_bits, const fopt_mapping* src_map, const fopt_mapping* dst_map) {
  bool ran = false;
  fopt_status st = guarded(ctx, [&] {
    require(out && prog && src_map && dst_map && n_in >= 0 && n_in <= 3, "fopt_reduce_map: bad arguments");
    require(prog->n_insn >= 0 && prog->n_insn <= 32, "fopt_reduce_map: program too long");
    for (int i = 0; i < n_in; ++i) require(inputs[i] != nullptr, "fopt_reduce_map: null input");
    // folds whose result does not depend on the order (or f32 sums outside exact-fold mode)
    int fold = -1;
    if (dtype == FOPT_F32) {
      if (op == FOPT_RED_MAX) fold = 2;
      else if (op == FOPT_RED_MIN) fold = 3;
      else if (!ctx->exact_fold && op == FOPT_RED_ADD) fold = 0;
      else if (!ctx->exact_fold && op == FOPT_RED_MUL) fold = 4;
    } else if (dtype == FOPT_I32) {
      if (op == FOPT_RED_ADD) fold = 10;
      else if (op == FOPT_RED_MAX) fold = 12;
      else if (op == FOPT_RED_MIN) fold = 13;
    }
    if (fold < 0) return;
    int64_t rows = 0, W = 0;
    if (!plain_row_reduce(ctx, src_map, dst_map, &rows, &W)) return;
    ran = launch_reduce_map_jit(ctx, prog, n_in, inputs, in_dtypes, bcast, fold, identity_bits, out, rows, W);
  });
  if (st == FOPT_OK && !ran) {
    ctx->err = "fopt_reduce_map: no fused kernel for this reduction";
    return FOPT_ERR_UNSUPPORTED;
  }
  return st;
}

// ---- contraction ----
static bool acc_type_of(int in_dt, int* acc) {
  switch (in_dt) {
    case FOPT_I8: case FOPT_I4: case FOPT_I5: case FOPT_I9: case FOPT_I32: *acc = FOPT_I32; return true;
    case FOPT_BF16: case FOPT_F8E4M3: case FOPT_F8E5M2: case FOPT_F32: *acc = FOPT_F32; return true;
    default: return false;
  }
}

// Detects a plain GEMM: out [M, N] row-major over two wheels, lhs [M, K] K-major, rhs [N, K]
// K-major, one fully-live contracted wheel. Fills M, N, K and leading dimensions.
static bool as_gemm(const FoldKPlan& p, int64_t* M, int64_t* N, int64_t* K, int64_t* lda, int64_t* ldb, int64_t* ldd,
                    int* scale_along_n) {
  if (p.residue.n != 1 || p.residue.live[0] != p.residue.extent[0]) return false;
  if (p.residue.stride[0][0] != 1 || p.residue.stride[1][0] != 1) return false;
  const KWalk& o = p.out;
  if (o.n != 2 || o.live[0] != o.extent[0] || o.live[1] != o.extent[1]) return false;
  // wheel 0 = N (inner, lhs stride 0), wheel 1 = M (rhs stride 0)
  if (o.stride[0][0] != 0 || o.stride[1][1] != 0) return false;
  *N = o.extent[0];
  *M = o.extent[1];
  *K = p.residue.extent[0];
  *lda = o.stride[0][1];
  *ldb = o.stride[1][0];
  *ldd = o.extent[0];
  if (*lda < *K || *ldb < *K) return false;
  *scale_along_n = o.stride[2][0] == 1 && o.stride[2][1] == 0;
  return true;
}

// Validates a contraction's arguments and returns its (cached) fold plan.
static std::shared_ptr<FoldKPlan> contraction_plan(fopt_ctx* ctx, fopt_dtype out_dtype, fopt_dtype in_dtype,
                                                   const fopt_mapping* lhs_map, const fopt_mapping* rhs_map,
                                                   const fopt_mapping* pre_reduce, const fopt_mapping* out_map,
                                                   const fopt_epilogue* epilogue) {
  require(lhs_map && rhs_map && pre_reduce && out_map, "fopt_contraction: null mapping");
  int acc;
  require(acc_type_of(in_dtype, &acc), "fopt_contraction: unsupported operand dtype");
  int ep_kind = epilogue ? epilogue->kind : 0;
  if (ep_kind == 4) {
    require(acc == FOPT_I32 && out_dtype == FOPT_F32, "SwiGLU epilogue maps an integer contraction to f32");
    require(epilogue->scale && epilogue->scale_axis && epilogue->row_scale,
            "SwiGLU epilogue needs row and channel scale vectors");
  } else if (ep_kind == 3 || ep_kind == 5) {
    require(acc == FOPT_I32 && out_dtype == FOPT_BF16, "dequant epilogue maps an integer contraction to bf16");
    require(epilogue->scale && epilogue->scale_axis && epilogue->row_scale,
            "dequant epilogue needs row and channel scale vectors");
    require(ep_kind == 3 || epilogue->residual, "residual epilogue needs the residual");
  } else if (ep_kind == 1) {
    require(acc == FOPT_I32, "requant epilogue needs an integer contraction");
    require(out_dtype == FOPT_I8, "requant epilogue commits i8");
    require(epilogue->scale && epilogue->scale_axis, "requant epilogue needs a scale vector and its axis");
  } else {
    require(out_dtype == in_dtype || out_dtype == acc, "fopt_contraction: out dtype must be the operand or accumulator type");
  }
  const bool scaled = ep_kind == 1 || ep_kind == 3 || ep_kind == 4 || ep_kind == 5;
  std::string extra_key = scaled ? std::string(epilogue->scale_axis) : "";
  std::string key = "c|" + lhs_map->key + "|" + rhs_map->key + "|" + pre_reduce->key + "|" + out_map->key + "|" + extra_key;
  {
    std::lock_guard<std::mutex> g(ctx->mu);
    auto it = ctx->folds.find(key);
    if (it != ctx->folds.end()) return it->second;
  }
  FoldPlan fp;
  // The four mappings may come from separate axis tables; re-parse against one shared table.
  auto table = std::make_shared<AxisTable>();
  auto adopt = [&](const Mapping& m) {
    for (size_t i = 0; i < m.axes->names.size(); ++i) table->intern(m.axes->names[i], m.axes->sizes[i]);
  };
  for (auto* h : {lhs_map, rhs_map, pre_reduce, out_map}) adopt(h->m);
  Mapping L = parse_mapping(lhs_map->m.to_string(), table), Rm = parse_mapping(rhs_map->m.to_string(), table),
          P = parse_mapping(pre_reduce->m.to_string(), table), O = parse_mapping(out_map->m.to_string(), table);
  Mapping X;
  if (scaled) X = parse_mapping(epilogue->scale_axis, table);
  if (!plan_contraction(L, Rm, P, O, fp, scaled ? &X : nullptr))
    throw Fail{FOPT_ERR_UNSUPPORTED, "contraction: mappings are not affine-factorisable"};
  auto kp = std::make_shared<FoldKPlan>(to_kfold(fp));
  std::lock_guard<std::mutex> g(ctx->mu);
  ctx->folds[key] = kp;
  return kp;
}

static void run_contraction(fopt_ctx* ctx, const FoldKPlan& kp, void* out, fopt_dtype out_dtype, const void* lhs,
                            const void* rhs, fopt_dtype in_dtype, int64_t lhs_elems, int64_t rhs_elems,
                            const fopt_epilogue* epilogue) {
  const int ep_kind = epilogue ? epilogue->kind : 0;
  const bool scaled = ep_kind == 1 || ep_kind == 3 || ep_kind == 4 || ep_kind == 5;
  int64_t M, N, K, lda, ldb, ldd;
  int scale_n = 0;
  if (as_gemm(kp, &M, &N, &K, &lda, &ldb, &ldd, &scale_n) && (!scaled || scale_n)) {
    if (ep_kind == 4) ldd = N / 2;  // the activation rows: half the interleaved product's columns
    if ((ep_kind != 4 || ldd == N / 2) &&
        launch_gemm_tc(ctx, out, out_dtype, lhs, rhs, in_dtype, M, N, K, lda, ldb, ldd, epilogue,
                       scaled ? epilogue->scale : nullptr, scale_n))
      return;
  }
  if (ep_kind == 4)
    throw Fail{FOPT_ERR_UNSUPPORTED, "SwiGLU epilogue needs a GEMM-shaped contraction with M % 256 and N % 256, "
                                     "scales along N, on the paired tensor-core kernel"};
  if (ep_kind == 3 || ep_kind == 5)
    throw Fail{FOPT_ERR_UNSUPPORTED, "dequant epilogue needs a GEMM-shaped contraction ([M, K] x [N, K] -> [M, N], "
                                     "M % 128, K % 128 bytes, N % 128, scales along N)"};
  launch_contraction_generic(ctx, kp, out, out_dtype, lhs, rhs, in_dtype, lhs_elems, rhs_elems, epilogue, nullptr,
                             ep_kind == 1 ? epilogue->scale : nullptr);
}

fopt_status fopt_contraction(fopt_ctx* ctx, void* out, fopt_dtype out_dtype, const void* lhs, const void* rhs,
                             fopt_dtype in_dtype, const fopt_mapping* lhs_map, const fopt_mapping* rhs_map,
                             const fopt_mapping* pre_reduce, const fopt_mapping* out_map,
                             const fopt_epilogue* epilogue) {
  return guarded(ctx, [&] {
    require(out && lhs && rhs, "fopt_contraction: null argument");
    auto kp = contraction_plan(ctx, out_dtype, in_dtype, lhs_map, rhs_map, pre_reduce, out_map, epilogue);
    run_contraction(ctx, *kp, out, out_dtype, lhs, rhs, in_dtype, lhs_map->m.size(), rhs_map->m.size(), epilogue);
  });
}

// The contraction on host buffers: operands in, result out, all in one call. A GEMM-shaped
// contraction with dense rows is pipelined: the rhs goes over once, then the lhs in row chunks on a
// copy stream, each chunk's GEMM on the compute stream as soon as its rows have landed, and each
// chunk of the result back on a second copy stream while later chunks are still coming in (PCIe
// carries both directions at once). Row chunks do not change any cell's sum, so the result is the
// one-shot contraction's. Host buffers should be pinned for the copies to overlap. On this pool the
// upload itself bounds the call (about 29 GB/s host -> device), so the pipeline hides the GEMM and
// the download behind it rather than shortening the upload.
fopt_status fopt_contraction_host(fopt_ctx* ctx, void* host_out, fopt_dtype out_dtype, const void* host_lhs,
                                  const void* host_rhs, fopt_dtype in_dtype, const fopt_mapping* lhs_map,
                                  const fopt_mapping* rhs_map, const fopt_mapping* pre_reduce,
                                  const fopt_mapping* out_map, const fopt_epilogue* epilogue) {
  return guarded(ctx, [&] {
    require(host_out && host_lhs && host_rhs, "fopt_contraction_host: null argument");
    require(!epilogue || (epilogue->kind != 4 && epilogue->kind != 5),
            "fopt_contraction_host: the SwiGLU and residual epilogues run on device storages");
    auto kp = contraction_plan(ctx, out_dtype, in_dtype, lhs_map, rhs_map, pre_reduce, out_map, epilogue);
    const int64_t lhs_elems = lhs_map->m.size(), rhs_elems = rhs_map->m.size(), out_elems = out_map->m.size();
    const size_t lb = (size_t)(lhs_elems * dtype_bits(in_dtype) + 7) / 8, rb = (size_t)(rhs_elems * dtype_bits(in_dtype) + 7) / 8;
    const size_t ob = (size_t)(out_elems * dtype_bits(out_dtype) + 7) / 8;
    void *dA = nullptr, *dB = nullptr, *dC = nullptr;
    cuda_check(cudaMallocAsync(&dA, std::max<size_t>(lb, 16), ctx->stream), "alloc");
    cuda_check(cudaMallocAsync(&dB, std::max<size_t>(rb, 16), ctx->stream), "alloc");
    cuda_check(cudaMallocAsync(&dC, std::max<size_t>(ob, 16), ctx->stream), "alloc");
    int64_t M, N, K, lda, ldb, ldd;
    int scale_n = 0;
    const int ep_kind = epilogue ? epilogue->kind : 0;
    const bool scaled = ep_kind == 1 || ep_kind == 3;
    const int ib = dtype_bits(in_dtype), obits = dtype_bits(out_dtype);
    const int64_t kRows = getenv("FOPT_HOST_ROWS") ? atoll(getenv("FOPT_HOST_ROWS")) : 512;
    const bool chunked = as_gemm(*kp, &M, &N, &K, &lda, &ldb, &ldd, &scale_n) && (!scaled || scale_n) &&
                         ib >= 8 && obits >= 8 && lda == K && ldd == N && M % kRows == 0 && M >= 2 * kRows &&
                         N % 128 == 0 && (K * ib / 8) % 128 == 0 &&
                         lb == (size_t)(M * K * ib / 8) && ob == (size_t)(M * N * obits / 8) &&
                         !getenv("FOPT_HOST_NO_PIPELINE");
    if (!chunked) {
      cuda_check(cudaMemcpyAsync(dA, host_lhs, lb, cudaMemcpyHostToDevice, ctx->stream), "h2d");
      cuda_check(cudaMemcpyAsync(dB, host_rhs, rb, cudaMemcpyHostToDevice, ctx->stream), "h2d");
      run_contraction(ctx, *kp, dC, out_dtype, dA, dB, in_dtype, lhs_elems, rhs_elems, epilogue);
      cuda_check(cudaMemcpyAsync(host_out, dC, ob, cudaMemcpyDeviceToHost, ctx->stream), "d2h");
    } else {
      for (auto* s : {&ctx->copy_in, &ctx->copy_out})
        if (!*s) cuda_check(cudaStreamCreateWithFlags(s, cudaStreamNonBlocking), "copy stream");
      auto event = [&]() {
        cudaEvent_t e;
        cuda_check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event");
        return e;
      };
      std::vector<cudaEvent_t> evs;
      auto record = [&](cudaStream_t s) {
        cudaEvent_t e = event();
        evs.push_back(e);
        cuda_check(cudaEventRecord(e, s), "event record");
        return e;
      };
      // the copies start after whatever the compute stream already holds (buffer reuse)
      cuda_check(cudaStreamWaitEvent(ctx->copy_in, record(ctx->stream), 0), "wait");
      cuda_check(cudaStreamWaitEvent(ctx->copy_out, evs.back(), 0), "wait");
      // one upload stream: two concurrent uploads measured 3.5x slower than one on this pool
      cuda_check(cudaMemcpyAsync(dB, host_rhs, rb, cudaMemcpyHostToDevice, ctx->copy_in), "h2d");
      const int64_t arow = K * ib / 8, crow = N * obits / 8;
      for (int64_t r0 = 0; r0 < M; r0 += kRows) {
        cuda_check(cudaMemcpyAsync((char*)dA + r0 * arow, (const char*)host_lhs + r0 * arow, kRows * arow,
                                   cudaMemcpyHostToDevice, ctx->copy_in), "h2d");
        cuda_check(cudaStreamWaitEvent(ctx->stream, record(ctx->copy_in), 0), "wait");
        fopt_epilogue ep{};
        if (epilogue) {
          ep = *epilogue;
          if (ep.row_scale) ep.row_scale += r0;
        }
        if (!launch_gemm_tc(ctx, (char*)dC + r0 * crow, out_dtype, (char*)dA + r0 * arow, dB, in_dtype, kRows, N, K,
                            lda, ldb, ldd, epilogue ? &ep : nullptr, scaled ? epilogue->scale : nullptr, scale_n))
          throw Fail{FOPT_ERR_UNSUPPORTED, "fopt_contraction_host: chunk not tensor-core shaped"};
        cuda_check(cudaStreamWaitEvent(ctx->copy_out, record(ctx->stream), 0), "wait");
        cuda_check(cudaMemcpyAsync((char*)host_out + r0 * crow, (char*)dC + r0 * crow, kRows * crow,
                                   cudaMemcpyDeviceToHost, ctx->copy_out), "d2h");
      }
      cuda_check(cudaStreamWaitEvent(ctx->stream, record(ctx->copy_out), 0), "wait");
      for (auto e : evs) cudaEventDestroy(e);  // released once their work completes
    }
    cudaFreeAsync(dA, ctx->stream);
    cudaFreeAsync(dB, ctx->stream);
    cudaFreeAsync(dC, ctx->stream);
  });
}

// ---- attention ----
fopt_status fopt_attention(fopt_ctx* ctx, void* o, const void* q, const void* k, const void* v, int32_t batch,
                           int32_t seq, int32_t hq, int32_t hkv, int32_t head_dim, float scale, int32_t causal,
                           float eps) {
  return guarded(ctx, [&] {
    require(o && q && k && v, "fopt_attention: null argument");
    require(head_dim == 128, "fopt_attention: head_dim must be 128");
    require(hkv > 0 && hq % hkv == 0, "fopt_attention: query heads must be a multiple of kv heads");
    require(batch > 0 && seq > 0, "fopt_attention: empty problem");
    launch_attention(ctx, o, q, k, v, batch, seq, hq, hkv, head_dim, scale, causal, eps);
  });
}

}  // extern "C"

// ---- byte equality (BufStorage PartialEq, buf.rs:38-41) ----
namespace {
__global__ void bytes_differ_kernel(const uint8_t* a, const uint8_t* b, size_t n, int32_t* flag) {
  size_t words = n / 16;
  const uint4* a4 = (const uint4*)a;
  const uint4* b4 = (const uint4*)b;
  bool aligned = ((uintptr_t)a % 16 == 0) && ((uintptr_t)b % 16 == 0);
  size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, step = (size_t)gridDim.x * blockDim.x;
  int diff = 0;
  if (aligned) {
    for (size_t i = tid; i < words; i += step) {
      uint4 x = a4[i], y = b4[i];
      diff |= (x.x != y.x) | (x.y != y.y) | (x.z != y.z) | (x.w != y.w);
    }
    for (size_t i = words * 16 + tid; i < n; i += step) diff |= a[i] != b[i];
  } else {
    for (size_t i = tid; i < n; i += step) diff |= a[i] != b[i];
  }
  if (__any_sync(0xffffffffu, diff) && (threadIdx.x & 31) == 0) atomicOr(flag, 1);
}
}  // namespace

extern "C" fopt_status fopt_equal(fopt_ctx* ctx, const void* a, const void* b, size_t bytes, int* equal) {
  return guarded(ctx, [&] {
    require(a && b && equal, "fopt_equal: null argument");
    int32_t* flag = (int32_t*)scratch(ctx, 16);
    cuda_check(cudaMemsetAsync(flag, 0, 4, ctx->stream), "equal flag");
    if (bytes) {
      int grid = (int)std::max<size_t>(1, std::min<size_t>((bytes / 16 + 255) / 256, 148 * 8));
      bytes_differ_kernel<<<grid, 256, 0, ctx->stream>>>((const uint8_t*)a, (const uint8_t*)b, bytes, flag);
      launched(ctx, "bytes_differ");
    }
    int32_t h = 0;
    cuda_check(cudaMemcpyAsync(&h, flag, 4, cudaMemcpyDeviceToHost, ctx->stream), "equal d2h");
    cuda_check(cudaStreamSynchronize(ctx->stream), "equal sync");
    *equal = h == 0;
  });
}

std::shared_ptr<FoldKPlan> fopt::reduce_plan(fopt_ctx* ctx, const fopt_mapping* src_map, const fopt_mapping* dst_map,
                                             int allow_broadcast) {
  return reduce_plan_cached(ctx, src_map, dst_map, allow_broadcast);
}
