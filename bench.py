"""Benchmark: the furiosa-opt emulator hot path on B200.

Default (headline) workload: config 2, the standalone int8 contraction M=N=K=4096 (i32 accumulate,
per-channel fp32 requant to i8), one step = one `contraction` call through the backend.
  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload gemm_i8|gemm_bf16|attention|
                  relayout|allreduce|mnist|decoder|decoder_tp] [--impl ours|reference]
Multi-GPU (torchrun, one rank per GPU): independent replicas of the step ("replicas only": the
contraction does not shard), except `allreduce`, the config-5 NCCL collective, and `decoder_tp`,
the config-4 block split over the GPUs (strong scaling).
`--impl reference` times the reference algorithm's CPU restatement (the oracle port: the emulator
itself is Rust + closed prebuilt libraries and cannot be built here) on this host's cores.
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def _pkg():
    if "furiosa_opt_b200" in sys.modules:
        return sys.modules["furiosa_opt_b200"]
    d = os.path.join(ROOT, "furiosa-opt_b200")
    spec = importlib.util.spec_from_file_location("furiosa_opt_b200", os.path.join(d, "__init__.py"),
                                                  submodule_search_locations=[d])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["furiosa_opt_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


class Clocks:
    """Samples nvidia-smi during the timed region (median SM clock under load, throttle reasons)."""

    def __init__(self, index: int):
        self.index, self.samples, self.proc = index, [], None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms",
                                          "50", "-i", str(self.index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def wait_first_sample(self, timeout=5.0):
        t0 = time.time()
        while self.proc and not self.samples and time.time() - t0 < timeout:
            time.sleep(0.02)

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 8:
                self.samples.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=2)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons}


# ---------------------------------------------------------------------------------------------
# workloads: each returns a dict with step(), per-step units, and metadata
# ---------------------------------------------------------------------------------------------
# DRAM bytes per launch of the step's dominant kernel, read + write, from one ncu capture of this
# workload (the summaries under profiles/ give the command); None where no capture was taken.
TRAFFIC = {
    "gemm_i8_4096x4096x4096": (33.6e6, "profiles/gemm_tc_i8_4096.md"),
    "attention_s2048": (25.2e6, "profiles/attention_tc2_s2048.md"),
}


def wl_gemm(fb, be, dtype: str, M=4096, N=4096, K=4096):
    rng = np.random.default_rng(42)
    ax = dict(M=M, N=N, K=K)
    exprs = ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]")
    L, R, P, O = (fb.Mapping(e, ax) for e in exprs)
    if dtype == "i8":
        a = rng.integers(-128, 128, M * K, dtype=np.int64).astype(np.int8)
        b = rng.integers(-128, 128, N * K, dtype=np.int64).astype(np.int8)
    else:
        a = fb.dtypes.f32_to_bf16_bits(rng.standard_normal(M * K).astype(np.float32))
        b = fb.dtypes.f32_to_bf16_bits(rng.standard_normal(N * K).astype(np.float32))
    scale = rng.uniform(0.001, 0.01, N).astype(np.float32)
    A, B = be.from_vec(L, a, dtype), be.from_vec(R, b, dtype)
    S = be.from_vec(fb.Mapping("[N]", ax), scale, "f32")
    out_dt = "i8" if dtype == "i8" else "bf16"
    ops = 2.0 * M * N * K
    OUT = be.zeroed(O, out_dt)

    def issue():
        if dtype == "i8":
            return be.contraction_requant(A, B, L, R, P, O, S, "N", out=OUT)
        return be.contraction(A, B, L, R, P, O, out=OUT)

    # the step is captured once and replayed, so the timed region holds the GEMM kernel and not the
    # host's plan lookup and tensor-map encoding (FOPT_NO_GRAPH=1 issues every step from the host)
    state = {}

    def step():
        if os.environ.get("FOPT_NO_GRAPH"):
            return issue()
        if "graph" not in state:
            if not state.get("eager"):
                state["eager"] = True
                return issue()
            state["graph"] = be.capture(issue)
        return state["graph"].launch()

    # e2e: host (pinned) inputs -> device -> contraction -> host result, every step
    import torch

    ha = torch.from_numpy(a.view(np.uint8)).pin_memory()
    hb = torch.from_numpy(b.view(np.uint8)).pin_memory()
    hout = torch.empty(M * N * (1 if dtype == "i8" else 2), dtype=torch.uint8).pin_memory()
    lib = fb._lib.lib()

    ep = fb.backend._ep(1, S, "N") if dtype == "i8" else None

    def e2e_step():
        # the public host-buffer call: operands in, contraction, result out (pipelined in row chunks)
        return be.contraction_host(ha, hb, L, R, P, O, dtype, out_dt, ep=ep, out=hout)

    return dict(step=step, e2e_step=e2e_step, units=ops, unit="TOPS" if dtype == "i8" else "TFLOP/s",
                scale=1e12, metric=f"{'int8' if dtype == 'i8' else 'bf16'} GEMM "
                                   f"{'TOPS' if dtype == 'i8' else 'TFLOP/s'} (M=N=K={M})",
                h2d=ha.numel() + hb.numel(), d2h=hout.numel(), bound="tensor",
                e2e_api="B200.contraction_host -> fopt_contraction_host (pinned host buffers, row-chunk pipeline)",
                algo_bytes=None, workload=f"gemm_{dtype}_{M}x{N}x{K}", dtype=dtype,
                extra={"out_dtype": out_dt, "epilogue": "per-channel requant" if dtype == "i8" else "bf16 narrow"},
                cpu=lambda rows: cpu_gemm(a, b, scale, dtype, M, N, K, rows),
                config={"M": M, "N": N, "K": K, "layout": "lhs [M, K], rhs [N, K], out [M, N]",
                        "cuda_graph": not os.environ.get("FOPT_NO_GRAPH")})


def cpu_gemm(a, b, scale, dtype, M, N, K, rows):
    import oracle
    from oracle import ref_m

    ax = dict(M=M, N=N, K=K)
    rl, rr, rp, ro = (ref_m(e, **ax) for e in ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]"))
    # only the per-cell fold is timed (the read plans correspond to the reference's sequence() setup)
    if dtype == "i8":
        oracle.contract(a.tobytes(), b.tobytes(), "i8", "i8", rl, rr, rp, ro, ep_kind=1, scale=scale,
                        scale_axis="N", out_cells=rows * N)
    else:
        oracle.contract(a.tobytes(), b.tobytes(), "bf16", "bf16", rl, rr, rp, ro, out_cells=rows * N)
    dt = oracle.last_fold_seconds
    return 2.0 * rows * N * K / dt, f"{rows} of {M} output rows ({rows * N} cells, full K={K})"


def wl_attention(fb, be, S=2048, Hq=32, Hkv=8, D=128):
    rng = np.random.default_rng(42)
    q = fb.dtypes.f32_to_bf16_bits(rng.standard_normal(S * Hq * D).astype(np.float32))
    k = fb.dtypes.f32_to_bf16_bits(rng.standard_normal(S * Hkv * D).astype(np.float32))
    v = fb.dtypes.f32_to_bf16_bits(rng.standard_normal(S * Hkv * D).astype(np.float32))
    mq = fb.Mapping("[S, H, D]", dict(S=S, H=Hq, D=D))
    mk = fb.Mapping("[S, H, D]", dict(S=S, H=Hkv, D=D))
    Q, Kt, V = be.from_vec(mq, q, "bf16"), be.from_vec(mk, k, "bf16"), be.from_vec(mk, v, "bf16")
    OUT = be.zeroed(mq, "bf16")

    def step():
        return be.attention(Q, Kt, V, 1, S, Hq, Hkv, D, causal=True, out=OUT)

    flops = 4.0 * S * S * D * Hq / 2  # causal half
    return dict(step=step, units=S, unit="tokens/s", scale=1.0, flops=flops, bound="tensor",
                metric="attention prefill tokens/s (Llama-3-8B shape, S=2048, causal)", workload="attention_s2048",
                dtype="bf16", config={"S": S, "Hq": Hq, "Hkv": Hkv, "D": D, "causal": True})


def wl_relayout(fb, be, R=8192, C=8192):
    rng = np.random.default_rng(1)
    ax = dict(R=R, C=C)
    S, D = fb.Mapping("[R, C]", ax), fb.Mapping("[C, R]", ax)
    x = fb.dtypes.f32_to_bf16_bits(rng.standard_normal(R * C).astype(np.float32))
    X = be.from_vec(S, x, "bf16")
    Y = be.zeroed(D, "bf16")

    def step():
        be.transpose(Y, X, S, D)
        return Y

    return dict(step=step, units=2.0 * R * C * 2, unit="GB/s", scale=1e9, bound="hbm",
                metric="relayout GB/s ([R, C] -> [C, R] bf16, 128 MiB)", workload="relayout_bf16_8192x8192",
                dtype="bf16", config={"R": R, "C": C})


def wl_allreduce(fb, be, rank, world, count=8 * 2048 * 4096):
    """Config 5: all-reduce of an 8x2048x4096 bf16 activation (N(0,1) per rank) over the Chip axis."""
    if world > 1:
        fb.dist.init_comm(be, rank, world)
    rng = np.random.default_rng(100 + rank)
    m = fb.Mapping("[E]", dict(E=count))
    x = be.from_vec(m, fb.dtypes.f32_to_bf16_bits(rng.standard_normal(count).astype(np.float32)), "bf16")

    def step():
        if world > 1:
            fb.dist.allreduce(be, x)
        return x

    nbytes = 2 * count
    bus = 2.0 * (world - 1) / world * nbytes if world > 1 else 0.0
    return dict(step=step, units=bus, unit="GB/s", scale=1e9, bound="nvlink", aggregate=False,
                metric="all-reduce bus bandwidth (8x2048x4096 bf16 per rank)", workload="allreduce_bf16_128MiB",
                dtype="bf16", config={"elements_per_rank": count, "bytes_per_rank": nbytes,
                                      "busbw": "bytes * 2(n-1)/n / t"})


def allreduce_sweep(fb, be, world, stream, steps=5):
    """1 KiB .. 1 GiB message sweep (x2 steps), bus bandwidth per size."""
    import torch

    out = []
    size = 1024
    buf = be.zeroed(fb.Mapping("[E]", dict(E=(1 << 30) // 2)), "bf16")
    lib = fb._lib.lib()
    st = stream  # the stream the library launches on
    while size <= (1 << 30):
        n = size // 2
        for _ in range(2):
            lib.fopt_allreduce(be.ctx, buf.ptr, n, fb._lib.DTYPES["bf16"])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(steps):
            lib.fopt_allreduce(be.ctx, buf.ptr, n, fb._lib.DTYPES["bf16"])
        e1.record(st)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t[0])
        out.append({"bytes": size, "us": round(ms * 1e3, 2),
                    "busbw_gbs": round(2.0 * (world - 1) / world * size / (ms * 1e-3) / 1e9, 1)})
        size *= 2
    return out


def wl_mnist(fb, be, B=64, I=784, H=128, O=10):
    """Config 1: MNIST-shaped int8 MLP forward (latency-bound). Unit: images/s."""
    x, w1, w2, s1 = fb.workloads.mnist_inputs(0, B, I, H, O)
    ax = dict(B=B, I=I, H=H, O=O)
    m = lambda e: fb.Mapping(e, ax)
    X, W1, W2, S1 = (be.from_vec(m("[B, I]"), x, "i8"), be.from_vec(m("[H, I]"), w1, "i8"),
                     be.from_vec(m("[O, H]"), w2, "i8"), be.from_vec(m("[H]"), s1, "f32"))

    fwd = lambda: fb.workloads.mnist_int8_forward(be, X, W1, W2, S1, B, I, H, O)  # noqa: E731
    out_bytes = fwd().nbytes
    step, e2e_step, hx, hout = graphed_step(fb, be, fwd, X, out_bytes)
    return dict(step=step, e2e_step=e2e_step, h2d=hx.numel(), d2h=hout.numel(),
                e2e_api="fopt_h2d -> captured forward (fopt_graph_launch) -> fopt_d2h (pinned host buffers)",
                units=B, unit="images/s", scale=1.0, bound="latency", flops=2.0 * B * (I * H + H * O),
                metric="MNIST-shaped int8 MLP forward, images/s (64x784 -> 128 -> 10)", workload="mnist_int8_mlp",
                dtype="i8", config={"B": B, "I": I, "H": H, "O": O, "cuda_graph": not os.environ.get("FOPT_NO_GRAPH")})


def graphed_step(fb, be, forward, X, out_bytes):
    """A step that runs `forward` once eagerly (kernels compiled, workspaces sized), then captures
    it into a CUDA graph and replays the graph every later step: the same kernels without the host
    work of issuing them (FOPT_NO_GRAPH=1 issues every step from the host). The end-to-end step
    copies the input X in from pinned host memory and the result out."""
    import torch

    use_graph = not os.environ.get("FOPT_NO_GRAPH")
    state = {}

    def step():
        if not use_graph:
            return forward()
        if "graph" not in state:
            if not state.get("eager"):
                state["eager"] = True
                return forward()
            state["graph"] = be.capture(forward)
        return state["graph"].launch()

    hx = torch.from_numpy(X.to_numpy().view(np.uint8).copy()).pin_memory()
    hout = torch.empty(out_bytes, dtype=torch.uint8).pin_memory()
    lib = fb._lib.lib()

    def e2e_step():
        fb._lib.check(lib.fopt_h2d(be.ctx, X.ptr, C.c_void_p(hx.data_ptr()), hx.numel()), be.ctx)
        out = step()
        fb._lib.check(lib.fopt_d2h(be.ctx, C.c_void_p(hout.data_ptr()), out.ptr, hout.numel()), be.ctx)

    return step, e2e_step, hx, hout


def wl_decoder(fb, be, batch=8, seq=512, Hq=32, Hkv=8, F=14336):
    """Config 4: W8A8 Llama-3-8B decoder block over 8 x 512 tokens. Unit: tokens/s."""
    T, H = batch * seq, Hq * 128
    blk = fb.workloads.DecoderBlockW8A8(be, T, H, Hq, Hkv, F, batch, seq, seed=0)
    rng = np.random.default_rng(1)
    X = be.from_vec(blk.m("[T, H]"), fb.dtypes.f32_to_bf16_bits(rng.standard_normal(T * H).astype(np.float32)),
                    "bf16")

    step, e2e_step, hx, hout = graphed_step(fb, be, lambda: blk.forward(X), X, T * H * 2)
    return dict(step=step, e2e_step=e2e_step, h2d=hx.numel(), d2h=hout.numel(),
                e2e_api="fopt_h2d -> captured block (fopt_graph_launch) -> fopt_d2h (pinned host buffers)",
                units=T, unit="tokens/s", scale=1.0, bound="tensor", dtype="i8",
                flops=blk.gemm_ops() + blk.attention_flops(),
                metric="W8A8 decoder block tokens/s (Llama-3-8B shape, 8 x 512 tokens)", workload="decoder_w8a8",
                config={"batch": batch, "seq": seq, "hidden": H, "ffn": F, "heads": Hq, "kv_heads": Hkv,
                        "gemm_ops": blk.gemm_ops(), "attention_flops": blk.attention_flops(),
                        "cuda_graph": not os.environ.get("FOPT_NO_GRAPH")})


def wl_decoder_tp(fb, be, rank, world, batch=8, seq=512, Hq=32, Hkv=8, F=14336):
    """Config 4 tensor-parallel over the ranks (strong scaling: the same 8 x 512-token block, heads and
    FFN columns split across GPUs, NCCL between the halves). Unit: tokens/s of the whole block."""
    T, H = batch * seq, Hq * 128
    if world > 1:
        fb.dist.init_comm(be, rank, world)
    else:
        fb.dist.init_comm(be, 0, 1)
    blk = fb.workloads.DecoderBlockW8A8TP(be, T, H, Hq, Hkv, F, batch, seq, rank, world, seed=0)
    rng = np.random.default_rng(1)
    X = be.from_vec(blk.m("[T, H]"), fb.dtypes.f32_to_bf16_bits(rng.standard_normal(T * H).astype(np.float32)),
                    "bf16")

    step, e2e_step, hx, hout = graphed_step(fb, be, lambda: blk.forward(X), X, T * H * 2)
    return dict(step=step, e2e_step=e2e_step, h2d=hx.numel(), d2h=hout.numel(),
                e2e_api="fopt_h2d -> captured block with its NCCL all-reduces (fopt_graph_launch) -> fopt_d2h",
                units=T, unit="tokens/s", scale=1.0, bound="tensor", dtype="i8", aggregate=False,
                scaling="strong", flops=blk.gemm_ops() + blk.attention_flops(),
                metric="W8A8 decoder block tokens/s, tensor-parallel (Llama-3-8B shape, 8 x 512 tokens)",
                workload="decoder_w8a8_tp",
                config={"batch": batch, "seq": seq, "hidden": H, "ffn": F, "heads": Hq, "kv_heads": Hkv,
                        "gemm_ops": blk.gemm_ops(), "attention_flops": blk.attention_flops()})


def bind_to_gpu_cpus(local: int) -> str:
    """Pins this process to the CPUs NVML reports as local to the GPU (a read-only query), so the
    pinned host buffers of the end-to-end steps sit on the GPU's NUMA node; host-to-device copies
    from the other socket's memory cross the inter-socket link. Returns what it did."""
    if os.environ.get("FOPT_NO_NUMA_BIND"):
        return "off"
    try:
        import pynvml

        pynvml.nvmlInit()
        try:
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            index = int(visible.split(",")[local]) if visible else local
            h = pynvml.nvmlDeviceGetHandleByIndex(index)
            words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = {w * 64 + b for w, word in enumerate(words) for b in range(64) if word >> b & 1}
        cpus &= set(range(os.cpu_count()))
        if not cpus:
            return "no affinity reported"
        os.sched_setaffinity(0, cpus)
        return f"{len(cpus)} GPU-local CPUs"
    except Exception as e:  # no NVML or no permission: run unbound
        return f"unbound ({type(e).__name__})"


def run_ours(args, rank, world, local):
    import torch

    numa = bind_to_gpu_cpus(local)
    fb = _pkg()
    torch.cuda.set_device(local)
    be = fb.B200(local)
    stream = torch.cuda.Stream()
    fb._lib.lib().fopt_set_stream(be.ctx, stream.cuda_stream)
    wl = {"gemm_i8": lambda: wl_gemm(fb, be, "i8"), "gemm_bf16": lambda: wl_gemm(fb, be, "bf16"),
          "attention": lambda: wl_attention(fb, be), "relayout": lambda: wl_relayout(fb, be),
          "allreduce": lambda: wl_allreduce(fb, be, rank, world), "mnist": lambda: wl_mnist(fb, be),
          "decoder": lambda: wl_decoder(fb, be),
          "decoder_tp": lambda: wl_decoder_tp(fb, be, rank, world)}[args.workload]()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")  # > 126 MB L2
    clk = Clocks(local).__enter__()  # sampling runs from before warm-up to the end of the timed steps
    clk.wait_first_sample()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            wl["step"]()
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        launches0 = be.launches
        durs = []
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        if True:
            torch.cuda.synchronize()
            wall0 = time.perf_counter()
            for i in range(args.steps):
                flush.zero_()
                ev[i][0].record(stream)
                wl["step"]()
                ev[i][1].record(stream)
            torch.cuda.synchronize()
            wall = time.perf_counter() - wall0
        clk.__exit__()
        launches = be.launches - launches0
        durs = [a.elapsed_time(b) for a, b in ev]
        e2e = None
        if "e2e_step" in wl:
            torch.cuda.synchronize()
            e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                    for _ in range(args.steps)]
            for i in range(args.steps):
                flush.zero_()
                e_ev[i][0].record(stream)
                wl["e2e_step"]()
                e_ev[i][1].record(stream)
            torch.cuda.synchronize()
            e2e_ms = statistics.mean(a.elapsed_time(b) for a, b in e_ev)
            e2e = e2e_ms
    ms = statistics.mean(durs)
    t = torch.tensor([ms, e2e or 0.0], device="cuda", dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms, e2e_ms = float(t[0]), float(t[1])
    sweep = allreduce_sweep(fb, be, world, stream) if (args.workload == "allreduce" and world > 1 and args.sweep) else None
    if rank != 0:
        return
    agg = world if wl.get("aggregate", True) else 1
    value = agg * wl["units"] / (ms * 1e-3) / wl["scale"]
    pk = peaks()
    if wl["bound"] == "latency":
        achieved = wl["flops"] / (ms * 1e-3) / 1e12
        roof = {"bound": "latency", "achieved": round(achieved, 4), "peak": None, "unit": "TOPS", "frac": None,
                "traffic": None, "peak_src": "launch/latency bound (13 M int-ops per forward)"}
    elif wl["bound"] == "nvlink":
        achieved = wl["units"] / (ms * 1e-3) / 1e9
        roof = {"bound": "nvlink", "achieved": round(achieved, 1), "peak": 770.0, "unit": "GB/s",
                "frac": round(achieved / 770.0, 3), "traffic": None,
                "peak_src": "measured peer copy 770 GB/s per direction (pool figure)"}
    elif wl["bound"] == "hbm":
        achieved = wl["units"] / (ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / pk["hbm_gbs"], 3), "traffic": None, "peak_src": pk["src"] + " copy"}
    else:
        flops = wl.get("flops", wl["units"])
        achieved = flops / (ms * 1e-3) / 1e12
        if wl.get("dtype") == "i8":
            peak, src = 2 * pk["bf16_tflops"], f"2x {pk['src']} bf16 cuBLAS burst (dense int8 rate = 2x bf16)"
        else:
            peak, src = pk["bf16_tflops"], f"{pk['src']} bf16 cuBLAS burst"
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(achieved / peak, 3), "traffic": None, "peak_src": src}
    tr = TRAFFIC.get(wl["workload"])
    if tr:
        roof["traffic"], roof["traffic_unit"], roof["traffic_src"] = tr[0], "bytes per launch (ncu)", tr[1]
    line = {"metric": wl["metric"], "value": round(value, 2), "unit": wl["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": wl.get("scaling", "weak"), "vs_baseline": None, "dtype": wl["dtype"],
            "data": "synthetic (seeded)",
            "config": {"workload": wl["workload"], **wl["config"], "l2": "flushed (256 MiB write) between steps",
                       "parallelism": (f"chip axis x{world} (NCCL)" if wl["bound"] == "nvlink" else
                                       f"tensor-parallel x{world} (NCCL)" if wl.get("scaling") == "strong" else
                                       f"replicas x{world}") if world > 1 else "1 GPU",
                       "host_cpus": numa},
            "roofline": roof, "gpu_launches": launches, "clocks": clk.summary(),
            "wall_s": round(wall, 4)}
    if e2e_ms:
        line["e2e"] = {"value": round(world * wl["units"] / (e2e_ms * 1e-3) / wl["scale"], 2), "unit": wl["unit"],
                       "h2d_bytes_per_step": wl["h2d"], "d2h_bytes_per_step": wl["d2h"],
                       "ms_per_step": round(e2e_ms, 4), "api": wl.get("e2e_api", "")}
    if args.workload == "allreduce" and world > 1 and args.sweep:
        line["sweep"] = sweep
    if "cpu" in wl and world == 1 and not args.no_cpu:
        rate, sample = wl["cpu"](args.cpu_rows)
        line["cpu_baseline"] = {"value": round(rate / wl["scale"], 4), "unit": wl["unit"],
                                "cores": os.cpu_count(), "kind": "port", "sample": sample}
    print(json.dumps(line), flush=True)


def run_reference(args, rank, world):
    """The reference algorithm on the host cores (the oracle port of BufStorage::contraction_in)."""
    if rank != 0:
        return
    fb = _pkg()
    M = N = K = 4096
    rng = np.random.default_rng(42)
    a = rng.integers(-128, 128, M * K, dtype=np.int64).astype(np.int8)
    b = rng.integers(-128, 128, N * K, dtype=np.int64).astype(np.int8)
    scale = rng.uniform(0.001, 0.01, N).astype(np.float32)
    rates = []
    for i in range(args.warmup + args.steps):
        rate, sample = cpu_gemm(a, b, scale, "i8", M, N, K, args.cpu_rows)
        if i >= args.warmup:
            rates.append(rate)
    v = statistics.mean(rates) / 1e12
    line = {"impl": "reference", "metric": "int8 GEMM TOPS (M=N=K=4096)", "value": round(v, 5), "unit": "TOPS",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "i8", "data": "synthetic (seeded)",
            "config": {"workload": "gemm_i8_4096x4096x4096", "M": M, "N": N, "K": K},
            "cpu_baseline": {"value": round(v, 5), "unit": "TOPS", "cores": os.cpu_count(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(v, 5), "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="gemm_i8")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-rows", type=int, default=512)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--sweep", action="store_true", help="allreduce: add the 1 KiB - 1 GiB size sweep")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import torch

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl")
    run_ours(args, rank, world, local)
    if world > 1:
        import torch

        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
