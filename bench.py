"""Benchmark: the furiosa-opt emulator hot path on B200.

Default (headline) workload: config 2, the standalone int8 contraction M=N=K=4096 (i32 accumulate,
per-channel fp32 requant to i8), one step = one `contraction` call through the backend. The default
run also measures the other configs, each as a sub-object of the one JSON line (`configs`): at one
GPU the bf16 GEMM, config 3 attention, config 4 decoder block, config 1 MNIST MLP and the layout
move, each with its roofline and its CPU-port baseline; at N > 1 GPUs config 5's all-reduce (bus
bandwidth at 128 MiB plus a 1 KiB - 1 GiB sweep, against the peer-to-peer bandwidth measured in the
same run) and a bit-exact self-check of the all-reduce and the chip shuffle. `--headline-only`
skips them.
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
    "relayout_bf16_8192x8192": (217.9e6, "profiles/relayout_tile_h_bf16_8192.md"),
    "relayout_padded_f32": (504.2e6, "profiles/relayout_pad_rows_f32.md"),
    "elementwise_f32_zip": (772.1e6, "profiles/fopt_ew_gen_zip_f32.md"),
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
                cpu=lambda rows, keep=None: cpu_gemm(a, b, scale, dtype, M, N, K, rows, keep),
                parity=lambda rows, cpu_bytes: gemm_parity(OUT, cpu_bytes, dtype, rows, N),
                config={"M": M, "N": N, "K": K, "layout": "lhs [M, K], rhs [N, K], out [M, N]",
                        "cuda_graph": not os.environ.get("FOPT_NO_GRAPH")})


def cpu_gemm(a, b, scale, dtype, M, N, K, rows, keep=None):
    """The oracle port's per-cell fold over the first `rows` output rows at full K (only the fold is
    timed: the read plans stand for the reference's sequence() setup). `keep` (a dict) receives the
    sample's output bytes, which the GPU result is compared with."""
    import oracle
    from oracle import ref_m

    ax = dict(M=M, N=N, K=K)
    rl, rr, rp, ro = (ref_m(e, **ax) for e in ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]"))
    if dtype == "i8":
        out = oracle.contract(a.tobytes(), b.tobytes(), "i8", "i8", rl, rr, rp, ro, ep_kind=1, scale=scale,
                              scale_axis="N", out_cells=rows * N)
    else:
        out = oracle.contract(a.tobytes(), b.tobytes(), "bf16", "bf16", rl, rr, rp, ro, out_cells=rows * N)
    dt = oracle.last_fold_seconds
    if keep is not None:
        keep["bytes"] = out
    return 2.0 * rows * N * K / dt, f"{rows} of {M} output rows ({rows * N} cells, full K={K})"


def gemm_parity(out_storage, cpu_bytes, dtype, rows, N):
    """The GPU's first `rows` output rows against the CPU port's bytes for the same rows."""
    esz = 1 if dtype == "i8" else 2
    got = out_storage.to_bytes()[: rows * N * esz]
    if dtype == "i8":
        same = got == cpu_bytes
        return {"check": f"first {rows} of the output rows against the CPU port", "bit_exact": same,
                "result": "bit-exact" if same else "DIFFERS"}
    import numpy as np_

    g = (np_.frombuffer(got, np_.uint16).astype(np_.uint32) << 16).view(np_.float32)
    w = (np_.frombuffer(cpu_bytes, np_.uint16).astype(np_.uint32) << 16).view(np_.float32)
    err = np_.abs(g - w)
    ok = bool(np_.all(err <= 2 ** -7 * np_.abs(w) + 1e-3 * np_.abs(w).max()))
    return {"check": f"first {rows} output rows against the CPU port (tensor-core sum order)",
            "max_abs_err": float(err.max()), "max_abs_out": float(np_.abs(w).max()),
            "result": "within 1 bf16 ulp + 1e-3 max|out|" if ok else "OUT OF TOLERANCE"}


def wl_attention(fb, be, S=2048, Hq=32, Hkv=8, D=128):
    rng = np.random.default_rng(42)
    q = fb.dtypes.f32_to_bf16_bits(rng.standard_normal(S * Hq * D).astype(np.float32))
    k = fb.dtypes.f32_to_bf16_bits(rng.standard_normal(S * Hkv * D).astype(np.float32))
    v = fb.dtypes.f32_to_bf16_bits(rng.standard_normal(S * Hkv * D).astype(np.float32))
    mq = fb.Mapping("[S, H, D]", dict(S=S, H=Hq, D=D))
    mk = fb.Mapping("[S, H, D]", dict(S=S, H=Hkv, D=D))
    Q, Kt, V = be.from_vec(mq, q, "bf16"), be.from_vec(mk, k, "bf16"), be.from_vec(mk, v, "bf16")
    OUT = be.zeroed(mq, "bf16")

    def issue():
        return be.attention(Q, Kt, V, 1, S, Hq, Hkv, D, causal=True, out=OUT)

    # captured once and replayed like the other steps: the timed region holds the kernels, not the
    # host's tensor-map encoding (FOPT_NO_GRAPH=1 issues every step from the host)
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

    flops = 4.0 * S * S * D * Hq / 2  # causal half

    def cpu(_rows=None, keep=None):
        import oracle

        q1 = q.reshape(S, Hq, D)[:, 0].copy()
        k1, v1 = k.reshape(S, Hkv, D)[:, 0].copy(), v.reshape(S, Hkv, D)[:, 0].copy()
        t0 = time.perf_counter()
        oracle.attention_chain(q1, k1, v1, 1, S, 1, 1, D, True)
        dt = time.perf_counter() - t0
        return S / (dt * Hq), f"the reference's attention op chain for 1 of {Hq} query heads (S={S}, causal)"

    return dict(step=step, units=S, unit="tokens/s", scale=1.0, flops=flops, bound="tensor", cpu=cpu,
                metric="attention prefill tokens/s (Llama-3-8B shape, S=2048, causal)", workload="attention_s2048",
                dtype="bf16", config={"S": S, "Hq": Hq, "Hkv": Hkv, "D": D, "causal": True,
                                      "cuda_graph": not os.environ.get("FOPT_NO_GRAPH")})


def graph_step(be, issue):
    """A step that runs `issue` once eagerly (plans built, kernels compiled), then captures it as a
    CUDA graph and replays that: the timed region holds the kernels, not the host's work of issuing
    them (FOPT_NO_GRAPH=1 issues every step from the host)."""
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

    return step


def wl_relayout(fb, be, R=8192, C=8192):
    rng = np.random.default_rng(1)
    ax = dict(R=R, C=C)
    S, D = fb.Mapping("[R, C]", ax), fb.Mapping("[C, R]", ax)
    x = fb.dtypes.f32_to_bf16_bits(rng.standard_normal(R * C).astype(np.float32))
    X = be.from_vec(S, x, "bf16")
    Y = be.zeroed(D, "bf16")

    def issue():
        be.transpose(Y, X, S, D)
        return Y

    step = graph_step(be, issue)

    def cpu(_rows=None, keep=None):
        # the oracle's BufStorage::transpose copy loop (OpenMP over destination positions) on a
        # 2048 x 2048 corner of the same layout; only the copy loop is timed
        import oracle
        from oracle import ref_m

        r = c = 2048
        xs = x.reshape(R, C)[:r, :c].copy()
        oracle.transpose(bytes(r * c * 2), xs.tobytes(), "bf16", ref_m("[R, C]", R=r, C=c), ref_m("[C, R]", R=r, C=c))
        dt = oracle.last_transpose_seconds
        return 2.0 * r * c * 2 / dt, f"the port's transpose loop on a {r} x {c} bf16 tile of the same layout"

    def parity(_rows=None, _b=None):
        y = np.frombuffer(Y.to_bytes(), np.uint16).reshape(C, R)
        same = bool(np.array_equal(y, x.reshape(R, C).T))
        return {"check": "whole output against numpy's transpose", "bit_exact": same,
                "result": "bit-exact" if same else "DIFFERS"}

    return dict(step=step, units=2.0 * R * C * 2, unit="GB/s", scale=1e9, bound="hbm", cpu=cpu, parity=parity,
                metric="relayout GB/s ([R, C] -> [C, R] bf16, 128 MiB)", workload="relayout_bf16_8192x8192",
                dtype="bf16", config={"R": R, "C": C, "cuda_graph": not os.environ.get("FOPT_NO_GRAPH")})


def wl_relayout_padded(fb, be, R=1 << 20, D=61):
    """The padded-row move [R, D] -> [R, D # 64] (f32, 244 MiB live each way): a whole-row pitch
    change whose dead cells the move must leave alone (buf.rs:257-313 skips padding)."""
    rng = np.random.default_rng(2)
    ax = dict(R=R, D=D)
    S, Dm = fb.Mapping("[R, D]", ax), fb.Mapping("[R, D # 64]", ax)
    x = rng.standard_normal(R * D).astype(np.float32)
    X = be.from_vec(S, x, "f32")
    Y = be.zeroed(Dm, "f32")

    def issue():
        be.transpose(Y, X, S, Dm)
        return Y

    step = graph_step(be, issue)

    def parity(_rows=None, _b=None):
        y = Y.to_numpy().reshape(R, 64)
        same = bool(np.array_equal(y[:, :D], x.reshape(R, D)) and not y[:, D:].any())
        return {"check": "live cells against the source, dead cells untouched", "bit_exact": same,
                "result": "bit-exact" if same else "DIFFERS"}

    live = 4.0 * R * D
    return dict(step=step, units=2.0 * live, unit="GB/s", scale=1e9, bound="hbm", parity=parity,
                cpu=lambda rows=None, keep=None: (float("nan"), "not sampled"),
                metric="padded-row relayout GB/s ([R, D] -> [R, D # 64] f32, D = 61)",
                workload="relayout_padded_f32", dtype="f32", config={"R": R, "D": D, "bytes": "live read + live write",
                                                      "cuda_graph": not os.environ.get("FOPT_NO_GRAPH")})


def wl_elementwise(fb, be, n=64 << 20, dt="f32"):
    """A generated zip program over two inputs well above L2: f32 a * b + a (64 Mi elements, 768 MiB
    moved); bf16 the same in f32 with the bf16 rounding of the result (128 Mi elements, 768 MiB);
    i8 a + b clipped to [-128, 127] (256 Mi elements, 768 MiB)."""
    rng = np.random.default_rng(3)
    m = fb.Mapping("[E]", dict(E=n))
    p_ = fb.ops.Prog(2)
    if dt == "i8":
        av, bv = (rng.integers(-128, 128, n, dtype=np.int64).astype(np.int8) for _ in range(2))
        prog = p_.build(p_.emit("MINI", p_.emit("MAXI", p_.emit("ADD_FXP", 0, 1), p_.const_i32(-128)),
                                p_.const_i32(127)))
        desc, esz = "i8 a + b clipped to [-128, 127]", 1
    else:
        av, bv = (rng.standard_normal(n).astype(np.float32) for _ in range(2))
        if dt == "bf16":
            av, bv = fb.dtypes.f32_to_bf16_bits(av), fb.dtypes.f32_to_bf16_bits(bv)
            prog = p_.build(p_.emit("F32_TO_BF16", p_.emit("ADDF", p_.emit("MULF", 0, 1), 0)))
            desc, esz = "bf16 a * b + a (f32 arithmetic, bf16 result)", 2
        else:
            prog = p_.build(p_.emit("ADDF", p_.emit("MULF", 0, 1), 0))
            desc, esz = "f32 a * b + a", 4
    a = be.from_vec(m, av, dt)
    b = be.from_vec(m, bv, dt)
    OUT = be.zeroed(m, dt)
    lib = fb._lib.lib()
    ptrs = (C.c_void_p * 2)(a.addr, b.addr)
    dts = (C.c_int32 * 2)(fb._lib.DTYPES[dt], fb._lib.DTYPES[dt])

    def issue():
        fb._lib.check(lib.fopt_elementwise(be.ctx, C.byref(prog), 2, ptrs, dts, OUT.ptr, fb._lib.DTYPES[dt], n),
                      be.ctx)
        return OUT

    step = graph_step(be, issue)

    def parity(_rows=None, _b=None):
        import oracle

        k = 1 << 16
        insns = [(prog.insn[i].op, prog.insn[i].dst, prog.insn[i].a, prog.insn[i].b, prog.insn[i].c, prog.insn[i].imm_i)
                 for i in range(prog.n_insn)]
        want = oracle.elementwise(insns, prog.ret, [np.ascontiguousarray(av[:k]).tobytes(),
                                                    np.ascontiguousarray(bv[:k]).tobytes()], [dt, dt], dt, k)
        same = OUT.to_bytes()[: esz * k] == want
        return {"check": f"first {k} elements against the oracle", "bit_exact": same,
                "result": "bit-exact" if same else "DIFFERS"}

    name = "elementwise_f32_zip" if dt == "f32" else f"elementwise_{dt}_zip"
    return dict(step=step, units=3.0 * esz * n, unit="GB/s", scale=1e9, bound="hbm", parity=parity,
                cpu=lambda rows=None, keep=None: (float("nan"), "not sampled"),
                metric=f"generated elementwise program GB/s ({desc}, {n >> 20} Mi elements)",
                workload=name, dtype=dt,
                config={"elements": n, "bytes": "2 reads + 1 write", "cuda_graph": not os.environ.get("FOPT_NO_GRAPH")})


def wl_broadcast(fb, be, A=4096, B=16384):
    """A broadcast relayout [A] -> [A, B] (i32, 256 MiB written): `transpose` with a zero-stride
    source axis (buf.rs:257-313 with allow_broadcast), materialised into a preallocated output."""
    ax = dict(A=A, B=B)
    S, D = fb.Mapping("[A]", ax), fb.Mapping("[A, B]", ax)
    x = np.random.default_rng(4).integers(-2**31, 2**31 - 1, A).astype(np.int32)
    X = be.from_vec(S, x, "i32")
    Y = be.zeroed(D, "i32")

    def issue():
        be.transpose(Y, X, S, D, allow_broadcast=True)
        return Y

    step = graph_step(be, issue)

    def parity(_rows=None, _b=None):
        y = Y.to_numpy().reshape(A, B)
        same = bool(np.array_equal(y, np.repeat(x[:, None], B, axis=1)))
        return {"check": "whole output against numpy's repeat", "bit_exact": same,
                "result": "bit-exact" if same else "DIFFERS"}

    return dict(step=step, units=4.0 * A * B + 4.0 * A, unit="GB/s", scale=1e9, bound="hbm", parity=parity,
                cpu=lambda rows=None, keep=None: (float("nan"), "not sampled"),
                metric="broadcast relayout GB/s ([A] -> [A, B] i32, 256 MiB written)", workload="broadcast_i32",
                dtype="i32", config={"A": A, "B": B, "bytes": "source read + output written",
                                     "cuda_graph": not os.environ.get("FOPT_NO_GRAPH")})


def wl_chip_layout(fb, be, A=4096, B=16384):
    """The chip-shuffle example's HBM relayout (shuffle_slice_tests.rs: [A / 4 % 4, A / 16, A % 4, B]
    -> [A / 4 % 4, B, A % 4, A / 16]), scaled from A = 256, B = 4096 to 256 MiB of i32."""
    ax = dict(A=A, B=B)
    S = fb.Mapping("[A / 4 % 4, A / 16, A % 4, B]", ax)
    D = fb.Mapping("[A / 4 % 4, B, A % 4, A / 16]", ax)
    x = np.arange(A * B, dtype=np.int64).astype(np.int32)
    X = be.from_vec(S, x, "i32")
    Y = be.zeroed(D, "i32")

    def issue():
        be.transpose(Y, X, S, D)
        return Y

    step = graph_step(be, issue)

    def parity(_rows=None, _b=None):
        # source position of (a4, a16, a1, b) is ((a4 * (A/16) + a16) * 4 + a1) * B + b; the output
        # walks (a4, b, a1, a16)
        y = Y.to_numpy().reshape(4, B, 4, A // 16)
        src = x.reshape(4, A // 16, 4, B)
        same = bool(np.array_equal(y, src.transpose(0, 3, 2, 1)))
        return {"check": "whole output against numpy's axis permutation", "bit_exact": same,
                "result": "bit-exact" if same else "DIFFERS"}

    return dict(step=step, units=2.0 * 4 * A * B, unit="GB/s", scale=1e9, bound="hbm", parity=parity,
                cpu=lambda rows=None, keep=None: (float("nan"), "not sampled"),
                metric="chip-shuffle layout relayout GB/s (i32, 256 MiB each way)", workload="relayout_chip_layout_i32",
                dtype="i32", config={"A": A, "B": B, "src": S.expr, "dst": D.expr,
                                     "cuda_graph": not os.environ.get("FOPT_NO_GRAPH")})


def wl_allreduce(fb, be, rank, world, count=8 * 2048 * 4096, comm_ready=False):
    """Config 5: all-reduce of an 8x2048x4096 bf16 activation (N(0,1) per rank) over the Chip axis."""
    if world > 1 and not comm_ready:
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

    def cpu(_rows=None, keep=None):
        # the port's two per-cell folds with the requant epilogue (the same restatement the parity
        # test pins); only the folds are timed
        import oracle
        from oracle import ref_m

        mm = lambda e: ref_m(e, **ax)  # noqa: E731
        oracle.contract(x.tobytes(), w1.tobytes(), "i8", "i8", mm("[B, I]"), mm("[H, I]"), mm("[B, H, I]"),
                        mm("[B, H]"), ep_kind=1, scale=s1, scale_axis="H", clip_lo=0, clip_hi=127)
        t = oracle.last_fold_seconds
        h = oracle.contract(x.tobytes(), w1.tobytes(), "i8", "i8", mm("[B, I]"), mm("[H, I]"), mm("[B, H, I]"),
                            mm("[B, H]"), ep_kind=1, scale=s1, scale_axis="H", clip_lo=0, clip_hi=127)
        t = min(t, oracle.last_fold_seconds)
        logits = oracle.contract(h, w2.tobytes(), "i8", "i32", mm("[B, H]"), mm("[O, H]"), mm("[B, O, H]"),
                                 mm("[B, O]"))
        t += oracle.last_fold_seconds
        if keep is not None:
            keep["bytes"] = logits
        return B / t, f"the whole forward ({B} images), both folds"

    def parity(_rows=None, cpu_bytes=None):
        got = step().to_bytes()
        same = got == cpu_bytes
        return {"check": "logits of the whole batch against the CPU port", "bit_exact": same,
                "result": "bit-exact" if same else "DIFFERS"}

    return dict(step=step, e2e_step=e2e_step, h2d=hx.numel(), d2h=hout.numel(), cpu=cpu, parity=parity,
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

    def cpu(_rows=None, keep=None):
        # the port's per-cell int8 fold (the block's projections are 99.8 % of its operations) on a
        # 16-token x 1024-channel x K=4096 piece of the gate projection, scaled to the block's
        # projection operations per token
        import oracle
        from oracle import ref_m

        t, n, k = 16, 1024, H
        ax = dict(T=t, N=n, K=k)
        mm = lambda e: ref_m(e, **ax)  # noqa: E731
        wg = blk.host["wg"][0][:n]
        xq = np.random.default_rng(2).integers(-127, 128, t * k).astype(np.int8)
        oracle.contract(xq.tobytes(), wg.tobytes(), "i8", "i32", mm("[T, K]"), mm("[N, K]"), mm("[T, N, K]"),
                        mm("[T, N]"))
        rate = 2.0 * t * n * k / oracle.last_fold_seconds
        per_token = blk.gemm_ops() / T
        return rate / per_token, (f"per-cell int8 fold of a {t} x {n} x {k} projection piece, scaled by the "
                                  f"block's {per_token / 1e6:.0f} M projection ops per token")

    return dict(step=step, e2e_step=e2e_step, h2d=hx.numel(), d2h=hout.numel(), cpu=cpu,
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


class L2Flush:
    """Between timed steps: write a 256 MiB buffer (more than the 126 MB L2), then read another
    256 MiB buffer, so that L2 holds none of the step's data and no dirty lines: without the read,
    the write-back of the flush's own last 126 MB would land inside the next timed step."""

    HOW = "flushed between steps (256 MiB written, then 256 MiB of another buffer read)"

    def __init__(self):
        import torch

        self.w = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        self.r = torch.zeros(256 << 20, dtype=torch.uint8, device="cuda")

    def __call__(self):
        self.w.zero_()
        self.r.amax()


def measure(be, wl, stream, flush, steps, warmup, world, local):
    """W untimed warm-up steps, then exactly `steps` steps, each bracketed by CUDA events on the
    library's stream with L2 flushed before it (outside the events), clocks sampled throughout; the
    end-to-end step (host buffers in and out) is timed the same way afterwards. Returns the mean
    device times, max over ranks."""
    import torch

    clk = Clocks(local).__enter__()  # sampling runs from before warm-up to the end of the timed steps
    clk.wait_first_sample()
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            wl["step"]()
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        launches0 = be.launches
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        torch.cuda.synchronize()
        wall0 = time.perf_counter()
        for i in range(steps):
            flush()
            ev[i][0].record(stream)
            wl["step"]()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - wall0
        clk.__exit__()
        launches = be.launches - launches0
        durs = [a.elapsed_time(b) for a, b in ev]
        e2e = 0.0
        if "e2e_step" in wl:
            torch.cuda.synchronize()
            e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                    for _ in range(steps)]
            for i in range(steps):
                flush()
                e_ev[i][0].record(stream)
                wl["e2e_step"]()
                e_ev[i][1].record(stream)
            torch.cuda.synchronize()
            e2e = statistics.mean(a.elapsed_time(b) for a, b in e_ev)
    t = torch.tensor([statistics.mean(durs), e2e], device="cuda", dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return {"ms": float(t[0]), "e2e_ms": float(t[1]), "launches": launches, "clocks": clk.summary(), "wall": wall}


def int8_library_peak(stream, n=8192, reps=10):
    """cuBLASLt's int8 GEMM (torch._int_mm, i32 out) at n^3 on this GPU, best of `reps`: the measured
    int8 reference the headline GEMM is also reported against."""
    import torch

    try:
        with torch.cuda.stream(stream):
            a = torch.randint(-128, 128, (n, n), dtype=torch.int8, device="cuda")
            b = torch.randint(-128, 128, (n, n), dtype=torch.int8, device="cuda").t()  # column-major K x N
            for _ in range(3):
                torch._int_mm(a, b)
            best = None
            for _ in range(reps):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                torch._int_mm(a, b)
                e1.record(stream)
                torch.cuda.synchronize()
                ms = e0.elapsed_time(e1)
                best = ms if best is None else min(best, ms)
        del a, b
        return {"tops": round(2.0 * n ** 3 / (best * 1e-3) / 1e12, 1), "how": f"torch._int_mm (cuBLASLt) {n}^3, "
                f"best of {reps}, CUDA events"}
    except Exception as e:  # an int8 GEMM the library refuses on this build: reported, not fatal
        return {"tops": None, "how": f"torch._int_mm unavailable ({type(e).__name__})"}


def roofline(wl, ms, pk, int8_peak=None):
    if wl["bound"] == "latency":
        achieved = wl["flops"] / (ms * 1e-3) / 1e12
        return {"bound": "latency", "achieved": round(achieved, 4), "peak": None, "unit": "TOPS", "frac": None,
                "traffic": None, "peak_src": "launch/latency bound (13 M int-ops per forward)"}
    if wl["bound"] == "nvlink":
        achieved = wl["units"] / (ms * 1e-3) / 1e9
        peak = wl.get("link_peak")
        return {"bound": "nvlink", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 3) if peak else None, "traffic": None,
                "peak_src": wl.get("link_peak_src", "unmeasured")}
    if wl["bound"] == "hbm":
        achieved = wl["units"] / (ms * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / pk["hbm_gbs"], 3), "traffic": None, "peak_src": pk["src"] + " copy"}
    flops = wl.get("flops", wl["units"])
    achieved = flops / (ms * 1e-3) / 1e12
    if wl.get("dtype") == "i8":
        peak, src = 2 * pk["bf16_tflops"], f"2x {pk['src']} bf16 cuBLAS burst (dense int8 rate = 2x bf16)"
    else:
        peak, src = pk["bf16_tflops"], f"{pk['src']} bf16 cuBLAS burst"
    roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
            "frac": round(achieved / peak, 3), "traffic": None, "peak_src": src}
    if wl.get("dtype") == "i8" and int8_peak and int8_peak.get("tops"):
        roof["int8_library_peak"] = int8_peak["tops"]
        roof["frac_of_int8_library"] = round(achieved / int8_peak["tops"], 3)
        roof["int8_library_how"] = int8_peak["how"]
    return roof


def report(wl, meas, world, pk, args, int8_peak=None, cpu=True):
    """The JSON object for one workload: value, roofline, clocks, e2e, CPU baseline, parity."""
    ms, e2e_ms = meas["ms"], meas["e2e_ms"]
    agg = world if wl.get("aggregate", True) else 1
    roof = roofline(wl, ms, pk, int8_peak)
    tr = TRAFFIC.get(wl["workload"])
    if tr:
        roof["traffic"], roof["traffic_unit"], roof["traffic_src"] = tr[0], "bytes per launch (ncu)", tr[1]
    out = {"metric": wl["metric"], "value": round(agg * wl["units"] / (ms * 1e-3) / wl["scale"], 2),
           "unit": wl["unit"], "ms_per_step": round(ms, 4), "dtype": wl["dtype"],
           "config": {"workload": wl["workload"], **wl["config"]}, "roofline": roof,
           "gpu_launches": meas["launches"], "clocks": meas["clocks"], "wall_s": round(meas["wall"], 4)}
    if e2e_ms:
        out["e2e"] = {"value": round(world * wl["units"] / (e2e_ms * 1e-3) / wl["scale"], 2), "unit": wl["unit"],
                      "h2d_bytes_per_step": wl["h2d"], "d2h_bytes_per_step": wl["d2h"],
                      "ms_per_step": round(e2e_ms, 4), "api": wl.get("e2e_api", "")}
    keep = {}
    if "cpu" in wl and world == 1 and cpu and not args.no_cpu:
        rate, sample = wl["cpu"](args.cpu_rows, keep)
        if rate == rate:  # a sampled CPU baseline (NaN: none for this workload)
            out["cpu_baseline"] = {"value": round(rate / wl["scale"], 6), "unit": wl["unit"],
                                   "cores": os.cpu_count(), "kind": "port", "sample": sample}
    if "parity" in wl and cpu and not args.no_cpu and (
            "bytes" in keep or wl["workload"].startswith(("relayout", "elementwise", "broadcast"))):
        out["parity"] = wl["parity"](args.cpu_rows, keep.get("bytes"))
    return out


def collective_report(fb, be, rank, world, stream, flush, args, local):
    """Config 5 at N GPUs: the all-reduce of an 8 x 2048 x 4096 bf16 activation (bus bandwidth),
    the 1 KiB - 1 GiB sweep, the peer-to-peer bandwidth each GPU reaches to its neighbour in the same
    run (the NVLink roofline's denominator), and a bit-exact self-check of the all-reduce and the
    chip shuffle (`pattern[target] = source`, memory.rs:657-679)."""
    import torch
    import torch.distributed as dist

    fb.dist.init_comm(be, rank, world)
    # peer-to-peer: every rank sends 1 GiB to rank+1 while receiving from rank-1 (NCCL send/recv)
    n = 1 << 29
    sbuf = torch.empty(n, dtype=torch.bfloat16, device="cuda").normal_()
    rbuf = torch.empty_like(sbuf)

    def ring():
        ops_ = [dist.P2POp(dist.isend, sbuf, (rank + 1) % world), dist.P2POp(dist.irecv, rbuf, (rank - 1) % world)]
        for r in dist.batch_isend_irecv(ops_):
            r.wait()

    with torch.cuda.stream(stream):
        for _ in range(2):
            ring()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(5):
            ring()
        e1.record(stream)
        torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / 5], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    p2p = 2 * n / (float(t[0]) * 1e-3) / 1e9
    del sbuf, rbuf
    # bit-exact self-check: small integers sum exactly in bf16; the shuffle moves whole slabs
    cnt = 1 << 20
    m = fb.Mapping("[E]", dict(E=cnt))
    vals = [((np.arange(cnt) * (r + 3)) % 17 - 8).astype(np.float32) for r in range(world)]
    x = be.from_vec(m, fb.dtypes.f32_to_bf16_bits(vals[rank]), "bf16")
    fb.dist.allreduce(be, x)
    ar_ok = bool(np.array_equal(fb.dtypes.bf16_bits_to_f32(x.to_numpy()), np.sum(vals, axis=0)))
    pattern = [(tt + 1) % world for tt in range(world)]
    src = be.from_vec(m, fb.dtypes.f32_to_bf16_bits(vals[rank]), "bf16")
    dst = be.zeroed(m, "bf16")
    fb.dist.chip_shuffle(be, dst, src, pattern)
    sh_ok = bool(np.array_equal(dst.to_numpy(), fb.dtypes.f32_to_bf16_bits(vals[pattern[rank]])))
    ok = torch.tensor([int(ar_ok and sh_ok)], device="cuda")
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    # the config-5 all-reduce, timed like every other step
    wl = wl_allreduce(fb, be, rank, world, comm_ready=True)
    wl["link_peak"], wl["link_peak_src"] = round(p2p, 1), ("peer-to-peer NCCL send/recv to the neighbouring rank, "
                                                           "1 GiB, measured in this run (per direction)")
    meas = measure(be, wl, stream, flush, args.steps, args.warmup, world, local)
    sweep = allreduce_sweep(fb, be, world, stream)
    if rank != 0:
        return None
    rep = report(wl, meas, world, peaks(), args, cpu=False)
    rep["self_check"] = {"allreduce_bit_exact": ar_ok, "chip_shuffle_bit_exact": sh_ok,
                         "all_ranks_ok": bool(int(ok[0]))}
    rep["sweep"] = sweep
    rep["peer_to_peer_gbs"] = round(p2p, 1)
    rep["nccl_ranks"] = world
    return rep


SUB_CONFIGS = ("gemm_bf16", "attention", "decoder", "mnist", "relayout", "relayout_padded", "relayout_chip_layout",
               "broadcast", "elementwise", "elementwise_bf16", "elementwise_i8")


def run_ours(args, rank, world, local):
    import torch

    numa = bind_to_gpu_cpus(local)
    fb = _pkg()
    torch.cuda.set_device(local)
    be = fb.B200(local)
    stream = torch.cuda.Stream()
    fb._lib.lib().fopt_set_stream(be.ctx, stream.cuda_stream)
    make = {"gemm_i8": lambda: wl_gemm(fb, be, "i8"), "gemm_bf16": lambda: wl_gemm(fb, be, "bf16"),
            "attention": lambda: wl_attention(fb, be), "relayout": lambda: wl_relayout(fb, be),
            "allreduce": lambda: wl_allreduce(fb, be, rank, world), "mnist": lambda: wl_mnist(fb, be),
            "decoder": lambda: wl_decoder(fb, be), "relayout_padded": lambda: wl_relayout_padded(fb, be),
            "elementwise": lambda: wl_elementwise(fb, be),
            "elementwise_bf16": lambda: wl_elementwise(fb, be, 128 << 20, "bf16"),
            "elementwise_i8": lambda: wl_elementwise(fb, be, 256 << 20, "i8"),
            "broadcast": lambda: wl_broadcast(fb, be), "relayout_chip_layout": lambda: wl_chip_layout(fb, be),
            "decoder_tp": lambda: wl_decoder_tp(fb, be, rank, world)}
    wl = make[args.workload]()
    flush = L2Flush()
    meas = measure(be, wl, stream, flush, args.steps, args.warmup, world, local)
    sweep = allreduce_sweep(fb, be, world, stream) if (args.workload == "allreduce" and world > 1 and args.sweep) else None
    extra = not args.headline_only and args.workload == "gemm_i8"
    int8_peak = int8_library_peak(stream) if args.workload == "gemm_i8" and rank == 0 else None
    pk = peaks()
    line = None
    if rank == 0:
        rep = report(wl, meas, world, pk, args, int8_peak)
        line = {"metric": rep["metric"], "value": rep["value"], "unit": rep["unit"], "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": rep["ms_per_step"],
                "higher_is_better": True, "scaling": wl.get("scaling", "weak"), "vs_baseline": None,
                "dtype": rep["dtype"], "data": "synthetic (seeded)",
                "config": {**rep["config"], "l2": L2Flush.HOW,
                           "parallelism": (f"chip axis x{world} (NCCL)" if wl["bound"] == "nvlink" else
                                           f"tensor-parallel x{world} (NCCL)" if wl.get("scaling") == "strong" else
                                           f"replicas x{world}") if world > 1 else "1 GPU",
                           "host_cpus": numa}}
        for k in ("roofline", "gpu_launches", "clocks", "wall_s", "e2e", "cpu_baseline", "parity"):
            if k in rep:
                line[k] = rep[k]
        if sweep is not None:
            line["sweep"] = sweep
    del wl
    if extra:
        configs = {}
        if world == 1:
            for name in SUB_CONFIGS:
                try:
                    sub = make[name]()
                    m_ = measure(be, sub, stream, flush, args.steps, args.warmup, world, local)
                    configs[name] = report(sub, m_, world, pk, args)
                    del sub
                except Exception as e:  # one failing sub-config must not hide the headline
                    configs[name] = {"error": f"{type(e).__name__}: {e}"[:300]}
        else:
            try:
                rep = collective_report(fb, be, rank, world, stream, flush, args, local)
                if rank == 0:
                    configs["allreduce"] = rep
            except Exception as e:
                configs["allreduce"] = {"error": f"{type(e).__name__}: {e}"[:300]}
        if line is not None:
            line["configs"] = configs
    if line is not None:
        emit(line)


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
    emit(line)


# The result line goes to the process's original stdout; everything else written to file
# descriptor 1 during the run (NCCL's version banner, native library prints) is sent to stderr, so
# stdout holds exactly one JSON line.
_RESULT_FD = None


def emit(line):
    data = (json.dumps(line) + "\n").encode()
    if _RESULT_FD is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
        return
    while data:
        data = data[os.write(_RESULT_FD, data):]


def main():
    global _RESULT_FD
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="gemm_i8")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-rows", type=int, default=512)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--sweep", action="store_true", help="allreduce: add the 1 KiB - 1 GiB size sweep")
    ap.add_argument("--headline-only", action="store_true", help="skip the other configs' sub-objects")
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
