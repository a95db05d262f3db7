"""The BASELINE configs as op sequences through the `B200` backend (every op is one or more of the
`Backend` value ops, as the reference's engine stages issue them).

* `mnist_int8_forward` -- config 1: the MNIST-shaped int8 MLP of the reference's mnist example
  (furiosa-opt-examples/src/mnist/mod.rs:181-192: fc1 matmul -> requant / ReLU -> fc2 matmul -> host
  argmax), with int8 weights and activations and i32 accumulation.
* `DecoderBlockW8A8` -- config 4: a Llama-3-8B-shaped decoder block with int8 weights (per-channel
  scales) and int8 activations (per-token scales): RMSNorm -> QKV -> causal GQA attention -> O-proj
  -> residual -> RMSNorm -> gate/up -> SwiGLU -> down -> residual. The norm, quantisation and
  activation steps are vector-engine ops (map / zip / reduce / broadcast relayout); the projections
  are contractions with the fused dequant epilogue; attention is the fused kernel. Rotary position
  embedding is not part of the config and is omitted.
"""
from __future__ import annotations

import os

import numpy as np

from . import dtypes, ops
from ._lib import FOPT_ERR_UNSUPPORTED, FoptError
from .backend import B200, Mapping, Storage


# ---------------------------------------------------------------------------------------------
# config 1
# ---------------------------------------------------------------------------------------------
def mnist_int8_forward(be: B200, x: Storage, w1: Storage, w2: Storage, s1: Storage, B: int, I: int, H: int,
                       O: int) -> Storage:
    """x [B, I] i8, w1 [H, I] i8, w2 [O, H] i8, s1 [H] f32 (per-tensor scale, broadcast along H).
    Returns the i32 logits [B, O]; the caller takes the argmax on the host, as mnist_tests.rs:40-52."""
    ax = dict(B=B, I=I, H=H, O=O)
    m = lambda e: Mapping(e, ax)
    # fc1 + requant + ReLU (Clip to [0, 127]) fused into the contraction's epilogue
    h = be.contraction_requant(x, w1, m("[B, I]"), m("[H, I]"), m("[B, H, I]"), m("[B, H]"), s1, "H", lo=0, hi=127)
    return be.contraction_wide(h, w2, m("[B, H]"), m("[O, H]"), m("[B, O, H]"), m("[B, O]"))


def mnist_inputs(seed: int = 0, B: int = 64, I: int = 784, H: int = 128, O: int = 10):
    """Config 1 inputs: x ~ U[0,1) quantised to i8 (scale 1/127), weights U[-127, 127] from a seed."""
    rng = np.random.default_rng(seed)
    x = np.rint(rng.random((B, I), dtype=np.float32) * 127).astype(np.int8)
    w1 = rng.integers(-127, 128, (H, I)).astype(np.int8)
    w2 = rng.integers(-127, 128, (O, H)).astype(np.int8)
    s1 = np.full(H, 2.0 ** -12, np.float32)
    return x, w1, w2, s1


def _prog_bias(relu: bool):
    # bf16 matmul + bf16 bias in f32 (ClipBinaryOpF32::Add), optional Max 0, narrowed to bf16
    p = ops.Prog(2)
    y = p.emit("ADDF", p.emit("BF16_TO_F32", 0), p.emit("BF16_TO_F32", 1))
    if relu:
        y = p.emit("MAXF", y, p.const_f32(0.0))
    return p.build(p.emit("F32_TO_BF16", y))


MNIST_BF16_AXES = dict(X=800, H=256, C=16)


def mnist_bf16_forward(be: B200, x: Storage, w1: Storage, b1: Storage, w2: Storage, b2: Storage) -> Storage:
    """The reference's own bf16 MNIST forward (furiosa-opt-examples/src/mnist/mod.rs:1-192), one
    image: fc1 contraction (bf16 x bf16, f32 accumulation, narrowed to bf16: `fc1_matmul`), bias add
    and ReLU in f32 narrowed to bf16 (`fc1_relu`), fc2 contraction and bias add (`fc2`). Shapes
    x [X=800], w1 [H=256, X], b1 [H], w2 [C=16, H], b2 [C]; returns the bf16 logits [C]."""
    m = lambda e: Mapping(e, MNIST_BF16_AXES)
    h = be._contract(w1, x, m("[H, X]"), m("[X]"), m("[H, X]"), m("[H]"), "bf16")
    h = be.zip_with(h, b1, _prog_bias(True), "bf16")
    o = be._contract(w2, h, m("[C, H]"), m("[H]"), m("[C, H]"), m("[C]"), "bf16")
    return be.zip_with(o, b2, _prog_bias(False), "bf16")


# ---------------------------------------------------------------------------------------------
# config 4
# ---------------------------------------------------------------------------------------------
RMS_EPS = 1e-5


def _prog_rinv(hidden: int):
    # rinv = 1 / sqrt(ss / hidden + eps)
    p = ops.Prog(1)
    y = p.emit("MULF", 0, p.const_f32(1.0 / hidden))
    y = p.emit("ADDF", y, p.const_f32(RMS_EPS))
    y = p.emit("SQRT", y)
    y = p.emit("DIVF", p.const_f32(1.0), y)
    return p.build(y)


def _prog_scale3():
    p = ops.Prog(3)  # x * rinv * g
    return p.build(p.emit("MULF", p.emit("MULF", 0, 1), 2))


def _prog_abs():
    p = ops.Prog(1)
    return p.build(p.emit("AND", 0, p.const_i32(0x7FFFFFFF)))


def _prog_token_scale():
    # s = max(amax, tiny) / 127
    p = ops.Prog(1)
    y = p.emit("MAXF", 0, p.const_f32(1e-12))
    return p.build(p.emit("DIVF", y, p.const_f32(127.0)))


def _prog_quant():
    # q = Clip(FpToFxp(x / s, 31), -127, 127) -> i8
    p = ops.Prog(2)
    y = p.emit("DIVF", 0, 1)
    q = p.emit("FP_TO_FXP", y, imm=31)
    q = p.emit("MAXI", q, p.const_i32(-127))
    return p.build(p.emit("MINI", q, p.const_i32(127)))


def _prog_residual():
    # bf16 + bf16 -> bf16 (f32 add, RNE narrow)
    p = ops.Prog(2)
    return p.build(p.emit("F32_TO_BF16", p.emit("ADDF", 0, 1)))


def _prog_swiglu():
    # silu(g) * u = g * sigmoid(g) * u, in f32
    p = ops.Prog(2)
    s = p.emit("SIGMOID", 0)
    return p.build(p.emit("MULF", p.emit("MULF", 0, s), 1))


class DecoderBlockW8A8:
    """Weights: int8 [N, K] (K-major) with f32 per-channel scales; RMSNorm gains f32."""

    # Gate / up / SwiGLU as one GEMM with the activation in its epilogue (`B200.contraction_swiglu`,
    # bit-identical): off by default. At 8 x 512 tokens its epilogue (an exp and a correctly rounded
    # reciprocal per element) outlasts each tile's MMAs: 405 us against 344 us for the two
    # projections, which the smaller row program (105 against 160 us) only offsets.
    SWIGLU_EPILOGUE = bool(os.environ.get("FOPT_SWIGLU_EPILOGUE"))

    def __init__(self, be: B200, T: int, H: int, Hq: int, Hkv: int, F: int, batch: int, seq: int, seed: int = 0):
        assert T == batch * seq and H == Hq * 128
        self.be, self.T, self.H, self.Hq, self.Hkv, self.F = be, T, H, Hq, Hkv, F
        self.batch, self.seq = batch, seq
        # residual adds in the O and down projections' epilogues (off: separate elementwise ops)
        self.fuse_residual = not os.environ.get("FOPT_NO_RESIDUAL_EPILOGUE")
        self.KV = Hkv * 128
        rng = np.random.default_rng(seed)
        self.ax = dict(T=T, H=H, Q=H, V=self.KV, F=F)
        self.host = {}

        def wt(name, n, k):
            w = rng.integers(-127, 128, (n, k)).astype(np.int8)
            s = (rng.uniform(0.5, 1.5, n) / (127.0 * np.sqrt(k))).astype(np.float32)
            self.host[name] = (w, s)
            return be.from_buf(self.m(f"[{self._ax_n(n)}, {self._ax_k(k)}]"), w.tobytes(), "i8"), \
                be.from_vec(self.m(f"[{self._ax_n(n)}]"), s, "f32")

        self.wq, self.sq = wt("wq", H, H)
        self.wk, self.sk = wt("wk", self.KV, H)
        self.wv, self.sv = wt("wv", self.KV, H)
        self.wo, self.so = wt("wo", H, H)
        self.wg, self.sg = wt("wg", F, H)
        self.wu, self.su = wt("wu", F, H)
        self.wd, self.sd = wt("wd", H, F)
        # gate and up interleaved in groups of 128 channels for the fused SwiGLU projection
        self.fuse_swiglu = self.SWIGLU_EPILOGUE and F % 128 == 0
        if self.fuse_swiglu:
            (wg, sg), (wu, su) = self.host["wg"], self.host["wu"]
            wgu = np.stack([wg.reshape(F // 128, 128, H), wu.reshape(F // 128, 128, H)], 1).reshape(2 * F, H)
            sgu = np.stack([sg.reshape(F // 128, 128), su.reshape(F // 128, 128)], 1).reshape(2 * F)
            self.ax["G"] = 2 * F
            self.wgu = be.from_buf(self.m("[G, H]"), np.ascontiguousarray(wgu).tobytes(), "i8")
            self.sgu = be.from_vec(self.m("[G]"), sgu.astype(np.float32), "f32")
        g1 = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        g2 = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        self.host["g1"], self.host["g2"] = g1, g2
        # the gains broadcast over tokens once, at load time
        self.g1 = be.relayout(be.from_vec(self.m("[H]"), g1, "f32"), self.m("[H]"), self.m("[T, H]"), True)
        self.g2 = be.relayout(be.from_vec(self.m("[H]"), g2, "f32"), self.m("[H]"), self.m("[T, H]"), True)
        self.p_rinv_h = _prog_rinv(H)
        self.p_rinv_f = _prog_rinv(F)

    # axis naming: H (hidden) doubles as the K of the projections; V the kv width; F the FFN width
    def _ax_n(self, n):
        return {self.H: "Q", self.KV: "V", self.F: "F"}[n]

    def _ax_k(self, k):
        return {self.H: "H", self.F: "F"}[k]

    def m(self, e: str) -> Mapping:
        # parsed once per expression and axis table (a forward asks for the same few dozen)
        cache = self.__dict__.setdefault("_mappings", {})
        key = (e, tuple(sorted(self.ax.items())))
        if key not in cache:
            cache[key] = Mapping(e, self.ax)
        return cache[key]

    # ---- vector-engine steps ----
    def rmsnorm(self, x_f32: Storage, g: Storage) -> Storage:
        be, m = self.be, self.m
        sq = be.zip_with(x_f32, x_f32, ops.fp_binary("MulF"), "f32")
        ss = be.reduce(sq, "Add", 0.0, m("[T, H]"), m("[T]"))
        rinv = be.map(ss, self.p_rinv_h, "f32")
        rb = be.relayout(rinv, m("[T]"), m("[T, H]"), allow_broadcast=True)
        return be.zip3_with(x_f32, rb, g, _prog_scale3(), "f32")

    def quantize(self, x_f32: Storage, width: str, amax_hook=None):
        """Per-token symmetric int8: s[t] = max|x[t, :]| / 127, q = Clip(round(x / s), -127, 127).
        amax_hook (tensor parallelism): folds the per-token maxima of this rank's columns across ranks."""
        be, m = self.be, self.m
        a = be.map(x_f32, _prog_abs(), "f32")
        amax = be.reduce(a, "Max", 0.0, m(f"[T, {width}]"), m("[T]"))
        if amax_hook is not None:
            amax_hook(amax)
        s = be.map(amax, _prog_token_scale(), "f32")
        sb = be.relayout(s, m("[T]"), m(f"[T, {width}]"), allow_broadcast=True)
        q = be.zip_with(x_f32, sb, _prog_quant(), "i8")
        return q, s

    def proj(self, q: Storage, s_tok: Storage, w: Storage, s_w: Storage, k_ax: str, n_ax: str,
             residual: Storage = None) -> Storage:
        m = self.m
        return self.be.contraction_dequant(q, w, m(f"[T, {k_ax}]"), m(f"[{n_ax}, {k_ax}]"), m(f"[T, {n_ax}, {k_ax}]"),
                                           m(f"[T, {n_ax}]"), s_tok, s_w, n_ax, residual=residual)

    def proj_residual(self, q, s_tok, w, s_w, k_ax, n_ax, x):
        """x + proj(...), the residual add in the projection's epilogue when `fuse_residual`."""
        if self.fuse_residual:
            try:
                return self.proj(q, s_tok, w, s_w, k_ax, n_ax, residual=x)
            except FoptError as e:
                if e.status != FOPT_ERR_UNSUPPORTED:
                    raise
                self.fuse_residual = False
        return self.be.zip_with(x, self.proj(q, s_tok, w, s_w, k_ax, n_ax), _prog_residual(), "bf16")

    def forward(self, x: Storage) -> Storage:
        """x: bf16 [T, H] -> bf16 [T, H]."""
        be = self.be
        xf = be.map(x, ops.cast("bf16", "f32"), "f32")
        q, s = self.quantize(self.rmsnorm(xf, self.g1), "H")
        Q = self.proj(q, s, self.wq, self.sq, "H", "Q")
        K = self.proj(q, s, self.wk, self.sk, "H", "V")
        V = self.proj(q, s, self.wv, self.sv, "H", "V")
        att = be.attention(Q, K, V, self.batch, self.seq, self.Hq, self.Hkv, 128, causal=True)
        qa, sa = self.quantize(be.map(att, ops.cast("bf16", "f32"), "f32"), "H")
        h1 = self.proj_residual(qa, sa, self.wo, self.so, "H", "Q", x)
        h1f = be.map(h1, ops.cast("bf16", "f32"), "f32")
        q2, s2 = self.quantize(self.rmsnorm(h1f, self.g2), "H")
        act = None
        if self.fuse_swiglu:
            m = self.m
            try:
                act = be.contraction_swiglu(q2, self.wgu, m("[T, H]"), m("[G, H]"), m("[T, G, H]"), m("[T, G]"), s2,
                                            self.sgu, "G")
            except FoptError as e:
                if e.status != FOPT_ERR_UNSUPPORTED:
                    raise
                self.fuse_swiglu = False
        if act is None:
            g = self.proj(q2, s2, self.wg, self.sg, "H", "F")
            u = self.proj(q2, s2, self.wu, self.su, "H", "F")
            act = be.zip_with(g, u, _prog_swiglu(), "f32")
        q3, s3 = self.quantize(act, "F")
        return self.proj_residual(q3, s3, self.wd, self.sd, "F", "Q", h1)

    def gemm_ops(self) -> float:
        """Algorithmic int8 ops of the block's projections."""
        T, H, KV, F = self.T, self.H, self.KV, self.F
        return 2.0 * T * H * (H + 2 * KV + H + 3 * F)

    def attention_flops(self) -> float:
        return 4.0 * self.seq * self.seq * 128 * self.Hq / 2 * self.batch


def _prog_dequant():
    # FxpToFp(31) -> MulF(row scale) -> MulF(column scale) -> bf16: the dequant epilogue's order
    p = ops.Prog(3)
    y = p.emit("FXP_TO_FP", 0, imm=31)
    y = p.emit("MULF", p.emit("MULF", y, 1), 2)
    return p.build(p.emit("F32_TO_BF16", y))


class DecoderBlockW8A8TP(DecoderBlockW8A8):
    """The config-4 block tensor-parallel over `world` GPUs (one process each, NCCL communicator
    already initialised on `be`): query / kv heads and FFN columns split across ranks
    (column-parallel Q, K, V, gate, up; row-parallel O and down). Weights are the single-GPU block's
    (same seed) and each rank keeps its shard. The row-parallel projections sum their i32
    accumulators across ranks before the dequant (exact), and the per-token quantisation scales of
    the sharded activations take the maximum across ranks (exact), so the output is bit-identical to
    the single-GPU block's."""

    SWIGLU_EPILOGUE = False  # its gate / up are column-parallel slices

    def __init__(self, be: B200, T, H, Hq, Hkv, F, batch, seq, rank: int, world: int, seed: int = 0):
        if Hq % world or Hkv % world or F % world:
            raise ValueError("heads and FFN width must split evenly across ranks")
        super().__init__(be, T, H, Hq, Hkv, F, batch, seq, seed=seed)
        from . import dist
        self.dist, self.rank, self.world = dist, rank, world
        self.Hq_l, self.Hkv_l, self.F_l = Hq // world, Hkv // world, F // world
        Ql, KVl = self.Hq_l * 128, self.Hkv_l * 128
        self.ax.update(QL=Ql, VL=KVl, FL=self.F_l)
        h = self.host
        rows = lambda w, n: w[rank * n:(rank + 1) * n]  # noqa: E731
        cols = lambda w, n: np.ascontiguousarray(w[:, rank * n:(rank + 1) * n])  # noqa: E731
        up = lambda e, a, dt: be.from_buf(self.m(e), np.ascontiguousarray(a).tobytes(), dt)  # noqa: E731
        self.wq, self.sq = up("[QL, H]", rows(h["wq"][0], Ql), "i8"), up("[QL]", rows(h["wq"][1], Ql), "f32")
        self.wk, self.sk = up("[VL, H]", rows(h["wk"][0], KVl), "i8"), up("[VL]", rows(h["wk"][1], KVl), "f32")
        self.wv, self.sv = up("[VL, H]", rows(h["wv"][0], KVl), "i8"), up("[VL]", rows(h["wv"][1], KVl), "f32")
        self.wg, self.sg = up("[FL, H]", rows(h["wg"][0], self.F_l), "i8"), up("[FL]", rows(h["wg"][1], self.F_l), "f32")
        self.wu, self.su = up("[FL, H]", rows(h["wu"][0], self.F_l), "i8"), up("[FL]", rows(h["wu"][1], self.F_l), "f32")
        self.wo = up("[Q, QL]", cols(h["wo"][0], Ql), "i8")
        self.wd = up("[Q, FL]", cols(h["wd"][0], self.F_l), "i8")

    def _amax_across(self, amax: Storage) -> None:
        self.dist.allreduce(self.be, amax, "Max")

    def _row_parallel(self, q: Storage, s_tok: Storage, w: Storage, s_w: Storage, k_ax: str) -> Storage:
        be, m = self.be, self.m
        acc = be.contraction_wide(q, w, m(f"[T, {k_ax}]"), m(f"[Q, {k_ax}]"), m(f"[T, Q, {k_ax}]"), m("[T, Q]"))
        self.dist.allreduce(be, acc)  # i32 sums: exact
        rs = be.relayout(s_tok, m("[T]"), m("[T, Q]"), allow_broadcast=True)
        cs = be.relayout(s_w, m("[Q]"), m("[T, Q]"), allow_broadcast=True)
        return be.zip3_with(acc, rs, cs, _prog_dequant(), "bf16")

    def forward(self, x: Storage) -> Storage:
        be = self.be
        xf = be.map(x, ops.cast("bf16", "f32"), "f32")
        q, s = self.quantize(self.rmsnorm(xf, self.g1), "H")
        Q = self.proj(q, s, self.wq, self.sq, "H", "QL")
        K = self.proj(q, s, self.wk, self.sk, "H", "VL")
        V = self.proj(q, s, self.wv, self.sv, "H", "VL")
        att = be.attention(Q, K, V, self.batch, self.seq, self.Hq_l, self.Hkv_l, 128, causal=True)
        qa, sa = self.quantize(be.map(att, ops.cast("bf16", "f32"), "f32"), "QL", amax_hook=self._amax_across)
        o = self._row_parallel(qa, sa, self.wo, self.so, "QL")
        h1 = be.zip_with(x, o, _prog_residual(), "bf16")
        h1f = be.map(h1, ops.cast("bf16", "f32"), "f32")
        q2, s2 = self.quantize(self.rmsnorm(h1f, self.g2), "H")
        g = self.proj(q2, s2, self.wg, self.sg, "H", "FL")
        u = self.proj(q2, s2, self.wu, self.su, "H", "FL")
        act = be.zip_with(g, u, _prog_swiglu(), "f32")
        q3, s3 = self.quantize(act, "FL", amax_hook=self._amax_across)
        d = self._row_parallel(q3, s3, self.wd, self.sd, "FL")
        return be.zip_with(h1, d, _prog_residual(), "bf16")
