"""ORACLE (test infrastructure only): CPU restatements of the config-1 and config-4 op chains.

Config 1's integer projections fold through `ref_contract` (BufStorage::contraction_in,
buf.rs:401-447) with the vector-engine epilogues. Config 4's projections sum int8 x int8 products
exactly (float64 matrix products of integers below 2^53, the same i32 sums the wire-order fold
gives, since no sum of these sizes reaches 2^31) and then run the dequant epilogue chain
(FxpToFp at int width 31 = IEEE int -> f32, MulF row scale, MulF column scale, bf16 cast); the float
steps restate the vector-engine ops in numpy float32 in the same order (semantics.rs: MulF, AddF,
DivF, Sqrt, Sigmoid; float/mod.rs float_to_fixedpoint), with the f32 row sums folded in wire
order; attention uses the f32 online softmax `ref_attention`.
"""
from __future__ import annotations

import numpy as np

from . import attention, contract, elementwise
from .mapping_ref import ref_m


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    sub = ((u >> 23) & 0xFF) == 0
    hi = (u >> 16) & 0xFFFF
    up = ((u & 0x8000) != 0) & ((u & 0x17FFF) != 0)
    out = np.where(nan, 0x7FC0, np.where(sub, hi & 0x8000, hi + up))
    return (out & 0xFFFF).astype(np.uint16)


def _f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def mnist_ref(x, w1, w2, s1, B, I, H, O) -> np.ndarray:
    ax = dict(B=B, I=I, H=H, O=O)
    m = lambda e: ref_m(e, **ax)
    h = contract(x.tobytes(), w1.tobytes(), "i8", "i8", m("[B, I]"), m("[H, I]"), m("[B, H, I]"), m("[B, H]"),
                 ep_kind=1, scale=s1, scale_axis="H", clip_lo=0, clip_hi=127)
    logits = contract(h, w2.tobytes(), "i8", "i32", m("[B, H]"), m("[O, H]"), m("[B, O, H]"), m("[B, O]"))
    return np.frombuffer(logits, np.int32).reshape(B, O)


def _bias_insns(relu: bool):
    # the register program of the bias step: r2 = bf16->f32(r0), r3 = bf16->f32(r1), r4 = r2 + r3,
    # [r6 = max(r4, 0.0)], narrowed to bf16 (opcode numbers of the C ABI)
    ins = [(1, 2, 0, 0, 0, 0), (1, 3, 1, 0, 0, 0), (30, 4, 2, 3, 0, 0)]
    if relu:
        ins += [(71, 5, 0, 0, 0, 0), (36, 6, 4, 5, 0, 0)]
    ins += [(2, 7, 6 if relu else 4, 0, 0, 0)]
    return ins, 7


def mnist_bf16_ref(x: bytes, w1: bytes, b1: bytes, w2: bytes, b2: bytes) -> bytes:
    """bf16 MNIST forward of mnist/mod.rs (one image): fc1 = bf16(sum_x w1[h, x] * x[x]) with the f32
    fold in x order, bias + ReLU in f32 -> bf16, fc2 likewise, bias -> bf16. Returns logits [16] bf16."""
    ax = dict(X=800, H=256, C=16)
    m = lambda e: ref_m(e, **ax)
    h = contract(w1, x, "bf16", "bf16", m("[H, X]"), m("[X]"), m("[H, X]"), m("[H]"))
    ins, ret = _bias_insns(True)
    h = elementwise(ins, ret, [h, b1], ["bf16", "bf16"], "bf16", 256)
    o = contract(w2, h, "bf16", "bf16", m("[C, H]"), m("[H]"), m("[C, H]"), m("[C]"))
    ins, ret = _bias_insns(False)
    return elementwise(ins, ret, [o, b2], ["bf16", "bf16"], "bf16", 16)


def _round_half_away(y: np.ndarray) -> np.ndarray:
    y = y.astype(np.float64)
    return np.sign(y) * np.floor(np.abs(y) + 0.5)


def decoder_ref(x_bits: np.ndarray, host: dict, T, H, Hq, Hkv, F, batch, seq, eps=1e-5,
                att_override=None) -> np.ndarray:
    """The W8A8 block. `att_override` (bf16 bits [T, H]) replaces the attention output, so that the
    rest of the chain can be compared on the attention values a kernel produced."""
    KV = Hkv * 128

    def rmsnorm(x, g, width):
        ss = np.cumsum(x * x, axis=1, dtype=np.float32)[:, -1]  # sequential: the wire-order fold
        rinv = np.float32(1.0) / np.sqrt(ss * np.float32(1.0 / width) + np.float32(eps))
        return (x * rinv[:, None]) * g[None, :]

    def quant(x):
        amax = np.max(np.abs(x), axis=1)
        s = np.maximum(amax, np.float32(1e-12)) / np.float32(127.0)
        q = _round_half_away(x / s[:, None])
        return np.clip(q, -127, 127).astype(np.int8), s.astype(np.float32)

    def proj(q, s, name):
        w, sw = host[name]
        acc = q.astype(np.float64) @ w.astype(np.float64).T  # exact integer sums
        assert np.abs(acc).max() < 2 ** 31
        y = acc.astype(np.int32).astype(np.float32)  # FxpToFp(31): IEEE RNE int -> f32
        y = (y * s.astype(np.float32)[:, None]) * sw.astype(np.float32)[None, :]
        return _bf16_bits(y)

    x = _f32(x_bits).reshape(T, H)
    q, s = quant(rmsnorm(x, host["g1"], H))
    Q, K, V = proj(q, s, "wq"), proj(q, s, "wk"), proj(q, s, "wv")
    if att_override is None:
        att = attention(Q.reshape(-1), K.reshape(-1), V.reshape(-1), batch, seq, Hq, Hkv, 128, 128 ** -0.5, True)
    else:
        att = np.asarray(att_override, np.uint16).reshape(-1)
    qa, sa = quant(_f32(att).reshape(T, H))
    o = proj(qa, sa, "wo")
    h1 = _bf16_bits(x + _f32(o))
    h1f = _f32(h1)
    q2, s2 = quant(rmsnorm(h1f, host["g2"], H))
    g, u = _f32(proj(q2, s2, "wg")), _f32(proj(q2, s2, "wu"))
    act = (g * (np.float32(1.0) / (np.float32(1.0) + np.exp(-g)))) * u
    q3, s3 = quant(act)
    d = proj(q3, s3, "wd")
    return _bf16_bits(h1f + _f32(d))
