"""ORACLE -- test infrastructure only.

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg may import this package,
and only as the checker / the timed CPU restatement, never as the thing measured or shipped.

It restates the reference's CPU emulator (furiosa-opt-std/src/storage/buf.rs) on the host:
`mapping_ref` re-derives every cell's logical index from the open `M::map` semantics, this module
turns those into BufStorage's per-cell read plans, and `storage_ref.c` runs the reference's loops.

Parity pins: tests/test_oracle.py checks this oracle against the reference's own known-answer tests
(buf.rs:921-1258, float/bf16.rs:47-76, docs/src/mapping-tensors/mapping-expressions.md asserts,
furiosa-mapping-types/src/lib.rs:1374-1535). The reference itself cannot be built here (Rust is
absent and its mapping library is a closed prebuilt download), so there is no `oracle/_ref`.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import time

import numpy as np

from .mapping_ref import RefMapping, ref_m  # noqa: F401

HERE = os.path.dirname(os.path.abspath(__file__))
SO = os.path.join(HERE, "liboracle.so")
DT = {"i8": 0, "i16": 1, "i32": 2, "bf16": 3, "f32": 4, "i4": 5, "f8e4m3": 6, "f8e5m2": 7, "f4e2m1": 8, "i5": 9,
      "i9": 10}
BITS = {"i8": 8, "i16": 16, "i32": 32, "bf16": 16, "f32": 32, "i4": 4, "f8e4m3": 8, "f8e5m2": 8, "f4e2m1": 4,
        "i5": 8, "i9": 16}


def build() -> str:
    src = os.path.join(HERE, "storage_ref.c")
    if os.path.exists(SO) and os.path.getmtime(SO) >= os.path.getmtime(src):
        return SO
    cmd = ["gcc", "-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-shared", "-fPIC",
           "-include", "stdlib.h", src, "-o", SO, "-lm"]
    subprocess.run(cmd, check=True)
    return SO


_lib = None
last_fold_seconds = 0.0  # duration of the last ref_contract fold (the timed CPU loop)
last_transpose_seconds = 0.0  # duration of the last ref_transpose copy loop


def lib():
    global _lib
    if _lib is None:
        _lib = C.CDLL(build())
        _lib.ref_fxp_to_fp.restype = C.c_uint32
        _lib.ref_fxp_to_fp.argtypes = [C.c_int32, C.c_uint32]
        _lib.ref_fp_to_fxp.restype = C.c_int32
        _lib.ref_fp_to_fxp.argtypes = [C.c_uint32, C.c_uint32]
    return _lib


F8_OPS = {"f8e4m3_to_f32": 8, "f32_to_f8e4m3": 9, "f8e5m2_to_f32": 10, "f32_to_f8e5m2": 11, "f4e2m1_to_f8e4m3": 15}


def f8_convert(kind: str, words) -> np.ndarray:
    """One of the f8 conversions (float/f8e4.rs, float/f8e5.rs) or the f4e2m1 -> f8e4m3 lookup
    (scalar.rs:933-959) over an array of 32-bit words (f32 bit patterns or codes); returns uint32."""
    a = np.ascontiguousarray(np.asarray(words).astype(np.uint32))
    out = np.empty_like(a)
    lib().ref_f8_map(F8_OPS[kind], _p(a), _p(out), C.c_int64(a.size))
    return out


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _buf(b) -> np.ndarray:
    return np.frombuffer(bytes(b), dtype=np.uint8).copy()


def nbytes(dtype: str, n: int) -> int:
    return BITS[dtype] * n // 8


# ---------------------------------------------------------------------------------------------
# index matching
# ---------------------------------------------------------------------------------------------
def _keys(co: dict, axes: list, sizes: dict) -> np.ndarray:
    k = np.zeros(len(next(iter(co.values()))) if co else 0, dtype=np.int64)
    for a in axes:
        k = k * (sizes[a] + 1) + co[a]
    return k


class _Index:
    """Lookup from logical coordinates (over `axes`) to the lowest live wire position of `m`."""

    def __init__(self, m: RefMapping, axes: list):
        self.m, self.axes = m, axes
        st, co = m.cells()
        live = np.nonzero(st == 0)[0]
        if axes:
            keys = _keys({a: co[a][live] for a in axes}, axes, m.axes)
        else:
            keys = np.zeros(len(live), np.int64)
        order = np.lexsort((live, keys))
        self.keys, self.pos = keys[order], live[order]

    def find(self, co: dict, n: int) -> np.ndarray:
        if not self.axes:
            return np.full(n, self.pos[0] if len(self.pos) else -1, dtype=np.int64)
        q = _keys({a: np.asarray(co[a], np.int64) for a in self.axes}, self.axes, self.m.axes)
        i = np.searchsorted(self.keys, q)
        ok = (i < len(self.keys)) & (self.keys[np.minimum(i, len(self.keys) - 1)] == q)
        return np.where(ok, self.pos[np.minimum(i, len(self.keys) - 1)], -1)


# ---------------------------------------------------------------------------------------------
# ops
# ---------------------------------------------------------------------------------------------
def transpose(dst: bytes, src: bytes, dtype: str, Src: RefMapping, Dst: RefMapping, src_base: int = 0,
              dst_base: int = 0, allow_broadcast: bool = False) -> bytes:
    """BufStorage::transpose: each live dst position reads the src cell with the same logical index
    (axes absent from Src broadcast)."""
    s_axes = Src.idents()
    for a in s_axes:
        assert a in Dst.idents(), "transpose: Src must be covered by the dst stream"
    if not allow_broadcast:
        assert all(a in s_axes for a in Dst.idents()), "transpose: broadcast not allowed"
    st, co = Dst.cells()
    n = Dst.size
    idx = _Index(Src, s_axes)
    pos = idx.find(co, n) if n else np.zeros(0, np.int64)
    pos = np.where(st == 0, pos, -1).astype(np.int64)
    out = _buf(dst)
    s = _buf(src)
    global last_transpose_seconds
    t0 = time.perf_counter()
    lib().ref_transpose(_p(out), _p(s), DT[dtype], _p(pos), C.c_int64(n), C.c_int64(src_base), C.c_int64(dst_base))
    last_transpose_seconds = time.perf_counter() - t0
    return out.tobytes()


def _residue(P: RefMapping, kept: list):
    """Live positions of P whose kept coordinates are all 0, ascending: the carve residue walk.

    For a large P the kept axes are re-declared with size 1 first (same wire order of the residue
    cells when the kept axes are whole symbols), so only the residue positions are evaluated."""
    if P.size > (1 << 24) and kept:
        try:
            small = RefMapping(P.expr, {a: (1 if a in kept else n) for a, n in P.axes.items()})
            st, co = small.cells()
            rows = np.nonzero(st == 0)[0]
            return {a: co[a][rows] for a in small.idents() if a not in kept}
        except AssertionError:
            pass
    st, co = P.cells()
    sel = st == 0
    for a in kept:
        sel &= co[a] == 0
    rows = np.nonzero(sel)[0]
    return {a: co[a][rows] for a in P.idents() if a not in kept}


def _plan(X: RefMapping, O: RefMapping, residue: dict, n_res: int, n_out=None):
    """ReadPlan for operand X: base[o] (out cell o at the first residue coordinate) and delta[r]."""
    x_axes = X.idents()
    idx = _Index(X, x_axes)
    n_out = O.size if n_out is None else int(n_out)
    st, oco = O.cells(np.arange(n_out))
    co = {}
    for a in x_axes:
        if a in residue:
            co[a] = np.full(n_out, residue[a][0], np.int64)
        elif a in oco:
            co[a] = oco[a]
        else:
            co[a] = np.zeros(n_out, np.int64)
    base = idx.find(co, n_out)
    base = np.where(st == 0, base, -1).astype(np.int64)
    # delta from output cell 0's row, as buf.rs:721-729
    rco = {a: (residue[a] if a in residue else np.zeros(n_res, np.int64)) for a in x_axes}
    row = idx.find(rco, n_res)
    delta = (row - row[0]).astype(np.int64)
    return base, delta


def reduce(src: bytes, dtype: str, op: int, ident_bits: int, Src: RefMapping, Dst: RefMapping,
           allow_broadcast: bool = False) -> bytes:
    kept = [a for a in Dst.idents() if a in Src.idents()]
    if not allow_broadcast:
        assert all(a in Src.idents() for a in Dst.idents())
    res = _residue(Src, kept)
    n_res = len(next(iter(res.values()))) if res else 1
    if not res:
        res = {}
    base, delta = _plan(Src, Dst, res, n_res)
    out = np.zeros(nbytes(dtype, Dst.size) + 4, np.uint8)
    s = _buf(src)
    lib().ref_reduce(_p(out), _p(s), DT[dtype], op, C.c_uint32(ident_bits), _p(base), _p(delta),
                     C.c_int64(Dst.size), C.c_int64(len(delta)), C.c_int64(Src.size))
    return out[: nbytes(dtype, Dst.size)].tobytes()


def contract(lhs: bytes, rhs: bytes, in_dtype: str, out_dtype: str, L: RefMapping, R: RefMapping, P: RefMapping,
             O: RefMapping, ep_kind: int = 0, scale=None, scale_axis: str = None, int_width: int = 31,
             clip_lo: int = -128, clip_hi: int = 127, out_cells=None, row_scale=None, row_axis: str = None) -> bytes:
    """BufStorage::contraction_in. `out_cells` optionally restricts the fold to the first k output
    cells (the bounded CPU-baseline sample); the returned image then covers just those cells."""
    kept = O.idents()
    res = _residue(P, kept)
    n_res = len(next(iter(res.values())))
    n_out = O.size if out_cells is None else int(out_cells)
    bl, dl = _plan(L, O, res, n_res, n_out)
    br, dr = _plan(R, O, res, n_res, n_out)
    sidx = np.zeros(n_out, np.int64)
    sc = np.zeros(1, np.float32)
    ridx = np.zeros(n_out, np.int64)
    rs = np.zeros(1, np.float32)
    if ep_kind in (1, 3):
        _, oco = O.cells(np.arange(n_out))
        sidx = oco[scale_axis].astype(np.int64)
        sc = np.asarray(scale, np.float32)
        if ep_kind == 3:
            ridx = oco[row_axis].astype(np.int64)
            rs = np.asarray(row_scale, np.float32)
    out = np.zeros(nbytes(out_dtype, n_out) + 4, np.uint8)
    lb, rb = _buf(lhs), _buf(rhs)
    global last_fold_seconds
    t0 = time.perf_counter()
    lib().ref_contract(_p(out), DT[out_dtype], _p(lb), _p(rb), DT[in_dtype], _p(bl), _p(dl), _p(br), _p(dr),
                       C.c_int64(n_out), C.c_int64(n_res), C.c_int64(L.size), C.c_int64(R.size), ep_kind, _p(sc),
                       _p(sidx), int_width, clip_lo, clip_hi, _p(rs), _p(ridx))
    last_fold_seconds = time.perf_counter() - t0
    return out[: nbytes(out_dtype, n_out)].tobytes()


def elementwise(insns, ret: int, inputs, in_dtypes, out_dtype: str, n: int) -> bytes:
    """insns: list of (op, dst, a, b, c, imm) in the fopt_program encoding."""
    arr = np.array(insns, dtype=np.int32).reshape(-1, 6)
    bufs = [_buf(b) for b in inputs]
    ptrs = (C.c_void_p * max(len(bufs), 1))(*[b.ctypes.data for b in bufs])
    dts = (C.c_int * max(len(bufs), 1))(*[DT[d] for d in in_dtypes])
    out = np.zeros(nbytes(out_dtype, n) + 4, np.uint8)
    lib().ref_elementwise(len(insns), _p(arr), ret, len(bufs), ptrs, dts, _p(out), DT[out_dtype], C.c_int64(n))
    return out[: nbytes(out_dtype, n)].tobytes()


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, B: int, S: int, Hq: int, Hkv: int, D: int, scale: float,
              causal: bool = True, eps: float = 6.25e-8) -> np.ndarray:
    o = np.zeros(B * S * Hq * D, np.uint16)
    q, k, v = (np.ascontiguousarray(x, np.uint16) for x in (q, k, v))
    lib().ref_attention(_p(o), _p(q), _p(k), _p(v), B, S, Hq, Hkv, D, C.c_float(scale), int(causal), C.c_float(eps))
    return o


SQRT_HEAD_DIM = 11.313708  # attention.rs:9, sqrt(128) as the reference writes it


def attention_chain(q: np.ndarray, k: np.ndarray, v: np.ndarray, B: int, S: int, Hq: int, Hkv: int, D: int,
                    causal: bool = True, chunk: int = 512, sqrt_d: float = SQRT_HEAD_DIM,
                    eps: float = 6.25e-8) -> np.ndarray:
    """The reference's chunked attention op chain (attention.rs:32-392): bf16 logits divided by
    sqrt(D), max before masking, Min mask, EPS per chunk, bf16 weights, 16-key bf16 partials, bf16
    online rescale, final division. Returns bf16 bits [B, S, Hq, D]."""
    if S > 4096 * 1024 or min(chunk, S) > 4096 or D > 256:
        raise ValueError("attention_chain: chunk <= 4096 and D <= 256")
    o = np.zeros(B * S * Hq * D, np.uint16)
    q, k, v = (np.ascontiguousarray(x, np.uint16) for x in (q, k, v))
    lib().ref_attention_chain(_p(o), _p(q), _p(k), _p(v), B, S, Hq, Hkv, D, C.c_float(sqrt_d), int(causal),
                              C.c_float(eps), int(chunk))
    return o
