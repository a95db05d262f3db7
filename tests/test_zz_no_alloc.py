"""fopt_reduce_noalloc: the reduce for callers that cannot let the library allocate device memory
(a runtime that owns the device-memory budget through its own allocator, or a latency-critical loop
that cannot absorb cudaFree's implicit device synchronisation). It is called straight through the C
ABI and must agree with fopt_reduce on two calls in a row, since every call reuses the same fixed
device array. This file sorts last so a failure here never hides the other tests."""
import ctypes as C

import numpy as np
import pytest

import furiosa_opt_b200 as fb
from furiosa_opt_b200 import _lib

pytestmark = pytest.mark.gpu


def _noalloc(be, out, src, dtype, op, ident_bits, S, D, bc=0):
    st = _lib.lib().fopt_reduce_noalloc(be.ctx, out.ptr, src.ptr, _lib.DTYPES[dtype], op, ident_bits, S.handle,
                                        D.handle, bc)
    _lib.check(st, be.ctx)
    be.sync()


def _bits(v, dt):
    return int(np.asarray(v, {"i32": np.int32, "f32": np.float32}[dt]).view(np.uint32)) if dt != "bf16" else \
        int(fb.dtypes.f32_to_bf16_bits(np.asarray([v], np.float32))[0])


def test_reduce_noalloc_matches_reduce_twice():
    be = fb.B200(0)
    rng = np.random.default_rng(11)
    ops = ["Add", "AddSat", "Max", "Min"]
    cases = [
        ("[R, C]", "[C]", dict(R=300, C=96), "i32", 0, 0),                        # add over the outer axis
        ("[A, B # 8, C]", "[C, A]", dict(A=7, B=5, C=33), "i32", 2, -2 ** 31),    # max, padded residue
        ("[N, G, T]", "[N, G]", dict(N=4, G=8, T=2048), "f32", 0, 0.0),            # f32 add over a long row
        ("[N, G, T]", "[N, G]", dict(N=4, G=8, T=2048), "f32", 2, -np.inf),        # f32 max over a long row
        ("[R, C]", "[R]", dict(R=64, C=200), "bf16", 0, 0.0),                      # bf16 add along the row
        ("[R, C]", "[C]", dict(R=100, C=48), "bf16", 3, np.inf),                   # bf16 min over the outer axis
    ]
    was = be.exact_fold
    be.set_exact_fold(True)
    try:
        for src_e, dst_e, ax, dt, op, ident in cases:
            S, D = fb.Mapping(src_e, ax), fb.Mapping(dst_e, ax)
            for call in range(2):  # the second call reuses (and must fully overwrite) the same array
                if dt == "i32":
                    vals = rng.integers(-2 ** 20, 2 ** 20, S.size).astype(np.int32)
                elif dt == "f32":
                    vals = rng.standard_normal(S.size).astype(np.float32)
                else:
                    vals = fb.dtypes.f32_to_bf16_bits(rng.standard_normal(S.size).astype(np.float32))
                src = be.from_vec(S, vals, dt)
                ref = be.reduce(src, ops[op], ident, S, D).to_bytes()
                out = be.zeroed(D, dt)
                _noalloc(be, out, src, dt, op, _bits(ident, dt), S, D)
                # the same per-cell wire-order fold as fopt_reduce in exact mode: bit-identical (no signed
                # zeros or NaNs in these inputs, so the f32 max also agrees with the order-free warp fold)
                assert out.to_bytes() == ref, (src_e, dt, ops[op], call)
    finally:
        be.set_exact_fold(was)


def test_reduce_noalloc_refused_inside_capture():
    be = fb.B200(0)
    S, D = fb.Mapping("[R, C]", dict(R=64, C=32)), fb.Mapping("[C]", dict(C=32))
    src, out = be.zeroed(S, "i32"), be.zeroed(D, "i32")
    status = []

    def step():
        status.append(_lib.lib().fopt_reduce_noalloc(be.ctx, out.ptr, src.ptr, _lib.DTYPES["i32"], 0, 0, S.handle,
                                                     D.handle, 0))
        return be.zeroed(D, "i32")

    g = be.capture(step)
    g.close()
    assert status == [1]
    assert b"capture" in _lib.lib().fopt_last_error(be.ctx)
    _noalloc(be, out, src, "i32", 0, 0, S, D)  # the context is still usable after the refusal
    assert not out.to_numpy().any()


def test_reduce_noalloc_rejects_oversize():
    be = fb.B200(0)
    S, D = fb.Mapping("[R, C]", dict(R=40000, C=2)), fb.Mapping("[C]", dict(C=2))
    src, out = be.zeroed(S, "i32"), be.zeroed(D, "i32")
    st = _lib.lib().fopt_reduce_noalloc(be.ctx, out.ptr, src.ptr, _lib.DTYPES["i32"], 0, 0, S.handle, D.handle, 0)
    assert st == 1
    assert b"maximum" in _lib.lib().fopt_last_error(be.ctx)
