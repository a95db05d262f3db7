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


def test_reduce_noalloc_matches_reduce_twice():
    be = fb.B200(0)
    rng = np.random.default_rng(11)
    cases = [
        ("[R, C]", "[C]", dict(R=300, C=96), "i32", 0, 0),           # add over the outer axis
        ("[A, B # 8, C]", "[C, A]", dict(A=7, B=5, C=33), "i32", 2, 0x80000000),  # max, padded residue
        ("[N, G, T]", "[N, G]", dict(N=4, G=8, T=2048), "f32", 0, 0),  # f32 add over a long row
    ]
    for src_e, dst_e, ax, dt, op, ident in cases:
        S, D = fb.Mapping(src_e, ax), fb.Mapping(dst_e, ax)
        for call in range(2):  # the second call reuses (and must fully overwrite) the same array
            if dt == "i32":
                vals = rng.integers(-2 ** 20, 2 ** 20, S.size).astype(np.int32)
            else:
                vals = rng.standard_normal(S.size).astype(np.float32)
            src = be.from_vec(S, vals, dt)
            be.set_exact_fold(True)
            ref = be.reduce(src, ["Add", "AddSat", "Max", "Min"][op], 0, S, D).to_numpy() if op != 2 else \
                be.reduce(src, "Max", -2 ** 31, S, D).to_numpy()
            be.set_exact_fold(False)
            out = be.zeroed(D, dt)
            _noalloc(be, out, src, dt, op, ident, S, D)
            got = out.to_numpy()
            if dt == "i32":
                assert np.array_equal(got, ref), (src_e, call)
            else:
                # same per-cell wire-order fold as fopt_reduce's exact mode: bit-identical
                assert got.tobytes() == ref.tobytes(), (src_e, call)


def test_reduce_noalloc_rejects_oversize():
    be = fb.B200(0)
    S, D = fb.Mapping("[R, C]", dict(R=40000, C=2)), fb.Mapping("[C]", dict(C=2))
    src, out = be.zeroed(S, "i32"), be.zeroed(D, "i32")
    st = _lib.lib().fopt_reduce_noalloc(be.ctx, out.ptr, src.ptr, _lib.DTYPES["i32"], 0, 0, S.handle, D.handle, 0)
    assert st == 1
    assert b"maximum" in _lib.lib().fopt_last_error(be.ctx)
