"""CUDA-graph capture through the C ABI: memory ownership across captures."""
import ctypes as C

import numpy as np
import pytest

import furiosa_opt_b200 as fb
from furiosa_opt_b200 import _lib


@pytest.mark.gpu
def test_graph_memory_freed_inside_a_later_capture():
    """An allocation owned by one graph, freed while a second capture is open, is released once
    (when that capture ends) and not again when the first graph is destroyed; the context keeps
    working."""
    be = fb.B200(0)
    lib, ctx = _lib.lib(), be.ctx
    _lib.check(lib.fopt_capture_begin(ctx), ctx)
    p = C.c_void_p()
    _lib.check(lib.fopt_alloc(ctx, 1 << 20, C.byref(p)), ctx)  # owned by the first graph
    g1 = C.c_void_p()
    _lib.check(lib.fopt_capture_end(ctx, C.byref(g1)), ctx)
    _lib.check(lib.fopt_graph_launch(ctx, g1), ctx)
    _lib.check(lib.fopt_capture_begin(ctx), ctx)
    _lib.check(lib.fopt_free(ctx, p), ctx)  # not the second capture's: deferred to its end
    g2 = C.c_void_p()
    _lib.check(lib.fopt_capture_end(ctx, C.byref(g2)), ctx)
    _lib.check(lib.fopt_graph_destroy(ctx, g1), ctx)
    _lib.check(lib.fopt_graph_destroy(ctx, g2), ctx)
    be.sync()
    m = fb.Mapping("[N]", dict(N=4096))
    v = np.arange(4096, dtype=np.int32)
    assert np.array_equal(be.from_vec(m, v, "i32").to_numpy(), v)


@pytest.mark.gpu
def test_capture_rejects_a_nested_capture():
    be = fb.B200(0)
    lib, ctx = _lib.lib(), be.ctx
    _lib.check(lib.fopt_capture_begin(ctx), ctx)
    assert lib.fopt_capture_begin(ctx) != 0
    g = C.c_void_p()
    _lib.check(lib.fopt_capture_end(ctx, C.byref(g)), ctx)
    _lib.check(lib.fopt_graph_destroy(ctx, g), ctx)
