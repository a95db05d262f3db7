"""Edge cases at the ends of the size range, through the C ABI, against the oracle or numpy.

  * config 2's requant epilogue at its full size (M = N = K = 4096): the first 256 output rows
    byte-exact against the oracle's per-cell fold (the full i32 result is covered by the checksum
    properties in test_gpu_parity.py);
  * a relayout of more than 2^31 elements (the 64-bit index paths of the tile kernels);
  * degenerate contractions: one contracted element (K = 1), one output cell, a padded residue
    with one live element;
  * reduces of a single cell and of a single-element residue.
"""
import numpy as np
import pytest

import furiosa_opt_b200 as fb
import oracle
from oracle import ref_m

pytestmark = pytest.mark.gpu


def test_config2_requant_rows_full_size(b200):
    M = N = K = 4096
    ax = dict(M=M, N=N, K=K)
    exprs = ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]")
    L, R, P, O = (fb.Mapping(e, ax) for e in exprs)
    rl, rr, rp, ro = (ref_m(e, **ax) for e in exprs)
    rng = np.random.default_rng(42)
    a = rng.integers(-128, 128, M * K).astype(np.int8)
    b = rng.integers(-128, 128, N * K).astype(np.int8)
    scale = rng.uniform(0.001, 0.01, N).astype(np.float32)
    s = b200.from_vec(fb.Mapping("[N]", ax), scale, "f32")
    got = b200.contraction_requant(b200.from_vec(L, a, "i8"), b200.from_vec(R, b, "i8"), L, R, P, O, s, "N").to_bytes()
    rows = 256
    want = oracle.contract(a.tobytes(), b.tobytes(), "i8", "i8", rl, rr, rp, ro, ep_kind=1, scale=scale,
                           scale_axis="N", out_cells=rows * N)
    assert got[: rows * N] == want


def test_relayout_beyond_2_31_elements(b200):
    n = 46344  # n * n = 2 147 766 336 > 2^31, a multiple of 8 (the 8 x 8 byte-block tile path)
    ax = dict(A=n, B=n)
    S, D = fb.Mapping("[A, B]", ax), fb.Mapping("[B, A]", ax)
    x = np.random.default_rng(1).integers(0, 256, n * n, dtype=np.uint8).view(np.int8)
    src = b200.from_vec(S, x, "i8")
    t = b200.relayout(src, S, D)
    got = np.frombuffer(t.to_bytes(), np.int8).reshape(n, n)
    xs = x.reshape(n, n)
    for r in (0, 1, n // 2, n - 2, n - 1):  # whole rows of the result at both ends and the middle
        assert np.array_equal(got[r], xs[:, r]), r
    back = b200.relayout(t, D, S)
    assert back == src  # the device-side byte comparison over all 2.1 G elements


@pytest.mark.parametrize("dtype", ["i8", "bf16", "f32"])
def test_contraction_degenerate_shapes(b200, dtype):
    cases = [
        ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]", dict(M=64, K=1, N=64)),      # one contracted element
        ("[K]", "[K]", "[K]", "[1]", dict(K=777)),                                 # one output cell
        ("[M, K = 1 # 8]", "[K = 1 # 8, N]", "[M, K = 1 # 8, N]", "[M, N]", dict(M=5, K=1, N=3)),  # padded residue
    ]
    rng = np.random.default_rng(5)
    acc = {"i8": "i32", "bf16": "f32", "f32": "f32"}[dtype]
    for l, r, p, o, ax in cases:
        L, R, P, O = (fb.Mapping(e, ax) for e in (l, r, p, o))
        rl, rr, rp, ro = (ref_m(e, **ax) for e in (l, r, p, o))
        if dtype == "i8":
            lv, rv = rng.integers(-128, 128, L.size).astype(np.int8), rng.integers(-128, 128, R.size).astype(np.int8)
        elif dtype == "bf16":
            lv = fb.dtypes.f32_to_bf16_bits(rng.standard_normal(L.size).astype(np.float32))
            rv = fb.dtypes.f32_to_bf16_bits(rng.standard_normal(R.size).astype(np.float32))
        else:
            lv, rv = rng.standard_normal(L.size).astype(np.float32), rng.standard_normal(R.size).astype(np.float32)
        got = b200._contract(b200.from_vec(L, lv, dtype), b200.from_vec(R, rv, dtype), L, R, P, O, acc).to_bytes()
        want = oracle.contract(fb.dtypes.to_bytes(lv, dtype), fb.dtypes.to_bytes(rv, dtype), dtype, acc, rl, rr, rp,
                               ro)
        assert got == want, (l, r, o)


def test_reduce_degenerate_shapes(b200):
    rng = np.random.default_rng(6)
    for src_e, dst_e, ax in (("[A]", "[1]", dict(A=1)), ("[A, B]", "[A]", dict(A=300, B=1)),
                             ("[A, B # 4]", "[A]", dict(A=17, B=1)), ("[A]", "[1]", dict(A=100003))):
        S, D = fb.Mapping(src_e, ax), fb.Mapping(dst_e, ax)
        v = rng.integers(-2 ** 20, 2 ** 20, S.size).astype(np.int32)
        got = b200.reduce(b200.from_vec(S, v, "i32"), "Add", 0, S, D).to_bytes()
        want = oracle.reduce(v.tobytes(), "i32", 0, 0, ref_m(src_e, **ax), ref_m(dst_e, **ax))
        assert got == want, src_e


@pytest.mark.parametrize("dtype", ["f32", "i32"])
@pytest.mark.parametrize("R,D,E", [(1000, 61, 64), (33, 7, 8), (4097, 100, 128)])
def test_padded_rows_keep_dead_cells(b200, dtype, R, D, E):
    """[R, D] -> [R, D # E] onto a canvas: live cells from the source, dead cells keep the canvas
    (buf.rs:257-313 writes only live destination positions); ragged row counts."""
    ax = dict(R=R, D=D)
    S, Dm = fb.Mapping("[R, D]", ax), fb.Mapping(f"[R, D # {E}]", ax)
    rng = np.random.default_rng(R + D)
    x = rng.integers(-2 ** 31, 2 ** 31, R * D, dtype=np.int64).astype(np.int32)
    canvas = rng.integers(-2 ** 31, 2 ** 31, R * E, dtype=np.int64).astype(np.int32)
    if dtype == "f32":
        x, canvas = x.view(np.float32), canvas.view(np.float32)
    dst = b200.from_vec(Dm, canvas, dtype)
    b200.transpose(dst, b200.from_vec(S, x, dtype), S, Dm)
    got = np.frombuffer(dst.to_bytes(), np.int32).reshape(R, E)
    want = canvas.view(np.int32).reshape(R, E).copy()
    want[:, :D] = x.view(np.int32).reshape(R, D)
    assert np.array_equal(got, want)


def test_padded_rows_from_a_source_window(b200):
    """The same move reading a window of a larger source (rows 5.. of [R2, D]): the staged kernel's
    first aligned vector starts before the window."""
    R2, R, D, E = 300, 200, 61, 64
    base = fb.Mapping("[R, D]", dict(R=R2, D=D))
    win = fb.Mapping("[R, D]", dict(R=R, D=D))
    Dm = fb.Mapping(f"[R, D # {E}]", dict(R=R, D=D))
    x = np.arange(R2 * D, dtype=np.int32)
    dst = b200.zeroed(Dm, "i32")
    b200.transpose(dst, b200.from_vec(base, x, "i32"), win, Dm, src_offset={"R": 5}, src_map=base)
    got = dst.to_numpy().reshape(R, E)
    assert np.array_equal(got[:, :D], x.reshape(R2, D)[5:5 + R])
    assert not got[:, D:].any()
