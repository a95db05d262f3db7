"""Parity of the CUDA kernels (through the C ABI) against the CPU oracle on the same seeded inputs.

Bar: bit-exact for integer, layout and cast work; float folds within the tolerance stated per test.
"""
import struct

import numpy as np
import pytest

import furiosa_opt_b200 as fb
import oracle
from furiosa_opt_b200 import _lib, dtypes, ops
from oracle import ref_m

pytestmark = pytest.mark.gpu

RNG = np.random.default_rng(42)


def pair(expr, **axes):
    return fb.Mapping(expr, axes), ref_m(expr, **axes)


def rand_vals(dtype, n, rng=RNG):
    if dtype in ("i8", "i5"):
        return rng.integers(-128, 128, n).astype(np.int8)
    if dtype == "i4":
        return rng.integers(-8, 8, n).astype(np.int8)
    if dtype in ("i16", "i9"):
        return rng.integers(-32768, 32768, n).astype(np.int16)
    if dtype == "i32":
        return rng.integers(-2 ** 31, 2 ** 31, n, dtype=np.int64).astype(np.int32)
    if dtype == "bf16":
        return dtypes.f32_to_bf16_bits(rng.standard_normal(n).astype(np.float32))
    if dtype == "f32":
        return rng.standard_normal(n).astype(np.float32)
    raise ValueError(dtype)


# ---------------------------------------------------------------------------------------------
# known answers (buf.rs tests) through the B200 backend
# ---------------------------------------------------------------------------------------------
def test_known_matmul_and_reorder(b200):
    M, R = fb.Mapping, None
    ax = dict(M=2, K=3, N=2)
    L, Rm, P, O = (fb.Mapping(e, ax) for e in ("[M, K]", "[K, N]", "[M, K, N]", "[M, N]"))
    a = b200.from_vec(L, np.arange(1, 7, dtype=np.float32), "f32")
    b = b200.from_vec(Rm, np.arange(1, 7, dtype=np.float32), "f32")
    assert list(b200.contraction_prewidened(a, b, L, Rm, P, O).to_numpy()) == [22, 28, 49, 64]
    ai = b200.from_vec(L, np.arange(1, 7, dtype=np.int32), "i32")
    bi = b200.from_vec(Rm, np.arange(1, 7, dtype=np.int32), "i32")
    ON = fb.Mapping("[N, M]", ax)
    assert list(b200.contraction_prewidened(ai, bi, L, Rm, P, ON).to_numpy()) == [22, 49, 28, 64]


def test_known_padded_k(b200):
    ax = dict(M=2, K=2, N=2)
    L, Rm = fb.Mapping("[M, K = 2 # 4]", ax), fb.Mapping("[K = 2 # 4, N]", ax)
    P, O = fb.Mapping("[M, K = 2 # 4, N]", ax), fb.Mapping("[M, N]", ax)
    a = b200.from_vec(L, np.array([1, 2, 0, 0, 3, 4, 0, 0], np.int32), "i32")
    b = b200.from_vec(Rm, np.array([1, 2, 3, 4, 0, 0, 0, 0], np.int32), "i32")
    assert list(b200.contraction_prewidened(a, b, L, Rm, P, O).to_numpy()) == [7, 10, 15, 22]


def test_known_i8_wraps_once(b200):
    ax = dict(M=1, K=100, N=1)
    L, Rm, P, O = (fb.Mapping(e, ax) for e in ("[M, K]", "[K, N]", "[M, K, N]", "[M, N]"))
    a = b200.from_vec(L, np.full(100, 100, np.int8), "i8")
    out = b200.contraction(a, a.clone(), L, Rm, P, O).to_numpy()
    assert out[0] == np.int32(1_000_000).astype(np.int8)


def test_known_cross_slice(b200):
    ax = dict(M=1, K=2, N=1)
    L, Rm, P, O = (fb.Mapping(e, ax) for e in ("[M, K]", "[K, N]", "[M, K, N]", "[M, N]"))
    bf = lambda v: (np.asarray(v, np.float32).view(np.uint32) >> 16).astype(np.uint16)
    part = b200.contraction(b200.from_vec(L, bf([1.0, 2 ** -8]), "bf16"), b200.from_vec(Rm, bf([1.0, 1.0]), "bf16"),
                            L, Rm, P, O).to_numpy()[0]
    assert part == 0x3F80
    S = fb.Mapping("[Slice, M, N]", dict(Slice=3, M=1, N=1))
    D = fb.Mapping("[M, N]", dict(M=1, N=1))
    b200.set_exact_fold(True)
    cross = b200.reduce(b200.from_vec(S, np.full(3, part, np.uint16), "bf16"), "Add", 0.0, S, D).to_numpy()[0]
    b200.set_exact_fold(False)
    assert cross == 0x4040


def test_known_reduce_and_transpose_large(b200):
    S, D = fb.Mapping("[R, C]", dict(R=256, C=512)), fb.Mapping("[C]", dict(C=512))
    data = (np.arange(256 * 512) % 5).astype(np.int32)
    got = b200.reduce(b200.from_vec(S, data, "i32"), "Add", 0, S, D).to_numpy()
    assert np.array_equal(got, data.reshape(256, 512).sum(0))
    S2, D2 = fb.Mapping("[Big, Small]", dict(Big=1 << 20, Small=4)), fb.Mapping("[Big]", dict(Big=1 << 20))
    d2 = (np.arange((1 << 20) * 4) % 7).astype(np.int32)
    assert np.array_equal(b200.reduce(b200.from_vec(S2, d2, "i32"), "Add", 0, S2, D2).to_numpy(),
                          d2.reshape(-1, 4).sum(1))
    Sr, Dr = fb.Mapping("[R, C]", dict(R=512, C=256)), fb.Mapping("[C, R]", dict(R=512, C=256))
    t = np.arange(512 * 256, dtype=np.int32)
    assert np.array_equal(b200.relayout(b200.from_vec(Sr, t, "i32"), Sr, Dr).to_numpy(),
                          t.reshape(512, 256).T.reshape(-1))


# ---------------------------------------------------------------------------------------------
# relayout
# ---------------------------------------------------------------------------------------------
RELAYOUTS = [
    ("[A, B]", "[B, A]", dict(A=4, B=8), False),
    ("[R, C]", "[C, R]", dict(R=96, C=80), False),
    ("[R, C]", "[C, R]", dict(R=512, C=384), False),
    ("[A, B, C]", "[C, A, B]", dict(A=3, B=5, C=7), False),
    ("[A, B, C]", "[B, A, C]", dict(A=16, B=24, C=64), False),
    ("[A, B, C]", "[A, C, B]", dict(A=3, B=36, C=20), False),  # batched tiles, extents not multiples of 128
    ("[A, B, C]", "[A, C, B]", dict(A=2, B=200, C=136), False),  # batched 8-byte-unit tiles, ragged edges
    ("[A]", "[B, A # 6]", dict(A=4, B=3), True),
    ("[C, D]", "[C, D # 64]", dict(C=13, D=61), False),
    ("[C, D # 64]", "[D, C]", dict(C=13, D=61), False),
    # partly live destination rows (vectorised rows path): live widths not a multiple of the vector,
    # permuted outer wheels, a strided innermost source wheel
    ("[C, D]", "[C, D # 48]", dict(C=37, D=33), False),
    ("[A, B, D]", "[B, A, D # 32]", dict(A=5, B=7, D=29), False),
    ("[D, C]", "[C, D # 32]", dict(C=9, D=20), False),
    ("[B]", "[B / 64, B % 32, B / 32 % 2]", dict(B=512), False),
    ("[A, B]", "[A / 4, B, A % 4]", dict(A=16, B=12), False),
    ("[H, X]", "[X / 8, H, X % 8]", dict(H=10, X=64), False),
    ("[M, K = 2 # 4]", "[K = 2 # 4, M]", dict(M=3, K=2), False),
    ("[A, B]", "[[A, B] # 100]", dict(A=7, B=13), False),
    ("[A / 4 % 4, A % 4, B]", "[A % 4, A / 4 % 4, B]", dict(A=16, B=64), False),
    ("[N, G, T]", "[N, T / 8, G, T % 8]", dict(N=4, G=16, T=128), False),
    ("[T]", "[T, H]", dict(T=24, H=64), True),  # broadcast along the innermost axis
    ("[H]", "[T, H]", dict(T=24, H=64), True),
]


@pytest.mark.parametrize("dtype", ["i8", "bf16", "i32", "i4"])
@pytest.mark.parametrize("src,dst,axes,bc", RELAYOUTS)
def test_relayout_parity(b200, src, dst, axes, bc, dtype):
    S, rs = pair(src, **axes)
    D, rd = pair(dst, **axes)
    if dtype == "i4" and (S.size % 2 or D.size % 2):
        pytest.skip("sub-byte element count must be byte-aligned")
    vals = rand_vals(dtype, S.size)
    canvas = rand_vals(dtype, D.size)
    src_s = b200.from_vec(S, vals, dtype)
    dst_s = b200.from_vec(D, canvas, dtype)
    b200.transpose(dst_s, src_s, S, D, allow_broadcast=bc)
    want = oracle.transpose(dtypes.to_bytes(canvas, dtype), dtypes.to_bytes(vals, dtype), dtype, rs, rd,
                            allow_broadcast=bc)
    assert dst_s.to_bytes() == want


def test_relayout_window(b200):
    # a tile write into a view of the base mapping (view.rs:178-189 -> window_base, buf.rs:760-781)
    ax = dict(A=4, B=8)
    base = fb.Mapping("[A, B]", ax)
    tile_dst = fb.Mapping("[A, B = 2 # 8]", ax)
    src_m, rsrc = pair("[B = 2, A]", **ax)
    vals = rand_vals("i32", src_m.size)
    canvas = np.zeros(32, np.int32)
    d = b200.from_vec(base, canvas, "i32")
    s = b200.from_vec(src_m, vals, "i32")
    b200.transpose(d, s, src_m, tile_dst, dst_offset={"B": 4}, dst_map=base)
    got = d.to_numpy().reshape(4, 8)
    want = np.zeros((4, 8), np.int32)
    v = vals.reshape(2, 4)  # [B=2, A]
    want[:, 4:6] = v.T
    assert np.array_equal(got, want)


# ---------------------------------------------------------------------------------------------
# elementwise
# ---------------------------------------------------------------------------------------------
def _ew_case(b200, prog, in_dtypes, out_dtype, n=4098, values=None):
    mp = fb.Mapping("[E]", dict(E=n))
    vals = values or [rand_vals(d, n) for d in in_dtypes]
    ins = [b200.from_vec(mp, v, d) for v, d in zip(vals, in_dtypes)]
    out = b200._ew(prog, ins, out_dtype).to_bytes()
    insns = [(prog.insn[i].op, prog.insn[i].dst, prog.insn[i].a, prog.insn[i].b, prog.insn[i].c, prog.insn[i].imm_i)
             for i in range(prog.n_insn)]
    want = oracle.elementwise(insns, prog.ret, [dtypes.to_bytes(v, d) for v, d in zip(vals, in_dtypes)], in_dtypes,
                              out_dtype, n)
    return out, want


EXACT = [
    (ops.cast("bf16", "f32"), ["bf16"], "f32"), (ops.cast("f32", "bf16"), ["f32"], "bf16"),
    (ops.cast("i8", "i32"), ["i8"], "i32"), (ops.cast("i32", "i8"), ["i32"], "i8"),
    (ops.cast("i32", "i16"), ["i32"], "i16"), (ops.cast("i4", "i32"), ["i4"], "i32"),
    (ops.cast("i32", "i4"), ["i32"], "i4"), (ops.cast_relu(), ["f32"], "bf16"),
    (ops.fxp_to_fp(31), ["i32"], "f32"), (ops.fxp_to_fp(8), ["i32"], "f32"), (ops.fp_to_fxp(31), ["f32"], "i32"),
    (ops.fp_to_fxp(4), ["f32"], "i32"),
    *[(ops.fp_binary(n), ["f32", "f32"], "f32") for n in ("AddF", "SubF", "MulF", "DivF")],
    (ops.fp_binary("SubF", "Mode10"), ["f32", "f32"], "f32"),
    *[(ops.clip_f32(n), ["f32", "f32"], "f32") for n in ("Add", "Min", "Max", "AbsMin", "AbsMax")],
    *[(ops.clip_i32(n), ["i32", "i32"], "i32") for n in ("AddFxp", "AddFxpSat", "Min", "Max", "AbsMin", "AbsMax")],
    *[(ops.fxp_binary(n), ["i32", "i32"], "i32") for n in ("SubFxp", "SubFxpSat", "LeftShift", "LeftShiftSat",
                                                            "MulFxp", "MulInt", "LogicRightShift", "ArithRightShift")],
    *[(ops.logic_i32(n), ["i32", "i32"], "i32") for n in ("BitAnd", "BitOr", "BitXor")],
    (ops.fp_ternary("FmaF"), ["f32", "f32", "f32"], "f32"),
    (ops.fp_unary("Sqrt"), ["f32"], "f32"),
    (ops.select(), ["i32", "f32", "f32"], "f32"),
    (ops.requant_i32_to_i8(0.0037, relu=True), ["i32"], "i8"),
    (ops.with_const_f32(ops.CLIP_F32, "Max", 0.0), ["f32"], "f32"),
]


@pytest.fixture(params=["generated", "interpreter"])
def ew_path(request, monkeypatch):
    """Runs an elementwise test through the NVRTC-generated kernel and through the interpreter."""
    if request.param == "interpreter":
        monkeypatch.setenv("FOPT_EW_NO_JIT", "1")
    else:
        monkeypatch.delenv("FOPT_EW_NO_JIT", raising=False)
    return request.param


def _check_path(path, before, in_dtypes, out_dtype):
    n = _lib.lib().fopt_elementwise_jit_launches() - before
    packed = "i4" in in_dtypes or out_dtype == "i4"
    assert n == (1 if path == "generated" and not packed else 0)


@pytest.mark.parametrize("case", range(len(EXACT)))
def test_elementwise_exact(b200, ew_path, case):
    prog, ins, out_dt = EXACT[case]
    before = _lib.lib().fopt_elementwise_jit_launches()
    got, want = _ew_case(b200, prog, ins, out_dt)
    _check_path(ew_path, before, ins, out_dt)
    if out_dt in ("f32", "bf16"):
        g = np.frombuffer(got, np.uint32 if out_dt == "f32" else np.uint16)
        w = np.frombuffer(want, np.uint32 if out_dt == "f32" else np.uint16)
        # NaN payloads may differ only where both are NaN
        fg = g.view(np.float32) if out_dt == "f32" else dtypes.bf16_bits_to_f32(g)
        fw = w.view(np.float32) if out_dt == "f32" else dtypes.bf16_bits_to_f32(w)
        both_nan = np.isnan(fg) & np.isnan(fw)
        assert np.array_equal(g[~both_nan], w[~both_nan])
    else:
        assert got == want


@pytest.mark.parametrize("path", ["generated", "interpreter"])
def test_lazy_broadcast_elementwise(b200, monkeypatch, path):
    """A broadcast made by relayout stays unwritten when only elementwise ops read it: a per-row
    value ([T] -> [T, W]) and a repeated row ([W] -> [T, W]) read through the broadcast index give
    the same bits as the written-out broadcast; without generated kernels the broadcast is written
    out first, with the same result; and its bytes, when asked for, are the relayout's."""
    if path == "interpreter":
        monkeypatch.setenv("FOPT_EW_NO_JIT", "1")
    else:
        monkeypatch.delenv("FOPT_EW_NO_JIT", raising=False)
    T, W = 24, 72
    ax = dict(T=T, W=W)
    big, rows, cols = fb.Mapping("[T, W]", ax), fb.Mapping("[T]", ax), fb.Mapping("[W]", ax)
    x = rand_vals("f32", T * W)
    r = rand_vals("f32", T)
    c = rand_vals("f32", W)
    X = b200.from_vec(big, x, "f32")
    R = b200.relayout(b200.from_vec(rows, r, "f32"), rows, big, allow_broadcast=True)
    Cb = b200.relayout(b200.from_vec(cols, c, "f32"), cols, big, allow_broadcast=True)
    assert R.lazy is not None and Cb.lazy is not None
    got = b200.zip3_with(X, R, Cb, ops.fp_ternary("FmaF"), "f32").to_numpy().reshape(T, W)
    # FmaF(a, b, c) = fma(a, b, c) on the written-out operands
    want = np.frombuffer(oracle.elementwise([(34, 3, 0, 1, 2, 0)], 3, [x.tobytes(), np.repeat(r, W).tobytes(),
                                                                      np.tile(c, T).tobytes()],
                                            ["f32", "f32", "f32"], "f32", T * W), np.float32).reshape(T, W)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    if path == "generated":
        assert R.lazy is not None and Cb.lazy is not None  # read through, never written out
    assert np.array_equal(R.to_numpy().reshape(T, W), np.repeat(r, W).reshape(T, W))
    assert np.array_equal(Cb.to_numpy().reshape(T, W), np.tile(c, T).reshape(T, W))


@pytest.mark.parametrize("op,ident", [("Add", 0.0), ("Max", float("-inf")), ("Min", float("inf"))])
def test_fused_map_reduce(b200, monkeypatch, op, ident):
    """Engine-chain fusion: a deferred map (here |x| * s with s a lazy per-row broadcast) folded by a
    row reduction without being written matches writing it and reducing (bit-exact for Max / Min;
    Add reassociates, within the n-eps bound of the non-exact reduce)."""
    T, W = 96, 4096 + 256
    ax = dict(T=T, W=W)
    big, rows = fb.Mapping("[T, W]", ax), fb.Mapping("[T]", ax)
    x = rand_vals("f32", T * W)
    r = np.abs(rand_vals("f32", T)) + 0.5
    p = ops.Prog(2)
    prog = p.build(p.emit("MULF", p.emit("AND", 0, p.const_i32(0x7FFFFFFF)), 1))
    X = b200.from_vec(big, x, "f32")
    Rb = b200.relayout(b200.from_vec(rows, r, "f32"), rows, big, allow_broadcast=True)
    lazy = b200.zip_with(X, Rb, prog, "f32")
    assert lazy.lazy is not None
    before = _lib.lib().fopt_elementwise_jit_launches()
    got = b200.reduce(lazy, op, ident, big, rows).to_numpy()
    assert _lib.lib().fopt_elementwise_jit_launches() == before + 1  # the fused kernel, nothing else
    assert lazy.lazy is not None  # the mapped values were never written
    vals = np.abs(x).reshape(T, W) * r[:, None]
    if op == "Add":
        want = vals.astype(np.float64).sum(1)
        assert np.all(np.abs(got - want) <= 1e-5 * np.abs(vals).sum(1) + 1e-6)
    else:
        want = vals.max(1) if op == "Max" else vals.min(1)
        assert np.array_equal(got, want.astype(np.float32))
    # and the same values through the unfused path
    monkeypatch.setenv("FOPT_NO_FUSION", "1")
    be2 = fb.B200(0)
    X2 = be2.from_vec(big, x, "f32")
    R2 = be2.relayout(be2.from_vec(rows, r, "f32"), rows, big, allow_broadcast=True)
    plain = be2.reduce(be2.zip_with(X2, R2, prog, "f32"), op, ident, big, rows).to_numpy()
    if op != "Add":
        assert np.array_equal(got, plain)


def test_deferred_values_survive_inplace_writes(b200):
    """A deferred elementwise value reads its inputs as they were when it was made: an in-place
    write into an input first makes the deferred value take its values."""
    ax = dict(N=4096)
    m = fb.Mapping("[N]", ax)
    x = rand_vals("f32", 4096)
    X = b200.from_vec(m, x, "f32")
    doubled = b200.zip_with(X, X, ops.fp_binary("AddF"), "f32")
    assert doubled.lazy is not None
    b200.transpose(X, b200.from_vec(m, np.zeros(4096, np.float32), "f32"), m, m)  # overwrite X in place
    assert doubled.lazy is None
    assert np.array_equal(doubled.to_numpy(), (x + x).astype(np.float32))


@pytest.mark.parametrize("n", [1, 7, 8, 9, 4096 * 37 + 3])
@pytest.mark.parametrize("case", [0, 1, 3, 4])
def test_elementwise_sizes(b200, ew_path, case, n):
    """Tails shorter than one 8-element group and grid-stride sizes, in both elementwise paths."""
    prog, ins, out_dt = EXACT[case]
    got, want = _ew_case(b200, prog, ins, out_dt, n=n)
    if out_dt == "f32":
        g, w = np.frombuffer(got, np.float32), np.frombuffer(want, np.float32)
        ok = (g.view(np.uint32) == w.view(np.uint32)) | (np.isnan(g) & np.isnan(w))
        assert ok.all()
    elif out_dt == "bf16":
        g, w = dtypes.bf16_bits_to_f32(np.frombuffer(got, np.uint16)), dtypes.bf16_bits_to_f32(np.frombuffer(want, np.uint16))
        assert ((np.frombuffer(got, np.uint16) == np.frombuffer(want, np.uint16)) | (np.isnan(g) & np.isnan(w))).all()
    else:
        assert got == want


@pytest.mark.parametrize("name", ["Exp", "NegExp", "Tanh", "Sigmoid", "Log", "Sin", "Cos"])
def test_elementwise_transcendental(b200, ew_path, name):
    # libm vs CUDA: within 2 ulp-ish relative (1e-6) / 1e-6 absolute
    before = _lib.lib().fopt_elementwise_jit_launches()
    got, want = _ew_case(b200, ops.fp_unary(name), ["f32"], "f32")
    _check_path(ew_path, before, ["f32"], "f32")
    g, w = np.frombuffer(got, np.float32), np.frombuffer(want, np.float32)
    fin = np.isfinite(w)
    assert np.array_equal(np.isnan(g), np.isnan(w))
    assert np.allclose(g[fin], w[fin], rtol=1e-6, atol=1e-6)


# ---------------------------------------------------------------------------------------------
# reduce
# ---------------------------------------------------------------------------------------------
REDUCES = [
    ("[R, C]", "[C]", dict(R=64, C=96)),
    ("[R, C]", "[R]", dict(R=64, C=300)),
    ("[A, B, C]", "[A, C]", dict(A=5, B=7, C=9)),
    ("[A, B # 8, C]", "[C, A]", dict(A=3, B=5, C=4)),
    ("[N, G, T]", "[N, G]", dict(N=4, G=8, T=2048)),
]


@pytest.mark.parametrize("op,ident", [("Add", 0), ("AddSat", 0), ("Max", -2 ** 31), ("Min", 2 ** 31 - 1)])
@pytest.mark.parametrize("src,dst,axes", REDUCES)
def test_reduce_i32_exact(b200, src, dst, axes, op, ident):
    S, rs = pair(src, **axes)
    D, rd = pair(dst, **axes)
    vals = rand_vals("i32", S.size)
    if op != "AddSat":
        vals = (vals >> 8).astype(np.int32)
    got = b200.reduce(b200.from_vec(S, vals, "i32"), op, ident, S, D).to_bytes()
    code = {"Add": 0, "AddSat": 1, "Max": 2, "Min": 3}[op]
    want = oracle.reduce(vals.tobytes(), "i32", code, ident & 0xFFFFFFFF, rs, rd)
    assert got == want


@pytest.mark.parametrize("src,dst,axes", REDUCES)
def test_reduce_f32(b200, src, dst, axes):
    S, rs = pair(src, **axes)
    D, rd = pair(dst, **axes)
    vals = rand_vals("f32", S.size)
    want = np.frombuffer(oracle.reduce(vals.tobytes(), "f32", 0, 0, rs, rd), np.float32)
    got = b200.reduce(b200.from_vec(S, vals, "f32"), "Add", 0.0, S, D).to_numpy()
    # fast mode reassociates: |err| <= 1e-5 * sum|x| per cell (n * eps bound)
    absum = np.frombuffer(oracle.reduce(np.abs(vals).tobytes(), "f32", 0, 0, rs, rd), np.float32)
    assert np.all(np.abs(got - want) <= 1e-5 * absum + 1e-6)
    b200.set_exact_fold(True)
    exact = b200.reduce(b200.from_vec(S, vals, "f32"), "Add", 0.0, S, D).to_bytes()
    b200.set_exact_fold(False)
    assert exact == want.tobytes()
    mx = b200.reduce(b200.from_vec(S, vals, "f32"), "Max", float("-inf"), S, D).to_bytes()
    assert mx == oracle.reduce(vals.tobytes(), "f32", 2, 0xFF800000, rs, rd)


# ---------------------------------------------------------------------------------------------
# contraction
# ---------------------------------------------------------------------------------------------
CONTRACTIONS = [
    # (lhs, rhs, pre_reduce, out, axes)
    ("[M, K]", "[K, N]", "[M, K, N]", "[M, N]", dict(M=33, K=70, N=19)),
    ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]", dict(M=128, K=256, N=128)),
    ("[M, K]", "[N, K]", "[M, N, K]", "[N, M]", dict(M=40, K=64, N=24)),
    ("[K, M]", "[K, N]", "[K, M, N]", "[M, N]", dict(M=16, K=48, N=20)),
    ("[M, K = 5 # 8]", "[K = 5 # 8, N]", "[M, K = 5 # 8, N]", "[M, N]", dict(M=6, K=5, N=7)),
    ("[M, K]", "[K]", "[M, K]", "[M]", dict(M=50, K=64)),
    ("[B, M, K]", "[K, N]", "[B, M, K, N]", "[B, M, N]", dict(B=3, M=8, K=32, N=16)),
    # tensor-core shapes (M % 128, N % 128, K % 128 bytes): several tiles per CTA ring
    ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]", dict(M=256, K=512, N=512)),
    ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]", dict(M=384, K=1024, N=384)),
    # fewer tiles than SM pairs and a long K: the paired kernel splits each tile into K-ranges
    ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]", dict(M=256, K=2048, N=512)),
]


@pytest.mark.parametrize("dtype,out", [("i8", "i32"), ("i8", "i8"), ("i4", "i32"), ("i32", "i32"), ("bf16", "f32"),
                                       ("bf16", "bf16"), ("f32", "f32")])
@pytest.mark.parametrize("case", range(len(CONTRACTIONS)))
def test_contraction_parity(b200, case, dtype, out):
    l, r, p, o, ax = CONTRACTIONS[case]
    (L, rl), (R, rr), (P, rp), (O, ro) = (pair(e, **ax) for e in (l, r, p, o))
    if dtype == "i4" and (L.size % 2 or R.size % 2):
        pytest.skip("odd i4 count")
    lv, rv = rand_vals(dtype, L.size), rand_vals(dtype, R.size)
    if dtype == "i32":
        lv, rv = (lv >> 20).astype(np.int32), (rv >> 20).astype(np.int32)
    a, b = b200.from_vec(L, lv, dtype), b200.from_vec(R, rv, dtype)
    got = b200._contract(a, b, L, R, P, O, out).to_bytes()
    want = oracle.contract(dtypes.to_bytes(lv, dtype), dtypes.to_bytes(rv, dtype), dtype, out, rl, rr, rp, ro)
    if dtype in ("bf16", "f32"):
        g = np.frombuffer(got, np.float32) if out == "f32" else dtypes.bf16_bits_to_f32(np.frombuffer(got, np.uint16))
        w = np.frombuffer(want, np.float32) if out == "f32" else dtypes.bf16_bits_to_f32(np.frombuffer(want, np.uint16))
        # tensor-core paths sum in a different order: |err| <= 2^-6 relative-to-|sum| bound, max-abs reported
        k = rl.size * rr.size // max(ro.size, 1)
        tol = 1e-5 * np.sqrt(max(k, 1)) * 8 + (2 ** -7 if out == "bf16" else 0) * np.abs(w)  # 1 bf16 ulp
        assert np.all(np.abs(g - w) <= tol + 1e-5), f"max abs err {np.max(np.abs(g - w))}"
    else:
        assert got == want


def test_contraction_requant_epilogue(b200):
    ax = dict(M=64, K=192, N=96)
    (L, rl), (R, rr), (P, rp), (O, ro) = (pair(e, **ax) for e in ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]"))
    lv, rv = rand_vals("i8", L.size), rand_vals("i8", R.size)
    scale = RNG.uniform(0.001, 0.01, 96).astype(np.float32)
    sm = fb.Mapping("[N]", dict(N=96))
    s = b200.from_vec(sm, scale, "f32")
    got = b200.contraction_requant(b200.from_vec(L, lv, "i8"), b200.from_vec(R, rv, "i8"), L, R, P, O, s, "N")
    want = oracle.contract(lv.tobytes(), rv.tobytes(), "i8", "i8", rl, rr, rp, ro, ep_kind=1, scale=scale,
                           scale_axis="N")
    assert got.to_bytes() == want


# ---------------------------------------------------------------------------------------------
# transmute / gather / scatter
# ---------------------------------------------------------------------------------------------
def test_transmute(b200):
    ax = dict(A=5, B=6)
    S = fb.Mapping("[A, B # 8]", ax)
    D = fb.Mapping("[[A, B] # 32]", ax)
    vals = rand_vals("i32", S.size)
    got = b200.transmute(b200.from_vec(S, vals, "i32"), S, D).to_numpy()
    rs, rd = ref_m("[A, B # 8]", **ax), ref_m("[[A, B] # 32]", **ax)
    live = vals[rs.cells()[0] == 0]
    want = np.zeros(D.size, np.int32)
    want[rd.cells()[0] == 0] = live
    assert np.array_equal(got, want)


def test_gather_rows(b200):
    # table [T, E] rows indexed by idx [I] -> out [I, E] (buf.rs:524-576, unscaled indices)
    ax = dict(T=50, E=16, I=20)
    Src, Dst = fb.Mapping("[T, E]", ax), fb.Mapping("[I, E]", ax)
    payload, axis, Idx = fb.Mapping("[E]", ax), fb.Mapping("[T]", ax), fb.Mapping("[I]", ax)
    table = rand_vals("bf16", Src.size)
    idx = RNG.integers(0, 50, 20).astype(np.int32)
    out = b200.zeroed(Dst, "bf16")
    b200.gather(b200.from_vec(Src, table, "bf16"), out, b200.from_vec(Idx, idx, "i32"), Src, Dst, payload, axis, Idx)
    assert np.array_equal(out.to_numpy().reshape(20, 16), table.reshape(50, 16)[idx])
    # scaled: byte offsets of payload-sized rows
    out2 = b200.zeroed(Dst, "bf16")
    b200.gather(b200.from_vec(Src, table, "bf16"), out2, b200.from_vec(Idx, idx * 32, "i32"), Src, Dst, payload, axis,
                Idx, scaled=True)
    assert np.array_equal(out2.to_numpy(), out.to_numpy())


def test_scatter_last_write_wins(b200):
    ax = dict(K=6, E=8, T=4)
    Src, Dst = fb.Mapping("[K, E]", ax), fb.Mapping("[T, E]", ax)
    payload, key, axis = fb.Mapping("[E]", ax), fb.Mapping("[K]", ax), fb.Mapping("[T]", ax)
    src = rand_vals("i32", Src.size)
    idx = np.array([1, 3, 1, 0, 3, 1], np.int32)
    canvas = rand_vals("i32", Dst.size)
    dst = b200.from_vec(Dst, canvas, "i32")
    b200.scatter(b200.from_vec(Src, src, "i32"), dst, b200.from_vec(key, idx, "i32"), Src, Dst, payload, key, axis)
    want = canvas.reshape(4, 8).copy()
    for k in range(6):  # serial, key order (buf.rs:512-519)
        want[idx[k]] = src.reshape(6, 8)[k]
    assert np.array_equal(dst.to_numpy().reshape(4, 8), want)


def test_gather_rejects_negative_index(b200):
    ax = dict(T=4, E=4, I=2)
    Src, Dst = fb.Mapping("[T, E]", ax), fb.Mapping("[I, E]", ax)
    with pytest.raises(fb._lib.FoptError):
        b200.gather(b200.zeroed(Src, "i32"), b200.zeroed(Dst, "i32"),
                    b200.from_vec(fb.Mapping("[I]", ax), np.array([0, -1], np.int32), "i32"), Src, Dst,
                    fb.Mapping("[E]", ax), fb.Mapping("[T]", ax), fb.Mapping("[I]", ax))


# ---------------------------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------------------------
@pytest.fixture(params=["paired", "one_tile", "split_rows"])
def attn_kernel(request, monkeypatch):
    """Each tcgen05 attention kernel, forced: the two-query-tile kernel (FOPT_ATTN_PAIRED; the default
    beyond S = 1024 when S % 256 == 0), the one-tile kernel (FOPT_ATTN_ONE_TILE, which also serves odd
    block counts) and the persistent kernel with two threads per row (FOPT_ATTN_SPLIT_ROWS; the
    default up to S = 1024)."""
    monkeypatch.delenv("FOPT_ATTN_ONE_TILE", raising=False)
    monkeypatch.delenv("FOPT_ATTN_SPLIT_ROWS", raising=False)
    monkeypatch.delenv("FOPT_ATTN_PAIRED", raising=False)
    if request.param == "paired":
        monkeypatch.setenv("FOPT_ATTN_PAIRED", "1")
    elif request.param == "one_tile":
        monkeypatch.setenv("FOPT_ATTN_ONE_TILE", "1")
    elif request.param == "split_rows":
        monkeypatch.setenv("FOPT_ATTN_SPLIT_ROWS", "1")
    return request.param


def _attention_check(b200, q, k, v, B, S, Hq, Hkv, causal, D=128, chain=True):
    """Checks the kernel against two restatements and prints the errors:
      * the plain f32 online softmax (oracle.attention): 2 bf16 ulps of the value plus 1e-2;
      * the reference's own op chain (oracle.attention_chain, attention.rs:32-392), which rounds the
        logits, the weights, the 16-key partials and the running output to bf16 and adds EPS per
        512-key chunk: 2^-5 |w| + 0.04. For N(0, 1) inputs at D = 128 the chain's own distance from
        exact attention is about 0.017 (max abs), and the kernel's (f32 logits, bf16 P) is below
        0.008, so the bound holds both with room. Not applied when the logits reach magnitudes where
        the chain's bf16 logits are coarse (chain=False)."""
    mq = fb.Mapping("[B, S, H, D]", dict(B=B, S=S, H=Hq, D=D))
    mk = fb.Mapping("[B, S, H, D]", dict(B=B, S=S, H=Hkv, D=D))
    o = b200.attention(b200.from_vec(mq, q, "bf16"), b200.from_vec(mk, k, "bf16"), b200.from_vec(mk, v, "bf16"), B, S,
                       Hq, Hkv, D, causal=causal).to_numpy()
    g = dtypes.bf16_bits_to_f32(o)
    want = oracle.attention(q, k, v, B, S, Hq, Hkv, D, D ** -0.5, causal)
    w = dtypes.bf16_bits_to_f32(want)
    err = np.abs(g - w)
    rel = err / np.maximum(np.abs(w), 2 ** -4)
    print(f"attention B={B} S={S} Hq={Hq} Hkv={Hkv} causal={causal}: vs f32 online softmax max abs {err.max():.3g}, "
          f"max rel (|w| >= 1/16 floor) {rel.max():.3g}")
    assert np.all(err <= 2 ** -7 * np.abs(w) + 1e-2), f"max abs err {err.max()}"
    if chain:
        wc = dtypes.bf16_bits_to_f32(oracle.attention_chain(q, k, v, B, S, Hq, Hkv, D, causal))
        errc = np.abs(g - wc)
        relc = errc / np.maximum(np.abs(wc), 2 ** -4)
        print(f"  vs the reference chain: max abs {errc.max():.3g}, max rel {relc.max():.3g}")
        assert np.all(errc <= 2 ** -5 * np.abs(wc) + 0.04), f"max abs err vs chain {errc.max()}"


def test_attention_growing_scores(b200, attn_kernel):
    """Keys whose magnitude grows along the sequence, so a row's running max keeps rising by more
    than 2^8 between key blocks: every rescaling path of the online softmax runs."""
    B, S, Hq, Hkv, D = 1, 1024, 4, 2, 128
    rng = np.random.default_rng(21)
    q = dtypes.f32_to_bf16_bits(rng.standard_normal(B * S * Hq * D).astype(np.float32))
    grow = (1.0 + np.arange(S, dtype=np.float32) / 32.0)[None, :, None, None]
    k = dtypes.f32_to_bf16_bits((rng.standard_normal((B, S, Hkv, D)).astype(np.float32) * grow).reshape(-1))
    v = dtypes.f32_to_bf16_bits(rng.standard_normal(B * S * Hkv * D).astype(np.float32))
    _attention_check(b200, q, k, v, B, S, Hq, Hkv, True, chain=False)


@pytest.mark.parametrize("B,S,Hq,Hkv,causal", [(1, 128, 4, 2, True), (1, 200, 8, 2, True), (1, 96, 2, 2, False),
                                               (1, 512, 8, 2, True), (2, 384, 4, 1, True), (2, 256, 4, 4, False),
                                               (1, 1024, 8, 2, False)])
def test_attention_parity(b200, attn_kernel, B, S, Hq, Hkv, causal):
    """S % 128 == 0 runs a tcgen05 kernel (multi-block online softmax, GQA, batches); other S the
    CUDA-core kernel."""
    D = 128
    q = rand_vals("bf16", B * S * Hq * D)
    k = rand_vals("bf16", B * S * Hkv * D)
    v = rand_vals("bf16", B * S * Hkv * D)
    _attention_check(b200, q, k, v, B, S, Hq, Hkv, causal, D)


def test_attention_config3_shape(b200, attn_kernel):
    """Config 3 at its own shape: Llama-3-8B prefill, batch 1, seq 2048, 32 query / 8 KV heads,
    D = 128, bf16 N(0, 1), causal, scale 1/sqrt(128)."""
    B, S, Hq, Hkv, D = 1, 2048, 32, 8, 128
    rng = np.random.default_rng(2048)
    q = dtypes.f32_to_bf16_bits(rng.standard_normal(B * S * Hq * D).astype(np.float32))
    k = dtypes.f32_to_bf16_bits(rng.standard_normal(B * S * Hkv * D).astype(np.float32))
    v = dtypes.f32_to_bf16_bits(rng.standard_normal(B * S * Hkv * D).astype(np.float32))
    _attention_check(b200, q, k, v, B, S, Hq, Hkv, True, D)


@pytest.fixture(params=["pair256", "pair128", "single"])
def gemm_tile(request, monkeypatch):
    """Runs a tensor-core GEMM test through each kernel shape: CTA pairs on 256 x 256 or 256 x 128
    tiles, and the single-CTA kernel."""
    monkeypatch.delenv("FOPT_GEMM_1SM", raising=False)
    monkeypatch.delenv("FOPT_GEMM_BN", raising=False)
    if request.param == "single":
        monkeypatch.setenv("FOPT_GEMM_1SM", "1")
    else:
        monkeypatch.setenv("FOPT_GEMM_BN", request.param[4:])
    return request.param


@pytest.mark.parametrize("shape", [(2048, 256, 2560), (512, 384, 384), (512, 2048, 2560), (256, 2048, 256)])
def test_gemm_tc_requant_large_grid(b200, gemm_tile, shape):
    # more tiles than SMs: exercises the persistent tile loop and both TMEM accumulators; the second
    # shape has N % 256 != 0, so the paired kernel runs 256 x 128 tiles whatever is asked; the last
    # two fill less than one wave over the SM pairs with K long enough, so their tiles run split into K-ranges
    M, K, N = shape
    ax = dict(M=M, K=K, N=N)
    (L, rl), (R, rr), (P, rp), (O, ro) = (pair(e, **ax) for e in ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]"))
    lv, rv = rand_vals("i8", L.size), rand_vals("i8", R.size)
    scale = RNG.uniform(0.001, 0.01, N).astype(np.float32)
    s = b200.from_vec(fb.Mapping("[N]", dict(N=N)), scale, "f32")
    got = b200.contraction_requant(b200.from_vec(L, lv, "i8"), b200.from_vec(R, rv, "i8"), L, R, P, O, s, "N")
    want = oracle.contract(lv.tobytes(), rv.tobytes(), "i8", "i8", rl, rr, rp, ro, ep_kind=1, scale=scale,
                           scale_axis="N")
    assert got.to_bytes() == want


@pytest.mark.parametrize("dtype,K", [("i8", 4096), ("bf16", 4096), ("i8", 16384), ("bf16", 12288)])
def test_gemm_full_size_properties(b200, gemm_tile, dtype, K):
    """Config 2 at full size (M=N=K=4096), and long-K shapes whose last wave runs split into K-ranges:
    size-independent checks instead of the slow oracle -- exact row / column checksums (linearity)
    of the i32 result and 8 sampled rows in full."""
    M = N = 4096
    ax = dict(M=M, N=N, K=K)
    L, R, P, O = (fb.Mapping(e, ax) for e in ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]"))
    rng = np.random.default_rng(7)
    if dtype == "i8":
        a = rng.integers(-128, 128, M * K).astype(np.int8)
        b = rng.integers(-128, 128, N * K).astype(np.int8)
        out = b200.contraction_wide(b200.from_vec(L, a, "i8"), b200.from_vec(R, b, "i8"), L, R, P, O).to_numpy()
        D = out.reshape(M, N).astype(np.int64)
        A, B = a.reshape(M, K).astype(np.int64), b.reshape(N, K).astype(np.int64)
        assert np.array_equal(D.sum(1), A @ B.sum(0))
        assert np.array_equal(D.sum(0), B @ A.sum(0))
        rows = rng.choice(M, 8, replace=False)
        assert np.array_equal(D[rows], A[rows] @ B.T)
    else:
        a = dtypes.f32_to_bf16_bits(rng.standard_normal(M * K).astype(np.float32))
        b = dtypes.f32_to_bf16_bits(rng.standard_normal(N * K).astype(np.float32))
        out = b200.contraction_wide(b200.from_vec(L, a, "bf16"), b200.from_vec(R, b, "bf16"), L, R, P, O).to_numpy()
        D = out.reshape(M, N).astype(np.float64)
        A = dtypes.bf16_bits_to_f32(a).reshape(M, K).astype(np.float64)
        B = dtypes.bf16_bits_to_f32(b).reshape(N, K).astype(np.float64)
        rows = rng.choice(M, 8, replace=False)
        ref = A[rows] @ B.T
        # f32 accumulation of K N(0,1) products: |err| <= 1e-4 * sqrt(K) * rms
        assert np.max(np.abs(D[rows] - ref)) <= 1e-4 * np.sqrt(K) * 2, np.max(np.abs(D[rows] - ref))
        # a row sum adds N such errors, which add up like a random walk
        assert np.allclose(D.sum(1), A @ B.sum(0), rtol=1e-3, atol=max(1.0, 2e-4 * np.sqrt(K) * np.sqrt(N)))


@pytest.fixture(params=["tensor_core", "generic"])
def contract_path(request, monkeypatch):
    """Runs a contraction test through the tensor-core GEMM and through the generic fold kernel."""
    if request.param == "generic":
        monkeypatch.setenv("FOPT_DISABLE_TC", "1")
    else:
        monkeypatch.delenv("FOPT_DISABLE_TC", raising=False)
    return request.param


@pytest.mark.parametrize("iw", [31, 24])
def test_gemm_tc_requant_ties_and_saturation(b200, contract_path, iw):
    """Requant on values that hit exact .5 ties (round half away from zero), huge and negative scales
    (saturation into the Clip), NaN scales (saturate by sign, then clip) and infinite scales times a
    zero accumulator (the x86 default NaN, which is negative)."""
    ax = dict(M=256, K=256, N=256)
    (L, rl), (R, rr), (P, rp), (O, ro) = (pair(e, **ax) for e in ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]"))
    lv, rv = rand_vals("i8", L.size), rand_vals("i8", R.size)
    scale = np.tile(np.array([0.5, 0.25, -0.5, 1e30, -1e30, 0.0078125, 1.5, -0.125], np.float32), 32)
    scale[7] = np.float32("nan")
    scale[15] = -np.float32("nan")
    scale[16], scale[17] = np.float32("inf"), -np.float32("inf")  # 0 * inf: the x86 default NaN is negative
    lv = lv.copy()
    lv.reshape(256, 256)[::7] = 0  # zero rows: accumulators of exactly 0
    s = b200.from_vec(fb.Mapping("[N]", dict(N=256)), scale, "f32")
    for lo, hi in ((-128, 127), (-20, 50)):
        got = b200.contraction_requant(b200.from_vec(L, lv, "i8"), b200.from_vec(R, rv, "i8"), L, R, P, O, s, "N",
                                       int_width=iw, lo=lo, hi=hi)
        want = oracle.contract(lv.tobytes(), rv.tobytes(), "i8", "i8", rl, rr, rp, ro, ep_kind=1, scale=scale,
                               scale_axis="N", int_width=iw, clip_lo=lo, clip_hi=hi)
        assert got.to_bytes() == want


def test_gemm_tc_requant_near_ties(b200, contract_path):
    """Round half away from zero next to the ties: accumulators -128 .. 127 (one per row) times
    scales within an ulp of k + 1/2 over small integers, and of 1/3, 2/3, 1/7."""
    M, K, N = 256, 128, 256
    ax = dict(M=M, K=K, N=N)
    (L, rl), (R, rr), (P, rp), (O, ro) = (pair(e, **ax) for e in ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]"))
    a = np.zeros((M, K), np.int8)
    a[:, 0] = np.arange(-128, 128)  # acc[m, n] = a[m, 0] * 1
    b = np.zeros((N, K), np.int8)
    b[:, 0] = 1
    base = []
    for num in (0.5, 1.5, 2.5, 0.25, 0.75, 1 / 3, 2 / 3, 1 / 7, 1.0, 0.1):
        f = np.float32(num)
        base += [f, np.nextafter(f, np.float32(0)), np.nextafter(f, np.float32(2))]
    scale = np.resize(np.array(base, np.float32), N)
    scale[1::2] *= -1
    s = b200.from_vec(fb.Mapping("[N]", dict(N=N)), scale, "f32")
    got = b200.contraction_requant(b200.from_vec(L, a.reshape(-1), "i8"), b200.from_vec(R, b.reshape(-1), "i8"),
                                   L, R, P, O, s, "N", lo=-128, hi=127)
    want = oracle.contract(a.tobytes(), b.tobytes(), "i8", "i8", rl, rr, rp, ro, ep_kind=1, scale=scale,
                           scale_axis="N", clip_lo=-128, clip_hi=127)
    assert got.to_bytes() == want


@pytest.mark.parametrize("iw", [0, 1, 4, 16, 24, 30, 31])
def test_fp_to_fxp_edges(b200, iw):
    """float_to_fixedpoint on ties, near-saturation and tiny values (float/mod.rs:99-111)."""
    rng = np.random.default_rng(iw)
    scale = 2.0 ** (31 - iw)
    ties = ((np.arange(-64, 64) + 0.5) / scale).astype(np.float32)
    near = (np.array([2 ** 31 - 128, 2 ** 31, 2 ** 31 + 256, -2 ** 31, -2 ** 31 - 256, 2 ** 24 + 1]) / scale)
    vals = np.concatenate([ties, near.astype(np.float32), rng.standard_normal(3000).astype(np.float32) * 100,
                           np.array([0.0, -0.0, 1e-30, -1e-30, np.inf, -np.inf, np.nan], np.float32)])
    vals = vals.astype(np.float32)
    got, want = _ew_case(b200, ops.fp_to_fxp(iw), ["f32"], "i32", n=len(vals), values=[vals])
    assert got == want


# ---------------------------------------------------------------------------------------------
# host I/O
# ---------------------------------------------------------------------------------------------
def test_from_safetensors_streams_to_device(b200, tmp_path):
    """HostTensor::from_safetensors + to_hbm in one step: bytes land unchanged (a 40 MiB tensor
    crosses several pinned staging chunks), the shape is checked against the mapping's pair-split
    sizes, and the byte count against the mapping's image."""
    import json
    import struct
    rng = np.random.default_rng(9)
    big = rng.integers(0, 2 ** 16, 20 * 1024 * 1024, dtype=np.int64).astype(np.uint16)  # bf16 bits
    small = rng.standard_normal((24, 16)).astype(np.float32)
    header = {"big": {"dtype": "BF16", "shape": [5120, 4096], "data_offsets": [0, big.nbytes]},
              "small": {"dtype": "F32", "shape": [24, 16], "data_offsets": [big.nbytes, big.nbytes + small.nbytes]}}
    text = json.dumps(header).encode()
    p = tmp_path / "w.safetensors"
    p.write_bytes(struct.pack("<Q", len(text)) + text + big.tobytes() + small.tobytes())
    with fb.SafeTensors(str(p)) as st:
        B = b200.from_safetensors(st, "big", fb.Mapping("[R, C]", dict(R=5120, C=4096)))
        S = b200.from_safetensors(st, "small", fb.Mapping("[A, B]", dict(A=24, B=16)), dtype="f32")
        with pytest.raises(ValueError):
            b200.from_safetensors(st, "small", fb.Mapping("[B, A]", dict(A=24, B=16)))
    assert B.to_bytes() == big.tobytes()
    assert S.to_bytes() == small.tobytes()


@pytest.mark.parametrize("shape", [(1024, 512, 768), (96, 64, 40)])
def test_contraction_host_buffers(b200, shape):
    """One call from host buffers to a host result: the row-chunk pipeline (GEMM shape) and the plain
    path (other shapes) give the device contraction's bytes, for requant and plain i32 outputs."""
    M, K, N = shape
    ax = dict(M=M, K=K, N=N)
    L, R, P, O = (fb.Mapping(e, ax) for e in ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]"))
    rng = np.random.default_rng(M)
    a = rng.integers(-128, 128, M * K).astype(np.int8)
    b = rng.integers(-128, 128, N * K).astype(np.int8)
    scale = rng.uniform(0.001, 0.01, N).astype(np.float32)
    S = b200.from_vec(fb.Mapping("[N]", ax), scale, "f32")
    A, B = b200.from_vec(L, a, "i8"), b200.from_vec(R, b, "i8")
    want_rq = b200.contraction_requant(A, B, L, R, P, O, S, "N").to_bytes()
    want_w = b200.contraction_wide(A, B, L, R, P, O).to_bytes()
    ep = fb.backend._ep(1, S, "N")
    assert b200.contraction_host(a, b, L, R, P, O, "i8", "i8", ep=ep).tobytes() == want_rq
    assert b200.contraction_host(a, b, L, R, P, O, "i8", "i32").tobytes() == want_w


# ---------------------------------------------------------------------------------------------
# row programs (engine-chain fusion across a row reduction)
# ---------------------------------------------------------------------------------------------
def _rms_quant_chain(be, x_bf16, g_f32, T, Wd):
    """RMSNorm then per-token int8 quantisation, as the decoder block writes it."""
    from furiosa_opt_b200 import workloads as Wl
    ax = dict(T=T, H=Wd)
    m = lambda e: fb.Mapping(e, ax)  # noqa: E731
    x = be.from_vec(m("[T, H]"), x_bf16, "bf16")
    g = be.relayout(be.from_vec(m("[H]"), g_f32, "f32"), m("[H]"), m("[T, H]"), True)
    xf = be.map(x, ops.cast("bf16", "f32"), "f32")
    sq = be.zip_with(xf, xf, ops.fp_binary("MulF"), "f32")
    ss = be.reduce(sq, "Add", 0.0, m("[T, H]"), m("[T]"))
    rinv = be.map(ss, Wl._prog_rinv(Wd), "f32")
    xn = be.zip3_with(xf, be.relayout(rinv, m("[T]"), m("[T, H]"), True), g, Wl._prog_scale3(), "f32")
    amax = be.reduce(be.map(xn, Wl._prog_abs(), "f32"), "Max", 0.0, m("[T, H]"), m("[T]"))
    s = be.map(amax, Wl._prog_token_scale(), "f32")
    q = be.zip_with(xn, be.relayout(s, m("[T]"), m("[T, H]"), True), Wl._prog_quant(), "i8")
    return q, s, ss, rinv


@pytest.fixture
def row_toggle(b200):
    saved = b200.row_fusion
    yield b200
    b200.row_fusion = saved


@pytest.mark.parametrize("T,Wd", [(96, 4096), (7, 4360), (33, 2048 * 16), (5, 8)])
def test_row_program_rmsnorm_quant_matches_unfused(row_toggle, T, Wd):
    """One row program (one launch) computes the bits of the unfused chain: the quantised values,
    the token scales and the intermediate per-row sums and reciprocals it writes out. Widths cover
    a partial last group of 2048, a width whose held value exceeds the register budget (read again
    from cache instead) and a single 8-element group."""
    be = row_toggle
    rng = np.random.default_rng(T + Wd)
    x = dtypes.f32_to_bf16_bits((rng.standard_normal(T * Wd) * rng.uniform(0.1, 4, T).repeat(Wd)).astype(np.float32))
    x[:Wd] = dtypes.f32_to_bf16_bits(np.zeros(Wd, np.float32))  # an all-zero row: the scale clamps
    g = (1.0 + 0.1 * rng.standard_normal(Wd)).astype(np.float32)
    be.row_fusion = True
    before = _lib.lib().fopt_elementwise_jit_launches()
    q, s, ss, rinv = _rms_quant_chain(be, x, g, T, Wd)
    fused = [q.to_bytes(), s.to_bytes(), ss.to_bytes(), rinv.to_bytes()]
    assert _lib.lib().fopt_elementwise_jit_launches() == before + 1
    be.row_fusion = False
    q2, s2, ss2, rinv2 = _rms_quant_chain(be, x, g, T, Wd)
    assert fused == [q2.to_bytes(), s2.to_bytes(), ss2.to_bytes(), rinv2.to_bytes()]
    # and against the arithmetic in numpy (f32 sums reassociate: scale within 1e-5 relative)
    xf = dtypes.bf16_bits_to_f32(x).reshape(T, Wd).astype(np.float64)
    want_ss = (xf * xf).sum(1)
    assert np.allclose(np.frombuffer(fused[2], np.float32), want_ss, rtol=1e-4, atol=1e-30)


def test_row_program_i32_folds_and_loads(row_toggle):
    """i32 folds (wrapping Add, Min), a per-row value already written out (a LOAD slot) and a
    repeated-row leaf, at a width that is not a multiple of 2048."""
    be = row_toggle
    T, Wd = 40, 3000
    ax = dict(T=T, H=Wd)
    m = lambda e: fb.Mapping(e, ax)  # noqa: E731
    rng = np.random.default_rng(11)
    a = rng.integers(-2**31, 2**31, T * Wd, dtype=np.int64).astype(np.int32)
    c = rng.integers(-1000, 1000, Wd).astype(np.int32)
    off = rng.integers(-50, 50, T).astype(np.int32)

    def chain():
        A = be.from_vec(m("[T, H]"), a, "i32")
        Cb = be.relayout(be.from_vec(m("[H]"), c, "i32"), m("[H]"), m("[T, H]"), True)
        Ob = be.relayout(be.from_vec(m("[T]"), off, "i32"), m("[T]"), m("[T, H]"), True)
        v = be.zip3_with(A, Cb, Ob, _add3(), "i32")
        tot = be.reduce(v, "Add", 0, m("[T, H]"), m("[T]"))
        lo = be.reduce(v, "Min", 2**31 - 1, m("[T, H]"), m("[T]"))
        p = ops.Prog(2)
        d = be.zip_with(tot, lo, p.build(p.emit("SUB_FXP", 0, 1)), "i32")
        p = ops.Prog(2)
        out = be.zip_with(v, be.relayout(d, m("[T]"), m("[T, H]"), True), p.build(p.emit("XOR", 0, 1)), "i16")
        return out.to_bytes(), tot.to_bytes(), lo.to_bytes()

    be.row_fusion = True
    fused = chain()
    be.row_fusion = False
    assert fused == chain()
    v = (a.reshape(T, Wd).astype(np.int64) + c[None, :] + off[:, None]).astype(np.int32)
    assert np.array_equal(np.frombuffer(fused[1], np.int32), v.astype(np.int64).sum(1).astype(np.int32))
    assert np.array_equal(np.frombuffer(fused[2], np.int32), v.min(1))


def _add3():
    p = ops.Prog(3)
    return p.build(p.emit("ADD_FXP", p.emit("ADD_FXP", 0, 1), 2))


def test_row_program_falls_back_through_origin(row_toggle, monkeypatch):
    """With row programs off, a value composed from more than 3 leaves runs through its origin
    (its deferred inputs written first) and matches the chain run op by op."""
    be = row_toggle
    T, Wd = 16, 256
    rng = np.random.default_rng(2)
    x = dtypes.f32_to_bf16_bits(rng.standard_normal(T * Wd).astype(np.float32))
    g = rng.uniform(0.5, 1.5, Wd).astype(np.float32)
    be.row_fusion = False
    q, s, _, _ = _rms_quant_chain(be, x, g, T, Wd)
    monkeypatch.setenv("FOPT_NO_FUSION", "1")
    eager = fb.B200(0)
    q2, s2, _, _ = _rms_quant_chain(eager, x, g, T, Wd)
    # the eager chain sums its squares with the general reduce (another f32 order): scales agree
    # to rounding, quantised values within one step
    assert np.allclose(s.to_numpy(), s2.to_numpy(), rtol=1e-5)
    d = np.abs(q.to_numpy().astype(np.int32) - q2.to_numpy().astype(np.int32))
    assert d.max() <= 1 and (d > 0).mean() < 1e-3


def test_decoder_block_row_programs_bit_exact(row_toggle):
    """The decoder block with row programs equals the block without them bit for bit, in fewer
    launches."""
    from furiosa_opt_b200 import workloads as Wl
    be = row_toggle
    batch, seq, Hq, Hkv, F = 2, 128, 4, 2, 1024
    T, H = batch * seq, Hq * 128
    blk = Wl.DecoderBlockW8A8(be, T, H, Hq, Hkv, F, batch, seq, seed=3)
    x = dtypes.f32_to_bf16_bits(np.random.default_rng(5).standard_normal(T * H).astype(np.float32))
    outs, launches = [], []
    for on in (True, False):
        be.row_fusion = on
        n0 = be.launches
        outs.append(blk.forward(be.from_vec(blk.m("[T, H]"), x, "bf16")).to_bytes())
        launches.append(be.launches - n0)
    assert outs[0] == outs[1]
    assert launches[0] < launches[1], launches


def test_row_program_quantise_near_ties(row_toggle):
    """Per-token quantisation through a row program (its division by the per-row scale runs as a
    reciprocal product with an exact fallback near rounding ties) equals the unfused chain's exact
    division bit for bit, on values placed within a few ulps of half-integer quotients, exact
    ties, zeros, huge values and rows whose scale is 0 or NaN."""
    from furiosa_opt_b200 import workloads as Wl
    be = row_toggle
    T, Wd = 64, 1024
    rng = np.random.default_rng(21)
    x = (rng.standard_normal((T, Wd)) * rng.uniform(0.01, 100, (T, 1))).astype(np.float32)
    amax = np.abs(x).max(1)
    s = np.maximum(amax, np.float32(1e-12)) / np.float32(127)
    k = rng.integers(-127, 127, (T, Wd)).astype(np.float32) + np.float32(0.5)
    near = (k * s[:, None]).astype(np.float32)
    ulps = rng.integers(-3, 4, (T, Wd)).astype(np.int32)
    near = (near.view(np.int32) + ulps).view(np.float32)
    pick = rng.random((T, Wd)) < 0.5
    x = np.where(pick, near, x).astype(np.float32)
    x[:, 0] = amax  # keep each row's max where it was, so the scale stays s
    x[1, :] = 0.0
    x[2, 5] = np.float32(3e38)
    x[3, :] = np.nan
    ax = dict(T=T, H=Wd)
    m = lambda e: fb.Mapping(e, ax)  # noqa: E731

    def chain():
        X = be.from_vec(m("[T, H]"), x.reshape(-1), "f32")
        a = be.map(be.map(X, Wl._prog_abs(), "f32"), ops.Prog(1).build(0), "f32")
        mx = be.reduce(a, "Max", 0.0, m("[T, H]"), m("[T]"))
        sc = be.map(mx, Wl._prog_token_scale(), "f32")
        xd = be.map(X, ops.Prog(1).build(0), "f32")  # a deferred value, so the chain stays lazy
        q = be.zip_with(xd, be.relayout(sc, m("[T]"), m("[T, H]"), True), Wl._prog_quant(), "i8")
        return q.to_bytes(), sc.to_bytes()

    be.row_fusion = True
    before = _lib.lib().fopt_elementwise_jit_launches()
    fused = chain()
    assert _lib.lib().fopt_elementwise_jit_launches() == before + 1
    be.row_fusion = False
    assert fused == chain()
