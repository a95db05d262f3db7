"""Pins the CPU oracle to the reference's own known-answer tests (no GPU needed).

Every expected value below is transcribed from the reference test it cites; the oracle must
reproduce each one before it is trusted as the parity checker for the CUDA kernels.
"""
import os
import struct

import numpy as np
import pytest

import oracle
from oracle import ref_m

# ---------------------------------------------------------------------------------------------
# mapping semantics: docs/src/mapping-tensors/mapping-expressions.md asserts
# ---------------------------------------------------------------------------------------------


def test_doc_symbol():  # mapping-expressions.md:94-101
    E = ref_m("[A]", A=8)
    for i in range(8):
        assert E.map(i) == {"A": i}
    assert E.map(8) == "OutOfBounds"


def test_doc_pair():  # mapping-expressions.md:131-141
    E = ref_m("[A, B]", A=8, B=512)
    assert E.map(0) == {"A": 0, "B": 0}
    assert E.map(511) == {"A": 0, "B": 511}
    assert E.map(512) == {"A": 1, "B": 0}
    assert E.map(519) == {"A": 1, "B": 7}
    assert E.map(4096) == "OutOfBounds"


def test_doc_identity():  # mapping-expressions.md:163-166
    E = ref_m("[1]")
    assert E.map(0) == {}
    assert E.map(1) == "OutOfBounds"


def test_doc_padding():  # mapping-expressions.md:191-198
    E = ref_m("[C, D # 64]", C=13, D=61)
    assert E.map(0) == {"C": 0, "D": 0}
    assert E.map(60) == {"C": 0, "D": 60}
    for i in (61, 62, 63):
        assert E.map(i) == ("Padding", 2)  # PaddingKind::Top
    assert E.map(64) == {"C": 1, "D": 0}


def test_doc_resize():  # mapping-expressions.md:243-249
    E = ref_m("[C, D = 2]", C=2, D=3)
    assert [E.map(i) for i in range(4)] == [{"C": 0, "D": 0}, {"C": 0, "D": 1}, {"C": 1, "D": 0}, {"C": 1, "D": 1}]
    assert E.map(4) == "OutOfBounds"


def test_doc_stride_modulo():  # mapping-expressions.md:300-323
    E = ref_m("[B / 64, B % 64]", B=512)
    F = ref_m("[B]", B=512)
    assert E.map(130) == {"B": 130}
    for i in range(512):
        assert E.map(i) == F.map(i)
    assert E.map(512) == "OutOfBounds"
    D1 = ref_m("B / 64", B=512)
    assert [D1.map(i) for i in range(8)] == [{"B": 64 * i} for i in range(8)]
    assert D1.map(8) == "OutOfBounds"


def test_doc_nested_stride():  # mapping-expressions.md:361-381
    E = ref_m("[B / 64, B % 32, B / 32 % 2]", B=512)
    assert E.map(67) == {"B": 97}
    for i in range(8):
        for j in range(32):
            for k in range(2):
                assert E.map(64 * i + 2 * j + k) == {"B": 64 * i + j + 32 * k}
    assert E.map(512) == "OutOfBounds"


def test_doc_padding_kinds():  # mapping-expressions.md:208-216
    assert ref_m("[A #{0} 8]", A=5).map(6) == ("Padding", 1)
    assert ref_m("[A #{!} 8]", A=5).map(6) == ("Padding", 0)
    assert ref_m("[A #{*} 8]", A=5).map(6) == ("Padding", 2)


def test_doc_equivalences():  # mapping-expressions.md: Equivalent Mappings
    A, B = 4, 6
    base = ref_m("[A, B]", A=A, B=B)
    for e in ("[[A, B] / 1]", "[[A, B] # 24]", "[[A, B] = 24]", "[1, [A, B]]", "[[A, B], 1]"):
        m = ref_m(e, A=A, B=B)
        assert [m.map(i) for i in range(24)] == [base.map(i) for i in range(24)], e
    # a zero coordinate is the same index as an absent one (mapping-expressions.md:111-112)
    nz = lambda c: {k: v for k, v in c.items() if v} if isinstance(c, dict) else c
    assert [nz(ref_m("[[A, B] / 6]", A=A, B=B).map(i)) for i in range(4)] == [nz(ref_m("A", A=A).map(i)) for i in range(4)]
    assert [nz(ref_m("[[A, B] % 6]", A=A, B=B).map(i)) for i in range(6)] == [nz(ref_m("B", B=B).map(i)) for i in range(6)]


# ---------------------------------------------------------------------------------------------
# float rules: furiosa-opt-std/src/float/bf16.rs:47-76, cast.rs:451-467
# ---------------------------------------------------------------------------------------------
def _ew(op, a_bits, dt_in="f32", dt_out="f32", imm=0):
    insns = [(op, 1, 0, 0, 0, imm)]
    src = np.asarray(a_bits, dtype=np.uint32 if dt_in in ("f32", "i32") else np.uint16).tobytes()
    out = oracle.elementwise(insns, 1, [src], [dt_in], dt_out, len(a_bits))
    return np.frombuffer(out, dtype=np.uint32 if dt_out in ("f32", "i32") else np.uint16)


F32_MIN_POS = 0x00800000


def test_bf16_subnormals_flush():  # bf16.rs:47-60
    half_min = struct.unpack("<I", struct.pack("<f", struct.unpack("<f", struct.pack("<I", F32_MIN_POS))[0] / 2))[0]
    r = _ew(2, [half_min, half_min | 0x80000000, F32_MIN_POS], "f32", "bf16")
    assert r[0] == 0x0000 and r[1] == 0x8000 and r[2] != 0
    w = _ew(1, [0x0001, 0x8001], "bf16", "f32")
    assert w[0] == 0 and w[1] == 0x80000000


def test_bf16_nan_canonical():  # bf16.rs:65-68
    assert _ew(2, [0x7FA00001], "f32", "bf16")[0] == 0x7FC0
    assert _ew(1, [0x7F81], "bf16", "f32")[0] == 0x7FC00000


def test_bf16_zero_and_normal():  # bf16.rs:72-76
    neg0 = 0x80000000
    r = _ew(2, [neg0, struct.unpack("<I", struct.pack("<f", 1.5))[0]], "f32", "bf16")
    assert r[0] == 0x8000 and r[1] == 0x3FC0
    w = _ew(1, [0xC020], "bf16", "f32")  # -2.5
    assert struct.unpack("<f", struct.pack("<I", int(w[0])))[0] == -2.5


def test_bf16_narrow_rne():  # cast.rs:451-467
    one_ulp = 2.0 ** -7
    vals = [1.0 + one_ulp / 2, 1.0 + one_ulp * 1.5, 1.0 + one_ulp * 0.75]
    bits = [struct.unpack("<I", struct.pack("<f", v))[0] for v in vals]
    r = _ew(2, bits, "f32", "bf16")
    got = [struct.unpack("<f", struct.pack("<I", int(x) << 16))[0] for x in r]
    assert got == [1.0, 1.0 + 2 * one_ulp, 1.0 + one_ulp]


def test_fixedpoint_roundtrip():  # float/mod.rs:99-139 (integers exact through iw=31)
    lib = oracle.lib()
    for v in (0, 1, -1, 7, 1 << 20, (1 << 24) + 1, -(1 << 30), 2 ** 31 - 1, -(2 ** 31)):
        f = struct.unpack("<f", struct.pack("<I", lib.ref_fxp_to_fp(v, 31)))[0]
        assert f == float(np.float32(v)), v
    assert lib.ref_fp_to_fxp(struct.unpack("<I", struct.pack("<f", 2.5))[0], 31) == 3  # half away from zero
    assert lib.ref_fp_to_fxp(struct.unpack("<I", struct.pack("<f", -2.5))[0], 31) == -3
    assert lib.ref_fp_to_fxp(0x7FC00000, 31) == 2 ** 31 - 1  # +NaN saturates high
    assert lib.ref_fp_to_fxp(struct.unpack("<I", struct.pack("<f", 0.5))[0], 0) == 2 ** 30  # Q31


def test_i32_accumulator_wraps():  # cast.rs:420-427, 431-447
    M, K, N = 1, 256, 1
    L, R = ref_m("[M, K]", M=M, K=K), ref_m("[K, N]", K=K, N=N)
    P, O = ref_m("[M, K, N]", M=M, K=K, N=N), ref_m("[M, N]", M=M, N=N)
    a = np.full(K, 100, np.int8).tobytes()
    wide = np.frombuffer(oracle.contract(a, a, "i8", "i32", L, R, P, O), np.int32)
    assert wide[0] == 256 * 100 * 100
    narrow = np.frombuffer(oracle.contract(a, a, "i8", "i8", L, R, P, O), np.int8)
    assert narrow[0] == np.int32(2_560_000).astype(np.int8)


# ---------------------------------------------------------------------------------------------
# storage: furiosa-opt-std/src/storage/buf.rs tests
# ---------------------------------------------------------------------------------------------
MKN = dict(M=2, K=3, N=2)


def _mkn(out="[M, N]", **ax):
    ax = ax or MKN
    return (ref_m("[M, K]", **ax), ref_m("[K, N]", **ax), ref_m("[M, K, N]", **ax), ref_m(out, **ax))


def test_contraction_matches_matmul():  # buf.rs:921-936
    L, R, P, O = _mkn()
    a = np.arange(1, 7, dtype=np.float32).tobytes()
    assert list(np.frombuffer(oracle.contract(a, a, "f32", "f32", L, R, P, O), np.float32)) == [22, 28, 49, 64]


def test_contraction_reordered_out():  # buf.rs:1066-1079
    L, R, P, O = _mkn("[N, M]")
    a = np.arange(1, 7, dtype=np.int32).tobytes()
    assert list(np.frombuffer(oracle.contract(a, a, "i32", "i32", L, R, P, O), np.int32)) == [22, 49, 28, 64]


def test_contraction_padded_contracted_axis():  # buf.rs:1086-1103
    ax = dict(M=2, K=2, N=2)
    L, R = ref_m("[M, K = 2 # 4]", **ax), ref_m("[K = 2 # 4, N]", **ax)
    P, O = ref_m("[M, K = 2 # 4, N]", **ax), ref_m("[M, N]", **ax)
    l = np.array([1, 2, 0, 0, 3, 4, 0, 0], np.int32).tobytes()
    r = np.array([1, 2, 3, 4, 0, 0, 0, 0], np.int32).tobytes()
    assert list(np.frombuffer(oracle.contract(l, r, "i32", "i32", L, R, P, O), np.int32)) == [7, 10, 15, 22]


def test_contraction_i8_wraps_once():  # buf.rs:1135-1146
    ax = dict(M=1, K=100, N=1)
    L, R, P, O = _mkn(**ax)
    a = np.full(100, 100, np.int8).tobytes()
    assert np.frombuffer(oracle.contract(a, a, "i8", "i8", L, R, P, O), np.int8)[0] == np.int32(1_000_000).astype(np.int8)


def test_contraction_bf16_wide_accumulator():  # buf.rs:1154-1176
    from_f = lambda v: (np.asarray(v, np.float32).view(np.uint32) >> 16).astype(np.uint16)  # exact values
    ax = dict(M=1, K=256, N=1)
    L, R, P, O = _mkn(**ax)
    lhs = from_f([1.0] + [1.0 / 128] * 255).tobytes()
    rhs = from_f([1.0] * 256).tobytes()
    got = np.frombuffer(oracle.contract(lhs, rhs, "bf16", "bf16", L, R, P, O), np.uint16)[0]
    gotf = struct.unpack("<f", struct.pack("<I", int(got) << 16))[0]
    assert abs(gotf - 2.9921875) <= 2.9921875 * 2 ** -7


def test_cross_slice_narrows_per_lane():  # buf.rs:1190-1232
    ax = dict(M=1, K=2, N=1)
    L, R, P, O = _mkn(**ax)
    bf = lambda v: (np.asarray(v, np.float32).view(np.uint32) >> 16).astype(np.uint16)
    part = np.frombuffer(oracle.contract(bf([1.0, 2 ** -8]).tobytes(), bf([1.0, 1.0]).tobytes(), "bf16", "bf16",
                                         L, R, P, O), np.uint16)[0]
    assert part == 0x3F80  # 1.0
    three = np.full(3, part, np.uint16).tobytes()
    s = ref_m("[Slice, M, N]", Slice=3, M=1, N=1)
    d = ref_m("[M, N]", M=1, N=1)
    cross = np.frombuffer(oracle.reduce(three, "bf16", 0, 0, s, d), np.uint16)[0]
    assert cross == 0x4040  # 3.0
    axg = dict(M=1, K=6, N=1)
    Lg, Rg, Pg, Og = _mkn(**axg)
    g = np.frombuffer(oracle.contract(bf([1.0, 2 ** -8] * 3).tobytes(), bf([1.0] * 6).tobytes(), "bf16", "bf16",
                                      Lg, Rg, Pg, Og), np.uint16)[0]
    assert struct.unpack("<f", struct.pack("<I", int(g) << 16))[0] == 3.015625


def test_reduce_large_split():  # buf.rs:968-979
    src = ref_m("[R, C]", R=256, C=512)
    dst = ref_m("[C]", C=512)
    data = (np.arange(256 * 512) % 5).astype(np.int32)
    got = np.frombuffer(oracle.reduce(data.tobytes(), "i32", 0, 0, src, dst), np.int32)
    assert np.array_equal(got, data.reshape(256, 512).sum(0))


def test_reduce_wide_out_thin():  # buf.rs:987-1002
    src = ref_m("[Big, Small]", Big=1 << 20, Small=4)
    dst = ref_m("[Big]", Big=1 << 20)
    data = (np.arange((1 << 20) * 4) % 7).astype(np.int32)
    got = np.frombuffer(oracle.reduce(data.tobytes(), "i32", 0, 0, src, dst), np.int32)
    assert np.array_equal(got, data.reshape(-1, 4).sum(1))


def test_contraction_large_split():  # buf.rs:1009-1030
    ax = dict(M=128, K=4, N=512)
    L, R, P, O = _mkn(**ax)
    lhs = (np.arange(128 * 4) % 5).astype(np.int32)
    rhs = (np.arange(4 * 512) % 3).astype(np.int32)
    got = np.frombuffer(oracle.contract(lhs.tobytes(), rhs.tobytes(), "i32", "i32", L, R, P, O), np.int32)
    assert np.array_equal(got, (lhs.reshape(128, 4) @ rhs.reshape(4, 512)).reshape(-1))


def test_transpose_large_split():  # buf.rs:1038-1059
    src, dst = ref_m("[R, C]", R=512, C=256), ref_m("[C, R]", R=512, C=256)
    data = np.arange(512 * 256, dtype=np.int32)
    got = np.frombuffer(oracle.transpose(bytes(512 * 256 * 4), data.tobytes(), "i32", src, dst), np.int32)
    assert np.array_equal(got, data.reshape(512, 256).T.reshape(-1))


def test_reduce_f32_close_to_serial():  # buf.rs:1240-1258
    src, dst = ref_m("[R, C]", R=256, C=512), ref_m("[C]", C=512)
    data = ((np.arange(256 * 512) % 13) * 0.5 + 0.25).astype(np.float32)
    got = np.frombuffer(oracle.reduce(data.tobytes(), "f32", 0, 0, src, dst), np.float32)
    want = data.astype(np.float64).reshape(256, 512).sum(0)
    assert np.all(np.abs(got - want) <= 1e-4 * np.maximum(np.abs(want), 1.0))


def test_transpose_broadcast_and_padding():  # buf.rs:268-313 (broadcast stride 0, write holes skipped)
    src = ref_m("[A]", A=4)
    dst = ref_m("[B, A # 6]", A=4, B=3)
    data = np.arange(1, 5, dtype=np.int32)
    canvas = np.full(18, -1, np.int32)
    got = np.frombuffer(oracle.transpose(canvas.tobytes(), data.tobytes(), "i32", src, dst, allow_broadcast=True),
                        np.int32)
    assert list(got) == [1, 2, 3, 4, -1, -1] * 3
    with pytest.raises(AssertionError):
        oracle.transpose(canvas.tobytes(), data.tobytes(), "i32", src, dst, allow_broadcast=False)


def test_fxp_to_fp_iw31_is_ieee_rne():
    """fixedpoint_to_float at int_width 31 equals IEEE round-to-nearest-even int -> f32, the fact
    the GEMM epilogue's fast path rests on (float/mod.rs:113-159)."""
    lib = oracle.lib()
    rng = np.random.default_rng(3)
    vals = np.concatenate([rng.integers(-2 ** 31, 2 ** 31, 200000, dtype=np.int64),
                           np.array([0, 1, -1, 2 ** 24, 2 ** 24 + 1, 2 ** 24 + 3, -(2 ** 24 + 1), 2 ** 25 + 2,
                                     2 ** 31 - 1, -(2 ** 31), -(2 ** 31) + 1, 16777217, 33554435])])
    for v in vals:
        got = lib.ref_fxp_to_fp(int(v), 31)
        assert got == int(np.float32(np.int32(v)).view(np.uint32)), int(v)


# furiosa-opt-examples/data/mnist/mnist.safetensors, committed as a fixture
MNIST_DATA = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "mnist.safetensors")


def _safetensors(path):
    import json
    import struct
    with open(path, "rb") as fh:
        raw = fh.read()
    n = struct.unpack("<Q", raw[:8])[0]
    head = json.loads(raw[8:8 + n])
    body = raw[8 + n:]
    return {k: body[v["data_offsets"][0]:v["data_offsets"][1]] for k, v in head.items() if k != "__metadata__"}


def test_mnist_bf16_reference_known_answers():
    """The reference's own end-to-end known answers (furiosa-opt-examples/tests/mnist_tests.rs:7-53):
    with its bf16 weights, the restated forward classifies all ten test images as labelled (the
    argmax over the first ten logits, as the test takes)."""
    from oracle.workloads_ref import mnist_bf16_ref
    t = _safetensors(MNIST_DATA)
    for i in range(10):
        logits = mnist_bf16_ref(t[f"hw.image_{i}"], t["hw.fc1.weight"], t["fc1.bias"], t["hw.fc2.weight"],
                                t["hw.fc2.bias"])
        f = (np.frombuffer(logits, np.uint16).astype(np.uint32) << 16).view(np.float32)[:10]
        assert int(np.argmax(f)) == int(np.frombuffer(t[f"label_{i}"], np.int32)[0]), i


# ---- 8-bit floats (float/f8e4.rs, float/f8e5.rs, scalar.rs:933-959) ----
def _f8_tables():
    import json
    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "f8_tables.json")) as fh:
        return json.load(fh)


def test_oracle_f8e4_decode_matches_reference_table():
    """The oracle's E4M3 decode, built from the value-set definition, equals the reference's
    256-entry table (f8e4.rs:67-101) entry by entry, NaN codes included."""
    want = np.array(_f8_tables()["F8E4_TO_F32"], np.uint32)
    got = oracle.f8_convert("f8e4m3_to_f32", np.arange(256))
    assert np.array_equal(got, want)


def test_oracle_f4e2m1_lookup_matches_reference_table():
    want = np.array(_f8_tables()["F4E2M1_TO_F8E4"], np.uint32)
    assert np.array_equal(oracle.f8_convert("f4e2m1_to_f8e4m3", np.arange(16)), want)


def test_oracle_f8e4_round_trips_full_range():
    """f8e4.rs:107-121: from_f32(to_f32(code)) == code for every non-NaN code."""
    codes = np.arange(256)
    wide = oracle.f8_convert("f8e4m3_to_f32", codes)
    back = oracle.f8_convert("f32_to_f8e4m3", wide)
    keep = ~np.isnan(wide.view(np.float32))
    assert keep.sum() == 254 and np.array_equal(back[keep], codes[keep])


def test_oracle_f8_known_values():
    """F8E4_ONE = 0x38 (f8e4.rs:8, :123-130), F8E5_ONE = 0x3c (f8e5.rs:8), the cast.rs:400-407 round
    trips of [-2, -1, 0, 0.5, 1, 2], the NaN codes, and the saturation / overflow rules."""
    f = lambda v: np.array(v, np.float32).view(np.uint32)
    e4 = lambda v: int(oracle.f8_convert("f32_to_f8e4m3", f([v]))[0])
    e5 = lambda v: int(oracle.f8_convert("f32_to_f8e5m2", f([v]))[0])
    assert e4(1.0) == 0x38 and e4(-1.0) == 0xb8 and e5(1.0) == 0x3c
    for kind in ("f8e4m3", "f8e5m2"):
        vals = f([-2.0, -1.0, 0.0, 0.5, 1.0, 2.0])
        codes = oracle.f8_convert(f"f32_to_{kind}", vals)
        assert np.array_equal(oracle.f8_convert(f"{kind}_to_f32", codes), vals)
    assert e4(float("nan")) == 0x7f and e4(-float("nan")) == 0x7f and e5(float("nan")) == 0x7e
    assert e4(448.0) == 0x7e and e4(1e9) == 0x7e and e4(float("inf")) == 0x7e and e4(-float("inf")) == 0xfe
    assert e4(464.0) == 0x7e and e4(440.0) == 0x7e and e4(424.0) == 0x7d  # 440 ties to 448 (even); 424 to 416
    assert e5(57344.0) == 0x7b and e5(61440.0) == 0x7c and e5(float("inf")) == 0x7c
    # E5M2 normals round half UP (f8e5.rs:56-66): 1 + 2^-3 is a tie between 1 and 1.25 -> 1.25
    assert e5(1.125) == 0x3d
    # E5M2 subnormals round half away and clamp to 3 (f8e5.rs:50-54): 3.5 * 2^-16 -> code 3
    assert e5(3.5 * 2 ** -16) == 3 and e5(2.5 * 2 ** -16) == 3 and e5(0.5 * 2 ** -16) == 1
    # E4M3 ties to even in the subnormal range (f8e4.rs:32-55): 0.5 * 2^-9 -> 0, 1.5 * 2^-9 -> 2
    assert e4(0.5 * 2 ** -9) == 0 and e4(1.5 * 2 ** -9) == 2 and e4(2.5 * 2 ** -9) == 2
    # the E5M2 decode keeps the sign of a NaN (f8e5.rs:21-24)
    assert int(oracle.f8_convert("f8e5m2_to_f32", [0xfe])[0]) == 0xffc00000


def test_oracle_f8_contraction_decodes_operands():
    """f8 operands widen through the decode (cast.rs:193-217), not as raw codes: 1.0 x 1.0 over
    K = 32 is 32.0, which narrows to E4M3 code 0x60 and E5M2 code 0x50."""
    from oracle import ref_m
    ax = dict(A=2, K=32, R=2)
    L, R, P, O = (ref_m(e, **ax) for e in ("[A, K]", "[R, K]", "[A, R, K]", "[A, R]"))
    for kind, one, out_code in (("f8e4m3", 0x38, 0x60), ("f8e5m2", 0x3c, 0x50)):
        a = bytes([one]) * 64
        wide = np.frombuffer(oracle.contract(a, a, kind, "f32", L, R, P, O), np.float32)
        assert np.all(wide == 32.0)
        narrow = oracle.contract(a, a, kind, kind, L, R, P, O)
        assert narrow == bytes([out_code]) * 4
