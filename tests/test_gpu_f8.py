"""8-bit float element types through the B200 backend, byte-exact against the oracle.

The f8 rules are the reference's (furiosa-opt-std/src/float/f8e4.rs, float/f8e5.rs); the oracle
restates them step for step and is pinned to the reference's own table and tests in test_oracle.py.
Covered here: the four f8 casts and the f4e2m1 -> f8e4m3 lookup over every code and over f32
patterns dense around every rounding boundary, on the generated and the interpreted elementwise
paths; and the f8e4m3 / f8e5m2 contractions of contract_element_types.rs:60-96,166-200 (A = 8,
K8 = 32, R = 8, accumulating in f32), plus larger and narrowing (f8 out) shapes.
"""
import numpy as np
import pytest

import furiosa_opt_b200 as fb
import oracle
from furiosa_opt_b200 import dtypes, ops
from oracle import ref_m

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["generated", "interpreter"])
def ew_path(request, monkeypatch):
    if request.param == "interpreter":
        monkeypatch.setenv("FOPT_EW_NO_JIT", "1")
    else:
        monkeypatch.delenv("FOPT_EW_NO_JIT", raising=False)
    return request.param


def f32_boundary_patterns(seed=0) -> np.ndarray:
    """f32 bit patterns for the encoders: every exponent x the top 4 mantissa bits x low bits at and
    around the E4M3 (bit 20) and E5M2 (bit 21) rounding points, both signs, the specials, and a
    random spread."""
    rng = np.random.default_rng(seed)
    exp = np.arange(256, dtype=np.uint32) << 23
    top = np.arange(16, dtype=np.uint32) << 19
    low = np.array([0, 1, 0x7ffff, 0x80000, 0x80001, 0xfffff, 0x100000 - 1, 0x100000, 0x100001, 0x17ffff,
                    0x180000, 0x180001, 0x400000, 0x3fffff, 0x400001], np.uint32) & 0x7fffff
    grid = (exp[:, None, None] | top[None, :, None] | low[None, None, :]).reshape(-1)
    grid = grid & 0x7fffffff
    specials = np.array([0x7f800000, 0x7fc00000, 0x7f800001, 0x43e00000, 0x43e80000, 0x43f00000, 0x47600000,
                         0x47700000, 0x477fffff, 0x47800000, 0x38800000, 0x387fffff, 0x38600000, 0x3c800000,
                         0x3c7fffff, 0x3b000000, 0x3a800000, 0x3a800001, 1, 0x007fffff], np.uint32)
    rand = rng.integers(0, 2 ** 32, 200_000, dtype=np.uint64).astype(np.uint32)
    pos = np.concatenate([grid, specials])
    return np.concatenate([pos, pos | 0x80000000, rand])


def _run_cast(be, src_dt, dst_dt, words):
    n = words.size
    mp = fb.Mapping("[E]", dict(E=n))
    src = be.from_vec(mp, words.astype(dtypes.NP[src_dt]) if src_dt != "f32" else words.view(np.float32), src_dt)
    out = be._ew(ops.cast(src_dt, dst_dt), [src], dst_dt)
    return np.frombuffer(out.to_bytes(), np.uint32 if dst_dt == "f32" else np.uint8).astype(np.uint32)


@pytest.mark.parametrize("kind", ["f8e4m3", "f8e5m2"])
def test_f8_decode_every_code(b200, ew_path, kind):
    codes = np.tile(np.arange(256, dtype=np.uint32), 17)  # 4352 elements: several vectors per thread
    got = _run_cast(b200, kind, "f32", codes)
    want = oracle.f8_convert(f"{kind}_to_f32", codes)
    assert np.array_equal(got, want)  # NaN bit patterns included: the reference's are canonical


@pytest.mark.parametrize("kind", ["f8e4m3", "f8e5m2"])
def test_f8_encode_boundaries(b200, ew_path, kind):
    words = f32_boundary_patterns()
    got = _run_cast(b200, "f32", kind, words)
    want = oracle.f8_convert(f"f32_to_{kind}", words)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, [(hex(words[i]), hex(got[i]), hex(want[i])) for i in bad[:8]]


@pytest.mark.parametrize("kind", ["f8e4m3", "f8e5m2"])
def test_f8_round_trip_every_code(b200, kind):
    """narrow(widen(x)) == x for every non-NaN code (f8e4.rs:107-121, cast.rs:400-407)."""
    codes = np.arange(256, dtype=np.uint32)
    wide = _run_cast(b200, kind, "f32", codes)
    back = _run_cast(b200, "f32", kind, wide)
    nan = np.isnan(wide.view(np.float32))
    assert np.array_equal(back[~nan], codes[~nan])


def test_f4e2m1_lookup(b200):
    nib = np.tile(np.arange(16, dtype=np.uint32), 64)
    mp = fb.Mapping("[E]", dict(E=nib.size))
    src = b200.from_vec(mp, nib.astype(np.int8), "f4e2m1")
    got = np.frombuffer(b200._ew(ops.cast("f4e2m1", "f8e4m3"), [src], "f8e4m3").to_bytes(), np.uint8)
    assert np.array_equal(got.astype(np.uint32), oracle.f8_convert("f4e2m1_to_f8e4m3", nib))


def _f8_codes(rng, n, kind, spread):
    """Codes of finite values drawn N(0, spread) through the encoder (the reference samples f8 as
    from_f32 of a float draw, scalar.rs:450-455)."""
    v = (rng.standard_normal(n) * spread).astype(np.float32)
    return oracle.f8_convert(f"f32_to_{kind}", v.view(np.uint32)).astype(np.uint8)


F8_CONTRACTIONS = [
    # contract_element_types.rs: [A, K8] x [R, K8] -> [A, R], A = 8, K8 = 32, R = 8
    ("[A, K]", "[R, K]", "[A, R, K]", "[A, R]", dict(A=8, K=32, R=8)),
    ("[M, K]", "[K, N]", "[M, K, N]", "[M, N]", dict(M=33, K=70, N=19)),
    ("[M, K = 5 # 8]", "[K = 5 # 8, N]", "[M, K = 5 # 8, N]", "[M, N]", dict(M=6, K=5, N=7)),
    ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]", dict(M=256, K=512, N=256)),
    ("[B, M, K]", "[K, N]", "[B, M, K, N]", "[B, M, N]", dict(B=3, M=8, K=32, N=16)),
]


@pytest.mark.parametrize("kind", ["f8e4m3", "f8e5m2"])
@pytest.mark.parametrize("out", ["f32", "narrow"])
@pytest.mark.parametrize("case", range(len(F8_CONTRACTIONS)))
def test_f8_contraction(b200, kind, out, case):
    l, r, p, o, ax = F8_CONTRACTIONS[case]
    L, R, P, O = (fb.Mapping(e, ax) for e in (l, r, p, o))
    rl, rr, rp, ro = (ref_m(e, **ax) for e in (l, r, p, o))
    rng = np.random.default_rng(100 + case)
    lv, rv = _f8_codes(rng, L.size, kind, 2.0), _f8_codes(rng, R.size, kind, 2.0)
    out_dt = "f32" if out == "f32" else kind
    got = b200._contract(b200.from_vec(L, lv, kind), b200.from_vec(R, rv, kind), L, R, P, O, out_dt).to_bytes()
    want = oracle.contract(lv.tobytes(), rv.tobytes(), kind, out_dt, rl, rr, rp, ro)
    # the fold is the reference's sequential f32 sum in wire order: bit-exact
    assert got == want
    # and it is not the raw-code arithmetic: the f32 results carry real magnitudes
    if out == "f32" and case == 0:
        g = np.frombuffer(got, np.float32)
        assert np.abs(g).max() > 1.0


def test_f8_contraction_specials(b200):
    """Codes with infinities and NaNs (f8e5m2) and saturating sums (f8e4m3 narrows to 448)."""
    ax = dict(M=16, K=64, N=16)
    L, R, P, O = (fb.Mapping(e, ax) for e in ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]"))
    rl, rr, rp, ro = (ref_m(e, **ax) for e in ("[M, K]", "[N, K]", "[M, N, K]", "[M, N]"))
    rng = np.random.default_rng(7)
    for kind in ("f8e4m3", "f8e5m2"):
        lv = rng.integers(0, 256, L.size).astype(np.uint8)
        rv = rng.integers(0, 256, R.size).astype(np.uint8)
        for out_dt in ("f32", kind):
            got = b200._contract(b200.from_vec(L, lv, kind), b200.from_vec(R, rv, kind), L, R, P, O,
                                 out_dt).to_bytes()
            want = oracle.contract(lv.tobytes(), rv.tobytes(), kind, out_dt, rl, rr, rp, ro)
            if out_dt == "f32":
                g, w = np.frombuffer(got, np.float32), np.frombuffer(want, np.float32)
                both_nan = np.isnan(g) & np.isnan(w)  # NaN payloads of f32 arithmetic differ by ISA
                assert np.array_equal(np.isnan(g), np.isnan(w))
                assert np.array_equal(g.view(np.uint32)[~both_nan], w.view(np.uint32)[~both_nan])
            else:
                assert got == want
