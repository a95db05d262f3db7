"""The bf16 conversions of the vector engine (float/bf16.rs:16-40; opcodes BF16_TO_F32, F32_TO_BF16,
F32_TO_BF16_RELU) over every bf16 code and over f32 patterns at every rounding boundary of every
exponent, byte-exact against the oracle, on the generated and the interpreted elementwise paths.
Every row program, epilogue-free elementwise op and fused chain of the decoder goes through these."""
import numpy as np
import pytest

import furiosa_opt_b200 as fb
import oracle
from furiosa_opt_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["generated", "interpreter"])
def ew_path(request, monkeypatch):
    if request.param == "interpreter":
        monkeypatch.setenv("FOPT_EW_NO_JIT", "1")
    else:
        monkeypatch.delenv("FOPT_EW_NO_JIT", raising=False)
    return request.param


def _f32_patterns():
    hi = np.arange(1 << 16, dtype=np.uint32) << 16
    low = np.array([0, 1, 0x7FFF, 0x8000, 0x8001, 0xFFFF, 0x4000, 0xC000], np.uint32)
    grid = (hi[:, None] | low[None, :]).reshape(-1)
    rand = np.random.default_rng(9).integers(0, 2 ** 32, 1 << 20, dtype=np.uint64).astype(np.uint32)
    return np.concatenate([grid, rand])


def _run(be, prog, words, in_dt, out_dt):
    n = words.size
    mp = fb.Mapping("[E]", dict(E=n))
    src = be.from_vec(mp, words.view(np.float32) if in_dt == "f32" else words.astype(np.uint16), in_dt)
    out = be._ew(prog, [src], out_dt)
    return out.to_bytes()


def _want(op, words, in_dt, out_dt):
    data = words.astype(np.uint32).tobytes() if in_dt == "f32" else words.astype(np.uint16).tobytes()
    return oracle.elementwise([(op, 1, 0, 0, 0, 0)], 1, [data], [in_dt], out_dt, words.size)


def test_bf16_to_f32_every_code(b200, ew_path):
    codes = np.tile(np.arange(1 << 16, dtype=np.uint32), 2)
    assert _run(b200, ops.cast("bf16", "f32"), codes, "bf16", "f32") == _want(1, codes, "bf16", "f32")


def test_f32_to_bf16_boundaries(b200, ew_path):
    w = _f32_patterns()
    got = np.frombuffer(_run(b200, ops.cast("f32", "bf16"), w, "f32", "bf16"), np.uint16)
    want = np.frombuffer(_want(2, w, "f32", "bf16"), np.uint16)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, [(hex(w[i]), hex(got[i]), hex(want[i])) for i in bad[:8]]


def test_f32_to_bf16_relu_boundaries(b200, ew_path):
    w = _f32_patterns()
    got = np.frombuffer(_run(b200, ops.cast_relu(), w, "f32", "bf16"), np.uint16)
    want = np.frombuffer(_want(3, w, "f32", "bf16"), np.uint16)
    assert np.array_equal(got, want)
