"""CPU-side checks of the product library (no GPU): the C ABI loads and exports every declared
symbol, the C++ mapping parser agrees with the oracle's position semantics, and the planner's
odometer walks reproduce the oracle's per-position source offsets."""
import os
import re

import numpy as np
import pytest

import furiosa_opt_b200 as fb
import oracle
from furiosa_opt_b200 import _lib
from oracle import ref_m

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "fopt_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(fopt_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    syms = header_symbols()
    assert len(syms) >= 30
    for s in syms:
        assert hasattr(lib, s), f"libfopt_b200.so does not export {s}"
    bound = {n for n, _, _ in _lib.SIGNATURES}
    assert set(syms) <= bound, f"unbound symbols: {set(syms) - bound}"


EXPRS = [
    ("[A]", dict(A=8)),
    ("[A, B]", dict(A=8, B=16)),
    ("[C, D # 64]", dict(C=13, D=61)),
    ("[C, D = 2]", dict(C=2, D=3)),
    ("[B / 64, B % 64]", dict(B=512)),
    ("[B / 64, B % 32, B / 32 % 2]", dict(B=512)),
    ("[A / 8, B % 4 # 16]", dict(A=64, B=16)),
    ("[A #{0} 8, B #{!} 3]", dict(A=5, B=2)),
    ("[[A, B] / 3, 2]", dict(A=4, B=6)),
    ("[[A, B] % 12]", dict(A=4, B=6)),
    ("[4, A, 1]", dict(A=3)),
    ("[[A, B] # 30]", dict(A=4, B=6)),
    ("m![A / 4 % 4, A % 4, B]", dict(A=256, B=8)),
    ("[A = 6 # 8, B / 2]", dict(A=8, B=8)),
]


@pytest.mark.parametrize("expr,axes", EXPRS)
def test_parser_matches_oracle(expr, axes):
    m = fb.Mapping(expr, axes)
    r = ref_m(expr, **axes)
    assert m.size == r.size
    st, co = r.cells(np.arange(r.size + 2))
    for i in range(r.size + 2):
        s, c = m.eval(i)
        assert s == st[i], (expr, i)
        if s == 0:
            for a in r.idents():
                assert c[a] == co[a][i], (expr, i, a)


def test_parse_errors_are_reported():
    with pytest.raises(_lib.FoptError):
        fb.Mapping("[A / 3]", A=8)  # stride does not divide
    with pytest.raises(_lib.FoptError):
        fb.Mapping("[Q]", A=8)  # undeclared axis
    with pytest.raises(_lib.FoptError):
        fb.Mapping("[A # 4]", A=8)  # padding below size


def walk_offsets(desc: str, n: int):
    """Evaluates a planner walk ("walk{(extent[/live]:stride)...}") on the host."""
    wheels = []
    for w in re.findall(r"\(([^)]*)\)", desc):
        ext, stride = w.split(":")
        e, _, l = ext.partition("/")
        wheels.append((int(e), int(l or e), int(stride)))
    q = np.arange(n, dtype=np.int64)
    off = np.zeros(n, np.int64)
    live = np.ones(n, bool)
    for e, l, s in wheels:
        d = q % e
        q //= e
        live &= d < l
        off += d * s
    return np.where(live, off, -1)


RELAYOUTS = [
    ("[A, B]", "[B, A]", dict(A=4, B=8), False),
    ("[R, C]", "[C, R]", dict(R=48, C=40), False),
    ("[A, B, C]", "[C, A, B]", dict(A=3, B=5, C=7), False),
    ("[A]", "[B, A # 6]", dict(A=4, B=3), True),
    ("[C, D]", "[C, D # 64]", dict(C=13, D=61), False),
    ("[B]", "[B / 64, B % 32, B / 32 % 2]", dict(B=512), False),
    ("[A / 4 % 4, A % 4, B]", "[A / 16, A % 4, B]", dict(A=64, B=8), False),
    ("[A, B]", "[A / 4, B, A % 4]", dict(A=16, B=12), False),
    ("[H, X]", "[X / 8, H, X % 8]", dict(H=10, X=64), False),
    ("[M, K = 2 # 4]", "[K = 2 # 4, M]", dict(M=3, K=2), False),
]


@pytest.mark.parametrize("src,dst,axes,bc", RELAYOUTS)
def test_relayout_walk_matches_oracle(src, dst, axes, bc):
    S, D = fb.Mapping(src, axes), fb.Mapping(dst, axes)
    desc = fb.B200.describe_relayout(None, S, D, bc)
    if not desc.startswith("walk"):
        pytest.skip("table plan")
    got = walk_offsets(desc, D.size)
    rs, rd = ref_m(src, **axes), ref_m(dst, **axes)
    st, co = rd.cells()
    idx = oracle._Index(rs, rs.idents())
    want = np.where(st == 0, idx.find(co, rd.size), -1)
    live = want >= 0
    assert np.array_equal(got >= 0, live), desc
    assert np.array_equal(got[live], want[live]), desc


def test_relayout_rejects_uncovered_src():
    S, D = fb.Mapping("[A, B]", A=2, B=3), fb.Mapping("[A]", A=2)
    with pytest.raises(_lib.FoptError):
        fb.B200.describe_relayout(None, S, D, False)


def test_window_base():
    # buf.rs:760-781: the wire position of the offset's live cell
    base = fb.Mapping("[A, B # 8]", A=4, B=6)
    assert base.window_base({"A": 2, "B": 3}) == 2 * 8 + 3
    assert base.window_base({}) == 0


def _nvrtc():
    import ctypes as C
    for n in ("libnvrtc.so.12", "libnvrtc.so"):
        try:
            return C.CDLL(n)
        except OSError:
            continue
    pytest.skip("NVRTC not available")


def _nvrtc_compile(src: bytes):
    import ctypes as C
    nv = _nvrtc()
    prog_h = C.c_void_p()
    assert nv.nvrtcCreateProgram(C.byref(prog_h), src, b"t.cu", 0, None, None) == 0
    opts = (C.c_char_p * 3)(b"--gpu-architecture=sm_100a", b"--std=c++17", b"--fmad=false")
    rc = nv.nvrtcCompileProgram(prog_h, 3, opts)
    if rc != 0:
        n = C.c_size_t()
        nv.nvrtcGetProgramLogSize(prog_h, C.byref(n))
        log = C.create_string_buffer(n.value)
        nv.nvrtcGetProgramLog(prog_h, log)
        pytest.fail(log.value.decode()[-3000:])
    nv.nvrtcDestroyProgram(C.byref(prog_h))


@pytest.mark.parametrize("fold", [0, 2, 3, 4, 10, 12, 13])
def test_generated_reduce_kernels_compile(fold):
    """The fused map + row-reduce kernels fopt_reduce_map generates compile for sm_100a."""
    import ctypes as C
    from furiosa_opt_b200 import ops, workloads as W
    if fold >= 10:
        prog, ins = ops.fxp_binary("MulInt"), ["i32", "i8"]
    else:
        p = ops.Prog(3)
        prog, ins = p.build(p.emit("MULF", p.emit("MULF", 0, 1), 2)), ["bf16", "f32", "f32"]
    lib = _lib.lib()
    dts = (C.c_int * 3)(*[_lib.DTYPES[d] for d in ins] + [0] * (3 - len(ins)))
    need = C.c_size_t()
    assert lib.fopt_reduce_map_source(C.byref(prog), len(ins), dts, fold, None, 0, C.byref(need)) == 0
    buf = C.create_string_buffer(need.value)
    assert lib.fopt_reduce_map_source(C.byref(prog), len(ins), dts, fold, buf, need.value, None) == 0
    _nvrtc_compile(buf.value)


@pytest.mark.parametrize("case", ["cast_bf16_f32", "requant", "swiglu", "quant", "zip3_select", "i16_shift"])
def test_generated_elementwise_kernels_compile(case):
    """The kernels fopt_elementwise generates compile for sm_100a (NVRTC runs without a GPU)."""
    import ctypes as C
    from furiosa_opt_b200 import ops, workloads as W
    progs = {
        "cast_bf16_f32": (ops.cast("bf16", "f32"), ["bf16"], "f32"),
        "requant": (ops.requant_i32_to_i8(0.01, relu=True), ["i32"], "i8"),
        "swiglu": (W._prog_swiglu(), ["bf16", "bf16"], "f32"),
        "quant": (W._prog_quant(), ["f32", "f32"], "i8"),
        "zip3_select": (ops.select(), ["i32", "f32", "f32"], "bf16"),
        "i16_shift": (ops.fxp_binary("ArithRightShift"), ["i16", "i8"], "i16"),
    }
    prog, ins, out = progs[case]
    lib = _lib.lib()
    dts = (C.c_int * 3)(*[_lib.DTYPES[d] for d in ins])
    need = C.c_size_t()
    assert lib.fopt_elementwise_source(C.byref(prog), len(ins), dts, _lib.DTYPES[out], None, 0, C.byref(need)) == 0
    buf = C.create_string_buffer(need.value)
    assert lib.fopt_elementwise_source(C.byref(prog), len(ins), dts, _lib.DTYPES[out], buf, need.value, None) == 0
    nv = _nvrtc()
    prog_h = C.c_void_p()
    assert nv.nvrtcCreateProgram(C.byref(prog_h), buf.value, b"t.cu", 0, None, None) == 0
    opts = (C.c_char_p * 3)(b"--gpu-architecture=sm_100a", b"--std=c++17", b"--fmad=false")
    rc = nv.nvrtcCompileProgram(prog_h, 3, opts)
    if rc != 0:
        n = C.c_size_t()
        nv.nvrtcGetProgramLogSize(prog_h, C.byref(n))
        log = C.create_string_buffer(n.value)
        nv.nvrtcGetProgramLog(prog_h, log)
        pytest.fail(log.value.decode()[-3000:])
    size = C.c_size_t()
    assert nv.nvrtcGetCUBINSize(prog_h, C.byref(size)) == 0 and size.value > 0
    nv.nvrtcDestroyProgram(C.byref(prog_h))


def _run(prog, ins, dts, out_dt):
    import oracle
    insns = [(prog.insn[i].op, prog.insn[i].dst, prog.insn[i].a, prog.insn[i].b, prog.insn[i].c, prog.insn[i].imm_i)
             for i in range(prog.n_insn)]
    n = len(ins[0]) // 4
    return oracle.elementwise(insns, prog.ret, ins, dts, out_dt, n)


def test_program_composition_matches_sequential_programs():
    """Deferred elementwise values are evaluated inside their consumer's program (ops.inline + the
    register reassignment in Prog.build): composed results are bit-identical to running the
    producer, writing its f32 values and running the consumer."""
    from furiosa_opt_b200 import ops, workloads as W
    rng = np.random.default_rng(3)
    g, u, s = (rng.standard_normal(4096).astype(np.float32) for _ in range(3))
    s = np.abs(s) + 0.1
    sw, q = W._prog_swiglu(), W._prog_quant()
    act = _run(sw, [g.tobytes(), u.tobytes()], ["f32", "f32"], "f32")
    want = _run(q, [act, s.tobytes()], ["f32", "f32"], "i8")
    b = ops.Prog(3)
    p = b.build(ops.inline(b, q, [ops.inline(b, sw, [0, 1]), 2]))
    assert _run(p, [g.tobytes(), u.tobytes(), s.tobytes()], ["f32"] * 3, "i8") == want
    # a chain of 20 dependent steps: needs the register reassignment (more than 16 handed out)
    step = ops.Prog(1)
    step = step.build(step.emit("MULF", step.emit("ADDF", 0, step.const_f32(0.5)), step.const_f32(0.75)))
    b = ops.Prog(1)
    r = 0
    for _ in range(6):
        r = ops.inline(b, step, [r])
    chain = b.build(r)
    assert chain.n_insn <= 32
    ref = g.tobytes()
    for _ in range(6):
        ref = _run(step, [ref], ["f32"], "f32")
    assert _run(chain, [g.tobytes()], ["f32"], "f32") == ref


def _write_safetensors(path, tensors, metadata=None):
    """A safetensors file from {name: (dtype string, shape, raw bytes)} (the published layout)."""
    import json
    import struct
    header, blobs, off = {}, [], 0
    if metadata:
        header["__metadata__"] = metadata
    for name, (dt, shape, raw) in tensors.items():
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    text = json.dumps(header).encode()
    text += b" " * ((8 - len(text) % 8) % 8)
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(text)) + text + b"".join(blobs))


def test_safetensors_header_and_flat_shape(tmp_path):
    """The native safetensors reader: names, dtypes, shapes and byte counts from the header, escapes
    and metadata skipped; and the pair-split shapes the reference checks a tensor against."""
    rng = np.random.default_rng(0)
    w = rng.standard_normal((8, 12)).astype(np.float32)
    b = rng.integers(-128, 128, 40, dtype=np.int64).astype(np.int8)
    p = tmp_path / "t.safetensors"
    _write_safetensors(p, {'w"x': ("F32", (8, 12), w.tobytes()), "b": ("I8", (40,), b.tobytes())},
                       metadata={"format": "pt"})
    with fb.SafeTensors(str(p)) as st:
        assert len(st) == 2
        assert sorted(st.names()) == ["b", 'w"x']
        name, dt, shape, nbytes = st.info(st.index('w"x'))
        assert (dt, shape, nbytes) == ("F32", [8, 12], w.nbytes)
        assert st.info(st.index("b"))[1:] == ("I8", [40], 40)
        with pytest.raises(_lib.FoptError):
            st.index("missing")
    assert fb.Mapping("[H, X]", dict(H=256, X=800)).flat_shape() == [256, 800]
    assert fb.Mapping("[[A, B], C]", dict(A=2, B=3, C=5)).flat_shape() == [2, 3, 5]
    assert fb.Mapping("[A # 8, B]", dict(A=5, B=3)).flat_shape() == [8, 3]
    assert fb.Mapping("[A / 4]", dict(A=16)).flat_shape() == [4]
    bad = tmp_path / "bad.safetensors"
    bad.write_bytes(b"\x10\x00\x00\x00\x00\x00\x00\x00{not json at all")
    with pytest.raises(_lib.FoptError):
        fb.SafeTensors(str(bad))


def test_safetensors_reads_reference_mnist_header():
    """The reference example's own weights file parses, with the shapes its test loads them as."""
    with fb.SafeTensors(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "mnist.safetensors")) as st:
        info = {st.info(k)[0]: st.info(k)[1:3] for k in range(len(st))}
    assert info["hw.fc1.weight"] == ("BF16", [256, 800])
    assert info["hw.fc2.weight"] == ("BF16", [16, 256])
    assert info["hw.image_0"] == ("BF16", [800])
    assert info["label_0"] == ("I32", [1])


def _fake_backend(monkeypatch):
    """A B200 without a device: storages get fake addresses and every elementwise materialisation
    is lowered to a row program (or None) and recorded instead of run."""
    import ctypes as C
    import itertools
    from furiosa_opt_b200 import backend as B, rowfuse
    addrs = itertools.count(1)

    def fake_alloc(self, zero):
        self._ptr = C.c_void_p(next(addrs) << 16)

    monkeypatch.setattr(B.Storage, "_alloc", fake_alloc)
    monkeypatch.setattr(B.Storage, "__del__", lambda self: None)
    built = []
    monkeypatch.setattr(B.B200, "_run_ew", lambda self, prog, leaves, out, origin=None: built.append(
        rowfuse.build_row_program(self, prog, leaves, out, origin)))
    be = B.B200.__new__(B.B200)
    be.ctx, be.device, be.eager_broadcast, be.fuse, be.row_fusion = None, 0, False, True, True
    return B, be, built


def _row_source(plan) -> bytes:
    import ctypes as C
    lib = _lib.lib()
    need = C.c_size_t()
    assert lib.fopt_row_program_source(C.byref(plan), None, 0, C.byref(need)) == 0
    buf = C.create_string_buffer(need.value)
    assert lib.fopt_row_program_source(C.byref(plan), buf, need.value, None) == 0
    return buf.value


def test_row_programs_lower_the_decoder_chains(monkeypatch):
    """RMSNorm -> per-token quantisation, the attention output's quantisation and SwiGLU ->
    quantisation each lower to one row program (leaves, held values, per-row slots) whose generated
    kernel compiles for sm_100a."""
    from furiosa_opt_b200 import ops, workloads as Wl
    B, be, built = _fake_backend(monkeypatch)
    T, H, F = 64, 4096, 14336
    blk = Wl.DecoderBlockW8A8.__new__(Wl.DecoderBlockW8A8)
    blk.be, blk.T, blk.H, blk.F = be, T, H, F
    blk.ax = dict(T=T, H=H, Q=H, V=1024, F=F)
    blk.p_rinv_h = Wl._prog_rinv(H)
    FOLD, SCALAR = _lib.ROW_FOLD, _lib.ROW_SCALAR

    # RMSNorm then quantisation: x (bf16) and the gain (a repeated row) are the leaves; x stays in
    # registers raw (its f32 cast is recomputed, not held); slots: sum of squares, 1 / rms,
    # max |x_n|, token scale; one warp per row
    x = B.Storage(be, "bf16", T * H)
    g = be.relayout(B.Storage(be, "f32", H), blk.m("[H]"), blk.m("[T, H]"), True)
    q, s = blk.quantize(blk.rmsnorm(be.map(x, ops.cast("bf16", "f32"), "f32"), g), "H")
    plan = built[-1].plan
    assert (plan.n_leaves, plan.n_held, plan.n_slots, plan.rows, plan.row_len) == (2, 0, 4, T, H)
    assert [plan.slot[j].kind for j in range(4)] == [FOLD, SCALAR, FOLD, SCALAR]
    assert plan.leaf_bcast[1] == -H and built[-1].slot_nodes[3] is s
    src = _row_source(plan)
    assert b"NW = 8, RPC = 1" in src  # 64 rows: the whole CTA on a row
    _nvrtc_compile(src)

    # the attention output: one fold (max |x|), then the scale
    att = B.Storage(be, "bf16", T * H)
    qa, sa = blk.quantize(be.map(att, ops.cast("bf16", "f32"), "f32"), "H")
    plan = built[-1].plan
    assert (plan.n_leaves, plan.n_held, plan.n_slots) == (1, 0, 2)
    assert [plan.slot[j].kind for j in range(2)] == [FOLD, SCALAR]
    _nvrtc_compile(_row_source(plan))

    # SwiGLU then quantisation over F: the activation is computed once and held between the passes
    gate, up = B.Storage(be, "bf16", T * F), B.Storage(be, "bf16", T * F)
    q3, s3 = blk.quantize(be.zip_with(gate, up, Wl._prog_swiglu(), "f32"), "F")
    plan = built[-1].plan
    assert (plan.n_leaves, plan.n_held, plan.n_slots, plan.row_len) == (2, 1, 2, F)
    src = _row_source(plan)
    assert b"NW = 8, RPC = 1" in src
    _nvrtc_compile(src)


def test_row_programs_decline_without_a_reduction(monkeypatch):
    """A zip with a broadcast of a value written out is no row program."""
    from furiosa_opt_b200 import ops, workloads as Wl
    B, be, built = _fake_backend(monkeypatch)
    T, H = 8, 64
    ax = dict(T=T, H=H)
    x = B.Storage(be, "f32", T * H)
    sb = be.relayout(B.Storage(be, "f32", T), fb.Mapping("[T]", ax), fb.Mapping("[T, H]", ax), True)
    be.zip_with(x, sb, Wl._prog_quant(), "i8")
    assert built == [None]


def test_row_program_without_room_for_held_values(monkeypatch):
    """A SwiGLU -> quantisation chain over 32768-wide rows would need 128 registers to hold its
    activation: the plan holds nothing (the passes recompute it from the leaves) and still
    compiles."""
    from furiosa_opt_b200 import workloads as Wl
    B, be, built = _fake_backend(monkeypatch)
    T, F = 16, 32768
    blk = Wl.DecoderBlockW8A8.__new__(Wl.DecoderBlockW8A8)
    blk.be, blk.T, blk.F = be, T, F
    blk.ax = dict(T=T, F=F)
    gate, up = B.Storage(be, "bf16", T * F), B.Storage(be, "bf16", T * F)
    blk.quantize(be.zip_with(gate, up, Wl._prog_swiglu(), "f32"), "F")
    plan = built[-1].plan
    assert (plan.n_leaves, plan.n_held, plan.n_slots, plan.row_len) == (2, 0, 2, F)
    _nvrtc_compile(_row_source(plan))


def test_residual_epilogue_checks_its_operand(monkeypatch):
    """contraction_dequant's fused residual must be bf16 laid out as the output."""
    B, be, built = _fake_backend(monkeypatch)
    ax = dict(M=256, N=256, K=128)
    m = lambda e: fb.Mapping(e, ax)  # noqa: E731
    a, w = B.Storage(be, "i8", 256 * 128), B.Storage(be, "i8", 256 * 128)
    s_row, s_col = B.Storage(be, "f32", 256), B.Storage(be, "f32", 256)
    for bad in (B.Storage(be, "f32", 256 * 256), B.Storage(be, "bf16", 256 * 128)):
        with pytest.raises(ValueError):
            be.contraction_dequant(a, w, m("[M, K]"), m("[N, K]"), m("[M, N, K]"), m("[M, N]"), s_row, s_col, "N",
                                   residual=bad)


@pytest.mark.parametrize("case", ["held_warp_per_row", "i32_load_slot", "i8_leaf", "f32_wide"])
def test_row_program_layouts_compile(monkeypatch, case):
    """Row plans across the generator's layouts compile for sm_100a: held values with one warp per
    row (unrolled, no CTA barrier), i32 folds with a LOAD slot and an i16 output, i8 leaves, and
    f32 leaves at a width with a partial last group of 2048."""
    from furiosa_opt_b200 import ops, workloads as Wl
    B, be, built = _fake_backend(monkeypatch)
    if case == "held_warp_per_row":
        T, F = 32768, 1024
        blk = Wl.DecoderBlockW8A8.__new__(Wl.DecoderBlockW8A8)
        blk.be, blk.T, blk.F, blk.ax = be, T, F, dict(T=T, F=F)
        gate, up = B.Storage(be, "bf16", T * F), B.Storage(be, "bf16", T * F)
        blk.quantize(be.zip_with(gate, up, Wl._prog_swiglu(), "f32"), "F")
        plan = built[-1].plan
        assert plan.n_held == 1
        src = _row_source(plan)
        assert b"NW = 1, RPC = 8" in src
    else:
        T, Wd = 64, {"i32_load_slot": 3000, "i8_leaf": 4096, "f32_wide": 6144 + 8}[case]
        ax = dict(T=T, H=Wd)
        m = lambda e: fb.Mapping(e, ax)  # noqa: E731
        if case == "i32_load_slot":
            A = B.Storage(be, "i32", T * Wd)
            off = be.relayout(B.Storage(be, "i32", T), m("[T]"), m("[T, H]"), True)
            p = ops.Prog(2)
            v = be.zip_with(A, off, p.build(p.emit("ADD_FXP", 0, 1)), "i32")
            lo = be.reduce(v, "Min", 2**31 - 1, m("[T, H]"), m("[T]"))
            p = ops.Prog(2)
            be.zip_with(v, be.relayout(lo, m("[T]"), m("[T, H]"), True), p.build(p.emit("XOR", 0, 1)), "i16")
        else:
            dt = "i8" if case == "i8_leaf" else "f32"
            X = B.Storage(be, dt, T * Wd)
            xf = be.map(X, ops.cast("i8", "f32") if dt == "i8" else ops.Prog(1).build(0), "f32")
            mx = be.reduce(be.map(xf, Wl._prog_abs(), "f32"), "Max", 0.0, m("[T, H]"), m("[T]"))
            sc = be.map(mx, Wl._prog_token_scale(), "f32")
            be.zip_with(xf, be.relayout(sc, m("[T]"), m("[T, H]"), True), Wl._prog_quant(), "i8")
        plan = built[-1].plan
        src = _row_source(plan)
    _nvrtc_compile(src)


def test_composition_cache_returns_the_fresh_composition(monkeypatch):
    """A memoised composition is the program a fresh composition builds, byte for byte."""
    from furiosa_opt_b200 import backend as Bk, ops, workloads as Wl
    B, be, built = _fake_backend(monkeypatch)
    n = 64
    x, y = B.Storage(be, "bf16", n), B.Storage(be, "f32", n)
    xf = be.map(x, ops.cast("bf16", "f32"), "f32")
    z = be.zip_with(xf, y, Wl._prog_swiglu(), "f32")
    first = bytes(z.lazy[1])
    Bk._COMPOSED.clear()
    again = be.zip_with(be.map(x, ops.cast("bf16", "f32"), "f32"), y, Wl._prog_swiglu(), "f32")
    assert bytes(again.lazy[1]) == first
    hit = be.zip_with(be.map(x, ops.cast("bf16", "f32"), "f32"), y, Wl._prog_swiglu(), "f32")
    assert hit.lazy[1] is again.lazy[1]


def test_captured_storages_are_released_by_their_graph(monkeypatch):
    """A storage allocated while a step is captured frees itself only during that capture; after it
    ends the graph owns the memory. Storages from outside a capture free normally."""
    import ctypes as C
    import itertools
    from furiosa_opt_b200 import backend as Bk
    addrs, freed = itertools.count(1), []

    class FakeLib:
        def _give(self, ctx, nbytes, out):
            out._obj.value = next(addrs) << 16
            return 0

        fopt_alloc = fopt_alloc_uninit = _give

        def fopt_free(self, ctx, p):
            freed.append(p.value)
            return 0

    monkeypatch.setattr(Bk._lib, "lib", lambda: FakeLib())
    be = Bk.B200.__new__(Bk.B200)
    be.ctx, be._capturing = None, object()
    inside, dies_inside = Bk.Storage(be, "f32", 16), Bk.Storage(be, "f32", 16)
    a_inside = dies_inside._ptr.value
    dies_inside.__del__()  # freed during the capture: a free node of the graph
    assert freed == [a_inside]
    be._capturing = None
    inside.__del__()  # outlives the capture: the graph's to release
    assert freed == [a_inside]
    outside = Bk.Storage(be, "f32", 16)
    a_outside = outside._ptr.value
    outside.__del__()
    assert freed == [a_inside, a_outside]
    for s_ in (inside, dies_inside, outside):
        s_._ptr = C.c_void_p()


def test_ctypes_structs_match_the_c_abi():
    """The Python mirror's ctypes structs have the C ABI's sizes."""
    import ctypes as C
    sizes = (C.c_size_t * 4)()
    assert _lib.lib().fopt_struct_sizes(sizes, 4) == 0
    assert list(sizes) == [C.sizeof(_lib.Program), C.sizeof(_lib.Epilogue), C.sizeof(_lib.RowSlot),
                           C.sizeof(_lib.RowPlan)]


def test_magic_add_rounds_like_rint():
    """The quantising division's fast path (`qdiv_fxp_fast`, `ew_ops.cuh`) rounds y with |y| < 4096
    by adding 1.5 * 2^23 in f32 (round to nearest even) and reads the integer from the low bits of
    the sum: checked here against rint in f32 arithmetic, over every f32 in the binades near the
    half-integers that matter (|y| < 8, and the last binade below 4096) plus random values."""
    magic = np.float32(12582912.0)

    def check(y):
        y = y[np.abs(y) < 4096].astype(np.float32)
        big = (y + magic).astype(np.float32)
        r = (big - magic).astype(np.float32)
        assert np.array_equal(r, np.rint(y))
        assert np.array_equal(big.view(np.int32) - 0x4B400000, np.rint(y).astype(np.int32))

    lo = np.arange(0, 0x41000000, 61, dtype=np.uint32).view(np.float32)  # 0 <= y < 8, every 61st code
    check(lo)
    check(-lo)
    top = np.arange(0x45000000, 0x45800000, dtype=np.uint32).view(np.float32)  # 2048 <= y < 4096, all
    check(top)
    check(-top)
    halves = (np.arange(-4096, 4096, dtype=np.float32) + np.float32(0.5))
    check(halves)  # exact ties go to even, as rint
    check(np.random.default_rng(5).uniform(-4096, 4096, 1 << 20).astype(np.float32))
