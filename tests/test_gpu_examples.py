"""The reference's shipped examples, run through the B200 backend and checked against each
example's own answer (furiosa-opt-examples/tests/*.rs).

Each test restates the example's device function as the sequence of Backend calls the reference's
CPU backend makes for it (HBM / DM moves and tile views are `transpose` with window offsets,
`Tensor::transpose` -> `Backend::transpose`; vector-engine stages are `map` / `zip_with` /
`reduce`; contraction stages are `contraction`), with the same mappings, then compares the result
with the answer the example's test computes. Where the test draws its inputs from Rust's SmallRng,
the inputs here come from a seeded numpy generator instead: each of these answers is computed from
the inputs themselves, so any inputs of the same shape and range check the same thing.
"""
import numpy as np
import pytest

import furiosa_opt_b200 as fb
import oracle
from furiosa_opt_b200 import dtypes, ops, workloads as W

pytestmark = pytest.mark.gpu


def M(expr, **axes):
    return fb.Mapping(expr, axes)


# ---- transpose_tests.rs:9-38 (src/transpose.rs:10-20) -------------------------------------------
def test_transpose_simple(b200):
    ax = dict(A=8, B=16, C=32)
    total = 8 * 16 * 32
    hbm = b200.to_hbm(np.arange(total, dtype=np.float32), M("[A, B, C]", **ax), "f32")
    inter = b200.relayout(hbm, M("[A, B, C]", **ax), M("[A, C, B]", **ax))       # [A, B, C] -> [A, C, B]
    out = b200.relayout(inter, M("[A, C, B]", **ax), M("[C, A, B]", **ax))       # [A, C, B] -> [C, A, B]
    expected = [a * 16 * 32 + b * 32 + c for c in range(32) for a in range(8) for b in range(16)]
    assert np.array_equal(out.to_numpy(), np.array(expected, np.float32))


# ---- shuffle_slice_tests.rs:6-35 (src/cluster_chip_shuffle_slice.rs:5-19), chip = 4 in one buffer --
def test_chip_shuffle(b200):
    ax = dict(A=256, B=4096)
    host = M("[A, B]", **ax)
    hbm_map = M("[A / 4 % 4, A / 16, A % 4, B]", **ax)            # HbmTensor<i32, m![A/4%4], m![A/16, A%4, B]>
    hbm2_map = M("[A / 4 % 4, B, A % 4, A / 16]", **ax)           # to_hbm::<.., m![B, A % 4, A / 16]>
    dm_map = M("[A / 4 % 4, A / 2 % 2, B % 16, B / 16 % 16, B / 256, A % 2, A / 16]", **ax)
    t = b200.to_hbm(np.arange(256 * 4096, dtype=np.int32), host, "i32", hbm_map)
    t = b200.relayout(t, hbm_map, hbm2_map)
    dm = b200.relayout(t, hbm2_map, dm_map)
    shuffled = fb.dist.chip_shuffle_local(b200, dm, 4, [1, 2, 3, 0])
    back = b200.relayout(shuffled, dm_map, hbm_map)
    got = b200.from_hbm(back, hbm_map, "i32", host)
    x = np.arange(256 * 4096, dtype=np.int64)
    a16, a4, a1, b = x // 4096 // 16, (x // 4096 % 16) // 4, x // 4096 % 4, x % 4096
    out_a4 = np.array([1, 2, 3, 0])[a4]
    expected = a16 * 4096 * 16 + out_a4 * 4096 * 4 + a1 * 4096 + b
    assert np.array_equal(got, expected.astype(np.int32))


def test_cluster_shuffle(b200):
    """dm_cluster_shuffle (memory.rs:1183-1206): `pattern[target] = source` over the Cluster axis of
    a DM tensor [Chip, Cluster, Slice, Element], on 2 chips x 2 clusters with [1, 0] (the swap the
    reference's doc names), against numpy."""
    ax = dict(A=512, B=64)
    dm = M("[A / 256, A / 128 % 2, A % 128, B]", **ax)              # Chip 2, Cluster 2, Slice 128, [B]
    x = np.random.default_rng(11).integers(-2**31, 2**31 - 1, 512 * 64).astype(np.int32)
    d = b200.from_vec(dm, x, "i32")
    out = fb.dist.cluster_shuffle_local(b200, d, 2, 2, [1, 0])
    want = x.reshape(2, 2, 128, 64)[:, [1, 0]].reshape(-1)
    assert np.array_equal(out.to_numpy(), want)
    with pytest.raises(ValueError):
        fb.dist.cluster_shuffle_local(b200, d, 2, 2, [0, 0])


# ---- pe_count_tests.rs (src/pe_count.rs): output == input + 1 on every device topology ----------
PE_CONFIGS = {
    # name: (axis, size, DM mapping = Chip, Cluster, Slice, Element)
    "one_pe_add": ("P1", 256, "[1, 1, P1 / 4, P1 % 4]"),
    "two_pe_add": ("P2", 512, "[1, 1, P2 / 4, P2 % 4]"),
    "four_pe_add": ("P4", 1024, "[1, 1, P4 / 4, P4 % 4]"),
    "eight_pe_add": ("P8", 2048, "[1, P8 / 1024, P8 / 4 % 256, P8 % 4]"),
    "two_chip_add": ("P2C", 4096, "[P2C / 2048, P2C / 1024 % 2, P2C / 4 % 256, P2C % 4]"),
    "four_chip_add": ("P4C", 8192, "[P4C / 2048, P4C / 1024 % 2, P4C / 4 % 256, P4C % 4]"),
}


@pytest.mark.parametrize("name", list(PE_CONFIGS))
def test_pe_count_add(b200, name):
    axis, n, dm = PE_CONFIGS[name]
    ax = {axis: n}
    host, hbm = M(f"[{axis}]", **ax), M(f"[{axis} / 2048, {axis} % 2048]" if n > 2048 else f"[{axis}]", **ax)
    dm_map = M(dm, **ax)
    # collect::<m![1], m![P % 4 # 8]>: the packet padded to 8 lanes
    collect = M(dm.replace(f"{axis} % 4]", f"{axis} % 4 # 8]"), **ax)
    x = np.arange(n, dtype=np.int32)
    t = b200.to_hbm(x, host, "i32", hbm)
    d = b200.relayout(t, hbm, dm_map)                       # to_dm
    c = b200.relayout(d, dm_map, collect)                   # fetch / collect
    v = b200.map(c, ops.with_const_i32(ops.FXP_BINARY, "AddFxp", 1), "i32")  # vector_fxp(AddFxp, 1)
    r = b200.relayout(v, collect, dm_map)                   # commit_trim::<m![P % 4]>
    out = b200.relayout(r, dm_map, hbm)                     # to_hbm
    assert np.array_equal(b200.from_hbm(out, hbm, "i32", host), x + 1)


# ---- binary_add_tests.rs (src/binary_add.rs): i32(lhs) + i32(rhs) ------------------------------
def test_binary_add_2048(b200):
    ax = dict(A=2048)
    rng = np.random.default_rng(42)
    lhs = rng.integers(-128, 128, 2048).astype(np.int8)
    rhs = rng.integers(-128, 128, 2048).astype(np.int8)
    hbm, dm = M("[A]", **ax), M("[1 # 2, A / 8, A % 8]", **ax)   # Cluster m![1 # 2], Slice [A/8], [A%8]
    l_dm = b200.relayout(b200.from_vec(hbm, lhs, "i8"), hbm, dm)
    r_dm = b200.relayout(b200.from_vec(hbm, rhs, "i8"), hbm, dm)
    li = b200.map(l_dm, ops.cast("i8", "i32"), "i32")     # fetch_cast::<i32>
    ri = b200.map(r_dm, ops.cast("i8", "i32"), "i32")
    s = b200.zip_with(ri, li, ops.clip_i32("AddFxp"), "i32")  # group1 + group0
    out = b200.relayout(s, dm, hbm)
    assert np.array_equal(out.to_numpy(), lhs.astype(np.int32) + rhs.astype(np.int32))


# ---- broadcast.rs: [A] -> [A, B] broadcast on an HBM-to-HBM move ------------------------------
def test_view_broadcast(b200):
    ax = dict(A=512, B=4)
    src = b200.from_vec(M("[A]", **ax), np.arange(512, dtype=np.int32), "i32")
    out = b200.relayout(src, M("[A]", **ax), M("[A, B]", **ax), allow_broadcast=True)
    assert np.array_equal(out.to_numpy(), np.repeat(np.arange(512, dtype=np.int32), 4))


# ---- commit_view_tile_answer_tests.rs (src/commit_view_tile.rs): swap the two X-halves ----------
def test_commit_view_swap_halves(b200):
    ax = dict(A=8, X=32)
    ramp = dtypes.f32_to_bf16_bits(np.arange(8 * 32, dtype=np.float32))
    hbm = M("[A, X]", **ax)
    base = M("[1 # 2, 1 # 256, A, X]", **ax)                      # Chip, Cluster, Slice, [A, X]
    x = b200.relayout(b200.from_vec(hbm, ramp, "bf16"), hbm, base)
    half_src = M("[1 # 2, 1 # 256, A, X = 16 # 32]", **ax)        # tile::<m![X], 16, m![A, X = 16 # 32]>
    half_dst = M("[1 # 2, 1 # 256, A, X = 16 #{!} 32]", **ax)     # the write side's down padding
    swapped = b200.zeroed(base, "bf16")
    b200.transpose(swapped, x, half_src, half_dst, src_offset={"X": 0}, dst_offset={"X": 16}, src_map=base,
                   dst_map=base)
    b200.transpose(swapped, x, half_src, half_dst, src_offset={"X": 16}, dst_offset={"X": 0}, src_map=base,
                   dst_map=base)
    got = b200.relayout(swapped, base, hbm).to_numpy().reshape(8, 32)
    r = ramp.reshape(8, 32)
    assert np.array_equal(got, np.concatenate([r[:, 16:], r[:, :16]], axis=1))


# ---- tile_tests.rs (src/tile.rs) ----------------------------------------------------------------
def test_tile_simple(b200):
    ax = dict(A=512, B=32)
    rng = np.random.default_rng(42)
    x = rng.integers(-128, 128, 512 * 32).astype(np.int8)
    base_in, base_out = M("[A, B]", **ax), M("[B, A]", **ax)
    inp = b200.from_vec(base_in, x, "i8")
    out = b200.zeroed(base_out, "i8")
    src_tile, dst_tile = M("[A, 1 # 32]", **ax), M("[1 #{!} 32, A]", **ax)
    for b in range(32):  # input.tile::<m![B], 1, m![A, 1 # 32]>(b) -> output.tile::<.., m![1 #{!} 32, A]>(b)
        b200.transpose(out, inp, src_tile, dst_tile, src_offset={"B": b}, dst_offset={"B": b}, src_map=base_in,
                       dst_map=base_out)
    assert np.array_equal(out.to_numpy(), x.reshape(512, 32).T.reshape(-1))


def test_tile_window_commit(b200):
    ax = dict(D=64)
    inp = b200.from_vec(M("[D]", **ax), np.arange(64, dtype=np.float32), "f32")
    base = M("[1 # 256, D]", **ax)                                # Chip, Cluster = 1, Slice = 1 # 256, [D]
    t = b200.relayout(inp, M("[D]", **ax), base)
    result = b200.zeroed(base, "f32")
    b200.transpose(result, t, M("[1 # 256, D = 32 # 64]", **ax), M("[1 # 256, D = 32 #{!} 64]", **ax),
                   src_offset={"D": 0}, dst_offset={"D": 32}, src_map=base, dst_map=base)
    got = b200.relayout(result, base, M("[D]", **ax)).to_numpy()
    assert np.all(got[:32] == 0.0), "out-of-tile cells must stay unwritten"
    assert np.array_equal(got[32:], np.arange(32, dtype=np.float32))


def test_tile_size_gt1_chunk_swap(b200):
    ax = dict(L=768, A=512)
    x = dtypes.f32_to_bf16_bits(np.random.default_rng(3).standard_normal(768 * 512).astype(np.float32))
    base = M("[L, A]", **ax)
    inp, out = b200.from_vec(base, x, "bf16"), b200.zeroed(base, "bf16")
    src_t, dst_t = M("[L = 256 # 768, A]", **ax), M("[L = 256 #{!} 768, A]", **ax)
    for s, d in ((0, 256), (256, 0), (512, 512)):
        b200.transpose(out, inp, src_t, dst_t, src_offset={"L": s}, dst_offset={"L": d}, src_map=base, dst_map=base)
    r = x.reshape(768, 512)
    assert np.array_equal(out.to_numpy().reshape(768, 512), np.concatenate([r[256:512], r[:256], r[512:]]))


def test_tile_inner_digit(b200):
    ax = dict(L=768)
    x = dtypes.f32_to_bf16_bits(np.arange(768, dtype=np.float32))
    base = M("[L]", **ax)
    inp, out = b200.from_vec(base, x, "bf16"), b200.zeroed(base, "bf16")
    b200.transpose(out, inp, M("[L / 96, L % 96 = 2 # 96]", **ax), M("[L / 96, L % 96 = 2 #{!} 96]", **ax),
                   src_offset={"L": 0}, dst_offset={"L": 4}, src_map=base, dst_map=base)
    want = np.zeros(768, np.uint16)
    for o in range(8):  # the 8 outer L / 96 positions, a 2-cell window at stride 96
        want[o * 96 + 4: o * 96 + 6] = x[o * 96: o * 96 + 2]
    assert np.array_equal(out.to_numpy(), want)


# ---- scatter_gather_tests.rs (src/scatter_gather.rs:53-64): cache[index] = data -----------------
def test_scatter_minimal(b200):
    ax = dict(K=512, D=128, C=612)
    data = dtypes.f32_to_bf16_bits(np.arange(1, 512 * 128 + 1, dtype=np.float32))
    hbm = M("[K, D]", **ax)
    dm = M("[1 # 2, K / 2, K % 2, D]", **ax)                       # DmTensor<Cluster = 1 # 2, [K/2], [K%2, D]>
    d = b200.relayout(b200.from_vec(hbm, data, "bf16"), hbm, dm)
    index = b200.from_vec(M("[K]", **ax), np.arange(512, dtype=np.int32) * 128 * 2, "i32")  # byte offsets
    out = b200.zeroed(M("[C, D]", **ax), "bf16")
    b200.scatter(d, out, index, dm, M("[C, D]", **ax), M("[D]", **ax), M("[K]", **ax), M("[C]", **ax), scaled=True)
    got = dtypes.bf16_bits_to_f32(out.to_numpy())
    i = np.arange(612 * 128)
    want = np.where(i < 512 * 128, i + 1, 0).astype(np.float32)
    want = dtypes.bf16_bits_to_f32(dtypes.f32_to_bf16_bits(want))
    assert np.array_equal(got, want)


def test_gather_minimal(b200):
    """gather_minimal (scatter_gather.rs:66-80), the inverse of the scatter: rows of a [K, D] table at
    byte-offset indices into [G, D]."""
    ax = dict(K=512, D=128, G=512)
    rng = np.random.default_rng(8)
    table = dtypes.f32_to_bf16_bits(rng.standard_normal(512 * 128).astype(np.float32))
    idx = rng.permutation(512).astype(np.int32)
    out_dm = M("[1 # 2, G / 2, G % 2, D]", **ax)
    out = b200.zeroed(out_dm, "bf16")
    b200.gather(b200.from_vec(M("[K, D]", **ax), table, "bf16"), out,
                b200.from_vec(M("[G]", **ax), idx * 256, "i32"), M("[K, D]", **ax), out_dm, M("[D]", **ax),
                M("[K]", **ax), M("[G]", **ax), scaled=True)
    got = b200.relayout(out, out_dm, M("[G, D]", **ax)).to_numpy().reshape(512, 128)
    assert np.array_equal(got, table.reshape(512, 128)[idx])


# ---- mnist_tests.rs: the reference's bf16 MLP on its own weights and images, labels checked ------
def test_mnist_reference_weights_labels(b200):
    import os

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "mnist.safetensors")
    m = lambda e: fb.Mapping(e, W.MNIST_BF16_AXES)  # noqa: E731
    with fb.SafeTensors(path) as st:
        w1 = b200.from_safetensors(st, "hw.fc1.weight", m("[H, X]"))
        b1 = b200.from_safetensors(st, "fc1.bias", m("[H]"))
        w2 = b200.from_safetensors(st, "hw.fc2.weight", m("[C, H]"))
        b2 = b200.from_safetensors(st, "hw.fc2.bias", m("[C]"))
        for i in range(10):
            img = b200.from_safetensors(st, f"hw.image_{i}", m("[X]"))
            logits = dtypes.bf16_bits_to_f32(W.mnist_bf16_forward(b200, img, w1, b1, w2, b2).to_numpy())
            label = int(b200.from_safetensors(st, f"label_{i}", fb.Mapping("[E]", dict(E=1))).to_numpy()[0])
            assert int(np.argmax(logits[:10])) == label, f"image_{i}"


# ---- contract_element_types_answer_tests.rs:18-54 and the other element-type kernels ----------
def _contract(b200, lhs, rhs, dt, out_dt, A=8, R=8, K=32):
    ax = dict(A=A, K=K, R=R)
    L, Rm, P, O = (M(e, **ax) for e in ("[A, K]", "[R, K]", "[A, R, K]", "[A, R]"))
    return b200._contract(b200.from_vec(L, lhs, dt), b200.from_vec(Rm, rhs, dt), L, Rm, P, O, out_dt).to_numpy()


def test_i8_contract_answer(b200):
    rng = np.random.default_rng(42)
    x = rng.integers(-8, 8, 8 * 32).astype(np.int8)
    w = rng.integers(-8, 8, 8 * 32).astype(np.int8)
    got = _contract(b200, x, w, "i8", "i32")
    want = x.reshape(8, 32).astype(np.int32) @ w.reshape(8, 32).astype(np.int32).T
    assert np.array_equal(got.reshape(8, 8), want)


def test_i4_contract_answer(b200):
    rng = np.random.default_rng(43)
    x = rng.integers(-8, 8, 8 * 64).astype(np.int8)
    w = rng.integers(-8, 8, 8 * 64).astype(np.int8)
    got = _contract(b200, x, w, "i4", "i32", K=64)
    assert np.array_equal(got.reshape(8, 8), x.reshape(8, 64).astype(np.int32) @ w.reshape(8, 64).astype(np.int32).T)


def test_zero_point_sub_contract_answer(b200):
    """fetch_zero_point_sub::<i9>(3) on the activation, then the i9 x i8 family contraction."""
    rng = np.random.default_rng(44)
    x = rng.integers(-128, 128, 8 * 32).astype(np.int8)
    w = rng.integers(-128, 128, 8 * 32).astype(np.int8)
    ax = dict(A=8, K=32, R=8)
    L, Rm, P, O = (M(e, **ax) for e in ("[A, K]", "[R, K]", "[A, R, K]", "[A, R]"))
    p = ops.Prog(1)
    sub = p.build(p.emit("SUB_FXP", 0, p.const_i32(3)))
    x9 = b200.map(b200.from_vec(L, x, "i8"), sub, "i9")       # i8 - zero point, staged as i9
    w9 = b200.map(b200.from_vec(Rm, w, "i8"), ops.cast("i8", "i9"), "i9")  # the i8 weight in the i9 family
    got = b200._contract(x9, w9, L, Rm, P, O, "i32").to_numpy().reshape(8, 8)
    want = (x.reshape(8, 32).astype(np.int32) - 3) @ w.reshape(8, 32).astype(np.int32).T
    assert np.array_equal(got, want)


@pytest.mark.parametrize("kind", ["f8e4m3", "f8e5m2"])
def test_f8_contract_answer(b200, kind):
    """f8 operands drawn as from_f32 of U(-1, 1) (scalar.rs:450-455, 552-556), accumulated in f32.
    Every product of two f8 values is exact in f32, and their sum over 32 terms needs fewer than 24
    significant bits unless a subnormal product appears, so the f32 fold equals the true sum up to
    one rounding of the running total: |err| <= 32 * 2^-24 * sum |terms|."""
    rng = np.random.default_rng(45)
    enc = lambda v: oracle.f8_convert(f"f32_to_{kind}", v.astype(np.float32).view(np.uint32)).astype(np.uint8)  # noqa
    x, w = enc(rng.uniform(-1, 1, 8 * 32)), enc(rng.uniform(-1, 1, 8 * 32))
    dec = lambda c: oracle.f8_convert(f"{kind}_to_f32", c).view(np.float32).astype(np.float64)  # noqa: E731
    xv, wv = dec(x).reshape(8, 32), dec(w).reshape(8, 32)
    got = _contract(b200, x, w, kind, "f32").reshape(8, 8).astype(np.float64)
    want = xv @ wv.T
    bound = 32 * 2.0 ** -24 * (np.abs(xv) @ np.abs(wv).T) + 1e-30
    assert np.all(np.abs(got - want) <= bound)


def test_bf16_contract_answer(b200):
    rng = np.random.default_rng(46)
    x = dtypes.f32_to_bf16_bits(rng.uniform(-1, 1, 8 * 16).astype(np.float32))
    w = dtypes.f32_to_bf16_bits(rng.uniform(-1, 1, 8 * 16).astype(np.float32))
    got = _contract(b200, x, w, "bf16", "f32", K=16).reshape(8, 8).astype(np.float64)
    xv = dtypes.bf16_bits_to_f32(x).astype(np.float64).reshape(8, 16)
    wv = dtypes.bf16_bits_to_f32(w).astype(np.float64).reshape(8, 16)
    assert np.all(np.abs(got - xv @ wv.T) <= 16 * 2.0 ** -24 * (np.abs(xv) @ np.abs(wv).T) + 1e-30)


# ---- transformer_tests.rs:290-389: two attention chunks through the chain, scalar oracle --------
SQRT_HEAD_DIM = 11.313708  # attention.rs:9
EPS = 6.25e-8              # attention.rs:12


class _Chain:
    """The decode attention kernel of attention.rs:32-392 as backend calls (one query per head)."""

    def __init__(self, be, N=8, G=2, D=128, T=512):
        self.be, self.N, self.G, self.D, self.T = be, N, G, D, T
        self.ax = dict(N=N, G=G, D=D, T=T)
        self.m = lambda e: fb.Mapping(e, self.ax)

    def prog(self, n_in, build):
        p = ops.Prog(n_in)
        return p.build(build(p))

    def qk_scaled(self, q, k):
        be, m = self.be, self.m
        s = be.contraction_wide(q, k, m("[N, G, D]"), m("[T, N, D]"), m("[N, G, T, D]"), m("[N, G, T]"))
        # vector_fp_div(SQRT_HEAD_DIM), then cast::<bf16>
        return be.map(s, self.prog(1, lambda p: p.emit("F32_TO_BF16", p.emit("DIVF", 0, p.const_f32(SQRT_HEAD_DIM)))),
                      "bf16")

    def row_max(self, qk):
        be, m = self.be, self.m
        return be.reduce(be.map(qk, ops.cast("bf16", "f32"), "f32"), "Max", -np.inf, m("[N, G, T]"), m("[N, G]"))

    def masked_exp(self, qk, mx, mask):
        be, m = self.be, self.m
        mb = be.relayout(mx, m("[N, G]"), m("[N, G, T]"), allow_broadcast=True)
        e = be.zip_with(qk, mb, self.prog(2, lambda p: p.emit("EXP", p.emit("SUBF", p.emit("BF16_TO_F32", 0), 1))),
                        "f32")
        kb = be.relayout(mask, m("[T]"), m("[N, G, T]"), allow_broadcast=True)
        return be.zip_with(e, kb, ops.clip_f32("Min"), "f32")  # vector_clip(Min, mask)

    def row_sum(self, e):
        be, m = self.be, self.m
        s = be.reduce(e, "Add", 0.0, m("[N, G, T]"), m("[N, G]"))
        return be.map(s, ops.with_const_f32(ops.CLIP_F32, "Add", EPS), "f32")

    def weighted_sum(self, e, v):
        be, m = self.be, self.m
        w = be.map(e, ops.cast("f32", "bf16"), "bf16")
        # per 16-key slice (SliceQV = m![N, T / 16]): the bf16 partial sum over T % 16 ...
        part = be.contraction(w, v, m("[N, G, T]"), m("[T, N, D]"), m("[N, T / 16, G, D, T % 16]"),
                              m("[N, T / 16, G, D]"))
        # ... then the inter-slice reduce in f32, narrowed to bf16
        pf = be.map(part, ops.cast("bf16", "f32"), "f32")
        tot = be.reduce(pf, "Add", 0.0, m("[N, T / 16, G, D]"), m("[N, G, D]"))
        return be.map(tot, ops.cast("f32", "bf16"), "bf16")

    def forward_first(self, q, k, v, mask):
        qk = self.qk_scaled(q, k)
        mx = self.row_max(qk)
        e = self.masked_exp(qk, mx, mask)
        return mx, self.row_sum(e), self.weighted_sum(e, v)

    def forward(self, q, k, v, mask, old_max, old_sum, old_out):
        be, m = self.be, self.m
        qk = self.qk_scaled(q, k)
        mx = be.zip_with(self.row_max(qk), old_max, ops.clip_f32("Max"), "f32")
        alpha = be.zip_with(mx, old_max, self.prog(2, lambda p: p.emit("EXP", p.emit("SUBF", 1, 0))), "f32")
        e = self.masked_exp(qk, mx, mask)
        es = self.row_sum(e)
        s = be.zip3_with(old_sum, alpha, es, self.prog(3, lambda p: p.emit("ADDF", p.emit("MULF", 0, 1), 2)), "f32")
        res = self.weighted_sum(e, v)
        ab = be.relayout(alpha, m("[N, G]"), m("[N, G, D]"), allow_broadcast=True)
        o = be.zip_with(old_out, ab, self.prog(2, lambda p: p.emit("F32_TO_BF16", p.emit("MULF", p.emit(
            "BF16_TO_F32", 0), 1))), "bf16")
        o = be.zip_with(o, res, self.prog(2, lambda p: p.emit("F32_TO_BF16", p.emit("ADDF", p.emit(
            "BF16_TO_F32", 0), p.emit("BF16_TO_F32", 1)))), "bf16")
        return mx, s, o


def test_attention_two_chunks_scalar_reference(b200):
    N, G, D, T = 8, 2, 128, 512
    rng = np.random.default_rng(0x00A77E17)
    bf = lambda n: dtypes.f32_to_bf16_bits(rng.uniform(-0.2, 0.2, n).astype(np.float32))  # noqa: E731
    q, k0, k1, v0, v1 = bf(N * G * D), bf(T * N * D), bf(T * N * D), bf(T * N * D), bf(T * N * D)
    ch = _Chain(b200, N, G, D, T)
    m = ch.m
    Q = b200.from_vec(m("[N, G, D]"), q, "bf16")
    K0, K1 = b200.from_vec(m("[T, N, D]"), k0, "bf16"), b200.from_vec(m("[T, N, D]"), k1, "bf16")
    V0, V1 = b200.from_vec(m("[T, N, D]"), v0, "bf16"), b200.from_vec(m("[T, N, D]"), v1, "bf16")
    mask = b200.from_vec(m("[T]"), np.ones(T, np.float32), "f32")
    mx, s, o = ch.forward_first(Q, K0, V0, mask)
    mx, s, o = ch.forward(Q, K1, V1, mask, mx, s, o)
    sums = s.to_numpy()
    out = dtypes.bf16_bits_to_f32(o.to_numpy())
    actual = dtypes.bf16_bits_to_f32(dtypes.f32_to_bf16_bits(out / np.repeat(sums, D)))
    # the test's scalar oracle (transformer_tests.rs:352-384), in float64
    qf = dtypes.bf16_bits_to_f32(q).astype(np.float64).reshape(N * G, D)
    kf = np.concatenate([dtypes.bf16_bits_to_f32(k).reshape(T, N, D) for k in (k0, k1)]).astype(np.float64)
    vf = np.concatenate([dtypes.bf16_bits_to_f32(v).reshape(T, N, D) for v in (v0, v1)]).astype(np.float64)
    want = np.zeros((N * G, D))
    want_max = np.zeros(N * G)
    for h in range(N * G):
        sc = kf[:, h // G] @ qf[h] / np.sqrt(D)
        want_max[h] = sc.max()
        w = np.exp(sc - sc.max())
        want[h] = w @ vf[:, h // G] / w.sum()
    diff = np.abs(actual - want.reshape(-1))
    print(f"attention two chunks: max abs err {diff.max():.3g} (test bound 0.12 + 0.12 |expected|)")
    assert np.all(diff <= 0.12 + 0.12 * np.abs(want.reshape(-1)))
    assert np.all(np.abs(mx.to_numpy() - want_max) < 0.1)


# ---- reshape_tests.rs (src/reshape.rs): a relabel of the DM layout across chip / cluster / slice ---
@pytest.mark.parametrize("variant", ["seven_axes", "four_axes"])
def test_reshape(b200, variant):
    ax = dict(A=256, B=4096)
    host = M("[A, B]", **ax)
    hbm_map = M("[A / 4 % 4, A / 16, A % 4, B]", **ax)
    hbm2_map = M("[A / 4 % 4, A % 4, B, A / 16]", **ax)
    dm_map = M("[A / 4 % 4, A / 2 % 2, B % 16, B / 16 % 16, B / 256, A % 2, A / 16]", **ax)
    t = b200.to_hbm(np.arange(256 * 4096, dtype=np.int32), host, "i32", hbm_map)
    t = b200.relayout(t, hbm_map, hbm2_map)
    dm = b200.relayout(t, hbm2_map, dm_map)
    if variant == "seven_axes":
        ax2 = dict(C=4, D=2, E=16, F=16, G=16, H=2, I=16)
        out_map = M("[C, D, E, F, G, H, I]", **ax2)
    else:
        ax2 = dict(C=4, D=2, E=256, F=512)
        out_map = M("[C, D, E, F]", **ax2)
    reshaped = b200.reshape(dm, dm_map, out_map)      # `unsafe { dm_tensor.reshape() }`: wire order kept
    got = reshaped.to_numpy()
    x = np.arange(256 * 4096, dtype=np.int64)
    a4 = x // (2 * 16 * 16 * 16 * 2 * 16)
    a2 = x % (2 * 16 * 16 * 16 * 2 * 16) // (16 * 16 * 16 * 2 * 16)
    b1 = x % (16 * 16 * 16 * 2 * 16) // (16 * 16 * 2 * 16)
    b16 = x % (16 * 16 * 2 * 16) // (16 * 2 * 16)
    b256 = x % (16 * 2 * 16) // (2 * 16)
    a1 = x % (2 * 16) // 16
    a16 = x % 16
    want = (a16 * 16 + a4 * 4 + a2 * 2 + a1) * 4096 + (b256 * 256 + b16 * 16 + b1)
    assert np.array_equal(got, want.astype(np.int32))


# ---- memset_tests.rs (src/memset.rs): a whole-region fill, then a DM relayout that reads it ------
MEMSETS = [("i32", 0, np.int32), ("i8", -1, np.int8), ("i16", 300, np.int16), ("f32", 1.5, np.float32),
           ("bf16", 1.0, None), ("f8e4m3", 1.0, None), ("i4", -1, np.int8), ("bf16", 3.0, None)]


@pytest.mark.parametrize("case", range(len(MEMSETS)))
def test_memset(b200, case):
    dt, value, npdt = MEMSETS[case]
    ax = dict(A=256, B=128)
    hbm, dm = M("[A, B]", **ax), M("[1 # 2, A, B]", **ax)          # Dm<D>: cluster m![1 # 2], slice [A], [B]
    relaid = M("[1 # 2, 1 # 2, A / 2, A % 2, B]", **ax)             # Relaid<D>
    out_map = M("[A / 2, A % 2, B]", **ax)
    n = 256 * 128
    rng = np.random.default_rng(case)
    if dt == "bf16":
        inp, fill = dtypes.f32_to_bf16_bits(rng.uniform(2, 100, n).astype(np.float32)), dtypes.f32_to_bf16_bits(
            np.array([value], np.float32))[0]
    elif dt == "f8e4m3":
        inp = oracle.f8_convert("f32_to_f8e4m3", np.full(n, 2.0, np.float32).view(np.uint32)).astype(np.uint8)
        fill = int(oracle.f8_convert("f32_to_f8e4m3", np.array([value], np.float32).view(np.uint32))[0])
    elif dt == "i4":
        inp, fill = (np.arange(n) % 7).astype(np.int8), np.int8(value)
    else:
        inp, fill = (np.arange(n) % 50 + 1).astype(npdt), npdt(value)
    store_dt = np.uint8 if dt == "f8e4m3" else (np.uint16 if dt == "bf16" else np.asarray(inp).dtype)
    d = b200.relayout(b200.from_vec(hbm, inp, dt), hbm, dm)                  # to_dm
    splat = b200.from_vec(dm, np.full(dm.size, fill, dtype=store_dt), dt)    # Tensor::splat(value)
    b200.transpose(d, splat, dm, dm, allow_broadcast=True)                    # memset: fill the live cells
    r = b200.relayout(d, dm, relaid)                                          # dm.to_dm(): reads the fill
    got = b200.from_hbm(b200.relayout(r, relaid, out_map), out_map, dt)       # to_hbm, to_host
    assert np.array_equal(got, np.full(n, fill, dtype=store_dt)), dt


# ---- fetch_commit_tests.rs (src/fetch_commit.rs): i8 [A, B] -> fetch_cast i32 -> [B, A] -----------
def test_fetch_commit_simple(b200):
    ax = dict(A=4096, B=8)
    hbm = M("[A, B]", **ax)
    dm = M("[1 # 2, A / 16, A / 8 % 2, A % 8, B]", **ax)          # Cluster m![1 # 2], [A / 16], [A/8%2, A%8, B]
    x = (np.arange(32768) % 256).astype(np.uint8).view(np.int8)   # (0..32768) as i8
    d = b200.relayout(b200.from_vec(hbm, x, "i8"), hbm, dm)
    c = b200.map(d, ops.cast("i8", "i32"), "i32")                 # fetch_cast::<i32>, collect, commit
    out = b200.relayout(c, dm, M("[B, A]", **ax))                 # to_hbm::<m![B, A]>
    a, b = np.meshgrid(np.arange(4096), np.arange(8))            # out[b, a] = ((a * 8 + b) as i8) as i32
    want = ((a * 8 + b) % 256).astype(np.uint8).view(np.int8).astype(np.int32).reshape(-1)
    assert np.array_equal(out.to_numpy(), want)


# ---- view_tests.rs (src/view.rs): three tile moves rotate each row of B by two -------------------
def test_view_simpl(b200):
    ax = dict(A=512, B=8)
    hbm, dm = M("[A, B]", **ax), M("[A / 256, A % 256, B]", **ax)
    inp = b200.relayout(b200.from_vec(hbm, np.arange(4096, dtype=np.int32), "i32"), hbm, dm)
    out = b200.zeroed(dm, "i32")
    for size, s, d in ((4, 0, 2), (2, 4, 6), (2, 6, 0)):
        b200.transpose(out, inp, M(f"[A / 256, A % 256, B = {size} # 8]", **ax),
                       M(f"[A / 256, A % 256, B = {size} #{{!}} 8]", **ax), src_offset={"B": s}, dst_offset={"B": d},
                       src_map=dm, dst_map=dm)
    got = b200.relayout(out, dm, hbm).to_numpy()
    want = np.array([8 * a + i for a in range(512) for i in (6, 7, 0, 1, 2, 3, 4, 5)], np.int32)
    assert np.array_equal(got, want)


def test_view_nested(b200):
    """view_nested (view.rs:41-67): a full copy, then a nested tile (132 of 264 of 528) copied onto
    itself; the output equals the input."""
    ax = dict(A=512, B=528)
    hbm, dm = M("[A, B]", **ax), M("[A / 256, A % 256, B]", **ax)
    x = np.random.default_rng(5).integers(-2**31, 2**31 - 1, 512 * 528).astype(np.int32)
    inp = b200.relayout(b200.from_vec(hbm, x, "i32"), hbm, dm)
    out = b200.zeroed(dm, "i32")
    b200.transpose(out, inp, dm, dm)
    b200.transpose(out, inp, M("[A / 256, A % 256, B = 132 # 528]", **ax),
                   M("[A / 256, A % 256, B = 132 #{!} 528]", **ax), src_offset={"B": 0}, dst_offset={"B": 0},
                   src_map=dm, dst_map=dm)
    assert np.array_equal(b200.relayout(out, dm, hbm).to_numpy(), x)


# ---- param_tests.rs (src/param.rs): a tuple / struct parameter passes through DM unchanged --------
def test_param_passthrough(b200):
    ax = dict(A=4096, B=8)
    hbm, dm = M("[A, B]", **ax), M("[1 # 2, A / 16, A / 8 % 2, A % 8, B]", **ax)
    x = (np.arange(32768) % 256).astype(np.uint8).view(np.int8)
    out = b200.relayout(b200.relayout(b200.from_vec(hbm, x, "i8"), hbm, dm), dm, hbm)
    assert np.array_equal(out.to_numpy(), x)


# ---- runtime_if_tests.rs (src/runtime_if.rs): the two arms write input + 1 and input + 2 ---------
def test_runtime_if_two_outputs(b200):
    ax = dict(W=1024)
    hbm, dm = M("[W]", **ax), M("[1, W / 4, W % 4]", **ax)        # Cluster m![1], Slice [W / 4], [W % 4]
    collect = M("[1, W / 4, W % 4 # 8]", **ax)                     # collect::<m![1], m![W % 4 # 8]>
    x = np.arange(1024, dtype=np.int32)
    d = b200.relayout(b200.from_vec(hbm, x, "i32"), hbm, dm)
    outs = []
    for c in (1, 2):                                              # if i == 0 { +1 } else { +2 }
        v = b200.map(b200.relayout(d, dm, collect), ops.with_const_i32(ops.FXP_BINARY, "AddFxp", c), "i32")
        view = b200.zeroed(dm, "i32")
        b200.transpose(view, v, collect, dm)                      # commit_trim::<m![W % 4]>, commit_view
        outs.append(b200.relayout(view, dm, hbm).to_numpy())
    assert np.array_equal(outs[0], x + 1) and np.array_equal(outs[1], x + 2)


# ---- runtime_if_scalar_tests.rs (src/runtime_if_scalar.rs): a runtime tile index copies both halves
def test_runtime_if_scalar_index(b200):
    ax = dict(A=512, B=32)
    hbm, dm = M("[A, B]", **ax), M("[A / 256, A % 256, B]", **ax)
    x = (np.arange(512 * 32) % 256).astype(np.uint8).view(np.int8)
    inp = b200.relayout(b200.from_vec(hbm, x, "i8"), hbm, dm)
    out = b200.zeroed(dm, "i8")
    for i in range(2):
        off = 0 if i == 0 else 16
        b200.transpose(out, inp, M("[A / 256, A % 256, B = 16 # 32]", **ax),
                       M("[A / 256, A % 256, B = 16 #{!} 32]", **ax), src_offset={"B": off}, dst_offset={"B": off},
                       src_map=dm, dst_map=dm)
    assert np.array_equal(b200.relayout(out, dm, hbm).to_numpy(), x)


# ---- host_tile_view_tests.rs (src/host_tile_view.rs): move one row of a table to another ---------
@pytest.mark.parametrize("moves", [[(3, 5)], [(0, 63), (32, 32), (63, 0), (3, 5)]])
def test_host_tile_move(b200, moves):
    ax = dict(C=64, H=64)
    base = M("[C, H]", **ax)
    table = dtypes.f32_to_bf16_bits(np.repeat(np.arange(64, dtype=np.float32), 64))   # row r holds r
    src = b200.from_vec(base, table, "bf16")
    out = b200.from_vec(base, dtypes.f32_to_bf16_bits(np.full(64 * 64, -1.0, np.float32)), "bf16")
    for s, d in moves:                                            # tile::<m![C], 1, SmallRow(Mut)>(row)
        b200.transpose(out, src, M("[1 # 64, H]", **ax), M("[1 #{!} 64, H]", **ax), src_offset={"C": s},
                       dst_offset={"C": d}, src_map=base, dst_map=base)
    got = dtypes.bf16_bits_to_f32(out.to_numpy()).reshape(64, 64)
    for r in range(64):
        want = next((float(s) for s, d in moves if d == r), -1.0)
        assert np.all(got[r] == want), f"row {r}"


# ---- memory_op_tests.rs (src/memory_op.rs) --------------------------------------------------------
def test_dm_relayout(b200):
    """dm_relayout: [A, B] -> DM [1 # 2, A, B] -> DM [1 # 2, 1 # 2, A / 2, A % 2, B] -> HBM
    [A / 2, A % 2, B], whose order is the input's (the example's test only runs it)."""
    ax = dict(A=256, B=4096)
    hbm = M("[A, B]", **ax)
    dm, relaid = M("[1 # 2, A, B]", **ax), M("[1 # 2, 1 # 2, A / 2, A % 2, B]", **ax)
    out_map = M("[A / 2, A % 2, B]", **ax)
    x = np.arange(256 * 4096, dtype=np.int32)
    r = b200.relayout(b200.relayout(b200.from_vec(hbm, x, "i32"), hbm, dm), dm, relaid)
    assert np.array_equal(b200.relayout(r, relaid, out_map).to_numpy(), x)


def test_commit_view_bottom_pad(b200):
    """commit_view_bottom_pad: an 8-wide [T, Q % 56 = 8] tensor committed into the first 8 of 56
    columns of a [T % 32, Q % 56] DM tile; the other 48 columns stay unwritten."""
    ax = dict(T=512, Q=896)
    hin = M("[T, Q % 56 = 8]", **ax)
    din = M("[1 # 2, T / 32 # 256, T % 32, Q % 56 = 8]", **ax)
    dres = M("[1 # 2, T / 32 # 256, T % 32, Q % 56]", **ax)
    x = np.random.default_rng(42).random(512 * 8).astype(np.float32)
    d = b200.relayout(b200.from_vec(hin, x, "f32"), hin, din)
    res = b200.zeroed(dres, "f32")
    b200.transpose(res, d, din, M("[1 # 2, T / 32 # 256, T % 32, Q % 56 = 8 #{!} 56]", **ax),
                   src_offset={}, dst_offset={"Q": 0}, src_map=din, dst_map=dres)
    got = b200.relayout(res, dres, M("[T, Q % 56]", **ax)).to_numpy().reshape(512, 56)
    assert np.array_equal(got[:, :8], x.reshape(512, 8)) and np.all(got[:, 8:] == 0)
