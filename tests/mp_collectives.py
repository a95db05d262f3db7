"""Run under torchrun (one rank per GPU): checks the Chip-axis collectives against numpy.
all-reduce: sum over ranks (bf16: exact for 2 ranks, since one rounding of the exact sum is the
reference's bf16 `+`; within 1 bf16 ulp per extra rank otherwise). chip shuffle: byte-exact."""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "tests"))
import conftest  # noqa: E402,F401  (binds the furiosa_opt_b200 package)
import furiosa_opt_b200 as fb  # noqa: E402

rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
torch.cuda.set_device(local)
dist.init_process_group("nccl")
be = fb.B200(local)
fb.dist.init_comm(be, rank, world)
n = 1 << 20
m = fb.Mapping("[E]", dict(E=n))
vals = [fb.dtypes.f32_to_bf16_bits(np.random.default_rng(r).standard_normal(n).astype(np.float32))
        for r in range(world)]
x = be.from_vec(m, vals[rank], "bf16")
fb.dist.allreduce(be, x)
got = fb.dtypes.bf16_bits_to_f32(x.to_numpy()).astype(np.float64)
exact = sum(fb.dtypes.bf16_bits_to_f32(v).astype(np.float64) for v in vals)
want = fb.dtypes.bf16_bits_to_f32(fb.dtypes.f32_to_bf16_bits(exact.astype(np.float32))).astype(np.float64)
if world == 2:
    assert np.array_equal(got, want), np.max(np.abs(got - want))
else:
    assert np.all(np.abs(got - exact) <= (world - 1) * 2 ** -7 * np.abs(exact) + 1e-6)
# chip shuffle: target t receives chip pattern[t]
pattern = [(t + 1) % world for t in range(world)]
src = be.from_vec(m, vals[rank], "bf16")
dst = be.zeroed(m, "bf16")
fb.dist.chip_shuffle(be, dst, src, pattern)
assert np.array_equal(dst.to_numpy(), vals[pattern[rank]])
# max / min / product folds over the Chip axis (f32, exact)
fv = [np.random.default_rng(100 + r).standard_normal(4096).astype(np.float32) for r in range(world)]
for op, fold in (("Max", np.maximum), ("Min", np.minimum)):
    y = be.from_vec(fb.Mapping("[E]", dict(E=4096)), fv[rank], "f32")
    fb.dist.allreduce(be, y, op)
    want_f = fv[0]
    for r in range(1, world):
        want_f = fold(want_f, fv[r])
    assert np.array_equal(y.to_numpy(), want_f), op
# the tensor-parallel decoder block: bit-identical to the single-GPU block (same weights)
from furiosa_opt_b200 import workloads as W  # noqa: E402
batch, seq, Hq, Hkv, F = 2, 128, 4, 2, 1024
T, H = batch * seq, Hq * 128
tp = W.DecoderBlockW8A8TP(be, T, H, Hq, Hkv, F, batch, seq, rank, world, seed=3)
one = W.DecoderBlockW8A8(be, T, H, Hq, Hkv, F, batch, seq, seed=3)
xb = fb.dtypes.f32_to_bf16_bits(np.random.default_rng(5).standard_normal(T * H).astype(np.float32))
got_tp = tp.forward(be.from_vec(tp.m("[T, H]"), xb, "bf16")).to_bytes()
got_one = one.forward(be.from_vec(one.m("[T, H]"), xb, "bf16")).to_bytes()
assert got_tp == got_one, "tensor-parallel block differs from the single-GPU block"
dist.barrier()
if rank == 0:
    print(f"collectives ok on {world} ranks")
dist.destroy_process_group()
