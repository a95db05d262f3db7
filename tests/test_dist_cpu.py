"""Host-side multi-rank logic on CPU: gloo ranks (no GPU) running the library's own host code.

  * the chip-shuffle peer plan (fopt_chip_shuffle_plan, the plan fopt_chip_shuffle executes over
    NCCL) drives a real exchange of slabs between 4 gloo ranks, which must realise
    `pattern[target] = source` (memory.rs:657-679, cluster_chip_shuffle_slice.rs:5-19);
  * the communicator rendezvous (dist.exchange_unique_id with the library's fopt_comm_unique_id on
    rank 0) delivers rank 0's id to every rank;
  * the bench's max-over-ranks timing reduction.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import furiosa_opt_b200 as fb


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shuffle_peers_plan():
    pattern = [1, 2, 3, 0]  # cluster_chip_shuffle_slice.rs:7-19: target t receives chip pattern[t]
    plans = [fb.dist.shuffle_peers(pattern, r) for r in range(4)]
    for r, (sends, recv) in enumerate(plans):
        assert recv == pattern[r]
        for t in sends:
            assert plans[t][1] == r
    assert fb.dist.shuffle_peers([0, 1, 2, 3], 2) == ([], 2)
    with pytest.raises(ValueError):
        fb.dist.shuffle_peers([0, 0, 1, 2], 0)
    with pytest.raises(ValueError):
        fb.dist.shuffle_peers([0, 1, 4, 2], 0)


def _worker(rank, world, port, pattern, q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)

    def bcast(buf):
        t = torch.tensor(list(buf), dtype=torch.uint8)
        dist.broadcast(t, 0)
        buf[:] = bytes(t.tolist())

    uid = fb.dist.exchange_unique_id(rank, world, bcast)
    # the chip shuffle plan, executed with gloo point-to-point in place of NCCL
    slab = torch.from_numpy((np.arange(4096, dtype=np.int32) + 100000 * rank))
    out = torch.zeros_like(slab)
    sends, frm = fb.dist.shuffle_peers(pattern, rank)
    reqs = [dist.isend(slab, t) for t in sends]
    if frm != rank:
        dist.recv(out, frm)
    else:
        out.copy_(slab)
    for r in reqs:
        r.wait()
    t = torch.tensor([float(rank + 1)])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)  # the bench's max-over-ranks timing reduction
    q.put((rank, uid, out.numpy().copy(), float(t)))
    dist.destroy_process_group()


@pytest.mark.parametrize("world,pattern", [(2, [1, 0]), (4, [1, 2, 3, 0]), (4, [2, 1, 3, 0])])
def test_gloo_ranks_run_the_library_plan(world, pattern):
    ctx = mp.get_context("fork")  # no CUDA state in this process
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, pattern, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    uids = {uid for _, uid, _, _ in got}
    assert len(uids) == 1 and len(next(iter(uids))) == 128 and any(next(iter(uids)))
    for rank, _, out, mx in got:
        assert np.array_equal(out, np.arange(4096, dtype=np.int32) + 100000 * pattern[rank])
        assert mx == float(world)
