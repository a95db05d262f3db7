"""Host-side multi-rank logic on CPU: 2 gloo ranks (no GPU). Checks the chip-shuffle peer plan is
consistent across ranks and that the NCCL-id rendezvous path delivers rank 0's bytes everywhere."""
import os
import socket

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
    with pytest.raises(ValueError):
        fb.dist.shuffle_peers([0, 0, 1, 2], 0)


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)

    def bcast(buf):
        t = torch.tensor(list(buf), dtype=torch.uint8)
        dist.broadcast(t, 0)
        buf[:] = bytes(t.tolist())

    # the id exchange without NCCL: rank 0 contributes a known pattern in place of a real id
    buf = bytearray(range(128)) if rank == 0 else bytearray(128)
    bcast(buf)
    t = torch.tensor([float(rank + 1)])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)  # the bench's max-over-ranks timing reduction
    q.put((rank, bytes(buf), float(t)))
    dist.destroy_process_group()


def test_gloo_rendezvous_two_ranks():
    ctx = mp.get_context("fork")  # no CUDA state in this process
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, buf, mx in got:
        assert buf == bytes(range(128))
        assert mx == 2.0
