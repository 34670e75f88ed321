"""The multi-GPU split on CPU: world-size-2 gloo ranks each take their
contiguous patch slice (bnns_to_c_b200.shard_range, the split the library's
bnn_forward_batch and bench.py's ranks use), run it through the CPU oracle,
and the gathered result must equal the unsharded batch bit for bit. No GPU
and no data-path collective: the gather exists only to check."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bnns_to_c_b200 as bn

GOLD = os.path.join(os.path.dirname(__file__), "golden")
N, H, W = 5, 16, 16


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(__file__))
    from oracle_util import OModel, synth
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lo, hi = bn.shard_range(N, rank, world)
    om = OModel(os.path.join(GOLD, "unet_c8_mixed_s1.blob"))
    x = synth(31, lo, hi - lo, 120, H, W)          # patches lo..hi-1 of the global batch
    mine = torch.from_numpy(om.forward_batch(x))
    sizes = [bn.shard_range(N, r, world) for r in range(world)]
    bufs = [torch.empty((h - l, 3, H, W)) for l, h in sizes]
    dist.all_gather(bufs, mine) if len({h - l for l, h in sizes}) == 1 else _gather_ragged(bufs, mine, rank)
    if rank == 0:
        q.put(torch.cat(bufs).numpy())
    dist.destroy_process_group()


def _gather_ragged(bufs, mine, rank):
    bufs[rank].copy_(mine)
    for r, b in enumerate(bufs):
        dist.broadcast(b, src=r)


def test_shard_range_partitions():
    for n in (0, 1, 5, 4096, 4097):
        for w in (1, 2, 3, 8):
            s = [bn.shard_range(n, r, w) for r in range(w)]
            assert s[0][0] == 0 and s[-1][1] == n
            assert all(s[i][1] == s[i + 1][0] for i in range(w - 1))
            assert max(h - l for l, h in s) - min(h - l for l, h in s) <= 1


def test_two_gloo_ranks_reproduce_unsharded_batch():
    from oracle_util import OModel, synth
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = OModel(os.path.join(GOLD, "unet_c8_mixed_s1.blob")).forward_batch(synth(31, 0, N, 120, H, W))
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
