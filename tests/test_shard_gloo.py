"""Row-sharded linear host logic on 2 CPU ranks (gloo): each rank computes its
row shard with the oracle, the all-gather reassembles y, and the result is
bit-identical to the unsharded linear (shard-count invariance, the property
the reference's thread-count test asserts, quant.rs:2063-2095)."""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, rows, q):
    sys.path[:0] = [REPO, os.path.join(REPO, "vitni-tensor_b200")]
    import torch
    import torch.distributed as dist
    from oracle import oracle as O
    from vtq import Q6_K, row_bytes, shard, synth
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n, batch = 512, 2
        w = synth.weight(Q6_K, "shard.w", rows, n)
        x = synth.activation("shard.x", batch, n)
        a, b = shard.row_range(rows, world, rank)
        rb = row_bytes(Q6_K, n)
        local = O.linear("q6_k_integer", x, w[a * rb:b * rb], batch, n, b - a)
        y = shard.gather_rows(torch.from_numpy(local), rows, batch).numpy()
        full = O.linear("q6_k_integer", x, w, batch, n, rows)
        q.put((rank, bool(np.array_equal(y.reshape(-1).view(np.uint32), full.view(np.uint32)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,rows", [(2, 64), (2, 37), (3, 50)])
def test_sharded_gather_is_bit_identical(world, rows):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, rows, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    results = dict(q.get(timeout=5) for _ in range(world))
    assert all(p.exitcode == 0 for p in procs)
    assert all(results[r] for r in range(world))


def test_row_ranges_cover_exactly():
    sys.path[:0] = [os.path.join(REPO, "vitni-tensor_b200")]
    from vtq import shard
    for rows in (1, 7, 4096, 32000, 11008):
        for world in (1, 2, 3, 4, 8):
            rr = shard.shard_rows(rows, world)
            assert rr[0][0] == 0 and rr[-1][1] == rows
            assert all(rr[i][1] == rr[i + 1][0] for i in range(world - 1))
            assert max(b - a for a, b in rr) - min(b - a for a, b in rr) <= 1
