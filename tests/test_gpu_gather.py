"""Fused row-shard all-gather (vtq_linear_gather / vtq_gather_wait) on 2 GPUs:
every rank computes its contiguous rows and stores them into every rank's full
y over NVLink; the gathered y must equal the oracle's full y bit for bit
(rows are independent reductions, src/ops/quant.rs:1373-1377). Skipped unless
the process sees at least two GPUs."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WORLD = 2
SHAPES = [(12, 4096, 1024), (14, 4096, 2000), (12, 11008, 512)]  # (dtype, in, rows)


def _rank(rank, port, q):
    import torch
    import torch.distributed as dist
    import vtq
    from vtq import synth, shard
    from oracle import oracle as O
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=WORLD)
        ctx = vtq.Context(rank)
        total = sum(r for _, _, r in SHAPES)
        gat = vtq.Gather(ctx, total)
        offs = [sum(r for _, _, r in SHAPES[:i]) for i in range(len(SHAPES))]
        ws, xs, refs = [], [], []
        for i, (dt, n, r) in enumerate(SHAPES):
            w = synth.weight(dt, f"gather.{i}", r, n, seed=i)
            x = synth.activation(f"gather.x.{i}", 1, n, seed=i)
            a, b = shard.row_range(r, WORLD, rank)
            ws.append((ctx.upload(dt, w, n, r, a, b), a))
            xs.append(torch.from_numpy(x).cuda())
            name = "q4_k_integer" if dt == 12 else "q6_k_integer"
            refs.append(O.linear(name, x, w, 1, n, r, 8))
        for step in range(4):  # counters keep growing across steps
            inline = step % 2 == 1  # odd steps: the last launch waits itself
            for i, (dt, n, r) in enumerate(SHAPES):
                last = i == len(SHAPES) - 1
                gat.linear(ws[i][0], xs[i].data_ptr(), ws[i][1], r, offs[i],
                           wait_signals=WORLD * len(SHAPES) if (inline and last) else 0)
            if not inline:
                gat.wait(WORLD * len(SHAPES))
            ctx.synchronize()
            class _View:  # zero-copy torch view of the gather buffer
                __cuda_array_interface__ = {"shape": (total,), "typestr": "<f4",
                                            "data": (gat.y_ptr, False), "version": 3}
            out = torch.as_tensor(_View(), device="cuda").cpu().numpy()
            for i, (dt, n, r) in enumerate(SHAPES):
                got = out[offs[i]:offs[i] + r]
                if not np.array_equal(got.view(np.uint32), refs[i].view(np.uint32)):
                    raise AssertionError(f"rank {rank} step {step} matrix {i}: gathered y differs")
        # The list form: one launch over every shard, one arrival signal per
        # launch, each launch waiting for the previous launch's arrivals.
        items = [(ws[i][0], xs[i].data_ptr(), offs[i] + ws[i][1]) for i in range(len(SHAPES))]
        for step in range(3):
            gat.linear_list(items, wait_signals=WORLD if step > 0 else 0)
        gat.wait(WORLD)
        ctx.synchronize()
        out = vtq._device_floats(gat.y_ptr, total)
        for i, (dt, n, r) in enumerate(SHAPES):
            got = out[offs[i]:offs[i] + r]
            if not np.array_equal(got.view(np.uint32), refs[i].view(np.uint32)):
                raise AssertionError(f"rank {rank} list launch matrix {i}: gathered y differs")
        dist.barrier()
        gat.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))


def test_fused_gather_two_gpus():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res
