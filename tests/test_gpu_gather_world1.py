"""The fused row-shard gather on ONE GPU (world 1: the rank gathers to
itself), so that the store / arrival counter / bounded-wait path runs on a
1-GPU box too; and the bounded wait running out.

The row split is the reference's (src/ops/quant.rs:1120-1143: rows are
independent reductions, so a shard's rows are the full result's rows); the
gathered y must equal the oracle's y bit for bit. Error convention: a wait
that runs out is reported as VTQ_ERR_TIMEOUT (no reference counterpart; the
reference's parallel linears cannot time out, src/error.rs:7-63), and leaves
the context usable."""
import numpy as np
import pytest

import vtq
from vtq import synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu

SHAPES = [(vtq.Q4_K, 4096, 1024), (vtq.Q6_K, 4096, 2000), (vtq.Q4_K, 11008, 512)]
NAME = {vtq.Q4_K: "q4_k_integer", vtq.Q6_K: "q6_k_integer"}


def _setup(ctx):
    import torch
    total = sum(r for _, _, r in SHAPES)
    gat = vtq.Gather(ctx, total)
    offs = [sum(r for _, _, r in SHAPES[:i]) for i in range(len(SHAPES))]
    ws, xs, refs = [], [], []
    for i, (dt, n, r) in enumerate(SHAPES):
        w = synth.weight(dt, f"gather1.{i}", r, n, seed=i)
        x = synth.activation(f"gather1.x.{i}", 1, n, seed=i)
        ws.append(ctx.upload(dt, w, n, r))
        xs.append(torch.from_numpy(x).cuda())
        refs.append(O.linear(NAME[dt], x, w, 1, n, r, 8))
    return gat, offs, ws, xs, np.concatenate(refs), total


@pytest.mark.parametrize("defer", [False, True])
def test_world1_gather_bit_exact(defer):
    import torch
    ctx = vtq.Context(0)
    gat, offs, ws, xs, ref, total = _setup(ctx)
    for step in range(4):  # counters keep growing across steps
        for i, (dt, n, r) in enumerate(SHAPES):
            last = i == len(SHAPES) - 1
            signals = (1 if defer else len(SHAPES)) if last else 0
            gat.linear(ws[i], xs[i].data_ptr(), 0, r, y_offset=offs[i],
                       wait_signals=signals, defer=defer and not last)
        ctx.synchronize()
        got = vtq._device_floats(gat.y_ptr, total)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), step
    # The separate wait kernel: one more step, then wait for its arrivals.
    for i, (dt, n, r) in enumerate(SHAPES):
        gat.linear(ws[i], xs[i].data_ptr(), 0, r, y_offset=offs[i])
    gat.wait(len(SHAPES))
    ctx.synchronize()
    gat.close()
    ctx.close()


def test_bounded_wait_runs_out_and_the_context_stays_usable():
    ctx = vtq.Context(0)
    gat, offs, ws, xs, ref, total = _setup(ctx)
    dt, n, r = SHAPES[0]
    gat.linear(ws[0], xs[0].data_ptr(), 0, r, y_offset=offs[0], wait_signals=1)
    ctx.synchronize()
    ctx.set_wait_limit(50_000_000)  # 50 ms
    gat.wait(5)  # five arrivals that nothing will send
    with pytest.raises(vtq.Timeout):
        ctx.synchronize()
    ctx.synchronize()  # the flag was reported once and cleared
    # The gather still works: the missing arrivals were not counted as seen.
    for i, (dt, n, r) in enumerate(SHAPES):
        gat.linear(ws[i], xs[i].data_ptr(), 0, r, y_offset=offs[i],
                   wait_signals=len(SHAPES) if i == len(SHAPES) - 1 else 0)
    ctx.synchronize()
    got = vtq._device_floats(gat.y_ptr, total)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    # And so does a plain linear on the same context.
    w = synth.weight(vtq.Q4_K, "gather1.0", 1024, 4096, seed=0)
    x = synth.activation("gather1.x.0", 1, 4096, seed=0)
    y = ctx.linear(ws[0], x, 1)
    assert np.array_equal(y.view(np.uint32), ref[:1024].view(np.uint32))
    gat.close()
    ctx.close()


def test_world1_list_gather_bit_exact():
    """vtq_linear_list_gather: one persistent launch over all three shards'
    matvecs (twice over), rows into the gather buffer, one arrival signal per
    launch, each launch waiting for the previous launch's arrival."""
    ctx = vtq.Context(0)
    gat, offs, ws, xs, ref, total = _setup(ctx)
    items = [(ws[i], xs[i].data_ptr(), offs[i]) for i in range(len(SHAPES))] * 2
    for step in range(4):
        gat.linear_list(items, wait_signals=1 if step > 0 else 0)
    gat.wait(1)  # the last launch's arrival
    ctx.synchronize()
    got = vtq._device_floats(gat.y_ptr, total)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    gat.close()
    ctx.close()
