"""vtq_linear_list: a run of integer k-quant linears in one persistent launch.

Every item's y must equal the oracle's linear (linear_q4_k_integer /
linear_q6_k_integer, src/ops/quant.rs:936-980, :1060-1146) bit for bit: for
independent items, for a chain whose x is an earlier item's y (wait_for, the
FFN up -> down order of forward_quantized.rs:540-575), for mixed formats and
row lengths, for fewer rows than CTAs, across repeated launches (the counters
must come back to zero) and under CUDA graph replay."""
import numpy as np
import pytest

import vtq
from vtq import synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu

NAME = {vtq.Q4_K: "q4_k_integer", vtq.Q6_K: "q6_k_integer"}


def bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32),
                          np.asarray(b, np.float32).view(np.uint32))


def _setup(ctx, shapes, tag):
    import torch
    ws, xs, ys, host = [], [], [], []
    for i, (dt, n, r) in enumerate(shapes):
        w = synth.weight(dt, f"list.{tag}.w{i}", r, n, seed=i)
        x = synth.activation(f"list.{tag}.x{i}", 1, n, seed=i)
        ws.append(ctx.upload(dt, w, n, r))
        xs.append(torch.from_numpy(x).cuda())
        ys.append(torch.full((r,), float("nan"), device="cuda"))
        host.append((w, x))
    return ws, xs, ys, host


@pytest.mark.parametrize("shapes", [
    [(vtq.Q4_K, 4096, 11008), (vtq.Q4_K, 11008, 4096)],          # the Llama-7B FFN pair
    [(vtq.Q6_K, 4096, 3000), (vtq.Q4_K, 256, 1), (vtq.Q6_K, 5632, 147),
     (vtq.Q4_K, 32768, 149), (vtq.Q6_K, 768, 13), (vtq.Q4_K, 2048, 300)],
    # 33..48 superblocks per row: 16-lane segments of 3 superblocks each.
    [(vtq.Q6_K, 8448, 700), (vtq.Q4_K, 12288, 301), (vtq.Q6_K, 9216, 37),
     (vtq.Q4_K, 11008, 1)],
])
def test_independent_items_bit_exact(ctx, shapes):
    import torch
    ws, xs, ys, host = _setup(ctx, shapes, len(shapes))
    items = [(w, x.data_ptr(), y.data_ptr()) for w, x, y in zip(ws, xs, ys)]
    for rep in range(3):  # counters reset by the kernel: repeated launches stay exact
        for y in ys:
            y.fill_(float("nan"))
        ctx.linear_list(items)
        torch.cuda.synchronize()
        for (dt, n, r), (w, x), y in zip(shapes, host, ys):
            ref = O.linear(NAME[dt], x, w, 1, n, r, 8)
            assert bits_equal(y.cpu().numpy(), ref), (rep, dt, n, r)


def test_chain_waits_for_the_earlier_item(ctx):
    """up (4096 -> 11008) then down (11008 -> 4096) reading up's y, then a
    Q6_K head reading down's y: each x is produced inside the same launch."""
    import torch
    shapes = [(vtq.Q4_K, 4096, 11008), (vtq.Q4_K, 11008, 4096), (vtq.Q6_K, 4096, 2000)]
    ws, xs, ys, host = _setup(ctx, shapes, "chain")
    items = [(ws[0], xs[0].data_ptr(), ys[0].data_ptr(), -1),
             (ws[1], ys[0].data_ptr(), ys[1].data_ptr(), 0),
             (ws[2], ys[1].data_ptr(), ys[2].data_ptr(), 1)]
    (w0, x0), (w1, _), (w2, _) = host
    r0 = O.linear("q4_k_integer", x0, w0, 1, 4096, 11008, 8)
    r1 = O.linear("q4_k_integer", r0, w1, 1, 11008, 4096, 8)
    r2 = O.linear("q6_k_integer", r1, w2, 1, 4096, 2000, 8)
    for rep in range(3):
        for y in ys:
            y.fill_(float("nan"))
        ctx.linear_list(items)
        torch.cuda.synchronize()
        for y, ref in zip(ys, (r0, r1, r2)):
            assert bits_equal(y.cpu().numpy(), ref), rep


def test_graph_replay_matches_eager(ctx):
    import torch
    shapes = [(vtq.Q4_K, 4096, 1024), (vtq.Q6_K, 1024, 4096), (vtq.Q4_K, 4096, 512)]
    ws, xs, ys, host = _setup(ctx, shapes, "graph")
    stream = torch.cuda.Stream()
    items = [(ws[0], xs[0].data_ptr(), ys[0].data_ptr(), -1),
             (ws[1], ys[0].data_ptr(), ys[1].data_ptr(), 0),
             (ws[2], ys[1].data_ptr(), ys[2].data_ptr(), 1)]
    (w0, x0), (w1, _), (w2, _) = host
    r0 = O.linear("q4_k_integer", x0, w0, 1, 4096, 1024, 8)
    r1 = O.linear("q6_k_integer", r0, w1, 1, 1024, 4096, 8)
    r2 = O.linear("q4_k_integer", r1, w2, 1, 4096, 512, 8)
    ctx.set_stream(stream.cuda_stream)
    try:
        with torch.cuda.stream(stream):
            ctx.linear_list(items)  # eager once (sets the kernel attributes)
            stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                ctx.linear_list(items)
                ctx.linear_list(items)
            for _ in range(3):
                for y in ys:
                    y.fill_(float("nan"))
                g.replay()
            stream.synchronize()
    finally:
        ctx.set_stream(None)
    for y, ref in zip(ys, (r0, r1, r2)):
        assert bits_equal(y.cpu().numpy(), ref)


def test_list_validation(ctx):
    w = ctx.upload(vtq.Q8_0, synth.weight(vtq.Q8_0, "list.q8", 4, 64), 64, 4)
    with pytest.raises(vtq.NotImplementedOp):
        ctx.linear_list([(w, 16, 16)])
    w4 = ctx.upload(vtq.Q4_K, synth.weight(vtq.Q4_K, "list.q4", 4, 256), 256, 4)
    with pytest.raises(vtq.InvalidArg):
        ctx.linear_list([(w4, 16, 16, 0)])  # wait_for must name an earlier item
    with pytest.raises(vtq.InvalidArg):
        ctx.linear_list([(w4, 16, 16)] * (vtq.LIST_MAX + 1))
    # Host pointers cannot name an earlier item's y as x.
    x = np.zeros(256, np.float32)
    y = np.zeros(8, np.float32)
    with pytest.raises(vtq.InvalidArg):
        ctx.linear_list([(w4, x.ctypes.data, y.ctypes.data),
                         (w4, x.ctypes.data, y.ctypes.data + 16, 0)],
                        host=True)


@pytest.mark.parametrize("pinned", [True, False])
def test_host_pointer_list(ctx, pinned):
    """VTQ_PTR_HOST: page-locked x / y are read and written in place by the
    kernel; pageable ones are staged. Both must equal the device-pointer run."""
    import torch
    shapes = [(vtq.Q4_K, 4096, 1100), (vtq.Q6_K, 2048, 300), (vtq.Q4_K, 11008, 77)]
    ws, xs, ys, host = _setup(ctx, shapes, "host")
    ctx.linear_list([(w, x.data_ptr(), y.data_ptr()) for w, x, y in zip(ws, xs, ys)])
    torch.cuda.synchronize()
    want = [y.cpu().numpy() for y in ys]
    for rep in range(2):
        if pinned:
            hx = [torch.from_numpy(x).pin_memory() for _, x in host]
            hy = [torch.full((r,), float("nan")).pin_memory() for _, _, r in shapes]
            ptrs = [(t.data_ptr(), u.data_ptr()) for t, u in zip(hx, hy)]
            out = lambda: [u.numpy() for u in hy]
        else:
            hx = [np.array(x) for _, x in host]
            hy = [np.full(r, np.nan, np.float32) for _, _, r in shapes]
            ptrs = [(t.ctypes.data, u.ctypes.data) for t, u in zip(hx, hy)]
            out = lambda: hy
        ctx.linear_list([(w, px, py) for w, (px, py) in zip(ws, ptrs)], host=True)
        for got, ref in zip(out(), want):
            assert bits_equal(got, ref), rep
