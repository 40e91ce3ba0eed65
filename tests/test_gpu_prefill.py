"""GPU parity for the batched (prefill) integer Q4_K linear: the tcgen05 GEMM
path that vtq_linear takes for Q4_K at batch >= 16, bit-exact against the CPU
oracle's linear_q4_k_integer (src/ops/quant.rs:936-980 with batch > 1: every
activation row quantised independently, every (b, o) its own fixed_tree)."""
import numpy as np
import pytest

import vtq
from vtq import synth
from oracle import oracle as O

from tests.test_gpu_parity import assert_bits

pytestmark = pytest.mark.gpu

CASES = [  # (in_feat, out_feat, batch)
    (256, 32, 128),     # one superblock, one tile
    (512, 45, 130),     # ragged rows and tokens
    (768, 100, 16),     # smallest batch on the GEMM path
    (2048, 33, 300),    # S = 8, three token tiles
    (4096, 96, 257),    # S = 16 (a power of two: the tree's root is one subtree)
    (5632, 40, 64),     # S = 22
    (14336, 64, 129),   # S = 56 (Mistral w2 rows)
    (11008, 37, 33),    # S = 43
]


@pytest.mark.parametrize("n,r,batch", CASES)
def test_q4k_batched_bit_exact(ctx, n, r, batch):
    w = synth.weight(vtq.Q4_K, f"pf.w.{n}x{r}", r, n, seed=7)
    x = synth.activation(f"pf.x.{n}", batch, n, seed=batch)
    wt = ctx.upload(vtq.Q4_K, w, n, r)
    got = ctx.linear(wt, x, batch)
    ref = O.linear("q4_k_integer", x, w, batch, n, r, 16)
    assert_bits(got, ref)


def test_q4k_batched_matches_per_row_matvec(ctx):
    """Batch 64 through the GEMM equals 64 separate batch-1 calls (matvec path)."""
    n, r, batch = 4096, 70, 64
    w = synth.weight(vtq.Q4_K, "pf.rows", r, n, seed=3)
    x = synth.activation("pf.rows.x", batch, n, seed=5)
    wt = ctx.upload(vtq.Q4_K, w, n, r)
    got = ctx.linear(wt, x, batch)
    rows = np.concatenate([ctx.linear(wt, x[b * n:(b + 1) * n], 1) for b in range(batch)])
    assert_bits(got, rows)


def test_q4k_batched_edge_activations(ctx):
    """Zero rows, NaN / infinity / subnormal entries and huge magnitudes."""
    n, r, batch = 1024, 48, 40
    w = synth.weight(vtq.Q4_K, "pf.edge", r, n, seed=11)
    x = synth.activation("pf.edge.x", batch, n, seed=2).reshape(batch, n).copy()
    x[0] = 0.0
    x[1, 5] = np.nan
    x[2, 7] = np.inf
    x[3, 300] = -np.inf
    x[4] = np.float32(1e-42)
    with np.errstate(over="ignore"):
        x[5] *= np.float32(3e38)
    x[6, :256] = np.nan
    x = x.reshape(-1)
    wt = ctx.upload(vtq.Q4_K, w, n, r)
    got = ctx.linear(wt, x, batch)
    ref = O.linear("q4_k_integer", x, w, batch, n, r, 16)
    assert_bits(got, ref, skip_nonfinite=True)


def test_q4k_batched_random_weight_bytes(ctx):
    """Arbitrary bytes: non-finite and subnormal fp16 d / dmin, every scale code."""
    n, r, batch = 2048, 64, 32
    rng = np.random.default_rng(9)
    w = rng.integers(0, 256, size=r * (n // 256) * 144, dtype=np.uint8)
    x = synth.activation("pf.rand.x", batch, n, seed=4)
    wt = ctx.upload(vtq.Q4_K, w, n, r)
    got = ctx.linear(wt, x, batch)
    ref = O.linear("q4_k_integer", x, w, batch, n, r, 16)
    assert_bits(got, ref, skip_nonfinite=True)


def test_config5_wk_full_size(ctx):
    """Config 5 shape: Mistral wk (1024 x 4096) at M = 512 tokens."""
    n, r, batch = 4096, 1024, 512
    w = synth.weight(vtq.Q4_K, "c5.wk", r, n, seed=0)
    x = synth.activation("c5.x.4096", batch, n, seed=0)
    wt = ctx.upload(vtq.Q4_K, w, n, r)
    got = ctx.linear(wt, x, batch)
    ref = O.linear("q4_k_integer", x, w, batch, n, r, 32)
    assert_bits(got, ref)


def test_device_api_with_caller_workspace(ctx):
    """vtq_linear_device_ws: the batched Q4_K path on caller-owned scratch gives
    the same bits as vtq_linear, and a too-small workspace is rejected."""
    import torch
    lib = vtq.load_library()
    n, r, b = 2048, 200, 40
    w = synth.weight(vtq.Q4_K, "ws.w", r, n)
    x = synth.activation("ws.x", b, n)
    ref = ctx.linear(ctx.upload(vtq.Q4_K, w, n, r), x, b)
    raw = torch.from_numpy(w).cuda()
    dst = torch.empty(lib.vtq_device_layout_bytes(vtq.Q4_K, n, r), dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert lib.vtq_device_repack(vtq.Q4_K, n, r, raw.data_ptr(), dst.data_ptr(), st) == vtq.OK
    need = lib.vtq_linear_device_workspace_bytes(vtq.Q4_K, n, b, 0)
    assert need >= b * n + b * (n // 256) * 4
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty(b * r, device="cuda")
    assert lib.vtq_linear_device_ws(vtq.Q4_K, dst.data_ptr(), n, r, dx.data_ptr(), n,
                                    dy.data_ptr(), r, b, 0, None, ws.data_ptr(), need - 256,
                                    st) == vtq.ERR_INVALID_ARG
    assert lib.vtq_linear_device_ws(vtq.Q4_K, dst.data_ptr(), n, r, dx.data_ptr(), n,
                                    dy.data_ptr(), r, b, 0, None, ws.data_ptr(), need,
                                    st) == vtq.OK
    torch.cuda.synchronize()
    assert np.array_equal(dy.cpu().numpy().view(np.uint32), ref.view(np.uint32))
