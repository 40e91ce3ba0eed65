"""GPU parity: every dtype arm of linear_dispatch through the C ABI, bit-exact
against the CPU oracle (the reference's arithmetic restated), at small odd
shapes and at the benchmark configurations' full sizes."""
import numpy as np
import pytest

import vtq
from vtq import synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def assert_bits(got, ref, skip_nonfinite=False):
    got = np.asarray(got, np.float32).reshape(-1)
    ref = np.asarray(ref, np.float32).reshape(-1)
    assert got.shape == ref.shape
    m = np.isfinite(ref) if skip_nonfinite else np.ones(ref.shape, bool)
    if skip_nonfinite:
        # NaN payloads are not part of the contract (quant.rs:2033-2044): a
        # non-finite reference must still be non-finite, infinities exactly.
        nf = ~m
        assert (~np.isfinite(got[nf])).all()
        inf = np.isinf(ref)
        assert np.array_equal(got[inf], ref[inf])
    bad = np.nonzero(got[m].view(np.uint32) != ref[m].view(np.uint32))[0]
    assert bad.size == 0, (f"{bad.size} mismatches; first at {bad[:5]}: "
                           f"got {got[m][bad[:5]]} ref {ref[m][bad[:5]]}")


ORACLE_NAME = {vtq.Q4_K: "q4_k_integer", vtq.Q6_K: "q6_k_integer"}


def oracle_linear(dtype, x, w, batch, n, r, q4k_float=False, threads=8):
    if dtype in (vtq.Q4_K, vtq.Q6_K) and not q4k_float:
        return O.linear(ORACLE_NAME[dtype], x, w, batch, n, r, threads)
    if dtype == vtq.Q4_K:
        return O.linear("q4_k_fused", x, w, batch, n, r, threads)
    out = []
    for b in range(batch):
        out.append(O.linear_dispatch(dtype, x[b * n:(b + 1) * n], w, n, r, threads=threads))
    return np.concatenate(out)


SMALL = [  # (dtype, in_feat, out_feat, batch)
    (vtq.Q4_K, 256, 1, 1), (vtq.Q4_K, 768, 13, 1), (vtq.Q4_K, 11008, 37, 1),
    (vtq.Q4_K, 14336, 150, 2), (vtq.Q4_K, 2048, 300, 9), (vtq.Q4_K, 4096, 1, 3),
    (vtq.Q6_K, 256, 1, 1), (vtq.Q6_K, 768, 13, 1), (vtq.Q6_K, 5632, 41, 1),
    (vtq.Q6_K, 14336, 150, 2), (vtq.Q6_K, 2048, 300, 9), (vtq.Q6_K, 4352, 3, 1),
    # Long rows and many rows per CTA: the ring holds fewer stages than there
    # are consumer warps, so warps start several ring laps apart.
    (vtq.Q4_K, 32768, 2000, 1), (vtq.Q6_K, 32768, 1200, 2), (vtq.Q4_K, 24576, 1500, 5),
    (vtq.Q8_0, 32, 1, 1), (vtq.Q8_0, 96, 17, 1), (vtq.Q8_0, 8224, 19, 2),
    (vtq.Q8_0, 4096, 33, 5), (vtq.Q8_0, 16416, 5, 1),
    (vtq.Q5_0, 32, 3, 1), (vtq.Q5_0, 1504, 21, 1), (vtq.Q5_0, 9216, 9, 1),
    (vtq.Q4_0, 64, 2, 1), (vtq.Q4_0, 2080, 23, 1), (vtq.Q4_0, 8192, 16, 2),
    (vtq.F32, 1, 1, 1), (vtq.F32, 37, 5, 1), (vtq.F32, 1000, 18, 2), (vtq.F32, 9000, 4, 1),
]


@pytest.mark.parametrize("dtype,n,r,batch", SMALL)
def test_small_shapes_bit_exact(ctx, dtype, n, r, batch):
    w = synth.weight(dtype, f"w{dtype}", r, n, seed=n + r)
    x = synth.activation("x", batch, n, seed=r)
    wt = ctx.upload(dtype, w, n, r)
    got = ctx.linear(wt, x, batch)
    assert_bits(got, oracle_linear(dtype, x, w, batch, n, r))


@pytest.mark.parametrize("n,r,batch", [(256, 3, 1), (4096, 40, 2), (14336, 17, 1), (8448, 9, 5)])
def test_q4k_float_mode_bit_exact(ctx, n, r, batch):
    w = synth.weight(vtq.Q4_K, "wf", r, n, seed=n)
    x = synth.activation("xf", batch, n)
    wt = ctx.upload(vtq.Q4_K, w, n, r)
    got = ctx.linear(wt, x, batch, q4k_float=True)
    assert_bits(got, oracle_linear(vtq.Q4_K, x, w, batch, n, r, q4k_float=True))


def lcg_bytes(seed, n):
    s = seed
    out = np.empty(n, np.uint8)
    for i in range(n):
        s = (s * 6364136223846793005 + 1) & 0xFFFFFFFFFFFFFFFF
        out[i] = (s >> 40) & 0xFF
    return out


@pytest.mark.parametrize("dtype,n,r", [(vtq.Q4_K, 4096, 3), (vtq.Q6_K, 1024, 5),
                                       (vtq.Q8_0, 256, 4), (vtq.Q5_0, 256, 4),
                                       (vtq.Q4_0, 256, 4)])
def test_random_bytes_including_nonfinite_scales(ctx, dtype, n, r):
    """Raw random bytes (the reference's fuzz style, quant.rs:2018-2044): f16
    scales may be Inf/NaN/subnormal. Finite reference outputs must match."""
    w = lcg_bytes(0xC0FFEE + dtype, r * vtq.row_bytes(dtype, n))
    x = synth.activation("xr", 1, n)
    wt = ctx.upload(dtype, w, n, r)
    assert_bits(ctx.linear(wt, x, 1), oracle_linear(dtype, x, w, 1, n, r), skip_nonfinite=True)


def test_activation_edge_cases(ctx):
    """NaN / -0.0 / subnormal / huge activations go through quantize_block_q8's
    exact rules (amax ignores NaN, 0*inf -> 0, saturating cast)."""
    n, r = 1024, 64
    x = synth.activation("xe", 1, n)
    x[3] = np.nan
    x[5] = -0.0
    x[256:512] = 0.0
    x[300] = 1e-40
    x[512:768] = -0.0
    x[800] = 3e38
    x[801] = -np.inf
    for dtype in (vtq.Q4_K, vtq.Q6_K):
        w = synth.weight(dtype, "we", r, n)
        wt = ctx.upload(dtype, w, n, r)
        assert_bits(ctx.linear(wt, x, 1), oracle_linear(dtype, x, w, 1, n, r),
                    skip_nonfinite=True)


@pytest.mark.parametrize("cfg", ["c1_q8_0_4096x4096", "c2_q4_k_llama7b_ffn",
                                 "c3_q6_k_head_4096x32000"])
def test_benchmark_configs_full_size_bit_exact(ctx, cfg):
    for dtype, n, r in synth.CONFIGS[cfg]:
        w = synth.weight(dtype, f"{cfg}.w.{n}x{r}", r, n)
        x = synth.activation(f"{cfg}.x.{n}", 1, n)
        wt = ctx.upload(dtype, w, n, r)
        got = ctx.linear(wt, x, 1)
        assert_bits(got, oracle_linear(dtype, x, w, 1, n, r))
        assert np.isfinite(got).all()


def test_row_shards_concatenate_to_the_full_result(ctx):
    """Row sharding (1/2/4/8 ranks) cannot change a row's reduction."""
    n, r = 4096, 32000
    w = synth.weight(vtq.Q6_K, "shard", r, n)
    x = synth.activation("shardx", 1, n)
    full = ctx.linear(ctx.upload(vtq.Q6_K, w, n, r), x)
    for world in (2, 4, 8):
        parts = []
        for rank in range(world):
            a, b = rank * r // world, (rank + 1) * r // world
            parts.append(ctx.linear(ctx.upload(vtq.Q6_K, w, n, r, a, b), x))
        assert_bits(np.concatenate(parts), full)


def test_reference_signature_entry_points(ctx):
    n, r, b = 512, 7, 2
    x = synth.activation("sig", b, n)
    for dtype, fn in ((vtq.Q4_K, vtq.linear_q4_k_integer), (vtq.Q6_K, vtq.linear_q6_k_integer),
                      (vtq.Q4_0, vtq.linear_q4_0)):
        w = synth.weight(dtype, "sigw", r, n)
        y = np.zeros(b * r, np.float32)
        fn(ctx, x, w, y, b, n, r)
        assert_bits(y, oracle_linear(dtype, x, w, b, n, r))
    w = synth.weight(vtq.Q4_K, "sigw", r, n)
    y = np.zeros(b * r, np.float32)
    vtq.linear_q4_k_fused(ctx, x, w, y, b, n, r)
    assert_bits(y, O.linear("q4_k_fused", x, w, b, n, r))
    for dtype in (vtq.Q8_0, vtq.Q5_0, vtq.F32, vtq.Q4_K, vtq.Q6_K, vtq.Q4_0):
        w = synth.weight(dtype, "disp", r, n)
        qt = vtq.QuantTensor((n, r), dtype, w.tobytes())
        assert_bits(vtq.linear_dispatch(ctx, x[:n], qt, n, r),
                    O.linear_dispatch(dtype, x[:n], w, n, r))


def test_errors_mirror_the_reference(ctx):
    y = np.zeros(4, np.float32)
    x = np.zeros(1024, np.float32)
    with pytest.raises(vtq.Internal, match="in_feat not a multiple of 256"):
        vtq.linear_q4_k_integer(ctx, x, np.zeros(1000, np.uint8), y, 1, 100, 1)
    with pytest.raises(vtq.Internal, match="weight shape mismatch"):
        vtq.linear_q6_k_integer(ctx, x, np.zeros(100, np.uint8), y, 1, 256, 1)
    with pytest.raises(vtq.Internal, match="weight blob length mismatch"):
        vtq.linear_q4_0(ctx, x, np.zeros(17, np.uint8), y, 1, 32, 1)
    with pytest.raises(vtq.NotImplementedOp, match="linear_dispatch"):
        vtq.linear_dispatch(ctx, x, vtq.QuantTensor((32, 1), 1, bytes(64)), 32, 1)
    with pytest.raises(vtq.Internal, match="weight blob too small"):
        vtq.linear_dispatch(ctx, x, vtq.QuantTensor((32, 2), vtq.Q8_0, bytes(34)), 32, 2)


def test_device_pointer_api_with_torch(ctx):
    import torch
    n, r, b = 4096, 1000, 3
    w = synth.weight(vtq.Q4_K, "dev", r, n)
    x = synth.activation("devx", b, n)
    lib = vtq.load_library()
    raw = torch.from_numpy(w).cuda()
    nb = lib.vtq_device_layout_bytes(vtq.Q4_K, n, r)
    dst = torch.empty(nb, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert lib.vtq_device_repack(vtq.Q4_K, n, r, raw.data_ptr(), dst.data_ptr(), st) == 0
    xd = torch.from_numpy(x).cuda()
    yd = torch.full((b * r,), float("nan"), device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.vtq_linear_device(vtq.Q4_K, dst.data_ptr(), n, r, xd.data_ptr(), n, yd.data_ptr(),
                                 r, b, 0, status.data_ptr(), st) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert_bits(yd.cpu().numpy(), oracle_linear(vtq.Q4_K, x, w, b, n, r))
