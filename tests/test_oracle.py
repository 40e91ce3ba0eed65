"""CPU oracle self-checks: the reference's published goldens and its own
property tests (src/ops/quant.rs:1567-2397, src/ops/matmul.rs:135-196),
restated, plus a cross-check against an independent numpy restatement."""
import numpy as np
import pytest

from oracle import oracle as O
from tests import numpy_ref as NR


def bits(v):
    return int(np.float32(v).view(np.uint32))


def lcg_bytes(seed, n):
    # src/ops/quant.rs:2022-2026: s = s*6364136223846793005+1; byte = (s >> 40) as u8
    out = np.empty(n, np.uint8)
    s = seed
    for i in range(n):
        s = (s * 6364136223846793005 + 1) & 0xFFFFFFFFFFFFFFFF
        out[i] = (s >> 40) & 0xFF
    return out


def ramp_x(n):
    # ((i * 7919) % 1000) as f32 / 500.0 - 1.0   (quant.rs:2027-2029)
    i = np.arange(n, dtype=np.int64)
    return ((i * 7919) % 1000).astype(np.float32) / np.float32(500.0) - np.float32(1.0)


def test_pinned_v2_reference_4096():
    a, b = O.lcg_pair(4096)
    assert bits(O.canonical_dot(a, b)) == 0x40CE39E1  # quant.rs:1571


def test_pinned_discriminating_reference_14336():
    a, b = O.lcg_pair(14336)
    assert bits(O.canonical_dot(a, b)) == 0xC1A3BF11  # quant.rs:1975-1990


def test_matmul_fnv_pinned():
    assert O.matmul_fnv_golden() == 0x8A428433686D13AF  # matmul.rs:135


def test_f16_known_constants():
    assert O.lib().or_f32_to_f16(1.0) == 0x3C00 and O.lib().or_f16_to_f32(0x3C00) == 1.0
    assert O.lib().or_f32_to_f16(-2.0) == 0xC000 and O.lib().or_f16_to_f32(0xC000) == -2.0
    assert O.lib().or_f32_to_f16(0.5) == 0x3800 and O.lib().or_f16_to_f32(0x3800) == 0.5
    assert O.lib().or_f16_to_f32(0) == 0.0


def test_f16_decode_matches_numpy_all_finite():
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([O.lib().or_f16_to_f32(int(v)) for v in h[::7]], np.float32)
    r = ref[::7]
    fin = np.isfinite(r)
    assert np.array_equal(got[fin].view(np.uint32), r[fin].view(np.uint32))


def f16le(v):
    return np.array([v], np.float16).view(np.uint8)


def test_q4_k_dequant_uniform_scale_one():  # quant.rs:1705-1749
    blk = np.zeros(144, np.uint8)
    blk[0:2] = f16le(1.0)
    blk[4:8] = 1
    blk[16:] = 0x10
    out = O.dequantize(O.Q4_K, blk)
    assert (out[0:32] == 0).all() and (out[32:64] == 1).all()
    assert (out[64:96] == 0).all() and (out[96:128] == 1).all() and (out[128:] == 0).all()


def test_q4_k_dequant_negative_min():  # quant.rs:1752-1767
    blk = np.zeros(144, np.uint8)
    blk[0:2] = f16le(1.0)
    blk[2:4] = f16le(2.0)
    blk[8] = 3
    out = O.dequantize(O.Q4_K, blk)
    assert np.allclose(out[:32], -6.0)


def test_q6_k_dequant_known_blocks():  # quant.rs:1770-1813
    blk = np.zeros(210, np.uint8)
    blk[192:208] = 1
    blk[208:210] = f16le(1.0)
    assert np.allclose(O.dequantize(O.Q6_K, blk), -32.0)
    blk[128] = 0b11_10_01_00
    out = O.dequantize(O.Q6_K, blk)
    assert (out[0], out[32], out[64], out[96]) == (-32.0, -16.0, 0.0, 16.0)


@pytest.mark.parametrize("in_feat,out_feat", [(256, 3), (512, 5), (1024, 7), (4096, 2),
                                              (8192, 2), (14336, 2)])
def test_fused_q4k_is_bit_identical_to_dequant_then_dot(in_feat, out_feat):
    # quant.rs:2013-2055: random bytes, skip non-finite references.
    w = lcg_bytes(0xC0FFEE, out_feat * in_feat // 256 * 144)
    x = ramp_x(in_feat)
    ref = O.linear("q4_k_cpu", x, w, 1, in_feat, out_feat)
    fused = O.linear("q4_k_fused", x, w, 1, in_feat, out_feat)
    fin = np.isfinite(ref)
    assert np.array_equal(ref[fin].view(np.uint32), fused[fin].view(np.uint32))


@pytest.mark.parametrize("in_feat,out_feat", [(256, 3), (1024, 5), (4096, 2), (8192, 2)])
def test_fused_q6k_is_bit_identical(in_feat, out_feat):  # quant.rs:2101-2128
    w = lcg_bytes(0xBEEF, out_feat * in_feat // 256 * 210).reshape(-1, 210)
    w[:, 208:210] = np.frombuffer((0x2E66).to_bytes(2, "little"), np.uint8)
    x = ramp_x(in_feat)
    ref = O.linear("q6_k_cpu", x, w, 1, in_feat, out_feat)
    fused = O.linear("q6_k_fused", x, w, 1, in_feat, out_feat)
    assert np.array_equal(ref.view(np.uint32), fused.view(np.uint32))


def test_parallel_matches_serial_at_every_thread_count():  # quant.rs:2063-2095
    in_feat, out_feat = 4096, 1024
    w = lcg_bytes(0xC0FFEE, out_feat * in_feat // 256 * 144).reshape(-1, 144)
    w[:, 0:2] = np.frombuffer((0x2E66).to_bytes(2, "little"), np.uint8)
    w[:, 2:4] = np.frombuffer((0x2666).to_bytes(2, "little"), np.uint8)
    x = ramp_x(in_feat)
    serial = O.linear("q4_k_fused", x, w, 1, in_feat, out_feat)
    iserial = O.linear("q4_k_integer", x, w, 1, in_feat, out_feat)
    for t in (1, 2, 3, 4, 7, 8, 16, 33):
        assert np.array_equal(serial.view(np.uint32),
                              O.linear("q4_k_fused", x, w, 1, in_feat, out_feat, t).view(np.uint32))
        assert np.array_equal(iserial.view(np.uint32),
                              O.linear("q4_k_integer", x, w, 1, in_feat, out_feat, t).view(np.uint32))


def test_integer_dot_agrees_with_float_on_same_activations():  # quant.rs:2192-2245
    for n in (256, 1024, 4096, 14336):
        w = lcg_bytes(0x13579, n // 256 * 144).reshape(-1, 144)
        w[:, 0:2] = np.frombuffer((0x2E66).to_bytes(2, "little"), np.uint8)
        w[:, 2:4] = np.frombuffer((0x2666).to_bytes(2, "little"), np.uint8)
        x = ramp_x(n)
        rt = np.empty(n, np.float32)
        for b in range(n // 256):
            q = O.quantize_block_q8(x[b * 256:(b + 1) * 256])
            rt[b * 256:(b + 1) * 256] = np.float32(q["d"]) * q["qs"].astype(np.float32)
        f = O.canonical_dot_q4k_fused(rt, w, n)
        i = O.integer_dot_q4k(x, w, n)
        assert abs(f - i) / max(abs(f), 1.0) < 1e-4
        if n == 256:
            assert bits(f) == bits(i)  # one superblock is entirely integer


def test_integer_q6k_agrees_with_float_on_same_activations():  # quant.rs:2293-2327
    for n in (256, 1024, 4096):
        w = lcg_bytes(0x2468, n // 256 * 210).reshape(-1, 210)
        w[:, 208:210] = np.frombuffer((0x2E66).to_bytes(2, "little"), np.uint8)
        x = ramp_x(n)
        rt = np.empty(n, np.float32)
        for b in range(n // 256):
            q = O.quantize_block_q8(x[b * 256:(b + 1) * 256])
            rt[b * 256:(b + 1) * 256] = np.float32(q["d"]) * q["qs"].astype(np.float32)
        yf = O.linear("q6_k_fused", rt, w, 1, n, 1)[0]
        yi = O.linear("q6_k_integer", x, w, 1, n, 1)[0]
        assert abs(yf - yi) / max(abs(yf), 1.0) < 1e-4


def test_canonical_fast_path_matches_spec():  # quant.rs:1900-1929
    for n in (1, 7, 8, 9, 63, 64, 65, 4096, 14336, 8193):
        a, b = O.lcg_pair(n)
        nch = (n + 8191) // 8192
        sums = []
        for c in range(nch):
            s, e = c * 8192, min((c + 1) * 8192, n)
            lanes = np.zeros(8, np.float32)
            for i in range(s, e):
                lanes[(i - s) % 8] = np.float32(lanes[(i - s) % 8] + np.float32(a[i] * b[i]))
            sums.append(O.fixed_tree(lanes))
        assert bits(O.fixed_tree(np.array(sums, np.float32))) == bits(O.canonical_dot(a, b))


def test_oracle_matches_numpy_restatement_q4k_q6k():
    rng = np.random.default_rng(5)
    for q6, n, r, bsz in ((False, 2048, 37, 2), (True, 1536, 29, 3), (False, 256, 5, 1),
                          (True, 5632, 7, 1)):
        bb = 210 if q6 else 144
        w = rng.integers(0, 256, size=r * n // 256 * bb, dtype=np.uint8).reshape(-1, bb)
        dpos = [208] if q6 else [0, 2]
        for p in dpos:  # finite scales
            w[:, p:p + 2] = np.array(np.abs(rng.standard_normal(len(w))) * 0.01,
                                     np.float16).view(np.uint8).reshape(-1, 2)
        x = rng.standard_normal(bsz * n).astype(np.float32)
        got = O.linear("q6_k_integer" if q6 else "q4_k_integer", x, w, bsz, n, r)
        ref = NR.linear_int(q6, x, w, bsz, n, r)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_quantize_block_edge_cases():
    x = np.zeros(256, np.float32)
    x[3] = np.nan
    x[4] = -0.0
    x[5] = 1e-40  # subnormal amax: 1/d overflows to inf; 0*inf = NaN -> 0, 1e-40*inf -> 127
    q = O.quantize_block_q8(x)
    assert q["d"] == np.float32(1e-40) / np.float32(127.0)
    expect = np.zeros(256, np.int8)
    expect[5] = 127
    assert np.array_equal(q["qs"], expect)
    with np.errstate(all="ignore"):
        d, qq = NR.quantize_blocks(x)
    assert np.array_equal(qq.astype(np.int8), expect)
    x = np.linspace(-3, 3, 256).astype(np.float32)
    q = O.quantize_block_q8(x)
    d, qq = NR.quantize_blocks(x)
    assert bits(q["d"]) == bits(d) and np.array_equal(q["qs"].astype(np.int32), qq)
    assert np.array_equal(q["bsums"], qq.reshape(8, 32).sum(axis=1))


def test_dispatch_errors():
    x = np.zeros(100, np.float32)
    with pytest.raises(O.OracleError) as e:
        O.linear_dispatch(O.Q4_K, x, np.zeros(144, np.uint8), 100, 1)
    assert e.value.status == 1
    with pytest.raises(O.OracleError) as e:
        O.linear_dispatch(1, x, np.zeros(200, np.uint8), 100, 1)
    assert e.value.status == 2
