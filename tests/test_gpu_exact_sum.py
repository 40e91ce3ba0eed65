"""The CTA-wide left-to-right fp32 sum (exact_sum.cuh) on the device against
the plain loop of rms_norm_slice (src/ops/rms_norm.rs:97-100), for the CTA
sizes the kernels use, term counts from 1 to past the model widths, and the
adversarial families of the host test."""
import numpy as np
import pytest

import vtq
from tests._exact_sum_cases import cases, serial

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nthr", [32, 256, 480, 512, 1024])
def test_device_sum_bit_exact(nthr):
    for n in (1, 7, 31, 32, 33, 255, 1000, 2048, 4096, 5632, 8192):
        rng = np.random.default_rng(n + nthr)
        v = rng.standard_normal((24, n)).astype(np.float32)
        v *= np.float32(10.0) ** rng.integers(-6, 6, (24, 1)).astype(np.float32)
        a = v * v
        got = vtq.exact_sum_device(a, nthr)
        ref = np.array([serial(r) for r in a], np.float32)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (nthr, n)


def test_device_sum_adversarial():
    cs = cases(seed=5, count=700)
    for kind, a in cs:
        got = vtq.exact_sum_device(a[None, :], 480)[0]
        ref = serial(a)
        assert got.view(np.uint32) == ref.view(np.uint32), (kind, a.size, got, ref)
