"""The run/crossing plan of the CTA-wide left-to-right sum (exact_sum.cuh),
evaluated step by step on the host, against the plain fp32 loop of
rms_norm_slice (src/ops/rms_norm.rs:97-100): identical bits on every case,
and no fallback except where the sum overflows."""
import numpy as np

import vtq
from tests._exact_sum_cases import cases, serial


def test_plan_matches_serial_sum():
    fallbacks = {}
    for kind, a in cases(seed=0, count=1400):
        got, fb = vtq.exact_sum_host(a)
        ref = serial(a)
        assert got.view(np.uint32) == ref.view(np.uint32), (kind, a.size, got, ref)
        fallbacks[kind] = fallbacks.get(kind, 0) + int(fb)
    assert all(v == 0 for k, v in fallbacks.items() if k != 6), fallbacks
    assert fallbacks[6] > 0  # overflow to inf takes the plain loop


def test_rmsnorm_width_has_few_crossings():
    # squares of 2048 normal values: the plan needs no fallback
    rng = np.random.default_rng(1)
    for _ in range(20):
        v = rng.standard_normal(2048).astype(np.float32) * np.float32(rng.uniform(1e-3, 1e3))
        got, fb = vtq.exact_sum_host(v * v)
        assert not fb and got.view(np.uint32) == serial(v * v).view(np.uint32)
