"""The software transcendentals (vtq_expf / vtq_sinf / vtq_cosf / vtq_powf and
the correctly rounded sqrtf) reproduce the reference's pinned cross-ISA sweep
hash (tests/transcendental_determinism.rs:14-67 of the reference) bit for bit."""
import ctypes

import blake3
import numpy as np

import vtq

PINNED = "0ae93cd6394c934bfb94a5803a0528193ba0c2330002162a0094062c294bc3d0"


def sweep_inputs():
    # x starts at -30.0 and advances by the f32 step 0.000123 while x <= 30.0,
    # accumulating in f32; then the 19 corner cases, in the reference's order.
    xs = []
    x = np.float32(-30.0)
    step = np.float32(0.000123)
    while x <= np.float32(30.0):
        xs.append(x)
        x = np.float32(x + step)
    corners = [0.0, -0.0, 1.0, -1.0, 0.5, -0.5, np.finfo(np.float32).tiny, 1e-20, 1e-10, 1e10,
               1e20, 87.0, 88.0, 88.7, -87.0, -88.0, -104.0, np.pi, np.e]
    return np.array(xs + [np.float32(c) for c in corners], np.float32)


def test_transcendental_sweep_hash_matches_reference():
    lib = vtq.load_library()
    xs = sweep_inputs()
    assert len(xs) == 489509
    out = np.zeros(len(xs) * 7, np.float32)
    lib.vtq_libm_sweep(xs.ctypes.data, len(xs), out.ctypes.data)
    assert blake3.blake3(out.tobytes()).hexdigest() == PINNED


def test_scalar_exports():
    lib = vtq.load_library()
    assert lib.vtq_expf(0.0) == 1.0
    assert lib.vtq_cosf(0.0) == 1.0 and lib.vtq_sinf(0.0) == 0.0
    assert lib.vtq_powf(10000.0, 0.0) == 1.0
    for v in (-3.5, 0.25, 7.0, 20.0):
        assert abs(lib.vtq_expf(v) - np.exp(np.float64(v))) <= 2e-7 * np.exp(v)
        assert abs(lib.vtq_sinf(v) - np.sin(np.float64(v))) < 2e-7
        assert abs(lib.vtq_powf(10000.0, v / 64) - 10000.0 ** (v / 64)) < 3e-7 * 10000.0 ** (v / 64)
