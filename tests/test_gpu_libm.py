"""The device build of the software transcendentals (used by the decode
kernels: expf in softmax and SiLU) reproduces the reference's pinned cross-ISA
sweep hash (tests/transcendental_determinism.rs:14-67) bit for bit."""
import blake3
import numpy as np
import pytest

import vtq
from tests.test_libm import PINNED, sweep_inputs

pytestmark = pytest.mark.gpu


def test_device_sweep_hash_matches_reference():
    lib = vtq.load_library()
    xs = sweep_inputs()
    out = np.zeros(len(xs) * 7, np.float32)
    assert lib.vtq_libm_sweep_device(xs.ctypes.data, len(xs), out.ctypes.data) == 0
    assert blake3.blake3(out.tobytes()).hexdigest() == PINNED
