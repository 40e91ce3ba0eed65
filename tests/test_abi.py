"""The C-ABI library loads on a machine without a GPU and exports every
symbol include/vtq.h declares; CPU-side argument validation."""
import ctypes
import os
import re

import numpy as np

import vtq

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for f in os.listdir(os.path.join(REPO, "include")):
        if f.endswith(".h"):
            src = open(os.path.join(REPO, "include", f)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(vtq_[a-z0-9_]+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol():
    lib = vtq.load_library()
    declared = declared_symbols()
    assert declared, "no declarations found"
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing
    assert declared == set(vtq.EXPORTS) | (declared - set(vtq.EXPORTS))


def test_layout_bytes_without_gpu():
    lib = vtq.load_library()
    assert lib.vtq_device_layout_bytes(vtq.Q4_K, 4096, 11008) == 11008 * 2304 + 16
    # Q6_K row 5632 = 22 superblocks = 4620 B -> pitch 4624
    assert lib.vtq_device_layout_bytes(vtq.Q6_K, 5632, 3) == 3 * 4624 + 16
    assert lib.vtq_device_layout_bytes(vtq.Q4_K, 100, 1) == -1
    assert lib.vtq_device_layout_bytes(99, 256, 1) == -1


def test_device_api_validates_before_touching_the_gpu():
    lib = vtq.load_library()
    # unsupported dtype -> NOT_IMPLEMENTED; bad in_feat -> INTERNAL; null -> INVALID_ARG
    assert lib.vtq_linear_device(1, None, 256, 1, None, 256, None, 1, 1, 0, None, None) == \
        vtq.ERR_NOT_IMPLEMENTED
    assert lib.vtq_linear_device(vtq.Q4_K, None, 100, 1, None, 100, None, 1, 1, 0, None, None) == \
        vtq.ERR_INTERNAL
    assert lib.vtq_linear_device(vtq.Q4_K, None, 256, 1, None, 256, None, 1, 1, 0, None, None) == \
        vtq.ERR_INVALID_ARG
    h = ctypes.c_void_p()
    assert lib.vtq_init(-1, ctypes.byref(h)) == vtq.ERR_GPU


def test_synthetic_generators_are_deterministic_and_well_formed():
    from vtq import synth
    from oracle import oracle as O
    a = synth.weight(vtq.Q4_K, "w", 3, 512)
    b = synth.weight(vtq.Q4_K, "w", 3, 512)
    assert np.array_equal(a, b)
    assert not np.array_equal(a, synth.weight(vtq.Q4_K, "w", 3, 512, seed=1))
    blk = a.reshape(-1, 144)
    from tests.numpy_ref import q4k_fields
    d, dmin, sc, m, q = q4k_fields(blk)
    assert (d >= 0).all() and np.isfinite(d).all() and (sc <= 63).all() and (m <= 63).all()
    # the packer inverts get_scale_min_k4 (quant.rs:268-276)
    sc_ref = synth.uniform_int("w.sc", 0, 6 * 8, 0, 63).reshape(6, 8)
    assert np.array_equal(sc, sc_ref)
    w6 = synth.weight(vtq.Q6_K, "h", 2, 256)
    from tests.numpy_ref import q6k_fields
    _, sc6, q6 = q6k_fields(w6)
    qref = synth.uniform_int("h.q", 0, 2 * 256, 0, 63).reshape(2, 256) - 32
    assert np.array_equal(q6, qref)
    deq = O.dequantize(O.Q6_K, w6)
    assert np.isfinite(deq).all()
    x = synth.activation("x", 2, 300)
    assert x.dtype == np.float32 and abs(float(x.mean())) < 0.2 and 0.8 < float(x.std()) < 1.2


def test_workspace_query_without_gpu():
    """Only integer Q4_K at batch >= 16 (the tensor-core path, sized on the
    GPU test side) needs scratch; every other linear needs none."""
    lib = vtq.load_library()
    assert lib.vtq_linear_device_workspace_bytes(vtq.Q4_K, 4096, 1, 0) == 0
    assert lib.vtq_linear_device_workspace_bytes(vtq.Q6_K, 4096, 32, 0) == 0
    assert lib.vtq_linear_device_workspace_bytes(vtq.Q4_K, 4096, 32, vtq.Q4K_FLOAT) == 0


def test_list_entry_points_validate_without_gpu():
    """vtq_linear_list / vtq_linear_list_gather reject a missing context or
    list before touching the device."""
    lib = vtq.load_library()
    assert lib.vtq_linear_list(None, None, 1, 0) == vtq.ERR_INVALID_ARG
    assert lib.vtq_linear_list_gather(None, None, 1, None, 0, 0) == vtq.ERR_INVALID_ARG
    assert lib.vtq_set_wait_limit(None, 1000) == vtq.ERR_INVALID_ARG
