"""ctypes binding of the CPU oracle (liboracle.so, built from vtq_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg as the checker. The product (libvtq.so and the
vtq package) never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")

F32, Q4_0, Q5_0, Q8_0, Q4_K, Q6_K = 0, 2, 6, 8, 12, 14


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _load():
    if not os.path.exists(LIB):
        build()
    lib = ctypes.CDLL(LIB)
    p, sz, f = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_float
    lib.or_canonical_dot.restype = f
    lib.or_canonical_dot.argtypes = [p, p, sz]
    lib.or_fixed_tree.restype = f
    lib.or_fixed_tree.argtypes = [p, sz]
    lib.or_f16_to_f32.restype = f
    lib.or_f16_to_f32.argtypes = [ctypes.c_uint16]
    lib.or_f32_to_f16.restype = ctypes.c_uint16
    lib.or_f32_to_f16.argtypes = [f]
    lib.or_matmul_fnv_golden.restype = ctypes.c_uint64
    lib.or_lcg_pair.argtypes = [sz, p, p]
    for nm in ("q4_0", "q5_0", "q8_0", "q4_k", "q6_k"):
        fn = getattr(lib, "or_dequantize_" + nm)
        fn.argtypes = [p, sz, p]
    lib.or_quantize_q8_0.argtypes = [p, sz, p]
    lib.or_quantize_q4_0.argtypes = [p, sz, p]
    lib.or_quantize_block_q8.argtypes = [p, sz, p]
    lib.or_dot_q4k_q8_block.restype = f
    lib.or_dot_q4k_q8_block.argtypes = [p, p, sz]
    lib.or_dot_q6k_q8_block.restype = f
    lib.or_dot_q6k_q8_block.argtypes = [p, p, sz]
    for nm in ("or_integer_dot_q4k", "or_canonical_dot_q4k_fused", "or_canonical_dot_q6k_fused"):
        getattr(lib, nm).argtypes = [p, p, sz, sz, p]
    for nm in ("q4_k_integer", "q6_k_integer", "q4_k_fused", "q6_k_fused", "q4_k_cpu",
               "q6_k_cpu", "q4_0_cpu"):
        getattr(lib, "or_linear_" + nm).argtypes = [p, p, sz, p, sz, sz, sz]
    for nm in ("q4_k_integer_parallel", "q6_k_integer_parallel", "q4_k_fused_parallel"):
        getattr(lib, "or_linear_" + nm).argtypes = [p, p, sz, p, sz, sz, sz, sz]
    lib.or_linear_dispatch.argtypes = [ctypes.c_int, p, p, sz, sz, sz, p, ctypes.c_int, sz]
    lib.or_rms_norm.argtypes = [p, p, sz, f, p]
    lib.or_argmax.restype = ctypes.c_uint32
    lib.or_argmax.argtypes = [p, sz]
    return lib


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def _f(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8(a):
    if isinstance(a, (bytes, bytearray)):
        return np.frombuffer(bytes(a), np.uint8)
    return np.ascontiguousarray(a).view(np.uint8).reshape(-1)


class OracleError(Exception):
    def __init__(self, status):
        super().__init__(f"oracle status {status}")
        self.status = status


def _chk(st):
    if st:
        raise OracleError(st)


# Q8Block as laid out in C: float d; int8 qs[256]; int32 bsums[8] (with padding).
Q8BLOCK = np.dtype([("d", np.float32), ("qs", np.int8, 256), ("bsums", np.int32, 8)],
                   align=True)


def canonical_dot(x, w) -> np.float32:
    x, w = _f(x), _f(w)
    return np.float32(lib().or_canonical_dot(x.ctypes.data, w.ctypes.data, x.size))


def fixed_tree(parts) -> np.float32:
    p = _f(parts).copy()
    return np.float32(lib().or_fixed_tree(p.ctypes.data, p.size))


def lcg_pair(n):
    a = np.empty(n, np.float32)
    b = np.empty(n, np.float32)
    lib().or_lcg_pair(n, a.ctypes.data, b.ctypes.data)
    return a, b


def dequantize(dtype, w) -> np.ndarray:
    w = _u8(w)
    numel, nbytes = {Q4_0: (32, 18), Q5_0: (32, 22), Q8_0: (32, 34), Q4_K: (256, 144),
                     Q6_K: (256, 210)}[dtype]
    out = np.empty(w.size // nbytes * numel, np.float32)
    name = {Q4_0: "q4_0", Q5_0: "q5_0", Q8_0: "q8_0", Q4_K: "q4_k", Q6_K: "q6_k"}[dtype]
    _chk(getattr(lib(), "or_dequantize_" + name)(w.ctypes.data, w.size, out.ctypes.data))
    return out


def quantize_block_q8(x):
    x = _f(x)
    out = np.zeros(1, Q8BLOCK)
    lib().or_quantize_block_q8(x.ctypes.data, x.size, out.ctypes.data)
    return out[0]


def dot_q4k_q8_block(w, blk, n=256) -> np.float32:
    w = _u8(w)
    b = np.array([blk], Q8BLOCK)
    return np.float32(lib().or_dot_q4k_q8_block(w.ctypes.data, b.ctypes.data, n))


def dot_q6k_q8_block(w, blk, n=256) -> np.float32:
    w = _u8(w)
    b = np.array([blk], Q8BLOCK)
    return np.float32(lib().or_dot_q6k_q8_block(w.ctypes.data, b.ctypes.data, n))


def _rowdot(name, x, w, n):
    x, w = _f(x), _u8(w)
    out = np.zeros(1, np.float32)
    _chk(getattr(lib(), name)(x.ctypes.data, w.ctypes.data, w.size, n, out.ctypes.data))
    return out[0]


def integer_dot_q4k(x, w, n):
    return _rowdot("or_integer_dot_q4k", x, w, n)


def canonical_dot_q4k_fused(x, w, n):
    return _rowdot("or_canonical_dot_q4k_fused", x, w, n)


def canonical_dot_q6k_fused(x, w, n):
    return _rowdot("or_canonical_dot_q6k_fused", x, w, n)


def linear(name, x, w, batch, in_feat, out_feat, threads=None) -> np.ndarray:
    """or_linear_<name>: e.g. name='q4_k_integer'; threads selects the _parallel twin."""
    x, w = _f(x), _u8(w)
    y = np.zeros(batch * out_feat, np.float32)
    if threads is None:
        _chk(getattr(lib(), "or_linear_" + name)(x.ctypes.data, w.ctypes.data, w.size,
                                                 y.ctypes.data, batch, in_feat, out_feat))
    else:
        _chk(getattr(lib(), "or_linear_" + name + "_parallel")(
            x.ctypes.data, w.ctypes.data, w.size, y.ctypes.data, batch, in_feat, out_feat,
            threads))
    return y


def linear_dispatch(dtype, x, w, in_feat, out_feat, q4k_float=False, threads=1) -> np.ndarray:
    x, w = _f(x), _u8(w)
    y = np.zeros(out_feat, np.float32)
    _chk(lib().or_linear_dispatch(dtype, x.ctypes.data, w.ctypes.data, w.size, in_feat, out_feat,
                                  y.ctypes.data, 1 if q4k_float else 0, threads))
    return y


def rms_norm(x, w, eps) -> np.ndarray:
    x, w = _f(x), _f(w)
    out = np.empty_like(x)
    lib().or_rms_norm(x.ctypes.data, w.ctypes.data, x.size, ctypes.c_float(eps), out.ctypes.data)
    return out


def argmax(x) -> int:
    x = _f(x)
    return int(lib().or_argmax(x.ctypes.data, x.size))


def matmul_fnv_golden() -> int:
    return int(lib().or_matmul_fnv_golden())
