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


# ---- decode step / run loop (vtq_oracle_decode.cpp) -------------------------

class _Tensor(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("bytes", ctypes.c_void_p), ("len", ctypes.c_size_t)]


class _Layer(ctypes.Structure):
    _fields_ = [("rms_att", ctypes.c_void_p), ("rms_ffn", ctypes.c_void_p)] + \
        [(n, _Tensor) for n in ("wq", "wk", "wv", "wo", "w1", "w2", "w3")] + \
        [(n, ctypes.c_void_p) for n in ("bq", "bk", "bv")] + \
        [(n, ctypes.c_int32) for n in ("bq_len", "bk_len", "bv_len")]


class _Model(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("dim", "hidden", "n_layers", "n_heads",
                                               "n_kv_heads", "vocab", "seq_len")] + \
        [("rope_theta", ctypes.c_float), ("rms_eps", ctypes.c_float),
         ("rope_neox", ctypes.c_int32), ("embd", _Tensor),
         ("rms_final", ctypes.c_void_p), ("wcls", _Tensor), ("layers", ctypes.c_void_p)]


def decode_run(gguf_blob: bytes, prompt, n_new: int, threads: int = 8, logits: bool = False):
    """The reference's run_quantized token loop on the CPU (oracle)."""
    import sys as _sys
    pkg = os.path.join(os.path.dirname(HERE), "vitni-tensor_b200")
    if pkg not in _sys.path:
        _sys.path.insert(0, pkg)
    from vtq import gguf as G
    g = G.read(gguf_blob)
    meta, ts = g["metadata"], g["tensors"]
    keep = []

    def addr(name):
        arr = np.frombuffer(ts[name][2], np.uint8)
        keep.append(arr)
        return arr.ctypes.data, arr.nbytes

    def tensor(name):
        p, n = addr(name)
        return _Tensor(ts[name][1], p, n)

    arch = meta["general.architecture"]
    m = _Model()
    m.dim = meta[f"{arch}.embedding_length"]
    m.hidden = meta[f"{arch}.feed_forward_length"]
    m.n_layers = meta[f"{arch}.block_count"]
    m.n_heads = meta[f"{arch}.attention.head_count"]
    m.n_kv_heads = meta.get(f"{arch}.attention.head_count_kv", m.n_heads)
    m.vocab = meta[f"{arch}.vocab_size"]
    m.seq_len = meta[f"{arch}.context_length"]
    m.rope_theta = meta.get(f"{arch}.rope.freq_base", 10000.0)
    m.rms_eps = meta.get(f"{arch}.attention.layer_norm_rms_epsilon", 1e-5)
    m.rope_neox = 1 if arch == "qwen2" else 0  # quant_weights.rs:151
    m.embd = tensor("token_embd.weight")
    m.rms_final = addr("output_norm.weight")[0]
    m.wcls = tensor("output.weight") if "output.weight" in ts else _Tensor(0, None, 0)
    layers = (_Layer * m.n_layers)()
    for l in range(m.n_layers):
        p = f"blk.{l}."
        layers[l].rms_att = addr(p + "attn_norm.weight")[0]
        layers[l].rms_ffn = addr(p + "ffn_norm.weight")[0]
        for fld, nm in (("wq", "attn_q"), ("wk", "attn_k"), ("wv", "attn_v"),
                        ("wo", "attn_output"), ("w1", "ffn_gate"), ("w2", "ffn_down"),
                        ("w3", "ffn_up")):
            setattr(layers[l], fld, tensor(p + nm + ".weight"))
        for fld, nm in (("bq", "attn_q"), ("bk", "attn_k"), ("bv", "attn_v")):
            if p + nm + ".bias" in ts:  # optional QKV bias (quant_weights.rs:172-174)
                a, n = addr(p + nm + ".bias")
                setattr(layers[l], fld, a)
                setattr(layers[l], fld + "_len", n // 4)
    m.layers = ctypes.cast(layers, ctypes.c_void_p)
    pr = np.ascontiguousarray(prompt, dtype=np.uint32)
    out = np.zeros(max(1, n_new), np.uint32)
    lg = np.zeros((len(pr) + n_new, m.vocab), np.float32) if logits else None
    fn = lib().or_decode_run
    fn.argtypes = [ctypes.POINTER(_Model), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    _chk(fn(ctypes.byref(m), pr.ctypes.data, len(pr), n_new, out.ctypes.data,
            lg.ctypes.data if lg is not None else None, threads))
    return out[:n_new].tolist(), lg
