"""Seeded synthetic inputs for the benchmark configurations.

The reference's measured configurations use real GGUF checkpoints that are not
available here; these generators produce inputs with the configurations'
shapes and value distributions instead:

* draws come from a counter-based splitmix64 stream keyed by (name, seed), so
  any tensor can be regenerated independently and in any order;
* normals are Box-Muller in float64, rounded to float32;
* f16 scales are numpy float16 (round to nearest even) of |N(0,1)| * scale.

Config 1: Q8_0  d = f16(|N|*0.02), qs uniform in [-127, 127].
Config 2: Q4_K  d, dmin = f16(|N|*0.01), 6-bit scales/mins uniform [0, 63],
          nibbles uniform [0, 15].
Config 3: Q6_K  d = f16(|N|*0.01), i8 scales uniform [-128, 127], 6-bit quants
          uniform [0, 63].
Activations: f32 N(0, 1).
"""
from __future__ import annotations

import hashlib

import numpy as np

from .formats import Q4_0, Q4_K, Q5_0, Q6_K, Q8_0, F32, row_bytes

_M = np.uint64(0xFFFFFFFFFFFFFFFF)


def _key(name: str, seed: int) -> np.uint64:
    h = hashlib.blake2b(f"{name}/{seed}".encode(), digest_size=8).digest()
    return np.uint64(int.from_bytes(h, "little"))


def splitmix64(name: str, seed: int, count: int, offset: int = 0) -> np.ndarray:
    """`count` 64-bit draws of stream (name, seed) starting at draw `offset`."""
    with np.errstate(over="ignore"):
        i = np.arange(offset + 1, offset + count + 1, dtype=np.uint64)
        z = _key(name, seed) + i * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def uniform_int(name: str, seed: int, count: int, lo: int, hi: int) -> np.ndarray:
    """Integers uniform in [lo, hi] (inclusive)."""
    span = np.uint64(hi - lo + 1)
    return (splitmix64(name, seed, count) % span).astype(np.int64) + lo


def normal(name: str, seed: int, count: int) -> np.ndarray:
    """float32 N(0, 1) draws (Box-Muller in float64)."""
    r = splitmix64(name, seed, 2 * ((count + 1) // 2))
    u = ((r >> np.uint64(11)).astype(np.float64) + 0.5) * (1.0 / (1 << 53))
    u1, u2 = u[0::2], u[1::2]
    rad = np.sqrt(-2.0 * np.log(u1))
    z = np.empty(2 * len(u1))
    z[0::2] = rad * np.cos(2 * np.pi * u2)
    z[1::2] = rad * np.sin(2 * np.pi * u2)
    return z[:count].astype(np.float32)


def _f16_bytes(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float16).view(np.uint8).reshape(-1, 2)


def pack_q4k_scales(sc: np.ndarray, m: np.ndarray) -> np.ndarray:
    """Invert get_scale_min_k4 (src/ops/quant.rs:268-276): [..., 8] 6-bit
    scales and mins -> [..., 12] bytes."""
    sc = sc.astype(np.uint8)
    m = m.astype(np.uint8)
    out = np.zeros(sc.shape[:-1] + (12,), np.uint8)
    out[..., 0:4] = sc[..., 0:4] | ((sc[..., 4:8] >> 4) << 6)
    out[..., 4:8] = m[..., 0:4] | ((m[..., 4:8] >> 4) << 6)
    out[..., 8:12] = (sc[..., 4:8] & 15) | ((m[..., 4:8] & 15) << 4)
    return out


def pack_q6k_quants(q: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """6-bit codes [..., 256] -> (ql [..., 128], qh [..., 64]) per the layout
    dequantize_q6_k reads (src/ops/quant.rs:337-386)."""
    q = q.astype(np.uint8)
    lead = q.shape[:-1]
    q = q.reshape(lead + (2, 4, 32))  # half, t (element offset 32t), l
    lo = q & 15
    hi = q >> 4
    ql = np.empty(lead + (2, 64), np.uint8)
    ql[..., 0:32] = lo[..., 0, :] | (lo[..., 2, :] << 4)
    ql[..., 32:64] = lo[..., 1, :] | (lo[..., 3, :] << 4)
    qh = hi[..., 0, :] | (hi[..., 1, :] << 2) | (hi[..., 2, :] << 4) | (hi[..., 3, :] << 6)
    return ql.reshape(lead + (128,)), qh.reshape(lead + (64,))


def q8_0_weight(name: str, rows: int, in_feat: int, seed: int = 0) -> np.ndarray:
    nb = rows * in_feat // 32
    blk = np.empty((nb, 34), np.uint8)
    blk[:, 0:2] = _f16_bytes(np.abs(normal(name + ".d", seed, nb)) * np.float32(0.02))
    blk[:, 2:] = uniform_int(name + ".qs", seed, nb * 32, -127, 127).astype(np.int8).view(
        np.uint8).reshape(nb, 32)
    return blk.reshape(-1)


def q4_k_weight(name: str, rows: int, in_feat: int, seed: int = 0) -> np.ndarray:
    nb = rows * in_feat // 256
    blk = np.empty((nb, 144), np.uint8)
    blk[:, 0:2] = _f16_bytes(np.abs(normal(name + ".d", seed, nb)) * np.float32(0.01))
    blk[:, 2:4] = _f16_bytes(np.abs(normal(name + ".dmin", seed, nb)) * np.float32(0.01))
    sc = uniform_int(name + ".sc", seed, nb * 8, 0, 63).reshape(nb, 8)
    mn = uniform_int(name + ".m", seed, nb * 8, 0, 63).reshape(nb, 8)
    blk[:, 4:16] = pack_q4k_scales(sc, mn)
    nib = uniform_int(name + ".q", seed, nb * 256, 0, 15).astype(np.uint8).reshape(nb, 4, 2, 32)
    blk[:, 16:] = (nib[:, :, 0, :] | (nib[:, :, 1, :] << 4)).reshape(nb, 128)
    return blk.reshape(-1)


def q6_k_weight(name: str, rows: int, in_feat: int, seed: int = 0) -> np.ndarray:
    nb = rows * in_feat // 256
    blk = np.empty((nb, 210), np.uint8)
    q = uniform_int(name + ".q", seed, nb * 256, 0, 63).reshape(nb, 256)
    blk[:, 0:128], blk[:, 128:192] = pack_q6k_quants(q)
    blk[:, 192:208] = uniform_int(name + ".sc", seed, nb * 16, -128, 127).astype(np.int8).view(
        np.uint8).reshape(nb, 16)
    blk[:, 208:210] = _f16_bytes(np.abs(normal(name + ".d", seed, nb)) * np.float32(0.01))
    return blk.reshape(-1)


def q5_0_weight(name: str, rows: int, in_feat: int, seed: int = 0) -> np.ndarray:
    nb = rows * in_feat // 32
    blk = np.empty((nb, 22), np.uint8)
    blk[:, 0:2] = _f16_bytes(np.abs(normal(name + ".d", seed, nb)) * np.float32(0.02))
    blk[:, 2:] = uniform_int(name + ".b", seed, nb * 20, 0, 255).astype(np.uint8).reshape(nb, 20)
    return blk.reshape(-1)


def q4_0_weight(name: str, rows: int, in_feat: int, seed: int = 0) -> np.ndarray:
    nb = rows * in_feat // 32
    blk = np.empty((nb, 18), np.uint8)
    blk[:, 0:2] = _f16_bytes(np.abs(normal(name + ".d", seed, nb)) * np.float32(0.02))
    blk[:, 2:] = uniform_int(name + ".b", seed, nb * 16, 0, 255).astype(np.uint8).reshape(nb, 16)
    return blk.reshape(-1)


def f32_weight(name: str, rows: int, in_feat: int, seed: int = 0) -> np.ndarray:
    return (normal(name, seed, rows * in_feat) * np.float32(0.02)).view(np.uint8)


WEIGHT_GEN = {Q8_0: q8_0_weight, Q4_K: q4_k_weight, Q6_K: q6_k_weight, Q5_0: q5_0_weight,
              Q4_0: q4_0_weight, F32: f32_weight}


def weight(dtype: int, name: str, rows: int, in_feat: int, seed: int = 0) -> np.ndarray:
    w = WEIGHT_GEN[dtype](name, rows, in_feat, seed)
    assert w.nbytes == rows * row_bytes(dtype, in_feat)
    return w


def activation(name: str, batch: int, in_feat: int, seed: int = 0) -> np.ndarray:
    return normal(name, seed, batch * in_feat)


# Matvec workloads of the benchmark (Q8_0 4096x4096, the Llama-7B FFN pair,
# the Q6_K output head): (dtype, in_feat, out_feat).
CONFIGS = {
    "c1_q8_0_4096x4096": [(Q8_0, 4096, 4096)],
    "c2_q4_k_llama7b_ffn": [(Q4_K, 4096, 11008), (Q4_K, 11008, 4096)],
    "c3_q6_k_head_4096x32000": [(Q6_K, 4096, 32000)],
}

# Config 5: one Mistral-7B layer's linears (wq, wk, wv, wo, w1, w3, w2) as
# batched Q4_K products at M = 512 prompt tokens.
PREFILL_CFG = "c5_q4_k_prefill_mistral"
PREFILL_M = 512
PREFILL_LINEARS = [  # (name, in_feat, out_feat)
    ("wq", 4096, 4096), ("wk", 4096, 1024), ("wv", 4096, 1024), ("wo", 4096, 4096),
    ("w1", 4096, 14336), ("w3", 4096, 14336), ("w2", 14336, 4096),
]
