"""GGUF v3 writer and reader for the quantized-decode configuration.

Layout as the reference parses it (src/model/gguf.rs:305-422): magic "GGUF",
u32 version, u64 tensor count, u64 metadata count, metadata key/values,
tensor infos (name, n_dims, u64 dims in GGML order [in, out], u32 type, u64
offset), padding to `general.alignment` (32), then the tensor data with every
offset aligned. The writer is deterministic: the same model dict gives the
same bytes (and therefore the same weights_hash).
"""
from __future__ import annotations

import struct

import numpy as np

from . import synth
from .formats import BLOCK, F32, Q4_K, Q6_K

# GGUF metadata value types (gguf.rs GgufValueType).
U8, I8, U16, I16, U32, I32, F32V, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
MAGIC = b"GGUF"


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, v) -> bytes:
    if vtype == U32:
        return struct.pack("<I", v)
    if vtype == I32:
        return struct.pack("<i", v)
    if vtype == F32V:
        return struct.pack("<f", v)
    if vtype == U64:
        return struct.pack("<Q", v)
    if vtype == STRING:
        return _str(v)
    if vtype == BOOL:
        return struct.pack("<B", 1 if v else 0)
    raise ValueError(f"unsupported metadata type {vtype}")


def write(metadata: list, tensors: list, alignment: int = 32) -> bytes:
    """metadata: [(key, vtype, value)]; tensors: [(name, ggml_shape, dtype, bytes)]."""
    out = bytearray(MAGIC)
    out += struct.pack("<IQQ", 3, len(tensors), len(metadata))
    for key, vtype, v in metadata:
        out += _str(key) + struct.pack("<I", vtype) + _value(vtype, v)
    offset = 0
    offsets = []
    for name, shape, dtype, data in tensors:
        offsets.append(offset)
        out += _str(name) + struct.pack("<I", len(shape))
        out += b"".join(struct.pack("<Q", d) for d in shape)
        out += struct.pack("<IQ", dtype, offset)
        offset += (len(data) + alignment - 1) // alignment * alignment
    out += bytes((-len(out)) % alignment)
    for (name, shape, dtype, data), off in zip(tensors, offsets):
        out += bytes(data)
        out += bytes((-len(data)) % alignment)
    return bytes(out)


def read(blob: bytes) -> dict:
    """Minimal reader: {'metadata': {key: value}, 'tensors': {name: (shape, dtype, memoryview)}}."""
    mv = memoryview(blob)
    pos = 0

    def take(n):
        nonlocal pos
        if pos + n > len(blob):
            raise ValueError("gguf: read past end")
        r = mv[pos:pos + n]
        pos += n
        return r

    def u32():
        return struct.unpack("<I", take(4))[0]

    def u64():
        return struct.unpack("<Q", take(8))[0]

    def string():
        return bytes(take(u64())).decode()

    def value(t):
        fmt = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<B", 10: "<Q",
               11: "<q", 12: "<d"}
        if t == STRING:
            return string()
        if t == ARRAY:
            et, n = u32(), u64()
            return [value(et) for _ in range(n)]
        f = fmt[t]
        return struct.unpack(f, take(struct.calcsize(f)))[0]

    if bytes(take(4)) != MAGIC:
        raise ValueError("gguf: bad magic")
    version = u32()
    nt, nm = u64(), u64()
    meta = {}
    for _ in range(nm):
        k = string()
        meta[k] = value(u32())
    infos = []
    for _ in range(nt):
        name = string()
        nd = u32()
        shape = [u64() for _ in range(nd)]
        dtype = u32()
        off = u64()
        infos.append((name, shape, dtype, off))
    align = meta.get("general.alignment", 32)
    pos = (pos + align - 1) // align * align
    base = pos
    tensors = {}
    for name, shape, dtype, off in infos:
        numel = int(np.prod(shape)) if shape else 1
        per, nb = BLOCK[dtype]
        size = numel // per * nb
        tensors[name] = (shape, dtype, mv[base + off: base + off + size])
    return {"version": version, "metadata": meta, "tensors": tensors}


# Config 4: a random-init Llama model with TinyLlama-1.1B shapes.
TINYLLAMA = dict(dim=2048, hidden=5632, layers=22, heads=32, kv_heads=4, vocab=32000,
                 seq_len=2048, rope_theta=10000.0, rms_eps=1e-5)
MODEL_ID = "vitni-b200-synthetic-tinyllama"


def synthetic_llama(cfg: dict = TINYLLAMA, seed: int = 0, embd_dtype: int = Q4_K,
                    shared_head: bool = False, arch: str = "llama",
                    qkv_bias: bool = False, wdtypes: dict = None) -> bytes:
    """Deterministic GGUF of the TinyLlama-shaped decode workload: attention/FFN-gate/up weights
    Q4_K, V / down / output head Q6_K, token_embd Q4_K, norms F32 = 1 + N(0, 0.02).
    arch="qwen2" writes the Qwen2 keys (the reference then uses NeoX RoPE,
    quant_weights.rs:151); qkv_bias adds F32 attn_q/k/v biases ~ N(0, 0.1);
    wdtypes overrides the format per role (attn_q, attn_k, attn_v, attn_output,
    ffn_gate, ffn_up, ffn_down, output), e.g. Q5_0 / Q8_0 as in Qwen2.5 files."""
    dt = {"attn_q": Q4_K, "attn_k": Q4_K, "attn_v": Q6_K, "attn_output": Q4_K,
          "ffn_gate": Q4_K, "ffn_up": Q4_K, "ffn_down": Q6_K, "output": Q6_K}
    dt.update(wdtypes or {})
    d, h, L = cfg["dim"], cfg["hidden"], cfg["layers"]
    hs = d // cfg["heads"]
    kv = cfg["kv_heads"] * hs
    meta = [
        ("general.architecture", STRING, arch),
        ("general.alignment", U32, 32),
        (f"{arch}.embedding_length", U32, d),
        (f"{arch}.feed_forward_length", U32, h),
        (f"{arch}.block_count", U32, L),
        (f"{arch}.attention.head_count", U32, cfg["heads"]),
        (f"{arch}.attention.head_count_kv", U32, cfg["kv_heads"]),
        (f"{arch}.context_length", U32, cfg["seq_len"]),
        (f"{arch}.vocab_size", U32, cfg["vocab"]),
        (f"{arch}.rope.freq_base", F32V, float(cfg["rope_theta"])),
        (f"{arch}.attention.layer_norm_rms_epsilon", F32V, float(cfg["rms_eps"])),
    ]
    tensors = []

    def mat(name, dtype, rows, cols):
        w = synth.weight(dtype, f"c4/{seed}/{name}", rows, cols, seed)
        tensors.append((name, [cols, rows], dtype, w.tobytes()))

    def norm(name, n):
        v = (np.float32(1.0) + synth.normal(f"c4/{seed}/{name}", seed, n) * np.float32(0.02))
        tensors.append((name, [n], F32, v.astype(np.float32).tobytes()))

    mat("token_embd.weight", embd_dtype, cfg["vocab"], d)
    for l in range(L):
        norm(f"blk.{l}.attn_norm.weight", d)
        mat(f"blk.{l}.attn_q.weight", dt["attn_q"], d, d)
        mat(f"blk.{l}.attn_k.weight", dt["attn_k"], kv, d)
        mat(f"blk.{l}.attn_v.weight", dt["attn_v"], kv, d)
        if qkv_bias:
            for nm, n in (("attn_q", d), ("attn_k", kv), ("attn_v", kv)):
                b = synth.normal(f"c4/{seed}/blk.{l}.{nm}.bias", seed, n) * np.float32(0.1)
                tensors.append((f"blk.{l}.{nm}.bias", [n], F32, b.astype(np.float32).tobytes()))
        mat(f"blk.{l}.attn_output.weight", dt["attn_output"], d, d)
        norm(f"blk.{l}.ffn_norm.weight", d)
        mat(f"blk.{l}.ffn_gate.weight", dt["ffn_gate"], h, d)
        mat(f"blk.{l}.ffn_up.weight", dt["ffn_up"], h, d)
        mat(f"blk.{l}.ffn_down.weight", dt["ffn_down"], d, h)
    norm("output_norm.weight", d)
    if not shared_head:
        mat("output.weight", dt["output"], cfg["vocab"], d)
    return write(meta, tensors)


def prompt_tokens(n: int = 16, vocab: int = 32000, seed: int = 0) -> list:
    """Config 4's prompt: n token ids uniform in [3, vocab - 1]."""
    return [int(t) for t in synth.uniform_int("c4/prompt", seed, n, 3, vocab - 1)]


def arch_string(cfg: dict, shared: bool = False) -> str:
    """arch_string (src/model/inference.rs:45-57)."""
    return (f"llama2c:dim={cfg['dim']},hidden={cfg['hidden']},layers={cfg['layers']},"
            f"heads={cfg['heads']},kv_heads={cfg['kv_heads']},vocab={cfg['vocab']},"
            f"seq={cfg['seq_len']},shared={'true' if shared else 'false'}")
