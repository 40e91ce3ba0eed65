"""The synthetic GGUF writer's architecture options, read back with the
project's GGUF reader (gguf.rs:305-422 layout): architecture-keyed metadata
(config.rs:141-165), optional F32 attn_q/k/v biases (quant_weights.rs:172-174)
and per-role weight formats."""
import numpy as np

import vtq
from vtq import gguf

CFG = dict(dim=256, hidden=512, layers=2, heads=4, kv_heads=2, vocab=300, seq_len=64,
           rope_theta=1e6, rms_eps=1e-6)


def test_qwen2_keys_biases_and_formats():
    blob = gguf.synthetic_llama(CFG, seed=1, arch="qwen2", qkv_bias=True,
                                wdtypes={"attn_q": vtq.Q5_0, "ffn_down": vtq.Q8_0})
    g = gguf.read(blob)
    meta, ts = g["metadata"], g["tensors"]
    assert meta["general.architecture"] == "qwen2"
    assert meta["qwen2.embedding_length"] == 256 and meta["qwen2.block_count"] == 2
    assert np.float32(meta["qwen2.rope.freq_base"]) == np.float32(1e6)
    assert np.float32(meta["qwen2.attention.layer_norm_rms_epsilon"]) == np.float32(1e-6)
    assert not any(k.startswith("llama.") for k in meta)
    kv = 2 * (256 // 4)
    for l in range(2):
        for nm, n in (("attn_q", 256), ("attn_k", kv), ("attn_v", kv)):
            dtype, raw = ts[f"blk.{l}.{nm}.bias"][1], ts[f"blk.{l}.{nm}.bias"][2]
            assert dtype == vtq.F32 and len(raw) == 4 * n
        assert ts[f"blk.{l}.attn_q.weight"][1] == vtq.Q5_0
        assert ts[f"blk.{l}.ffn_down.weight"][1] == vtq.Q8_0
        assert ts[f"blk.{l}.attn_k.weight"][1] == vtq.Q4_K  # default kept


def test_llama_default_unchanged():
    g = gguf.read(gguf.synthetic_llama(CFG, seed=1))
    assert g["metadata"]["general.architecture"] == "llama"
    assert not any(k.endswith(".bias") for k in g["tensors"])
