"""Qwen2 handling in the decode oracle (forward_quantized.rs:414-448 NeoX RoPE,
:807-813 QKV bias; quant_weights.rs:143-151 architecture parameters). The
reference's Qwen2 tests need a model file, so these are self-consistency
checks: at position 0 RoPE is the identity (cos 0 = 1, sin 0 = 0), so a file
keyed "qwen2" without biases must give the Llama logits there and differ
after; biases change the logits from position 0 on."""
import numpy as np

from oracle import oracle as O
from vtq import gguf

CFG = dict(dim=256, hidden=512, layers=2, heads=4, kv_heads=2, vocab=300, seq_len=64,
           rope_theta=1e6, rms_eps=1e-6)


def _logits(**kw):
    blob = gguf.synthetic_llama(CFG, seed=3, **kw)
    _, lg = O.decode_run(blob, [5, 6, 7, 8], 2, threads=4, logits=True)
    return lg


def test_neox_rope_identity_at_position_0():
    llama, qwen = _logits(), _logits(arch="qwen2")
    assert np.array_equal(llama[0].view(np.uint32), qwen[0].view(np.uint32))
    assert not np.array_equal(llama[1:], qwen[1:])


def test_qkv_bias_changes_position_0():
    plain, biased = _logits(arch="qwen2"), _logits(arch="qwen2", qkv_bias=True)
    assert not np.array_equal(plain[0], biased[0])
