"""Device decode session vs the CPU oracle of the reference's decode step:
per-step logits bit-exact, generated tokens and receipt digests identical
(the TinyLlama-shaped decode workload and smaller models through the same code)."""
import numpy as np
import pytest

import vtq
from vtq import gguf, receipt
from oracle import oracle as O

pytestmark = pytest.mark.gpu

SMALL = dict(dim=256, hidden=512, layers=2, heads=4, kv_heads=2, vocab=300, seq_len=64,
             rope_theta=10000.0, rms_eps=1e-5)


# (environment, expected vtq_decode_step_kind). Every path batches the prompt
# positions except "no_prefill", which runs them one token at a time.
STEP_PATHS = {"graph": ({}, 1), "persistent": ({"VTQ_DECODE_PERSISTENT": "1"}, 2),
              "unfused": ({"VTQ_DECODE_UNFUSED": "1"}, 0),
              "no_prefill": ({"VTQ_DECODE_NO_PREFILL": "1"}, 1)}


@pytest.fixture(params=list(STEP_PATHS))
def step_path(request, monkeypatch):
    env, kind = STEP_PATHS[request.param]
    for k in ("VTQ_DECODE_PERSISTENT", "VTQ_DECODE_UNFUSED", "VTQ_DECODE_NO_PREFILL"):
        monkeypatch.delenv(k, raising=False)
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    return kind


def run_both(blob, prompt, n_new, kind=None):
    sess = vtq.DecodeSession(blob)
    if kind is not None:
        assert sess.step_kind == kind, (sess.step_kind, kind)
    got, lg = sess.run(prompt, n_new, logits=True)
    again, _ = sess.run(prompt, n_new)  # a second run (graph without the logits log)
    sess.close()
    ref, rlg = O.decode_run(blob, prompt, n_new, threads=8, logits=True)
    return got, lg, again, ref, rlg


def assert_bits(a, b):
    bad = np.nonzero(a.reshape(-1).view(np.uint32) != b.reshape(-1).view(np.uint32))[0]
    assert bad.size == 0, f"{bad.size} logits differ; first {bad[:4]}"


@pytest.mark.parametrize("variant", ["q4k_embd", "q6k_embd", "shared_head", "mha", "qwen2",
                                     "qwen2_q5", "long_prompt"])
def test_small_models_bit_exact(variant, step_path):
    cfg = dict(SMALL)
    kw = {}
    kind = step_path
    if variant == "q6k_embd":
        kw["embd_dtype"] = vtq.Q6_K
    if variant == "shared_head":
        kw["shared_head"] = True
    if variant == "mha":
        cfg.update(kv_heads=4, hidden=768, layers=3)
    if variant.startswith("qwen2"):
        # Qwen2: NeoX RoPE, QKV bias, rope base 1e6, eps 1e-6 (quant_weights.rs:143-151)
        cfg.update(rope_theta=1e6, rms_eps=1e-6)
        kw.update(arch="qwen2", qkv_bias=True)
    if variant == "qwen2_q5":
        # Qwen2.5-style formats: the linears run on the canonical fp32 kernels,
        # so every step path falls back to the per-op graph (kind 0)
        kw["wdtypes"] = {"attn_q": vtq.Q5_0, "attn_k": vtq.Q5_0, "attn_v": vtq.Q8_0,
                         "attn_output": vtq.Q5_0, "ffn_gate": vtq.Q5_0, "ffn_up": vtq.Q5_0,
                         "ffn_down": vtq.Q8_0}
        kw["embd_dtype"] = vtq.Q8_0
        kind = 0
    n_prompt, n_new = 7, 9
    if variant == "long_prompt":  # 20 batched prompt rows: Q4_K linears on the GEMM
        n_prompt, n_new = 21, 4
    blob = gguf.synthetic_llama(cfg, seed=3, **kw)
    prompt = gguf.prompt_tokens(n_prompt, cfg["vocab"], seed=1)
    got, lg, again, ref, rlg = run_both(blob, prompt, n_new, kind)
    assert_bits(lg, rlg)
    assert got == ref and again == ref


def test_tinyllama_config4_receipt(step_path):
    cfg = gguf.TINYLLAMA
    blob = gguf.synthetic_llama(cfg)
    prompt = gguf.prompt_tokens(16, cfg["vocab"])
    got, lg, again, ref, rlg = run_both(blob, prompt, 64, step_path)
    assert_bits(lg, rlg)
    assert got == ref == again
    arch = gguf.arch_string(cfg)
    r_gpu = receipt.decode_receipt(gguf.MODEL_ID, blob, arch, prompt, 64, got)
    r_cpu = receipt.decode_receipt(gguf.MODEL_ID, blob, arch, prompt, 64, ref)
    assert r_gpu == r_cpu


def test_decode_errors():
    blob = gguf.synthetic_llama(SMALL, seed=3)
    with pytest.raises(vtq.Malformed):
        vtq.DecodeSession(b"NOPE" + blob[4:])
    with pytest.raises(vtq.Truncated):
        vtq.DecodeSession(blob[: len(blob) // 2])
    sess = vtq.DecodeSession(blob)
    with pytest.raises(vtq.Internal, match="exceeds seq_len"):
        sess.run([5] * 60, 10)
    with pytest.raises(vtq.Internal, match="must not be empty"):
        sess.run([], 3)
    sess.close()


def test_long_context_attention_bit_exact(monkeypatch):
    """seq_len 16384: the attention kernel's shared memory (3 head sizes plus one
    score per cached position, (3 * 64 + 16384) * 4 B = 66 KB) is above the
    48 KB default, so the session opts the kernel into the larger limit. The
    positions run are few; the allocation and the opt-in are what is tested."""
    for k in ("VTQ_DECODE_PERSISTENT", "VTQ_DECODE_UNFUSED", "VTQ_DECODE_NO_PREFILL"):
        monkeypatch.delenv(k, raising=False)
    cfg = dict(SMALL, seq_len=16384)
    blob = gguf.synthetic_llama(cfg, seed=5)
    prompt = gguf.prompt_tokens(6, cfg["vocab"], seed=2)
    got, lg, again, ref, rlg = run_both(blob, prompt, 5)
    assert_bits(lg, rlg)
    assert list(got) == list(ref) and list(again) == list(ref)
