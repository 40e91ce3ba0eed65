"""Receipt digest pinned to the reference's golden (src/cert/builder.rs:720-741)
and the GGUF writer/reader round trip for the decode configuration."""
import numpy as np

from vtq import gguf, receipt


def test_v2_digest_pinned():
    d = receipt.digest_v2([("model_id", b"tinyllama"), ("prompt_tokens", bytes([1, 0, 0, 0]))],
                          [("output_tokens", bytes([9, 0, 0, 0]))])
    assert d.hex() == "6d5f534cf69c441ba2832c6e63747a7989ccb5de9a2cc9dc528e5b8e0359cf1e"
    d1 = receipt.digest_v1([("model_id", b"tinyllama"), ("prompt_tokens", bytes([1, 0, 0, 0]))],
                           [("output_tokens", bytes([9, 0, 0, 0]))])
    assert d1 != d


def test_leb128_multibyte():
    assert receipt._leb128(0) == b"\x00" and receipt._leb128(127) == b"\x7f"
    assert receipt._leb128(128) == b"\x80\x01" and receipt._leb128(300) == b"\xac\x02"


def test_gguf_roundtrip_small():
    cfg = dict(dim=256, hidden=512, layers=2, heads=4, kv_heads=2, vocab=300, seq_len=64,
               rope_theta=10000.0, rms_eps=1e-5)
    blob = gguf.synthetic_llama(cfg)
    assert blob == gguf.synthetic_llama(cfg)  # deterministic
    g = gguf.read(blob)
    assert g["metadata"]["llama.embedding_length"] == 256
    assert g["metadata"]["general.architecture"] == "llama"
    shape, dtype, data = g["tensors"]["blk.1.ffn_down.weight"]
    assert shape == [512, 256] and dtype == gguf.Q6_K and len(data) == 256 * 2 * 210
    shape, dtype, data = g["tensors"]["output_norm.weight"]
    v = np.frombuffer(data, np.float32)
    assert dtype == gguf.F32 and v.shape == (256,) and abs(float(v.mean()) - 1.0) < 0.01
    assert gguf.arch_string(cfg) == ("llama2c:dim=256,hidden=512,layers=2,heads=4,kv_heads=2,"
                                     "vocab=300,seq=64,shared=false")
    toks = gguf.prompt_tokens(16, 300)
    assert len(toks) == 16 and min(toks) >= 3 and max(toks) <= 299


def test_receipt_json_matches_the_reference_binary_format():
    rc = {"model_digest": "ab" * 32, "regime": receipt.REGIME, "model_digest_v1": "cd" * 32,
          "weights_hash": "ef" * 32, "tokens": [5, 17, 3]}
    line = receipt.receipt_json(rc)
    assert line == ('{"model_digest":"' + "ab" * 32 + '","regime":"' + receipt.REGIME +
                    '","model_digest_v1":"' + "cd" * 32 + '","weights_hash":"' + "ef" * 32 +
                    '","tokens":[5,17,3]}')
    import json
    assert json.loads(line)["tokens"] == [5, 17, 3]
