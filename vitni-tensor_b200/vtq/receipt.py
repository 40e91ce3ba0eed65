"""vitnify-receipt digests (src/cert/builder.rs:347-597 of the reference).

The decode receipt binds I/O only (src/model/inference.rs:282-337):
inputs model_id, weights_hash, arch_hash, prompt_tokens, n_new_tokens;
outputs output_tokens, output_tokens_hash; no op / activation /
intervention records. v2 (shipped) prefixes the numerical regime string;
v1 is the frozen original format.
"""
from __future__ import annotations

import struct

import blake3

REGIME = "vitni-regime-1"  # builder.rs:440


def _leb128(v: int) -> bytes:
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _sections(inputs, outputs) -> bytes:
    def fields(fs):
        b = _leb128(len(fs))
        for name, data in fs:
            nb = name.encode()
            b += _leb128(len(nb)) + nb + _leb128(len(data)) + bytes(data)
        return b
    # inputs, outputs, then empty op / activation / intervention sections
    return fields(inputs) + fields(outputs) + _leb128(0) + _leb128(0) + _leb128(0)


def digest_v2(inputs, outputs) -> bytes:
    h = blake3.blake3(b"vitnify-receipt v2\x00")
    h.update(_leb128(len(REGIME)) + REGIME.encode())
    h.update(_sections(inputs, outputs))
    return h.digest()


def digest_v1(inputs, outputs) -> bytes:
    h = blake3.blake3(b"vitnify-receipt v1\x00")
    h.update(_sections(inputs, outputs))
    return h.digest()


def u32_le(tokens) -> bytes:
    return b"".join(struct.pack("<I", int(t)) for t in tokens)


def decode_receipt(model_id: str, gguf_blob: bytes, arch: str, prompt, n_new: int, generated):
    """The receipt JSON fields of the reference's receipt binary (src/bin/vitni-receipt.rs:43-55)."""
    weights_hash = blake3.blake3(gguf_blob).digest()
    inputs = [("model_id", model_id.encode()), ("weights_hash", weights_hash),
              ("arch_hash", blake3.blake3(arch.encode()).digest()),
              ("prompt_tokens", u32_le(prompt)), ("n_new_tokens", struct.pack("<I", n_new))]
    out_bytes = u32_le(generated)
    outputs = [("output_tokens", out_bytes), ("output_tokens_hash", blake3.blake3(out_bytes).digest())]
    return {"model_digest": digest_v2(inputs, outputs).hex(), "regime": REGIME,
            "model_digest_v1": digest_v1(inputs, outputs).hex(),
            "weights_hash": weights_hash.hex(), "tokens": [int(t) for t in generated]}


def receipt_json(rc: dict) -> str:
    """The receipt line exactly as the reference's binary prints it
    (src/bin/vitni-receipt.rs:46-53): compact JSON, this key order."""
    toks = ",".join(str(int(t)) for t in rc["tokens"])
    return ('{"model_digest":"%s","regime":"%s","model_digest_v1":"%s","weights_hash":"%s",'
            '"tokens":[%s]}' % (rc["model_digest"], rc["regime"], rc["model_digest_v1"],
                                rc["weights_hash"], toks))
