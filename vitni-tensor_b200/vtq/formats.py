"""GGML block formats the k-quant path consumes (src/model/gguf.rs:127-217 and
src/ops/quant.rs block layouts of the reference)."""
from __future__ import annotations

from dataclasses import dataclass

F32, F16, Q4_0, Q5_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 6, 8, 12, 14

# (elements per block, bytes per block)
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q5_0: (32, 22), Q8_0: (32, 34),
         Q4_K: (256, 144), Q6_K: (256, 210)}

NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q5_0: "Q5_0", Q8_0: "Q8_0", Q4_K: "Q4_K",
         Q6_K: "Q6_K"}


def row_bytes(dtype: int, in_feat: int) -> int:
    numel, nbytes = BLOCK[dtype]
    if in_feat % numel:
        raise ValueError(f"{NAMES[dtype]}: in_feat {in_feat} not a multiple of {numel}")
    return in_feat // numel * nbytes


@dataclass
class QuantTensor:
    """QuantTensor (src/model/quant_weights.rs:47-52): GGML-order shape [in, out],
    dtype tag and the row-major bytes."""
    shape: tuple
    dtype: int
    bytes: bytes
