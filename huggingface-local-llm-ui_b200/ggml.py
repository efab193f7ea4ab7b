"""GGML tensor types as the reference's GGUF parser knows them.

Mirrors ``GgmlDType`` (src/inference.rs:116-185): the numeric ids stored in a
GGUF tensor-info record, the number of elements per block and the bytes per
block.  A row of ``k`` elements of type ``t`` occupies
``(k // block_size(t)) * type_size(t)`` bytes (inference.rs:420, :579).
"""

F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q8_1 = 0, 1, 2, 3, 6, 7, 8, 9
Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, Q8_K, BF16 = 10, 11, 12, 13, 14, 15, 30

NAMES = {
    F32: "F32", F16: "F16", Q4_0: "Q4_0", Q4_1: "Q4_1", Q5_0: "Q5_0", Q5_1: "Q5_1",
    Q8_0: "Q8_0", Q8_1: "Q8_1", Q2_K: "Q2_K", Q3_K: "Q3_K", Q4_K: "Q4_K",
    Q5_K: "Q5_K", Q6_K: "Q6_K", Q8_K: "Q8_K", BF16: "BF16",
}

_BLOCK = {F32: 1, F16: 1, BF16: 1, Q4_0: 32, Q4_1: 32, Q5_0: 32, Q5_1: 32, Q8_0: 32,
          Q8_1: 32, Q2_K: 256, Q3_K: 256, Q4_K: 256, Q5_K: 256, Q6_K: 256, Q8_K: 256}
_SIZE = {F32: 4, F16: 2, BF16: 2, Q4_0: 18, Q4_1: 20, Q5_0: 22, Q5_1: 24, Q8_0: 34,
         Q8_1: 36, Q2_K: 84, Q3_K: 110, Q4_K: 144, Q5_K: 176, Q6_K: 210, Q8_K: 292}


def from_u32(v: int) -> int:
    """GgmlDType::from_u32 (inference.rs:136-155): unknown ids are an error."""
    if v not in _BLOCK:
        raise ValueError(f"unknown GGML data type in GGUF: {v}")
    return v


def block_size(t: int) -> int:
    return _BLOCK[from_u32(t)]


def type_size(t: int) -> int:
    return _SIZE[from_u32(t)]


def row_bytes(t: int, k: int) -> int:
    bs = block_size(t)
    if k % bs:
        raise ValueError(f"row length {k} is not a multiple of the {NAMES[t]} block ({bs})")
    return (k // bs) * type_size(t)
