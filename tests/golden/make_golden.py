"""Generate the dequantisation golden vectors in tests/golden/.

The reference engine (Rust, Windows-only) cannot be built here and ships no
test vectors.  These fixtures pin the oracle's restatement of
dequantize_slice (src/inference.rs:1347-1474) against gguf-py 0.19.0
(gguf.quants), llama.cpp's independent Python decoder of the same GGML block
formats, which evaluates the same f32 expressions in the same order:
Q4_K (d*sc)*q - dmin*m, Q6_K (d*sc)*q, Q8_0 d*q, Q5_K as Q4_K with the fifth
bit, Q4_0 d*(q-8).

Inputs are seeded random blocks plus hand-built edge cases:
  * f16 scales that are +-0, subnormal, the largest finite, +-inf and NaN,
  * every 6-bit scale/min code 0..63 in each of the 8 sub-block positions
    (exercising all branches of decode_q4k_scales),
  * all-zero and all-ones quant planes, and int8 codes -128/127.
Blocks whose expected output contains a NaN are stored too; the comparison
treats NaN == NaN (gguf-py's f16 -> f32 cast may quiet a signalling NaN,
so NaN payloads are not part of this pin).

Run:  python tests/golden/make_golden.py   (writes dequant_golden.npz)
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent

TYPES = {"Q4_K": (12, 144, 256), "Q6_K": (14, 210, 256), "Q8_0": (8, 34, 32),
         "Q5_K": (13, 176, 256), "Q4_0": (2, 18, 32)}

SPECIAL_F16 = np.array([0x0000, 0x8000, 0x0001, 0x03FF, 0x0200, 0x8001, 0x0400, 0x7BFF,
                        0xFBFF, 0x7C00, 0xFC00, 0x7E00, 0x3C00, 0x1400, 0x0155, 0x00FF],
                       dtype=np.uint16)


def pack_scales(sc, mn):
    out = np.zeros(12, np.uint8)
    out[0:4] = sc[0:4] | ((sc[4:8] >> 4) << 6)
    out[4:8] = mn[0:4] | ((mn[4:8] >> 4) << 6)
    out[8:12] = (sc[4:8] & 0x0F) | ((mn[4:8] & 0x0F) << 4)
    return out


def make_blocks(name: str, rng: np.random.Generator) -> np.ndarray:
    tid, ts, _ = TYPES[name]
    blocks = [rng.integers(0, 256, size=ts, dtype=np.uint8) for _ in range(48)]
    # make the random ones sane: finite f16 scales of plausible magnitude
    for b in blocks:
        d = np.float16(abs(rng.standard_normal()) * 1e-3).view(np.uint16)
        if name in ("Q4_K", "Q5_K"):
            dm = np.float16(abs(rng.standard_normal()) * 1e-3).view(np.uint16)
            b[0:2] = np.array([d], np.uint16).view(np.uint8)
            b[2:4] = np.array([dm], np.uint16).view(np.uint8)
        elif name == "Q6_K":
            b[208:210] = np.array([d], np.uint16).view(np.uint8)
        else:
            b[0:2] = np.array([d], np.uint16).view(np.uint8)
    # special f16 scale values
    for h in SPECIAL_F16:
        b = rng.integers(0, 256, size=ts, dtype=np.uint8)
        hb = np.array([h], np.uint16).view(np.uint8)
        if name in ("Q4_K", "Q5_K"):
            b[0:2] = hb
            b[2:4] = np.array([SPECIAL_F16[(int(h) * 7) % len(SPECIAL_F16)]], np.uint16).view(np.uint8)
        elif name == "Q6_K":
            b[208:210] = hb
        else:
            b[0:2] = hb
        blocks.append(b)
    if name in ("Q4_K", "Q5_K"):
        # every 6-bit code in every scale and min position
        for code in range(64):
            sc = np.array([(code + j * 9) % 64 for j in range(8)], np.uint8)
            mn = np.array([(63 - code + j * 5) % 64 for j in range(8)], np.uint8)
            b = rng.integers(0, 256, size=ts, dtype=np.uint8)
            b[0:2] = np.array([np.float16(0.0123).view(np.uint16)], np.uint16).view(np.uint8)
            b[2:4] = np.array([np.float16(0.00071).view(np.uint16)], np.uint16).view(np.uint8)
            b[4:16] = pack_scales(sc, mn)
            blocks.append(b)
    # extreme quant planes
    for fill in (0x00, 0xFF, 0x80, 0x7F):
        b = np.full(ts, fill, np.uint8)
        d16 = np.array([np.float16(0.5).view(np.uint16)], np.uint16).view(np.uint8)
        if name in ("Q4_K", "Q5_K"):
            b[0:2] = d16
            b[2:4] = d16
        elif name == "Q6_K":
            b[208:210] = d16
        else:
            b[0:2] = d16
        blocks.append(b)
    return np.stack(blocks)


def main() -> None:
    sys.path.insert(0, str(REPO))
    import gguf.quants as gq
    from gguf.constants import GGMLQuantizationType as QT
    import importlib.metadata as md

    rng = np.random.default_rng(0x5EED)
    out = {"gguf_version": np.array(md.version("gguf"))}
    f16_all = np.arange(65536, dtype=np.uint16)
    out["f16_bits"] = f16_all
    with np.errstate(invalid="ignore"):
        out["f16_as_f32"] = f16_all.view(np.float16).astype(np.float32)
    for name in TYPES:
        blocks = make_blocks(name, rng)
        with np.errstate(all="ignore"):
            ref = gq.dequantize(blocks.reshape(-1), getattr(QT, name)).astype(np.float32).reshape(-1)
        out[f"{name}_raw"] = blocks
        out[f"{name}_f32"] = ref
    np.savez_compressed(HERE / "dequant_golden.npz", **out)
    print("wrote", HERE / "dequant_golden.npz", {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
