"""Generates tests/golden/blocks.npz: GGUF block streams and their element
values as decoded by gguf-py 0.19.0 (llama.cpp's Python package, installed
in this image as `gguf`), an implementation of the same block formats that is
independent of both the reference and this repository.

gguf-py evaluates the same expressions in the same order as the reference's
get() decoders (Q8_0: q*d; Q4_K: (d*sc)*q - dmin*m; Q6_K: (d*sc)*q; BF16:
bits<<16), so its float32 results must match the oracle bit for bit.

Also stores small GEMV cases (raw blocks, x, and y computed in float64 from
the gguf-py decoded weights) used as tolerance fixtures.

Also writes tests/golden/blocks_more.npz with the remaining formats the
reference loads (F16, Q4_0, Q4_1, Q5_1, Q5_K, MXFP4), pinned the same way.

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
from gguf import GGMLQuantizationType as Q
from gguf.quants import dequantize, quantize

HERE = Path(__file__).resolve().parent
TYPES = {"F32": (Q.F32, 0), "BF16": (Q.BF16, 30), "Q8_0": (Q.Q8_0, 8), "Q4_K": (Q.Q4_K, 12), "Q6_K": (Q.Q6_K, 14)}
BLOCK = {"F32": (1, 4), "BF16": (1, 2), "Q8_0": (32, 34), "Q4_K": (256, 144), "Q6_K": (256, 210)}
FP16_FIELDS = {"Q8_0": [0], "Q4_K": [0, 2], "Q6_K": [208]}


def finite_f16(rng, n, scale):
    return (rng.standard_normal(n) * scale).astype(np.float16).view(np.uint16)


def random_blocks(name: str, nblocks: int, rng) -> np.ndarray:
    be, bb = BLOCK[name]
    if name == "F32":
        return rng.standard_normal(nblocks).astype(np.float32).view(np.uint8)
    if name == "BF16":
        return (rng.standard_normal(nblocks).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16).view(np.uint8)
    raw = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    for off in FP16_FIELDS[name]:
        raw[:, off:off + 2] = finite_f16(rng, nblocks, 0.01).view(np.uint8).reshape(nblocks, 2)
    return raw.reshape(-1)


def edge_blocks(name: str) -> np.ndarray:
    """Blocks built by hand around the decoders' edge codes."""
    be, bb = BLOCK[name]
    f16 = lambda v: np.array([v], dtype=np.float16).view(np.uint8)
    if name == "Q8_0":
        rows = []
        for d in [1.0, -0.5, 6.1e-5, 5.96e-8, 65504.0]:  # normal, negative, min normal, min subnormal, max
            b = np.zeros(bb, np.uint8)
            b[:2] = f16(d)
            b[2:] = np.array(list(range(-128, -112)) + list(range(112, 128)), dtype=np.int8).view(np.uint8)
            rows.append(b)
        return np.concatenate(rows)
    if name == "Q4_K":
        rows = []
        for d, dmin in [(1.0, 1.0), (0.01, 0.02), (6.1e-5, 5.96e-8), (-0.25, 0.5)]:
            b = np.zeros(bb, np.uint8)
            b[0:2] = f16(d)
            b[2:4] = f16(dmin)
            b[4:16] = np.array([63, 0, 0xC0 | 17, 0x80 | 5, 0, 63, 0x40 | 9, 0xC0 | 63, 0xF0, 0x0F, 0xA5, 0x5A],
                               dtype=np.uint8)  # 6-bit extremes and the j>=4 packed high bits
            b[16:] = np.arange(128, dtype=np.uint8) * 17  # nibbles 0..15 in both halves
            rows.append(b)
        return np.concatenate(rows)
    if name == "Q6_K":
        rows = []
        for d in [1.0, -0.125, 6.1e-5, 5.96e-8]:
            b = np.zeros(bb, np.uint8)
            b[:128] = np.arange(128, dtype=np.uint8) * 31
            b[128:192] = np.array([0x00, 0xFF, 0x1B, 0xE4] * 16, dtype=np.uint8)  # q6 = 0 and 63 and mixes
            b[192:208] = np.array([127, -128, -1, 1, 0, 64, -64, 5, 7, -9, 100, -100, 3, -3, 2, -2],
                                  dtype=np.int8).view(np.uint8)
            b[208:210] = f16(d)
            rows.append(b)
        return np.concatenate(rows)
    if name == "BF16":
        bits = np.array([0x0000, 0x8000, 0x3F80, 0xBF80, 0x0001, 0x7F7F, 0xFF7F, 0x7F80, 0xFF80, 0x0080],
                        dtype=np.uint16)
        return bits.view(np.uint8)
    return np.array([0.0, -0.0, 1.5, -2.25, 1e-40, 3.4e38], dtype=np.float32).view(np.uint8)


def gguf_decode(name: str, raw: np.ndarray) -> np.ndarray:
    qt = TYPES[name][0]
    if name == "F32":
        return raw.view(np.float32).copy()
    be, bb = BLOCK[name]
    return dequantize(raw.reshape(-1, bb), qt).reshape(-1).astype(np.float32)


def main() -> None:
    rng = np.random.default_rng(20261201)
    out = {}
    for name in TYPES:
        be, bb = BLOCK[name]
        nblocks = {"F32": 2048, "BF16": 2048, "Q8_0": 96, "Q4_K": 24, "Q6_K": 24}[name]
        raw = random_blocks(name, nblocks, rng)
        out[f"{name}_raw"] = raw
        out[f"{name}_vals"] = gguf_decode(name, raw)
        er = edge_blocks(name)
        out[f"{name}_edge_raw"] = er
        out[f"{name}_edge_vals"] = gguf_decode(name, er)
    # gguf-py's own Q8_0 quantizer (ggml-exact) on a known input, for the
    # build's quantizer to match.
    w = (rng.standard_normal(32 * 64) * 0.02).astype(np.float32)
    out["q8_0_quant_in"] = w
    out["q8_0_quant_out"] = quantize(w.reshape(-1, 32), Q.Q8_0).reshape(-1)
    # GEMV fixtures: rows x cols, y in float64 from the decoded weights.
    for name, rows, cols in [("Q8_0", 8, 256), ("Q4_K", 6, 512), ("Q6_K", 6, 512), ("BF16", 8, 64),
                             ("F32", 8, 64)]:
        be, bb = BLOCK[name]
        raw = random_blocks(name, rows * cols // be, rng)
        x = rng.standard_normal(cols).astype(np.float32)
        wv = gguf_decode(name, raw).astype(np.float64).reshape(rows, cols)
        out[f"gemv_{name}_raw"] = raw
        out[f"gemv_{name}_x"] = x
        out[f"gemv_{name}_y"] = (wv @ x.astype(np.float64)).astype(np.float64)
        out[f"gemv_{name}_shape"] = np.array([rows, cols])
    np.savez_compressed(HERE / "blocks.npz", **out)
    print("wrote", HERE / "blocks.npz", sum(v.nbytes for v in out.values()), "bytes")


# ---------------------------------------------------------------- the other formats the reference loads
# FloatTensorFactory.kt:7-23: F16, Q4_0, Q4_1, Q5_1, Q5_K, MXFP4 besides the five above.  Written to
# blocks_more.npz with a seed of their own, so blocks.npz stays as it is.
MORE = {"F16": (Q.F16, 1, 1, 2, []), "Q4_0": (Q.Q4_0, 2, 32, 18, [0]), "Q4_1": (Q.Q4_1, 3, 32, 20, [0, 2]),
        "Q5_1": (Q.Q5_1, 7, 32, 24, [0, 2]), "Q5_K": (Q.Q5_K, 13, 256, 176, [0, 2]),
        "MXFP4": (Q.MXFP4, 39, 32, 17, [])}


def more_random(name: str, nblocks: int, rng) -> np.ndarray:
    qt, _, be, bb, f16_fields = MORE[name]
    if name == "F16":
        return finite_f16(rng, nblocks, 1.0).view(np.uint8)
    raw = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    for off in f16_fields:
        raw[:, off:off + 2] = finite_f16(rng, nblocks, 0.01).view(np.uint8).reshape(nblocks, 2)
    if name == "MXFP4":
        raw[:, 0] = rng.integers(100, 140, size=nblocks)  # scales 2^-28 .. 2^11
    return raw.reshape(-1)


def more_edge(name: str) -> np.ndarray:
    qt, _, be, bb, _ = MORE[name]
    f16 = lambda v: np.array([v], dtype=np.float16).view(np.uint8)
    codes = np.arange(16, dtype=np.uint8) * 17  # every nibble value in both halves
    rows = []
    if name == "F16":
        bits = np.array([0x0000, 0x8000, 0x3C00, 0xBC00, 0x0001, 0x03FF, 0x0400, 0x7BFF, 0xFBFF, 0x7C00, 0xFC00],
                        dtype=np.uint16)
        return bits.view(np.uint8)
    if name == "Q4_0":
        for d in [1.0, -0.5, 6.1e-5, 5.96e-8, 65504.0]:
            b = np.zeros(bb, np.uint8)
            b[:2] = f16(d)
            b[2:] = codes
            rows.append(b)
    elif name in ("Q4_1", "Q5_1"):
        for (d, m), qh in zip([(1.0, -8.0), (0.01, 0.02), (6.1e-5, -5.96e-8), (-0.25, 0.5)],
                              [0x00000000, 0xFFFFFFFF, 0xAAAAAAAA, 0x0F0F00F0]):
            b = np.zeros(bb, np.uint8)
            b[0:2] = f16(d)
            b[2:4] = f16(m)
            if name == "Q5_1":
                b[4:8] = np.array([qh], dtype="<u4").view(np.uint8)
                b[8:] = codes
            else:
                b[4:] = codes
            rows.append(b)
    elif name == "Q5_K":
        for (d, dmin), hb in zip([(1.0, 1.0), (0.01, 0.02), (6.1e-5, 5.96e-8), (-0.25, 0.5)], [0x00, 0xFF, 0xA5, 0x3C]):
            b = np.zeros(bb, np.uint8)
            b[0:2] = f16(d)
            b[2:4] = f16(dmin)
            b[4:16] = np.array([63, 0, 0xC0 | 17, 0x80 | 5, 0, 63, 0x40 | 9, 0xC0 | 63, 0xF0, 0x0F, 0xA5, 0x5A],
                               dtype=np.uint8)
            b[16:48] = (np.arange(32, dtype=np.uint8) * 37) ^ hb  # the fifth bits of all eight sub-blocks
            b[48:] = np.arange(128, dtype=np.uint8) * 17
            rows.append(b)
    elif name == "MXFP4":
        for e in [0, 1, 2, 100, 127, 128, 200, 254]:
            b = np.zeros(bb, np.uint8)
            b[0] = e
            b[1:] = codes
            rows.append(b)
    return np.concatenate(rows)


def more_decode(name: str, raw: np.ndarray) -> np.ndarray:
    qt, _, be, bb, _ = MORE[name]
    if name == "F16":
        return raw.view(np.float16).astype(np.float32)
    return dequantize(raw.reshape(-1, bb), qt).reshape(-1).astype(np.float32)


def main_more() -> None:
    rng = np.random.default_rng(20261202)
    out = {}
    for name in MORE:
        _, tid, be, bb, _ = MORE[name]
        raw = more_random(name, {"F16": 2048}.get(name, 64 if be == 32 else 16), rng)
        out[f"{name}_raw"] = raw
        out[f"{name}_vals"] = more_decode(name, raw)
        er = more_edge(name)
        out[f"{name}_edge_raw"] = er
        out[f"{name}_edge_vals"] = more_decode(name, er)
        rows, cols = (6, 512)
        graw = more_random(name, rows * cols // be, rng)
        x = rng.standard_normal(cols).astype(np.float32)
        wv = more_decode(name, graw).astype(np.float64).reshape(rows, cols)
        out[f"gemv_{name}_raw"] = graw
        out[f"gemv_{name}_x"] = x
        out[f"gemv_{name}_y"] = wv @ x.astype(np.float64)
        out[f"gemv_{name}_shape"] = np.array([rows, cols])
    np.savez_compressed(HERE / "blocks_more.npz", **out)
    print("wrote", HERE / "blocks_more.npz", sum(v.nbytes for v in out.values()), "bytes")


if __name__ == "__main__":
    main()
    main_more()
