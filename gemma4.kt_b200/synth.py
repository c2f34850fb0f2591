"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (no public dataset or model file is involved).

All randomness comes from numpy's PCG64 (np.random.default_rng(seed)); the
quantizers are the C routines in csrc/g4_synth.c.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from ._lib import synth
from .floattensor import GGMLType


def quantize(ggml_type, w: np.ndarray, threads: int | None = None) -> np.ndarray:
    """fp32 weights (row-major, flat) -> GGUF block stream bytes."""
    w = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    t = GGMLType(int(ggml_type))
    n = w.size
    out = np.empty(t.byte_size_for(n), dtype=np.uint8)
    rc = synth().g4s_quantize(int(t), w.ctypes.data_as(C.c_void_p), n, out.ctypes.data_as(C.c_void_p),
                              threads or os.cpu_count() or 1)
    if rc != 0:
        raise ValueError(f"cannot quantize {n} elements as {t.name}")
    return out


def normal(rng: np.random.Generator, n: int, std: float = 0.02) -> np.ndarray:
    x = rng.standard_normal(n, dtype=np.float32)
    if std != 1.0:
        x *= np.float32(std)
    return x


def q8_0_random_blocks(rng: np.random.Generator, n_elems: int) -> np.ndarray:
    """Config-1 blocks: int8 q uniform in [-127, 127], fp16 d = |N(0, 0.02)| / 127."""
    nb = n_elems // 32
    blocks = np.empty((nb, 34), dtype=np.uint8)
    d = (np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.02) / np.float32(127)).astype(np.float16)
    blocks[:, :2] = d.view(np.uint8).reshape(nb, 2)
    q = rng.integers(-127, 128, size=(nb, 32), dtype=np.int16).astype(np.int8)
    blocks[:, 2:] = q.view(np.uint8)
    return blocks.reshape(-1)


def gemv_case(ggml_type, rows: int, cols: int, seed: int):
    """(weight bytes, x) for one GEMV-sweep case: W ~ N(0, 0.02) quantized, x ~ N(0, 1)."""
    rng = np.random.default_rng(seed)
    w = normal(rng, rows * cols)
    x = rng.standard_normal(cols, dtype=np.float32)
    return quantize(ggml_type, w), x


class MoeLayerData:
    """Host copy of one synthetic MoE layer (Q4_K experts by default).

    Tensor shapes follow ModelLoader.kt:223-232 / LlamaWeights.kt:50-65:
    gate_inp [dim, n_expert] F32, gate_up_exps [dim, 2*ff, n_expert],
    down_exps [ff, dim, n_expert], norms and scales F32.
    The scale and norm tensors are seeded draws, N(1, 0.1) for
    ffn_gate_inp.scale / pre_ffw_norm_2 / post_ffw_norm_2 and U(0.5, 1.5) for
    ffn_down_exps.scale, so that none of them is trivially 1.
    """

    def __init__(self, seed: int = 2, dim: int = 2816, n_expert: int = 128, n_used: int = 8, ff: int = 704,
                 expert_type=GGMLType.Q4_K, eps: float = 1e-6):
        rng = np.random.default_rng(seed)
        self.dim, self.n_expert, self.n_used, self.ff, self.eps = dim, n_expert, n_used, ff, eps
        self.expert_type = GGMLType(int(expert_type))
        self.gate_inp = normal(rng, n_expert * dim)  # F32 router
        self.gate_inp_scale = (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
        self.gate_up = quantize(self.expert_type, normal(rng, n_expert * 2 * ff * dim))
        self.down = quantize(self.expert_type, normal(rng, n_expert * dim * ff))
        self.down_scale = rng.uniform(0.5, 1.5, n_expert).astype(np.float32)
        self.pre_norm = (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
        self.post_norm = (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)

    def tokens(self, n_tokens: int, seed: int = 2) -> np.ndarray:
        """Residual-stream hidden states ~ N(0, 1), [n_tokens, dim]."""
        rng = np.random.default_rng(seed + 1000)
        return rng.standard_normal((n_tokens, self.dim), dtype=np.float32)


def random_blocks(ggml_type, n_elems: int, rng: np.random.Generator) -> np.ndarray:
    """Valid block streams for the formats without a quantizer here (F16, Q4_0,
    Q4_1, Q5_1, Q5_K, MXFP4): random code bytes, fp16 scale fields ~ N(0, 0.01)
    (Q4_1/Q5_1 minima and Q5_K mins included), MXFP4 exponents 2^-12..2^-4.
    Weights of roughly the magnitude of the quantized N(0, 0.02) ones."""
    from .floattensor import GGMLType

    t = GGMLType(int(ggml_type))
    nb = n_elems // t.block_size
    if nb * t.block_size != n_elems:
        raise ValueError("n_elems is not a whole number of blocks")
    f16 = lambda n: (rng.standard_normal(n) * 0.01).astype(np.float16).view(np.uint8).reshape(n, 2)
    if t == GGMLType.F16:
        return (rng.standard_normal(nb) * 0.02).astype(np.float16).view(np.uint8)
    raw = rng.integers(0, 256, size=(nb, t.type_size), dtype=np.uint8)
    fields = {GGMLType.Q4_0: [0], GGMLType.Q4_1: [0, 2], GGMLType.Q5_1: [0, 2], GGMLType.Q5_K: [0, 2]}
    if t == GGMLType.MXFP4:
        raw[:, 0] = rng.integers(116, 125, size=nb)
    elif t in fields:
        for off in fields[t]:
            raw[:, off:off + 2] = f16(nb)
        if t == GGMLType.Q4_0:  # |d|/8 per step, as a symmetric 4-bit quantizer would
            raw[:, 0:2] = (rng.standard_normal(nb) * 0.004).astype(np.float16).view(np.uint8).reshape(nb, 2)
    else:
        raise ValueError(f"no random block generator for {t.name}")
    return raw.reshape(-1)
