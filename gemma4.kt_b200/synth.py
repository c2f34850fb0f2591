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


def normal_fast(seed: int, stream: int, n: int, std: float = 0.02, threads: int | None = None) -> np.ndarray:
    """n N(0, std) float32 values from the C generator of g4_synth.c (xoshiro256**
    streams per 2^20-value chunk, seeded from (seed, stream, chunk); the result
    does not depend on the thread count).  For models too large for numpy's
    single-threaded generator."""
    out = np.empty(n, dtype=np.float32)
    rc = synth().g4s_normal(int(seed) & (2**64 - 1), int(stream) & (2**64 - 1), out.ctypes.data_as(C.c_void_p), n,
                            float(std), threads or os.cpu_count() or 1)
    if rc != 0:
        raise ValueError("g4s_normal failed")
    return out


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


class SharedMlpData:
    """Host copy of the shared-MLP half of a synthetic MoE layer (ffn_gate /
    ffn_up [dim, ff], ffn_down [ff, dim] N(0, 0.02) quantized; ffn_norm,
    post_ffw_norm_1, post_ffw_norm N(1, 0.1); layer output scale U(0.5, 1))."""

    def __init__(self, dim: int, ff: int, seed: int = 5, gate_type=GGMLType.Q8_0):
        rng = np.random.default_rng([seed, 77])
        self.dim, self.ff, self.gate_type = dim, ff, GGMLType(int(gate_type))
        self.ffn_gate = quantize(self.gate_type, normal(rng, dim * ff))
        self.ffn_up = quantize(self.gate_type, normal(rng, dim * ff))
        self.ffn_down = quantize(self.gate_type, normal(rng, dim * ff))
        self.ffn_norm = (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
        self.post_ffw_norm_1 = (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
        self.post_ffw_norm = (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
        self.layer_output_scale = float(np.float32(rng.uniform(0.5, 1.0)))


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


# ---------------------------------------------------------------------- whole models
from dataclasses import dataclass, field  # noqa: E402


@dataclass
class DecoderSpec:
    """Geometry of a synthetic Gemma-4-style decoder (the metadata keys of
    ModelLoader.kt:46-116 and the tensor set of ModelLoader.kt:154-261).

    Layer l uses sliding-window attention unless (l + 1) % swa_period == 0
    (swa_period 0: every layer full attention); the pattern is written as
    gemma4.attention.sliding_window_pattern.  The last shared_kv_layers layers
    reuse the KV cache of an earlier layer (LlamaConfiguration.kvSourceLayer).
    Layers listed in no_v_layers have no attn_v tensor (V = K, Llama.kt:176-181).
    n_expert > 0 makes every layer a MoE layer: shared dense FFN of width ff
    plus n_expert experts of width expert_ff (top n_expert_used)."""

    name: str
    n_layers: int
    dim: int
    n_heads: int
    n_kv_heads: int
    head_size: int
    ff: int
    vocab: int
    ctx_len: int = 4096
    wtype: int = GGMLType.Q8_0
    emb_type: int = GGMLType.Q8_0
    head_size_swa: int = 0          # 0: same as head_size
    sliding_window: int = 512
    swa_period: int = 5
    shared_kv_layers: int = 0
    no_v_layers: tuple = ()
    softcap: float = 30.0
    eps: float = 1e-6
    rope_theta: float = 1e6
    rope_theta_swa: float = 1e4
    tied_output: bool = True
    n_expert: int = 0
    n_expert_used: int = 0
    expert_ff: int = 0
    expert_type: int = GGMLType.Q4_K
    layer_scale: bool = True
    qk_temperature: bool = True     # q/k norm weights scaled by head_size^-1/4 (see SynthDecoder)
    fast_rng: bool = False          # matrices from normal_fast (all host threads) instead of numpy
    replicate_layers: bool = False  # layers > 0 reuse layer 0's matrices (benchmark models: same bytes per layer)
    extra: dict = field(default_factory=dict)

    def hs(self, layer: int) -> int:
        return (self.head_size_swa or self.head_size) if self.is_swa(layer) else self.head_size

    def is_swa(self, layer: int) -> bool:
        return self.swa_period > 0 and (layer + 1) % self.swa_period != 0


# The benchmark's configurations 4 and 5 (dense and MoE decoders).
C4_DENSE = DecoderSpec("C4 dense decoder", n_layers=35, dim=1536, n_heads=8, n_kv_heads=1, head_size=256, ff=6144,
                       vocab=262144)
C5_MOE = DecoderSpec("C5 MoE decoder", n_layers=30, dim=2816, n_heads=16, n_kv_heads=8, head_size=256, ff=2112,
                     vocab=262144, n_expert=128, n_expert_used=8, expert_ff=704, fast_rng=True)

# special tokens the reference tokenizer and chat format look up
# (GemmaTokenizer.kt:18-28, GemmaChatFormat.kt:6-13, Llama.kt:18)
SPECIAL_TOKENS = ["<pad>", "<eos>", "<bos>", "<unk>", "<mask>", "<|turn>", "<turn|>"]
N_SPECIAL = len(SPECIAL_TOKENS) + 256  # specials, then the 256 byte tokens <0x00>..<0xFF>


def vocabulary(n: int):
    """Token strings, scores and types of a synthetic vocabulary of n tokens."""
    tokens = list(SPECIAL_TOKENS) + [f"<0x{b:02X}>" for b in range(256)]
    tokens += [f"▁t{i}" for i in range(n - len(tokens))]
    scores = np.zeros(n, dtype=np.float32)
    scores[N_SPECIAL:] = -np.arange(n - N_SPECIAL, dtype=np.float32)
    types = np.ones(n, dtype=np.int32)
    types[:len(SPECIAL_TOKENS)] = 3  # control
    types[len(SPECIAL_TOKENS):N_SPECIAL] = 6  # byte
    return tokens, scores, types


class SynthDecoder:
    """Seeded random-init weights of a DecoderSpec, in GGUF form: `metadata`
    (gguf.Typed values) and `tensors` [(name, dims, GGMLType, block bytes)].
    Matrices are N(0, 0.02) quantized by the build's quantizers; norm weights
    N(1, 0.1); layer output scales U(0.5, 1); rope_freqs U(1, 2); router
    F32 N(0, 0.02); router input scales N(1, 0.1); expert output scales
    U(0.5, 1.5).  Every tensor draws from its own stream
    default_rng([seed, index]), so tensors can be made in any order.

    The attention of the reference has scale 1.0 (Llama.kt:198): the learned
    q/k norm weights set the temperature.  With weights near 1, scores of
    RMS-normalised q and k have a spread of about sqrt(head_size) (16 at 256)
    and the model is chaotic: the reference's own Vector-API and scalarDot
    modes (llama.VectorBitSize) stop agreeing within a few positions.  So
    by default (qk_temperature) the q and k norm weights are
    head_size^-1/4 * N(1, 0.1): scores of unit spread, the usual
    1/sqrt(head_size) temperature folded into the two norms."""

    def __init__(self, spec: DecoderSpec, seed: int, threads: int | None = None):
        from . import gguf as G

        self.spec, self.seed = spec, seed
        s = spec
        self._i = 0
        self._layer0 = {}
        self.tensors = []
        self.threads = threads
        tokens, scores, types = vocabulary(s.vocab)
        A, VT = G.arr, G.ValueType
        self.metadata = {
            "general.architecture": "gemma4",
            "general.name": f"synthetic {s.name} seed {seed}",
            "general.alignment": G.u32(32),
            "gemma4.context_length": G.u32(s.ctx_len),
            "gemma4.embedding_length": G.u32(s.dim),
            "gemma4.block_count": G.u32(s.n_layers),
            "gemma4.feed_forward_length": G.u32(s.ff),
            "gemma4.attention.head_count": G.u32(s.n_heads),
            "gemma4.attention.head_count_kv": G.u32(s.n_kv_heads),
            "gemma4.attention.key_length": G.u32(s.head_size),
            "gemma4.attention.value_length": G.u32(s.head_size),
            "gemma4.attention.key_length_swa": G.u32(s.head_size_swa or s.head_size),
            "gemma4.attention.value_length_swa": G.u32(s.head_size_swa or s.head_size),
            "gemma4.attention.sliding_window": G.u32(s.sliding_window),
            "gemma4.attention.sliding_window_pattern": A(VT.BOOL, [s.is_swa(l) for l in range(s.n_layers)]),
            "gemma4.attention.shared_kv_layers": G.u32(s.shared_kv_layers),
            "gemma4.attention.layer_norm_rms_epsilon": G.f32(s.eps),
            "gemma4.rope.freq_base": G.f32(s.rope_theta),
            "gemma4.rope.freq_base_swa": G.f32(s.rope_theta_swa),
            "gemma4.final_logit_softcapping": G.f32(s.softcap),
            "tokenizer.ggml.model": "gemma4",
            "tokenizer.ggml.tokens": A(VT.STRING, tokens),
            "tokenizer.ggml.scores": A(VT.FLOAT32, scores),
            "tokenizer.ggml.token_type": A(VT.INT32, types),
            "tokenizer.ggml.bos_token_id": G.u32(2),
            "tokenizer.ggml.eos_token_id": G.u32(1),
        }
        if s.n_expert:
            self.metadata.update({
                "gemma4.expert_count": G.u32(s.n_expert),
                "gemma4.expert_used_count": G.u32(s.n_expert_used),
                "gemma4.expert_feed_forward_length": G.u32(s.expert_ff),
            })
        self.metadata.update(s.extra)
        d = s.dim
        self._mat("token_embd.weight", s.emb_type, d, s.vocab)
        if not s.tied_output:
            self._mat("output.weight", s.wtype, d, s.vocab)
        self._f32("output_norm.weight", self._rng().normal(1.0, 0.1, d))
        self._f32("rope_freqs.weight", self._rng().uniform(1.0, 2.0, s.head_size // 2))
        for l in range(s.n_layers):
            hs = s.hs(l)
            p = f"blk.{l}."
            self._f32(p + "attn_norm.weight", self._rng().normal(1.0, 0.1, d))
            self._mat(p + "attn_q.weight", s.wtype, d, s.n_heads * hs)
            self._mat(p + "attn_k.weight", s.wtype, d, s.n_kv_heads * hs)
            if l not in s.no_v_layers:
                self._mat(p + "attn_v.weight", s.wtype, d, s.n_kv_heads * hs)
            self._mat(p + "attn_output.weight", s.wtype, s.n_heads * hs, d)
            qk = float(hs) ** -0.25 if s.qk_temperature else 1.0
            self._f32(p + "attn_q_norm.weight", qk * self._rng().normal(1.0, 0.1, hs))
            self._f32(p + "attn_k_norm.weight", qk * self._rng().normal(1.0, 0.1, hs))
            self._f32(p + "post_attention_norm.weight", self._rng().normal(1.0, 0.1, d))
            self._f32(p + "ffn_norm.weight", self._rng().normal(1.0, 0.1, d))
            self._mat(p + "ffn_gate.weight", s.wtype, d, s.ff)
            self._mat(p + "ffn_up.weight", s.wtype, d, s.ff)
            self._mat(p + "ffn_down.weight", s.wtype, s.ff, d)
            self._f32(p + "post_ffw_norm.weight", self._rng().normal(1.0, 0.1, d))
            if s.layer_scale:
                self._f32(p + "layer_output_scale.weight", self._rng().uniform(0.5, 1.0, 1))
            if s.n_expert:
                E, eff = s.n_expert, s.expert_ff
                self._f32(p + "post_ffw_norm_1.weight", self._rng().normal(1.0, 0.1, d))
                self._f32(p + "pre_ffw_norm_2.weight", self._rng().normal(1.0, 0.1, d))
                self._f32(p + "post_ffw_norm_2.weight", self._rng().normal(1.0, 0.1, d))
                self._mat(p + "ffn_gate_inp.weight", GGMLType.F32, d, E)
                self._f32(p + "ffn_gate_inp.scale", self._rng().normal(1.0, 0.1, d))
                self._mat(p + "ffn_gate_up_exps.weight", s.expert_type, d, 2 * eff, E)
                self._mat(p + "ffn_down_exps.weight", s.expert_type, eff, d, E)
                self._f32(p + "ffn_down_exps.scale", self._rng().uniform(0.5, 1.5, E))

    def _rng(self):
        r = np.random.default_rng([self.seed, self._i])
        self._i += 1
        return r

    def _f32(self, name, values):
        a = np.asarray(values, dtype=np.float32).reshape(-1)
        self.tensors.append((name, (a.size,), GGMLType.F32, a.view(np.uint8)))

    def _mat(self, name, t, *dims):
        if self.spec.replicate_layers and name.startswith("blk."):
            layer, suffix = name.split(".", 2)[1:]
            if layer != "0":
                _, d0, t0, raw0 = self._layer0[suffix]
                self.tensors.append((name, d0, t0, raw0))
                return
        n = 1
        for x in dims:
            n *= x
        if self.spec.fast_rng:
            w = normal_fast(self.seed, self._i, n, threads=self.threads)
            self._i += 1
        else:
            w = normal(self._rng(), n)
        raw = w.view(np.uint8) if int(t) == GGMLType.F32 else quantize(t, w, self.threads)
        self.tensors.append((name, tuple(dims), GGMLType(int(t)), raw))
        if self.spec.replicate_layers and name.startswith("blk.0."):
            self._layer0[name.split(".", 2)[2]] = self.tensors[-1]

    def tensor(self, name: str) -> np.ndarray:
        for n, _, _, raw in self.tensors:
            if n == name:
                return raw
        raise KeyError(name)

    def write(self, path) -> None:
        from .gguf import write_gguf

        write_gguf(path, self.metadata, self.tensors)

    def prompt(self, n: int, seed: int | None = None) -> np.ndarray:
        """n uniform random token ids outside the special and byte tokens."""
        rng = np.random.default_rng([self.seed if seed is None else seed, 999983])
        return rng.integers(N_SPECIAL, self.spec.vocab, size=n, dtype=np.int64).astype(np.int32)
