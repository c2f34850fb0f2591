"""Host-side mirror of gemma4.kt's model loading and decode loop, backed by the
GPU-resident decoder of libg4b200 (g4_model_* / g4_state_* / g4_decode_*).

Reference (lib/src/main/kotlin/io/github/lbenedetto/internal/):
  ModelLoader.loadModel       gguf/ModelLoader.kt:39-152   -> ModelConfig.from_metadata
  ModelLoader.loadWeights     gguf/ModelLoader.kt:154-261  -> DecoderModel (raw blocks to HBM)
  LlamaConfiguration          model/LlamaConfiguration.kt  -> ModelConfig
  Llama.forward               model/Llama.kt:105-408       -> DecoderState.step (one CUDA graph)
  Llama.generateTokens        model/Llama.kt:413-477       -> DecoderState.generate (greedy, GPU-resident)
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import check, lib
from .floattensor import Context, GGMLType


@dataclass
class ModelConfig:
    """LlamaConfiguration (LlamaConfiguration.kt:3-55) as ModelLoader derives it."""

    dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: list
    ff: list
    vocab: int
    ctx_len: int
    eps: float
    rope_theta: float
    rope_theta_swa: float
    head_size_full: int
    head_size_swa: int
    sliding_window: int
    logit_softcap: float
    is_swa: list
    n_layer_kv_from_start: int
    n_expert: int = 0
    n_expert_used: int = 0
    expert_ff: int = 0

    def head_size(self, l: int) -> int:
        return self.head_size_swa if self.is_swa[l] else self.head_size_full

    def kv_source_layer(self, l: int) -> int:
        """LlamaConfiguration.kvSourceLayer (LlamaConfiguration.kt:22-28)."""
        if l < self.n_layer_kv_from_start:
            return l
        return self.n_layer_kv_from_start - (2 if self.is_swa[l] else 1)

    @staticmethod
    def from_metadata(md: dict, tensor_dims: dict, context_length: int = -1) -> "ModelConfig":
        """ModelLoader.loadModel (ModelLoader.kt:39-139); tensor_dims: name -> dims."""
        ctx = int(md["gemma4.context_length"])
        if 0 <= context_length <= ctx:
            ctx = context_length
        n_layers = int(md["gemma4.block_count"])
        hf = int(md["gemma4.attention.key_length"])
        hsw = int(md["gemma4.attention.key_length_swa"])
        ffr = md["gemma4.feed_forward_length"]
        ff = [int(v) for v in ffr] if isinstance(ffr, (list, np.ndarray)) else [int(ffr)] * n_layers
        pat = md.get("gemma4.attention.sliding_window_pattern")
        if pat is not None:
            is_swa = [bool(v) for v in pat]
        else:
            is_swa = []
            for i in range(n_layers):
                qn = tensor_dims.get(f"blk.{i}.attn_q_norm.weight")
                is_swa.append(int(np.prod(qn)) == hsw if qn is not None else i % 5 != 4)
        n_heads = int(md["gemma4.attention.head_count"])
        n_kv = []
        for i in range(n_layers):
            kd = tensor_dims.get(f"blk.{i}.attn_k.weight")
            hs = hsw if is_swa[i] else hf
            n_kv.append(int(kd[1]) // hs if kd is not None else n_heads)
        shared = int(md.get("gemma4.attention.shared_kv_layers", 0))
        vocab = len(md["tokenizer.ggml.tokens"])
        def f32(key, default):  # FLOAT32 metadata, read as a Kotlin Float
            return float(np.float32(md.get(key, default)))

        return ModelConfig(
            dim=int(md["gemma4.embedding_length"]), n_layers=n_layers, n_heads=n_heads, n_kv_heads=n_kv, ff=ff,
            vocab=vocab, ctx_len=ctx, eps=f32("gemma4.attention.layer_norm_rms_epsilon", 1e-6),
            rope_theta=f32("gemma4.rope.freq_base", 1000000.0),
            rope_theta_swa=f32("gemma4.rope.freq_base_swa", 10000.0),
            head_size_full=hf, head_size_swa=hsw, sliding_window=int(md["gemma4.attention.sliding_window"]),
            logit_softcap=f32("gemma4.final_logit_softcapping", 0.0), is_swa=is_swa,
            n_layer_kv_from_start=n_layers - shared, n_expert=int(md.get("gemma4.expert_count", 0)),
            n_expert_used=int(md.get("gemma4.expert_used_count", 0)),
            expert_ff=int(md.get("gemma4.expert_feed_forward_length", 0)))


def layer_scales(cfg: ModelConfig, f32_tensor) -> np.ndarray:
    """ModelLoader.kt:179-188: blk.N.layer_output_scale.weight[0], else 1."""
    out = np.ones(cfg.n_layers, dtype=np.float32)
    for i in range(cfg.n_layers):
        t = f32_tensor(f"blk.{i}.layer_output_scale.weight")
        if t is not None:
            out[i] = t[0]
    return out


class TensorSource:
    """Uniform view over a GGUF file or an in-memory SynthDecoder:
    metadata, {name: (dims, type)}, raw block bytes and F32 views by name."""

    def __init__(self, metadata: dict, infos: dict, raw_fn):
        self.metadata, self.infos, self._raw = metadata, infos, raw_fn

    @staticmethod
    def from_gguf(f) -> "TensorSource":
        infos = {n: (ti.dims, ti.ggml_type) for n, ti in f.tensors.items()}
        return TensorSource(f.metadata, infos, f.tensor_bytes)

    @staticmethod
    def from_synth(m) -> "TensorSource":
        md = {k: (v.value if hasattr(v, "vtype") else v) for k, v in m.metadata.items()}
        infos = {n: (tuple(d), GGMLType(int(t))) for n, d, t, _ in m.tensors}
        by_name = {n: raw for n, _, _, raw in m.tensors}
        return TensorSource(md, infos, lambda n: by_name[n])

    def dims(self) -> dict:
        return {n: d for n, (d, _) in self.infos.items()}

    def has(self, name: str) -> bool:
        return name in self.infos

    def raw(self, name: str) -> np.ndarray:
        return self._raw(name)

    def type(self, name: str) -> GGMLType:
        return self.infos[name][1]

    def f32(self, name: str):
        if name not in self.infos:
            return None
        if self.infos[name][1] != GGMLType.F32:
            raise ValueError(f"Conversion to {self.infos[name][1].name}")
        return np.asarray(self._raw(name)).view(np.float32)

    def config(self, context_length: int = -1) -> ModelConfig:
        return ModelConfig.from_metadata(self.metadata, self.dims(), context_length)


class DecoderModel:
    """A model resident in HBM for the GPU decoder (g4_model): the mirror of
    ModelLoader.loadWeights (ModelLoader.kt:154-261), every tensor uploaded
    in its GGUF block layout (no dequantization)."""

    def __init__(self, ctx: Context, src: TensorSource, context_length: int = -1):
        from ._lib import ModelConfigStruct

        self.ctx = ctx
        self.cfg = cfg = src.config(context_length)
        self._arrays = [np.array(cfg.n_kv_heads, np.int32), np.array(cfg.ff, np.int32),
                        np.array(cfg.is_swa, np.uint8)]
        mc = ModelConfigStruct(cfg.dim, cfg.n_layers, cfg.n_heads, cfg.vocab, cfg.ctx_len, cfg.head_size_full,
                               cfg.head_size_swa, cfg.sliding_window, cfg.n_layer_kv_from_start, cfg.eps,
                               cfg.rope_theta, cfg.rope_theta_swa, cfg.logit_softcap, cfg.n_expert,
                               cfg.n_expert_used, cfg.expert_ff, *(a.ctypes.data for a in self._arrays))
        h = C.c_void_p()
        check(lib().g4_model_create(ctx.handle, C.byref(mc), C.byref(h)), ctx.handle, "g4_model_create")
        self.handle = h
        try:
            for name, (dims, t) in src.infos.items():
                raw = np.ascontiguousarray(np.asarray(src.raw(name)).view(np.uint8))
                n = 1
                for d in dims:
                    n *= int(d)
                check(lib().g4_model_set_tensor(h, name.encode(), int(t), raw.ctypes.data_as(C.c_void_p), raw.nbytes,
                                                n), ctx.handle, f"g4_model_set_tensor({name})")
            check(lib().g4_model_finalize(h), ctx.handle, "g4_model_finalize")
        except Exception:
            self.free()
            raise

    @staticmethod
    def load(ctx: Context, path, context_length: int = -1) -> "DecoderModel":
        """GemmaModel.load for a GGUF file (weights mmapped, then uploaded)."""
        from .gguf import GGUFFile

        return DecoderModel(ctx, TensorSource.from_gguf(GGUFFile(path)), context_length)

    def free(self) -> None:
        if getattr(self, "handle", None):
            lib().g4_model_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def new_state(self) -> "DecoderState":
        return DecoderState(self)

    def new_batch(self, n_max: int, max_positions: int) -> "DecoderBatch":
        return DecoderBatch(self, n_max, max_positions)


class DecoderState:
    """LlamaState on the device (KV cache, activations, step control)."""

    def __init__(self, model: DecoderModel):
        self.model = model
        h = C.c_void_p()
        check(lib().g4_state_create(model.handle, C.byref(h)), model.ctx.handle, "g4_state_create")
        self.handle = h

    def free(self) -> None:
        if getattr(self, "handle", None):
            lib().g4_state_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return int(lib().g4_state_stream(self.handle) or 0)

    def step(self, token: int, position: int, want_logits: bool = True):
        """Llama.forward: (logits or None, argmax token)."""
        lg = np.empty(self.model.cfg.vocab, np.float32) if want_logits else None
        nt = C.c_int(-1)
        check(lib().g4_decode_step(self.handle, int(token), int(position),
                                   lg.ctypes.data_as(C.c_void_p) if want_logits else None, C.byref(nt)),
              self.model.ctx.handle, "g4_decode_step")
        return lg, int(nt.value)

    def generate(self, tokens, n_generate: int, start_position: int = 0) -> np.ndarray:
        """Greedy Llama.generateTokens: tokens fed from start_position (tokens[0]
        normally <bos>), then n_generate argmax tokens fed back on the GPU."""
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.empty(max(n_generate, 1), np.int32)
        check(lib().g4_decode_greedy(self.handle, t.ctypes.data_as(C.c_void_p), t.size, int(start_position),
                                     int(n_generate), out.ctypes.data_as(C.c_void_p)),
              self.model.ctx.handle, "g4_decode_greedy")
        return out[:n_generate]

    def stage(self, tokens, positions) -> None:
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        check(lib().g4_decode_stage(self.handle, t.ctypes.data_as(C.c_void_p), p.ctypes.data_as(C.c_void_p), t.size),
              self.model.ctx.handle, "g4_decode_stage")

    def enqueue(self, n_steps: int) -> None:
        check(lib().g4_decode_enqueue(self.handle, int(n_steps)), self.model.ctx.handle, "g4_decode_enqueue")

    def read_tokens(self, first_step: int, n: int) -> np.ndarray:
        out = np.empty(n, np.int32)
        check(lib().g4_decode_read_tokens(self.handle, int(first_step), int(n), out.ctypes.data_as(C.c_void_p)),
              self.model.ctx.handle, "g4_decode_read_tokens")
        return out


class DecoderBatch:
    """Many sequences decoded together (g4_batch): one LlamaState's worth of
    KV cache per sequence, every step advances sequences 0..n-1 by one
    position each with the weight reads shared across them."""

    def __init__(self, model: DecoderModel, n_max: int, max_positions: int):
        self.model, self.n_max, self.max_positions = model, int(n_max), int(max_positions)
        h = C.c_void_p()
        check(lib().g4_batch_create(model.handle, self.n_max, self.max_positions, C.byref(h)), model.ctx.handle,
              "g4_batch_create")
        self.handle = h

    def free(self) -> None:
        if getattr(self, "handle", None):
            lib().g4_batch_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return int(lib().g4_batch_stream(self.handle) or 0)

    def expert_parallel(self) -> None:
        """Experts split over the ranks of the context's communicator
        (Context.dist_init); from now on every rank steps together."""
        check(lib().g4_batch_expert_parallel(self.handle), self.model.ctx.handle, "g4_batch_expert_parallel")

    def step(self, tokens, positions, want_logits: bool = True, slots=None):
        """Llama.forward for n rows (row i: tokens[i] at positions[i] of the
        sequence in slot slots[i], default i): (logits [n, vocab] or None,
        argmax [n]).  Rows of one slot at consecutive positions prefill a
        prompt chunk in one step."""
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        if t.shape != p.shape or t.ndim != 1:
            raise ValueError("tokens and positions must be 1-D and of equal length")
        s = None if slots is None else np.ascontiguousarray(slots, np.int32)
        if s is not None and s.shape != t.shape:
            raise ValueError("slots must match tokens")
        n = t.size
        lg = np.empty((n, self.model.cfg.vocab), np.float32) if want_logits else None
        nt = np.empty(n, np.int32)
        check(lib().g4_batch_step(self.handle, t.ctypes.data_as(C.c_void_p), p.ctypes.data_as(C.c_void_p),
                                  None if s is None else s.ctypes.data_as(C.c_void_p), n,
                                  lg.ctypes.data_as(C.c_void_p) if want_logits else None,
                                  nt.ctypes.data_as(C.c_void_p)),
              self.model.ctx.handle, "g4_batch_step")
        return lg, nt
