"""ctypes binding of the CPU oracle (oracle/libg4oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, as the checker of the CUDA path.  Nothing in the
product package imports it.  See g4_oracle.h for what it restates and how it
is pinned.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libg4oracle.so"
GEN = HERE / "libg4gen.so"
GEN_SRC = HERE.parent / "gemma4.kt_b200" / "csrc" / "g4_synth.c"

_lib = None
_gen = None


def build() -> Path:
    src = [HERE / "g4_oracle.c", HERE / "g4_oracle.h", HERE / "Makefile"]
    stale = not LIB.exists() or any(s.stat().st_mtime > LIB.stat().st_mtime for s in src)
    stale = stale or (GEN_SRC.exists() and (not GEN.exists() or GEN_SRC.stat().st_mtime > GEN.stat().st_mtime))
    if stale:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def quantize(ggml_type: int, w: np.ndarray, threads: int | None = None) -> np.ndarray:
    """fp32 weights -> GGUF block bytes with the benchmark-input generator
    (the same source as the package's synth.quantize, built under oracle/)."""
    global _gen
    if _gen is None:
        if not GEN.exists():
            build()
        _gen = C.CDLL(str(GEN))
        _gen.g4s_quantize.restype = C.c_int
        _gen.g4s_quantize.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_void_p, C.c_int]
        _gen.g4s_nbytes.restype = C.c_int64
        _gen.g4s_nbytes.argtypes = [C.c_int, C.c_int64]
    w = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    nb = _gen.g4s_nbytes(int(ggml_type), w.size)
    if nb < 0:
        raise ValueError(f"cannot quantize {w.size} elements as type {ggml_type}")
    out = np.empty(nb, dtype=np.uint8)
    if _gen.g4s_quantize(int(ggml_type), w.ctypes.data_as(C.c_void_p), w.size, out.ctypes.data_as(C.c_void_p),
                         threads or os.cpu_count() or 1):
        raise ValueError(f"cannot quantize {w.size} elements as type {ggml_type}")
    return out


class MoeW(C.Structure):
    _fields_ = [
        ("dim", C.c_int), ("n_expert", C.c_int), ("n_used", C.c_int), ("expert_ff", C.c_int),
        ("eps", C.c_float), ("gate_up_type", C.c_int), ("down_type", C.c_int),
        ("gate_inp", C.c_void_p), ("gate_inp_scale", C.c_void_p), ("gate_up_exps", C.c_void_p),
        ("down_exps", C.c_void_p), ("down_exps_scale", C.c_void_p), ("pre_ffw_norm_2", C.c_void_p),
        ("post_ffw_norm_2", C.c_void_p),
    ]


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = C.CDLL(str(LIB))
        vp, i, i64, f = C.c_void_p, C.c_int, C.c_int64, C.c_float
        sig = {
            "o_f16_to_f32": (f, [C.c_uint16]),
            "o_get": (f, [i, vp, i64]),
            "o_dequant": (None, [i, vp, i64, i64, vp]),
            "o_scalar_dot": (f, [i, vp, i64, vp, i]),
            "o_vector_dot": (f, [i, vp, i64, vp, i]),
            "o_matmul": (None, [i, vp, i64, vp, vp, i, i, i, i]),
            "o_gelu": (f, [f]),
            "o_rmsnorm": (None, [vp, vp, vp, i, f]),
            "o_softmax": (None, [vp, i]),
            "o_topk": (None, [vp, i, i, vp, vp]),
            "o_moe_token": (None, [C.POINTER(MoeW), vp, vp, vp, vp, vp, i]),
            "o_moe_router_logits": (None, [C.POINTER(MoeW), vp, vp]),
            "o_reset_topk_margin": (None, []),
            "o_note_topk_margin": (None, [vp, i, i]),
            "o_topk_margin": (C.c_double, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray) -> C.c_void_p:
    return a.ctypes.data_as(C.c_void_p)


def dequant(ggml_type: int, raw: np.ndarray, offset: int, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().o_dequant(int(ggml_type), _p(raw), offset, n, _p(out))
    return out


def matmul(ggml_type: int, raw: np.ndarray, x: np.ndarray, dim0: int, dim1: int, this_offset: int = 0,
           threads: int | None = None, vector: bool = True) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(dim0, dtype=np.float32)
    lib().o_matmul(int(ggml_type), _p(raw), this_offset, _p(x), _p(out), dim0, dim1,
                   threads or os.cpu_count() or 1, 1 if vector else 0)
    return out


def vector_dot(ggml_type: int, raw: np.ndarray, this_offset: int, x: np.ndarray, size: int) -> float:
    x = np.ascontiguousarray(x, dtype=np.float32)
    return float(lib().o_vector_dot(int(ggml_type), _p(raw), this_offset, _p(x), size))


def scalar_dot(ggml_type: int, raw: np.ndarray, this_offset: int, x: np.ndarray, size: int) -> float:
    x = np.ascontiguousarray(x, dtype=np.float32)
    return float(lib().o_scalar_dot(int(ggml_type), _p(raw), this_offset, _p(x), size))


def f16_to_f32(h: int) -> float:
    return float(lib().o_f16_to_f32(h))


def gelu(x: float) -> float:
    return float(lib().o_gelu(x))


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """Llama.rmsnorm (Llama.kt:27-37)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    lib().o_rmsnorm(_p(out), _p(x), _p(w), x.size, float(eps))
    return out


def ffn_moe_block(x: np.ndarray, moe: "MoeOracle", shared, eps: float) -> np.ndarray:
    """The FFN half of a MoE layer for one token, as Llama.forward runs it
    (Llama.kt:226-353) followed by the layer output scale (Llama.kt:393-397);
    returns the new residual stream.  shared: ffn_gate / ffn_up / ffn_down
    blocks of shared.gate_type, ffn_norm, post_ffw_norm_1, post_ffw_norm,
    layer_output_scale."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    dim, ff, t = x.size, shared.ff, int(shared.gate_type)
    h = rmsnorm(x, shared.ffn_norm, eps)                                   # :232
    hb = matmul(t, shared.ffn_gate, h, ff, dim)                            # :233
    hb2 = matmul(t, shared.ffn_up, h, ff, dim)                             # :234
    hb = np.array([gelu(float(v)) for v in hb], dtype=np.float32) * hb2    # :235-236
    xb = matmul(t, shared.ffn_down, hb, dim, ff)                           # :237
    xb = rmsnorm(xb, shared.post_ffw_norm_1, eps)                          # :238-243
    moe_out, _, _, _ = moe.token(x)                                        # :247-346 (state.x)
    xb = (xb + moe_out).astype(np.float32)                                 # :349
    xb = rmsnorm(xb, shared.post_ffw_norm, eps)                            # :352
    out = (x + xb).astype(np.float32)                                      # :353
    if shared.layer_output_scale != 1.0:
        out = (out * np.float32(shared.layer_output_scale)).astype(np.float32)  # :393-397
    return out


def softmax(x: np.ndarray) -> np.ndarray:
    y = np.array(x, dtype=np.float32, copy=True)
    lib().o_softmax(_p(y), y.size)
    return y


def topk(probs: np.ndarray, k: int):
    p = np.array(probs, dtype=np.float32, copy=True)
    idx = np.empty(k, dtype=np.int32)
    val = np.empty(k, dtype=np.float32)
    lib().o_topk(_p(p), p.size, k, _p(idx), _p(val))
    return idx, val


class MoeOracle:
    """Holds a MoeW view over host arrays of one MoE layer."""

    def __init__(self, d, gate_up_type: int, down_type: int, post_norm: bool = True):
        self._keep = [d.gate_inp, d.gate_inp_scale, d.gate_up, d.down, d.down_scale, d.pre_norm, d.post_norm]
        self.w = MoeW(d.dim, d.n_expert, d.n_used, d.ff, d.eps, int(gate_up_type), int(down_type),
                      _p(d.gate_inp).value, _p(d.gate_inp_scale).value, _p(d.gate_up).value, _p(d.down).value,
                      _p(d.down_scale).value, _p(d.pre_norm).value, _p(d.post_norm).value if post_norm else None)
        self.dim, self.k, self.e = d.dim, d.n_used, d.n_expert

    def token(self, x: np.ndarray, threads: int | None = None):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(self.dim, dtype=np.float32)
        idx = np.empty(self.k, dtype=np.int32)
        prob = np.empty(self.k, dtype=np.float32)
        logits = np.empty(self.e, dtype=np.float32)
        lib().o_moe_token(C.byref(self.w), _p(x), _p(out), _p(idx), _p(prob), _p(logits),
                          threads or os.cpu_count() or 1)
        return out, idx, prob, logits

    def router_logits(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(self.e, dtype=np.float32)
        lib().o_moe_router_logits(C.byref(self.w), _p(x), _p(out))
        return out


# ---------------------------------------------------------------------- whole model
class OTensor(C.Structure):
    _fields_ = [("type", C.c_int), ("data", C.c_void_p)]


class OLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("attn_norm", "attn_q_norm", "attn_k_norm", "post_attention_norm",
                                          "ffn_norm", "post_ffw_norm")] + \
               [(n, OTensor) for n in ("wq", "wk", "wv", "wo", "w1", "w2", "w3")] + \
               [(n, C.c_void_p) for n in ("post_ffw_norm_1", "pre_ffw_norm_2", "post_ffw_norm_2", "gate_inp_scale",
                                          "down_exps_scale")] + \
               [(n, OTensor) for n in ("gate_inp", "gate_up_exps", "down_exps")]


class OModel(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("dim", "n_layers", "n_heads", "vocab", "ctx_len", "head_size_full",
                                       "head_size_swa", "sliding_window", "n_layer_kv_from_start")] + \
               [(n, C.c_float) for n in ("eps", "rope_theta", "rope_theta_swa", "logit_softcap")] + \
               [(n, C.c_int) for n in ("n_expert", "n_expert_used", "expert_ff")] + \
               [(n, C.c_void_p) for n in ("n_kv_heads", "ff", "is_swa", "layer_scale", "rope_freqs")] + \
               [("tok_embd", OTensor), ("output", OTensor), ("output_norm", C.c_void_p),
                ("layers", C.POINTER(OLayer))]


def _model_lib():
    L = lib()
    if not getattr(L, "_model_sigs", False):
        L.o_state_new.restype = C.c_void_p
        L.o_state_new.argtypes = [C.POINTER(OModel)]
        L.o_state_free.restype = None
        L.o_state_free.argtypes = [C.c_void_p]
        L.o_forward.restype = C.POINTER(C.c_float)
        L.o_forward.argtypes = [C.POINTER(OModel), C.c_void_p, C.c_int, C.c_int, C.c_int]
        L.o_argmax.restype = C.c_int
        L.o_argmax.argtypes = [C.c_void_p, C.c_int]
        L.o_set_vector_api.restype = None
        L.o_set_vector_api.argtypes = [C.c_int]
        L.o_rope_table.restype = None
        L.o_rope_table.argtypes = [C.c_int, C.c_int, C.c_double, C.c_void_p, C.c_void_p, C.c_void_p]
        L._model_sigs = True
    return L


def reset_topk_margin() -> None:
    """Start a new routing-margin window (see topk_margin)."""
    lib().o_reset_topk_margin()


def topk_margin() -> float:
    """Smallest gap between the k-th and (k+1)-th router probability over the
    oracle's MoE tokens since reset_topk_margin (inf if none ran).  A gap at
    the level of fp32 rounding means the expert choice there is a tie that
    any implementation within the 1e-3 tolerance may break either way."""
    return float(lib().o_topk_margin())


def set_vector_api(on: bool) -> None:
    """Whole-model forward: Vector-API dot products (True, default) or the
    reference's scalarDot mode (llama.VectorBitSize=0)."""
    _model_lib().o_set_vector_api(1 if on else 0)


class ModelOracle:
    """Llama.forward restated on the CPU over a model's raw tensors
    (src: gemma4_kt_b200.model.TensorSource).  One state (KV cache) per
    instance; call step() with positions 0, 1, 2, ... like generateTokens."""

    def __init__(self, src, context_length: int = -1, threads: int | None = None):
        from gemma4_kt_b200.model import layer_scales  # host mirror of the loader's scale lookup

        cfg = src.config(context_length)
        self.cfg = cfg
        self.threads = threads or os.cpu_count() or 1
        keep = self._keep = []

        def ptr(a):
            if a is None:
                return None
            a = np.ascontiguousarray(a)
            keep.append(a)
            return a.ctypes.data

        def ten(name):
            if not src.has(name):
                return OTensor(0, None)
            return OTensor(int(src.type(name)), ptr(np.asarray(src.raw(name)).view(np.uint8)))

        def f32(name):
            v = src.f32(name)
            return ptr(v) if v is not None else None

        L = cfg.n_layers
        layers = (OLayer * L)()
        for i in range(L):
            p = f"blk.{i}."
            ly = layers[i]
            ly.attn_norm, ly.attn_q_norm = f32(p + "attn_norm.weight"), f32(p + "attn_q_norm.weight")
            ly.attn_k_norm = f32(p + "attn_k_norm.weight")
            ly.post_attention_norm, ly.ffn_norm = f32(p + "post_attention_norm.weight"), f32(p + "ffn_norm.weight")
            ly.post_ffw_norm = f32(p + "post_ffw_norm.weight")
            ly.wq, ly.wk, ly.wv = ten(p + "attn_q.weight"), ten(p + "attn_k.weight"), ten(p + "attn_v.weight")
            ly.wo = ten(p + "attn_output.weight")
            ly.w1, ly.w2, ly.w3 = ten(p + "ffn_gate.weight"), ten(p + "ffn_down.weight"), ten(p + "ffn_up.weight")
            if cfg.n_expert:
                ly.post_ffw_norm_1 = f32(p + "post_ffw_norm_1.weight")
                ly.pre_ffw_norm_2 = f32(p + "pre_ffw_norm_2.weight")
                ly.post_ffw_norm_2 = f32(p + "post_ffw_norm_2.weight")
                ly.gate_inp_scale = f32(p + "ffn_gate_inp.scale")
                ly.down_exps_scale = f32(p + "ffn_down_exps.scale")
                ly.gate_inp = ten(p + "ffn_gate_inp.weight")
                ly.gate_up_exps, ly.down_exps = ten(p + "ffn_gate_up_exps.weight"), ten(p + "ffn_down_exps.weight")
        keep.append(layers)
        m = OModel()
        m.dim, m.n_layers, m.n_heads, m.vocab, m.ctx_len = cfg.dim, L, cfg.n_heads, cfg.vocab, cfg.ctx_len
        m.head_size_full, m.head_size_swa, m.sliding_window = cfg.head_size_full, cfg.head_size_swa, cfg.sliding_window
        m.n_layer_kv_from_start = cfg.n_layer_kv_from_start
        m.eps, m.rope_theta, m.rope_theta_swa = cfg.eps, cfg.rope_theta, cfg.rope_theta_swa
        m.logit_softcap = cfg.logit_softcap
        m.n_expert, m.n_expert_used, m.expert_ff = cfg.n_expert, cfg.n_expert_used, cfg.expert_ff
        m.n_kv_heads = ptr(np.array(cfg.n_kv_heads, np.int32))
        m.ff = ptr(np.array(cfg.ff, np.int32))
        m.is_swa = ptr(np.array(cfg.is_swa, np.uint8))
        m.layer_scale = ptr(layer_scales(cfg, src.f32))
        m.rope_freqs = f32("rope_freqs.weight")
        m.tok_embd = ten("token_embd.weight")
        m.output = ten("output.weight")
        m.output_norm = f32("output_norm.weight")
        m.layers = layers
        self.m = m
        self.state = _model_lib().o_state_new(C.byref(m))

    def close(self):
        if self.state:
            _model_lib().o_state_free(self.state)
            self.state = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def step(self, token: int, position: int) -> np.ndarray:
        """Llama.forward: logits (a copy) for `token` at `position`."""
        p = _model_lib().o_forward(C.byref(self.m), self.state, int(token), int(position), self.threads)
        return np.ctypeslib.as_array(p, shape=(self.cfg.vocab,)).copy()

    def greedy(self, prompt, n_generate: int, bos: int = 2, collect_logits: bool = False):
        """Llama.generateTokens with the ARGMAX sampler, stop tokens ignored:
        BOS at position 0, prompt[i] at position i + 1, then n_generate greedy
        tokens.  Returns the generated ids (and every position's logits)."""
        token, out, logits = bos, [], []
        pos = 0
        for t in list(prompt):
            lg = self.step(token, pos)
            if collect_logits:
                logits.append(lg)
            token = int(t)
            pos += 1
        for _ in range(n_generate):
            lg = self.step(token, pos)
            if collect_logits:
                logits.append(lg)
            token = int(np.argmax(lg))  # first maximum, as FloatTensor.argmax
            out.append(token)
            pos += 1
        return (np.array(out, np.int32), logits) if collect_logits else np.array(out, np.int32)
