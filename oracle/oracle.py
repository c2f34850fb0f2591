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

_lib = None


def build() -> Path:
    src = [HERE / "g4_oracle.c", HERE / "g4_oracle.h", HERE / "Makefile"]
    if not LIB.exists() or any(s.stat().st_mtime > LIB.stat().st_mtime for s in src):
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


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
