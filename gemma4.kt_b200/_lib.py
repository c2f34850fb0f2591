"""ctypes binding of libg4b200.so (include/g4.h).

The product path is the CUDA library: if it is missing or cannot be loaded
this module raises instead of falling back to anything else.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libg4b200.so"
SYNTH_PATH = PKG / "libg4synth.so"

G4_OK = 0
ERRORS = {
    -1: "G4_E_ARG",
    -2: "G4_E_TYPE",
    -3: "G4_E_CUDA",
    -4: "G4_E_NOMEM",
    -5: "G4_E_DEVICE",
    -6: "G4_E_DIST",
}

# Every symbol include/g4.h declares, with its ctypes signature.
_vp, _i, _i64, _u64, _f = C.c_void_p, C.c_int, C.c_int64, C.c_uint64, C.c_float
SIGNATURES = {
    "g4_init": (_i, [_i, C.POINTER(_vp)]),
    "g4_destroy": (_i, [_vp]),
    "g4_last_error": (C.c_char_p, [_vp]),
    "g4_tensor_upload": (_i, [_vp, _i, _vp, _u64, _u64, C.POINTER(_vp)]),
    "g4_tensor_upload_rows": (_i, [_vp, _i, _vp, _u64, _u64, _u64, C.POINTER(_vp)]),
    "g4_tensor_free": (_i, [_vp]),
    "g4_tensor_device_ptr": (_vp, [_vp]),
    "g4_tensor_nbytes": (_u64, [_vp]),
    "g4_tensor_n_elems": (_u64, [_vp]),
    "g4_tensor_type": (_i, [_vp]),
    "g4_matmul": (_i, [_vp, _vp, _i64, _vp, _vp, _i, _i, _vp]),
    "g4_matmul_host": (_i, [_vp, _vp, _i64, _vp, _vp, _i, _i]),
    "g4_dequant": (_i, [_vp, _vp, _i64, _i64, _vp, _vp]),
    "g4_sync": (_i, [_vp, _vp]),
    "g4_moe_layer": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp, _vp]),
    "g4_moe_layer_host": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp]),
    "g4_moe_topk": (_i, [_vp, _vp, _i, _i, _i, _vp, _vp, _vp]),
    "g4_moe_layer_noalloc": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp, _vp]),
    "g4_moe_layer_ep": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp, _vp]),
    "g4_ffn_moe_block": (_i, [_vp, _vp, _vp, _i, _vp]),
    "g4_ffn_moe_block_host": (_i, [_vp, _vp, _vp, _i]),
    "g4_dist_unique_id": (_i, [_vp]),
    "g4_dist_init": (_i, [_vp, _i, _i, _vp]),
    "g4_dist_init_timeout": (_i, [_vp, _i, _i, _vp, _i]),
    "g4_dist_abort": (_i, [_vp]),
    "g4_dist_rank": (_i, [_vp]),
    "g4_dist_world": (_i, [_vp]),
    "g4_matmul_sharded": (_i, [_vp, _vp, _vp, _vp, _i, _i, _vp]),
    "g4_model_create": (_i, [_vp, _vp, C.POINTER(_vp)]),
    "g4_model_set_tensor": (_i, [_vp, C.c_char_p, _i, _vp, _u64, _u64]),
    "g4_model_finalize": (_i, [_vp]),
    "g4_model_free": (_i, [_vp]),
    "g4_state_create": (_i, [_vp, C.POINTER(_vp)]),
    "g4_state_free": (_i, [_vp]),
    "g4_decode_step": (_i, [_vp, _i, _i, _vp, _vp]),
    "g4_decode_greedy": (_i, [_vp, _vp, _i, _i, _i, _vp]),
    "g4_decode_stage": (_i, [_vp, _vp, _vp, _i]),
    "g4_decode_enqueue": (_i, [_vp, _i]),
    "g4_decode_read_tokens": (_i, [_vp, _i, _i, _vp]),
    "g4_state_stream": (_vp, [_vp]),
    "g4_batch_create": (_i, [_vp, _i, _i, C.POINTER(_vp)]),
    "g4_batch_free": (_i, [_vp]),
    "g4_batch_step": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp]),
    "g4_batch_stream": (_vp, [_vp]),
    "g4_batch_expert_parallel": (_i, [_vp]),
}


class G4Error(RuntimeError):
    pass


class MoeWeightsStruct(C.Structure):
    """g4_moe_weights (include/g4.h)."""

    _fields_ = [
        ("dim", C.c_int),
        ("n_expert", C.c_int),
        ("n_used", C.c_int),
        ("expert_ff", C.c_int),
        ("eps", C.c_float),
        ("gate_inp", C.c_void_p),
        ("gate_inp_scale", C.c_void_p),
        ("gate_up_exps", C.c_void_p),
        ("down_exps", C.c_void_p),
        ("down_exps_scale", C.c_void_p),
        ("pre_ffw_norm_2", C.c_void_p),
        ("post_ffw_norm_2", C.c_void_p),
    ]


class FfnMoeWeightsStruct(C.Structure):
    """g4_ffn_moe_weights (include/g4.h)."""

    _fields_ = [("moe", C.POINTER(MoeWeightsStruct)), ("ff", C.c_int)] + \
               [(n, C.c_void_p) for n in ("ffn_gate", "ffn_up", "ffn_down", "ffn_norm", "post_ffw_norm_1",
                                          "post_ffw_norm")] + [("layer_output_scale", C.c_float)]


class ModelConfigStruct(C.Structure):
    """g4_model_config (include/g4.h)."""

    _fields_ = [(n, C.c_int) for n in ("dim", "n_layers", "n_heads", "vocab", "ctx_len", "head_size_full",
                                       "head_size_swa", "sliding_window", "n_layer_kv_from_start")] + \
               [(n, C.c_float) for n in ("eps", "rope_theta", "rope_theta_swa", "logit_softcap")] + \
               [(n, C.c_int) for n in ("n_expert", "n_expert_used", "expert_ff")] + \
               [("n_kv_heads", C.c_void_p), ("ff", C.c_void_p), ("is_swa", C.c_void_p)]


_lib = None
_synth = None


def lib() -> C.CDLL:
    """Load libg4b200.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise G4Error(f"{LIB_PATH} is missing: run __graft_entry__.build() first")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def synth() -> C.CDLL:
    global _synth
    if _synth is None:
        if not SYNTH_PATH.exists():
            raise G4Error(f"{SYNTH_PATH} is missing: run __graft_entry__.build() first")
        S = C.CDLL(str(SYNTH_PATH))
        S.g4s_quantize.restype = C.c_int
        S.g4s_quantize.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_void_p, C.c_int]
        S.g4s_normal.restype = C.c_int
        S.g4s_normal.argtypes = [C.c_uint64, C.c_uint64, C.c_void_p, C.c_int64, C.c_double, C.c_int]
        S.g4s_nbytes.restype = C.c_int64
        S.g4s_nbytes.argtypes = [C.c_int, C.c_int64]
        _synth = S
    return _synth


def check(rc: int, ctx=None, what: str = "") -> None:
    if rc != G4_OK:
        msg = lib().g4_last_error(ctx)
        msg = msg.decode() if msg else ""
        raise G4Error(f"{what}: {ERRORS.get(rc, rc)}: {msg}")
