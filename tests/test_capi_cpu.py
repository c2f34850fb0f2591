"""C-ABI library and host-side logic, without a GPU: the library loads and
exports every symbol include/g4.h declares; type geometry; the synthetic
quantizers; error reporting when no device is present."""
import ctypes as C
import re

import numpy as np
import pytest

from oracle import oracle
from tests.conftest import ROOT, rel_l2


def declared_symbols():
    text = (ROOT / "include" / "g4.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(g4_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_expected_api():
    syms = declared_symbols()
    for s in ["g4_init", "g4_tensor_upload", "g4_matmul", "g4_matmul_host", "g4_dequant", "g4_moe_layer",
              "g4_moe_topk", "g4_dist_init", "g4_matmul_sharded", "g4_last_error"]:
        assert s in syms


def test_library_exports_every_declared_symbol(g4):
    L = g4.lib()
    for s in declared_symbols():
        assert hasattr(L, s), f"{s} missing from libg4b200.so"
    # and the Python binding covers every one of them
    from gemma4_kt_b200._lib import SIGNATURES

    assert sorted(SIGNATURES) == declared_symbols()


def test_init_without_device_reports_error(g4):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a device is present")
    h = C.c_void_p()
    rc = g4.lib().g4_init(0, C.byref(h))
    assert rc != 0 and not h.value
    assert b"device" in g4.lib().g4_last_error(None)
    with pytest.raises(g4.G4Error):
        g4.Context(0)


def test_ggml_type_geometry(g4):
    T = g4.GGMLType
    assert (T.Q8_0.block_size, T.Q8_0.type_size) == (32, 34)
    assert (T.Q4_K.block_size, T.Q4_K.type_size) == (256, 144)
    assert (T.Q6_K.block_size, T.Q6_K.type_size) == (256, 210)
    assert T.BF16.byte_size_for(10) == 20 and T.F32.byte_size_for(3) == 12
    assert T.Q4_K.byte_size_for(1536 * 262144) == 226_492_416
    with pytest.raises(ValueError):
        T.Q8_0.byte_size_for(33)
    assert [(t.block_size, t.type_size) for t in (T.F16, T.Q4_0, T.Q4_1, T.Q5_1, T.Q5_K, T.MXFP4)] == [
        (1, 2), (32, 18), (32, 20), (32, 24), (256, 176), (32, 17)]  # GGMLType.kt:17-55
    with pytest.raises(g4.UnsupportedOperation):
        T.from_id(10)  # Q2_K: FloatTensorFactory.create has no tensor class for it


def test_q8_0_quantizer_matches_ggml(golden):
    from gemma4_kt_b200 import synth

    got = synth.quantize(8, golden["q8_0_quant_in"])
    assert np.array_equal(got, golden["q8_0_quant_out"])


@pytest.mark.parametrize("t,tol", [(8, 0.01), (12, 0.12), (14, 0.04), (30, 0.005), (0, 0.0)])
def test_quantizers_roundtrip(t, tol):
    from gemma4_kt_b200 import synth

    rng = np.random.default_rng(5)
    w = (rng.standard_normal(256 * 64) * 0.02).astype(np.float32)
    raw = synth.quantize(t, w)
    back = oracle.dequant(t, raw, 0, w.size)
    assert rel_l2(back, w) <= tol + 1e-9


def test_synthetic_config1_blocks():
    from gemma4_kt_b200 import synth

    raw = synth.q8_0_random_blocks(np.random.default_rng(0), 2048 * 2048)
    assert raw.size == 2048 * 2048 // 32 * 34
    blocks = raw.reshape(-1, 34)
    q = blocks[:, 2:].view(np.int8)
    assert q.min() >= -127 and q.max() <= 127
    d = blocks[:, :2].copy().view(np.float16).astype(np.float32)
    assert np.all(d >= 0) and 0.00005 < float(d.mean()) < 0.0002  # E|N(0,0.02)|/127 = 1.26e-4
