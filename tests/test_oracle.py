"""Pins the CPU oracle: block decoders bit-exact against gguf-py's golden
vectors, hand-built edge blocks, and the 16-lane dot products against exact
float64 dots.  CPU only."""
import numpy as np
import pytest

from oracle import oracle
from tests.conftest import rel_l2

TYPE_IDS = {"F32": 0, "BF16": 30, "Q8_0": 8, "Q4_K": 12, "Q6_K": 14}


def same_bits(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    nan = np.isnan(a) & np.isnan(b)
    return bool(np.all(nan | (a.view(np.uint32) == b.view(np.uint32))))


@pytest.mark.parametrize("name", list(TYPE_IDS))
def test_dequant_matches_gguf_py(golden, name):
    raw, vals = golden[f"{name}_raw"], golden[f"{name}_vals"]
    got = oracle.dequant(TYPE_IDS[name], raw, 0, vals.size)
    assert same_bits(got, vals)


@pytest.mark.parametrize("name", list(TYPE_IDS))
def test_dequant_edge_blocks_match_gguf_py(golden, name):
    raw, vals = golden[f"{name}_edge_raw"], golden[f"{name}_edge_vals"]
    got = oracle.dequant(TYPE_IDS[name], raw, 0, vals.size)
    assert same_bits(got, vals)


@pytest.mark.parametrize("name", list(TYPE_IDS))
def test_dequant_with_offset(golden, name):
    raw, vals = golden[f"{name}_raw"], golden[f"{name}_vals"]
    off = 37
    got = oracle.dequant(TYPE_IDS[name], raw, off, vals.size - off)
    assert same_bits(got, vals[off:])


def test_f16_conversion_exact():
    # every binary16 bit pattern: compare with numpy's IEEE conversion
    h = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([oracle.f16_to_f32(int(v)) for v in h[::97]], np.float32)
    assert same_bits(got, ref[::97])
    for v in [0x0001, 0x03FF, 0x0400, 0x7BFF, 0x7C00, 0xFC00, 0x8001, 0x8000]:
        assert same_bits([oracle.f16_to_f32(v)], [np.array([v], np.uint16).view(np.float16)[0]])


@pytest.mark.parametrize("name", list(TYPE_IDS))
def test_gemv_fixture(golden, name):
    rows, cols = golden[f"gemv_{name}_shape"]
    raw, x, y = golden[f"gemv_{name}_raw"], golden[f"gemv_{name}_x"], golden[f"gemv_{name}_y"]
    got = oracle.matmul(TYPE_IDS[name], raw, x, int(rows), int(cols))
    assert rel_l2(got, y) < 1e-5
    got_s = oracle.matmul(TYPE_IDS[name], raw, x, int(rows), int(cols), vector=False)
    assert rel_l2(got_s, y) < 1e-5


@pytest.mark.parametrize("name,bs", [("Q8_0", 32), ("Q4_K", 256), ("Q6_K", 256), ("BF16", 1), ("F32", 1)])
@pytest.mark.parametrize("off,size", [(0, 512), (5, 500), (3, 20), (256, 256), (31, 257)])
def test_vector_dot_head_tail(golden, name, bs, off, size):
    """vectorDot splits unaligned heads/tails off to scalarDot (e.g.
    Q8_0FloatTensor.kt:50-54,137-139); the result must equal the exact dot."""
    raw, vals = golden[f"{name}_raw"], golden[f"{name}_vals"]
    if off + size > vals.size:
        pytest.skip("fixture too small")
    rng = np.random.default_rng(off * 1000 + size)
    x = rng.standard_normal(size).astype(np.float32)
    exact = float(np.dot(vals[off:off + size].astype(np.float64), x.astype(np.float64)))
    got = oracle.vector_dot(TYPE_IDS[name], raw, off, x, size)
    scale = float(np.sum(np.abs(vals[off:off + size].astype(np.float64) * x)))
    assert abs(got - exact) <= 1e-5 * scale + 1e-30


def test_softmax_topk_semantics():
    # ties go to the lowest index; probabilities are not renormalised (Llama.kt:280-293)
    logits = np.array([0.5, 2.0, 2.0, -1.0, 2.0, 0.1], np.float32)
    p = oracle.softmax(logits)
    assert abs(float(np.sum(p.astype(np.float64))) - 1.0) < 1e-6
    idx, val = oracle.topk(p, 4)
    assert list(idx) == [1, 2, 4, 0]
    assert same_bits(val, p[[1, 2, 4, 0]])


def test_gelu_and_rmsnorm():
    for v in [-3.0, -0.5, 0.0, 0.7, 2.5]:
        xd = float(np.float32(v))
        ref = 0.5 * xd * (1 + np.tanh(np.sqrt(2 / np.pi) * (xd + 0.044715 * xd ** 3)))
        assert same_bits([oracle.gelu(v)], [np.float32(ref)])


# ---------------------------------------------------------------- the other formats the reference loads
MORE_IDS = {"F16": 1, "Q4_0": 2, "Q4_1": 3, "Q5_1": 7, "Q5_K": 13, "MXFP4": 39}


@pytest.mark.parametrize("name", list(MORE_IDS))
@pytest.mark.parametrize("kind", ["", "edge_"])
def test_more_formats_dequant_match_gguf_py(golden_more, name, kind):
    """Q4_0/Q4_1/Q5_1/Q5_K/F16/MXFP4FloatTensor.get restated in the oracle, bit for bit."""
    raw, vals = golden_more[f"{name}_{kind}raw"], golden_more[f"{name}_{kind}vals"]
    got = oracle.dequant(MORE_IDS[name], raw, 0, vals.size)
    assert same_bits(got, vals)


@pytest.mark.parametrize("name", list(MORE_IDS))
def test_more_formats_gemv_fixture(golden_more, name):
    rows, cols = golden_more[f"gemv_{name}_shape"]
    raw, x, y = golden_more[f"gemv_{name}_raw"], golden_more[f"gemv_{name}_x"], golden_more[f"gemv_{name}_y"]
    got = oracle.matmul(MORE_IDS[name], raw, x, int(rows), int(cols))
    assert rel_l2(got, y) < 1e-5


def test_topk_margin():
    """The routing-margin probe the MoE decoder tests use to reject fixtures
    with router ties: the gap between the k-th and (k+1)-th probability."""
    p = np.array([0.1, 0.5, 0.2, 0.15, 0.05], np.float32)
    oracle.reset_topk_margin()
    assert oracle.topk_margin() == float("inf")
    oracle.lib().o_note_topk_margin(p.ctypes.data, p.size, 2)  # 0.2 - 0.15
    assert abs(oracle.topk_margin() - (np.float64(np.float32(0.2)) - np.float64(np.float32(0.15)))) < 1e-12
    oracle.lib().o_note_topk_margin(p.ctypes.data, p.size, 1)  # 0.5 - 0.2: larger, minimum kept
    assert abs(oracle.topk_margin() - 0.05) < 1e-7
    oracle.lib().o_note_topk_margin(p.ctypes.data, p.size, 4)  # 0.1 - 0.05
    assert abs(oracle.topk_margin() - 0.05) < 1e-7
    q = np.array([0.3, 0.3, 0.4], np.float32)  # an exact tie at the boundary
    oracle.lib().o_note_topk_margin(q.ctypes.data, q.size, 2)
    assert oracle.topk_margin() == 0.0
