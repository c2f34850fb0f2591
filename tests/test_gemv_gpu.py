"""GPU parity of the quantized GEMV (g4_matmul / g4_matmul_host / g4_dequant)
against the CPU oracle, through the C ABI.

Tolerance: fp32 outputs within 1e-3 relative L2 of the oracle's restatement
of the reference vectorDot (summation order differs); dequantized weights
bit-exact.
"""
import numpy as np
import pytest

from oracle import oracle
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3
T = {"F32": 0, "BF16": 30, "Q8_0": 8, "Q4_K": 12, "Q6_K": 14}


def dev_tensor(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_gemv(g4, ctx, t, raw, x, rows, cols, off=0):
    import torch

    n = raw.size // g4.GGMLType(t).type_size * g4.GGMLType(t).block_size
    w = g4.FloatTensorFactory.create(ctx, t, raw, n)
    y = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    w.matmul(dev_tensor(x), y, rows, cols, this_offset=off)
    ctx.sync()
    return y.cpu().numpy(), w


def bits_equal(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return bool(np.all((np.isnan(a) & np.isnan(b)) | (a.view(np.uint32) == b.view(np.uint32))))


@pytest.mark.parametrize("name", list(T))
@pytest.mark.parametrize("kind", ["", "_edge"])
def test_dequant_bit_exact_vs_gguf_py(g4, ctx, golden, name, kind):
    raw, vals = golden[f"{name}{kind}_raw"], golden[f"{name}{kind}_vals"]
    w = g4.FloatTensorFactory.create(ctx, T[name], raw, vals.size)
    out = w.dequant(0, vals.size)
    ctx.sync()
    assert bits_equal(out.cpu().numpy(), vals)
    off = 3
    out2 = w.dequant(off, vals.size - off)
    ctx.sync()
    assert bits_equal(out2.cpu().numpy(), vals[off:])


@pytest.mark.parametrize("name", list(T))
def test_gemv_golden_fixtures(g4, ctx, golden, name):
    rows, cols = (int(v) for v in golden[f"gemv_{name}_shape"])
    y, _ = run_gemv(g4, ctx, T[name], golden[f"gemv_{name}_raw"], golden[f"gemv_{name}_x"], rows, cols)
    assert rel_l2(y, golden[f"gemv_{name}_y"]) < TOL


SHAPES = [(1536, 1536), (6144, 1536), (1536, 6144), (2048, 2048), (64, 256), (2816, 2112), (100, 2816)]


@pytest.mark.parametrize("name", ["Q8_0", "Q4_K", "Q6_K", "BF16", "F32"])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_gemv_vs_oracle(g4, ctx, name, rows, cols):
    from gemma4_kt_b200 import synth

    if rows * cols % g4.GGMLType(T[name]).block_size:
        pytest.skip("matrix is not a whole number of blocks")
    raw, x = synth.gemv_case(T[name], rows, cols, seed=1)
    y, _ = run_gemv(g4, ctx, T[name], raw, x, rows, cols)
    ref = oracle.matmul(T[name], raw, x, rows, cols)
    assert rel_l2(y, ref) < TOL


def test_config1_q8_0_2048(g4, ctx):
    """Config 1: 2048x2048 Q8_0, int8 uniform [-127,127], d = |N(0,0.02)|/127, seed 0."""
    from gemma4_kt_b200 import synth

    rng = np.random.default_rng(0)
    raw = synth.q8_0_random_blocks(rng, 2048 * 2048)
    x = rng.standard_normal(2048, dtype=np.float32)
    y, _ = run_gemv(g4, ctx, 8, raw, x, 2048, 2048)
    assert rel_l2(y, oracle.matmul(8, raw, x, 2048, 2048)) < TOL


@pytest.mark.parametrize("name", ["Q4_K", "Q6_K", "Q8_0"])
def test_straddling_rows_expert_down(g4, ctx, name):
    """704-wide rows straddle 256-element super-blocks (the MoE down
    projection, Q4_KFloatTensor.kt:96-103,200-204), at an expert offset."""
    from gemma4_kt_b200 import synth

    n_exp, rows, cols = 3, 2816, 704
    rng = np.random.default_rng(7)
    raw = synth.quantize(T[name], synth.normal(rng, n_exp * rows * cols))
    x = rng.standard_normal(cols, dtype=np.float32)
    for e in range(n_exp):
        off = e * rows * cols
        y, _ = run_gemv(g4, ctx, T[name], raw, x, rows, cols, off)
        assert rel_l2(y, oracle.matmul(T[name], raw, x, rows, cols, this_offset=off)) < TOL


@pytest.mark.parametrize("name", ["Q4_K", "Q8_0", "Q6_K", "BF16"])
def test_generic_path_odd_shapes(g4, ctx, name):
    """Offsets off block boundaries and widths that are not multiples of 16
    take the generic kernel; results must still match vectorDot."""
    from gemma4_kt_b200 import synth

    rng = np.random.default_rng(11)
    n = 256 * 64
    raw = synth.quantize(T[name], synth.normal(rng, n))
    for rows, cols, off in [(7, 300, 5), (40, 100, 0), (3, 1000, 129), (1, 17, 3)]:
        x = rng.standard_normal(cols, dtype=np.float32)
        y, _ = run_gemv(g4, ctx, T[name], raw, x, rows, cols, off)
        assert rel_l2(y, oracle.matmul(T[name], raw, x, rows, cols, this_offset=off)) < TOL


def test_host_buffers_path(g4, ctx):
    from gemma4_kt_b200 import synth

    raw, x = synth.gemv_case(12, 1536, 1536, seed=3)
    w = g4.FloatTensorFactory.create(ctx, 12, raw, 1536 * 1536)
    out = np.zeros(1536, np.float32)
    w.matmul(x, out, 1536, 1536)
    assert rel_l2(out, oracle.matmul(12, raw, x, 1536, 1536)) < TOL


def test_deterministic(g4, ctx):
    from gemma4_kt_b200 import synth

    raw, x = synth.gemv_case(12, 6144, 1536, seed=4)
    a, w = run_gemv(g4, ctx, 12, raw, x, 6144, 1536)
    b, _ = run_gemv(g4, ctx, 12, raw, x, 6144, 1536)
    assert bits_equal(a, b)


@pytest.mark.parametrize("name", ["Q8_0", "Q4_K", "Q6_K", "BF16"])
def test_output_projection_full_size(g4, ctx, name):
    """262144 x 1536 (the tied-embedding logits projection) at full size; the
    oracle checks 2048 sampled rows through row offsets, and the whole output
    is checked against torch fp32 on the GPU-dequantized matrix."""
    import torch
    from gemma4_kt_b200 import synth

    rows, cols = 262144, 1536
    raw, x = synth.gemv_case(T[name], rows, cols, seed=1)
    y, w = run_gemv(g4, ctx, T[name], raw, x, rows, cols)
    rng = np.random.default_rng(1)
    for r0 in rng.choice(rows // 64, 32, replace=False) * 64:
        ref = oracle.matmul(T[name], raw, x, 64, cols, this_offset=int(r0) * cols)
        assert rel_l2(y[r0:r0 + 64], ref) < TOL
    full = w.dequant(0, rows * cols).view(rows, cols)
    yt = (full @ dev_tensor(x)).cpu().numpy()
    assert rel_l2(y, yt) < TOL
    del full
    torch.cuda.empty_cache()


def test_errors(g4, ctx):
    import torch

    raw = np.zeros(34 * 4, np.uint8)
    w = g4.FloatTensorFactory.create(ctx, 8, raw, 128)
    x = torch.zeros(64, device="cuda")
    y = torch.zeros(4, device="cuda")
    with pytest.raises(g4.G4Error):
        w.matmul(x, y, 4, 64)  # 256 elements > 128
    with pytest.raises(g4.UnsupportedOperation):
        g4.FloatTensorFactory.create(ctx, 10, raw, 128)  # Q2_K: no tensor class in FloatTensorFactory.create
    with pytest.raises(ValueError):
        g4.FloatTensorFactory.create(ctx, 8, raw, 100)  # not whole blocks
    w.matmul(x, y, 0, 64)  # dim0 = 0 is a no-op
    ctx.sync()


# ---------------------------------------------------------------- the other formats the reference loads
MORE = {"F16": 1, "Q4_0": 2, "Q4_1": 3, "Q5_1": 7, "Q5_K": 13, "MXFP4": 39}


@pytest.mark.parametrize("name", list(MORE))
@pytest.mark.parametrize("kind", ["", "edge_"])
def test_more_formats_dequant_bit_exact(g4, ctx, golden_more, name, kind):
    """g4_dequant of F16/Q4_0/Q4_1/Q5_1/Q5_K/MXFP4 blocks equals gguf-py's decode bit for bit."""
    raw, vals = golden_more[f"{name}_{kind}raw"], golden_more[f"{name}_{kind}vals"]
    w = g4.FloatTensorFactory.create(ctx, MORE[name], raw, vals.size)
    got = w.dequant(0, vals.size).cpu().numpy()
    assert bits_equal(got, vals)
    if vals.size > 40:
        assert bits_equal(w.dequant(37, vals.size - 37).cpu().numpy(), vals[37:])


@pytest.mark.parametrize("name", list(MORE))
def test_more_formats_gemv_fixture(g4, ctx, golden_more, name):
    rows, cols = (int(v) for v in golden_more[f"gemv_{name}_shape"])
    y, _ = run_gemv(g4, ctx, MORE[name], golden_more[f"gemv_{name}_raw"], golden_more[f"gemv_{name}_x"], rows,
                    cols)
    assert rel_l2(y, golden_more[f"gemv_{name}_y"]) < TOL


@pytest.mark.parametrize("name", list(MORE))
def test_more_formats_gemv_vs_oracle(g4, ctx, name):
    """1024 x 1536 random blocks, whole matrix and a row window at an element offset."""
    from gemma4_kt_b200 import synth

    rng = np.random.default_rng(11)
    rows, cols = 1024, 1536
    raw = synth.random_blocks(MORE[name], rows * cols, rng)
    x = rng.standard_normal(cols).astype(np.float32)
    y, _ = run_gemv(g4, ctx, MORE[name], raw, x, rows, cols)
    assert rel_l2(y, oracle.matmul(MORE[name], raw, x, rows, cols)) < TOL
    off = 100 * cols
    y2, _ = run_gemv(g4, ctx, MORE[name], raw, x, 300, cols, off=off)
    assert rel_l2(y2, oracle.matmul(MORE[name], raw, x, 300, cols, this_offset=off)) < TOL


@pytest.mark.parametrize("name", ["Q8_0", "Q4_K", "Q6_K"])
def test_int16_activation_precision(g4, ctx, name):
    """The quantized formats multiply int16 activations (per 32 columns, power-of-two
    scales).  With an outlier inside a block, an all-zero block and a block of tiny
    values the rounding stays near 6e-5 relative L2 (numpy restatement of the rule);
    the bound leaves a 4x margin and is 4x tighter than the general tolerance."""
    from gemma4_kt_b200 import synth

    rows, cols = 2048, 1536
    raw, x = synth.gemv_case(T[name], rows, cols, seed=6)
    x = x.copy()
    x[5], x[700] = 40.0, -25.0  # outliers set their blocks' scales
    x[64:96] = 0.0  # all-zero block
    x[256:288] *= 1e-20  # tiny values: their own small scale
    y, _ = run_gemv(g4, ctx, T[name], raw, x, rows, cols)
    assert rel_l2(y, oracle.matmul(T[name], raw, x, rows, cols)) < 2.5e-4
