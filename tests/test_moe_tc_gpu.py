"""GPU parity of the tensor-core grouped expert path (g4_moe_tc.cu) of
g4_moe_layer against the CPU oracle (Llama.kt:247-346), through the C ABI.

G4_MOE_TC=1 forces the tensor-core path whenever the layout allows it, =0
forbids it; the library reads the variable on every call.  The path rounds
weights and activations to fp16 before the fp32-accumulating products, so
outputs are compared within the 1e-3 relative L2 bar like every fp32 output.
"""
import numpy as np
import pytest

from oracle import oracle
from tests.conftest import rel_l2
from tests.test_moe_gpu import check_layer

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.fixture(scope="module")
def moe32():
    from gemma4_kt_b200 import synth

    return synth.MoeLayerData(seed=2, n_expert=32)


@pytest.mark.parametrize("n_tokens", [1, 3, 16, 64])
def test_tc_forced_vs_oracle(g4, ctx, moe32, n_tokens, monkeypatch):
    """Tiny batches leave most experts empty and give ragged token tiles."""
    monkeypatch.setenv("G4_MOE_TC", "1")
    check_layer(g4, ctx, moe32, n_tokens)


def test_tc_without_post_norm(g4, ctx, moe32, monkeypatch):
    monkeypatch.setenv("G4_MOE_TC", "1")
    check_layer(g4, ctx, moe32, 8, post_norm=False)


def _forward(g4, ctx, layer, x, n):
    import torch

    out = torch.empty((n, x.shape[1]), dtype=torch.float32, device="cuda")
    layer.forward(torch.from_numpy(x).cuda(), out, n)
    ctx.sync()
    return out.cpu().numpy()


@pytest.mark.parametrize("n_tokens", [64, 700])
def test_tc_matches_cuda_core_path(g4, ctx, moe32, n_tokens, monkeypatch):
    """Same layer, same tokens: tensor-core path vs the fp32 CUDA-core kernels
    (700 tokens: about 175 slots per expert, tiles split at the 128/256 caps)."""
    layer = g4.MoeLayer.upload(ctx, moe32)
    x = moe32.tokens(n_tokens)
    monkeypatch.setenv("G4_MOE_TC", "0")
    ref = _forward(g4, ctx, layer, x, n_tokens)
    monkeypatch.setenv("G4_MOE_TC", "1")
    got = _forward(g4, ctx, layer, x, n_tokens)
    errs = np.array([rel_l2(got[t], ref[t]) for t in range(n_tokens)])
    assert errs.max() < TOL, errs.max()
    # a second call on the same buffers gives the same result (no state leaks)
    again = _forward(g4, ctx, layer, x, n_tokens)
    np.testing.assert_array_equal(again, got)


def test_tc_full_geometry_wide_batch(g4, ctx):
    """The benchmark layer (128 experts, top-8, 2816/704, Q4_K) at 4096 tokens:
    about 256 slots per expert; sampled tokens vs the oracle."""
    from gemma4_kt_b200 import synth

    d = synth.MoeLayerData(seed=2)
    check_layer(g4, ctx, d, 4096, check_tokens=list(range(0, 4096, 257)))


def test_tc_full_geometry_256(g4, ctx):
    from gemma4_kt_b200 import synth

    d = synth.MoeLayerData(seed=2)
    check_layer(g4, ctx, d, 256, check_tokens=list(range(0, 256, 23)))
