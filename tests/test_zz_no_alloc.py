"""GPU test of g4_moe_layer_noalloc, the MoE entry point that allocates no
device memory (for hosts that cannot let the library call cudaMalloc once
they are running: all free HBM handed to the host's own pool, or no device-wide
synchronisation allowed inside a decode step).

It calls the entry point through the C ABI twice in a row, with different
tokens, and checks each output against g4_moe_layer's: same top-k selection,
outputs within the 1e-3 relative L2 tolerance of the other MoE tests.  It also
checks that a batch larger than the fixed work array is refused with an error.
Kept in a file of its own, collected last.
"""
import ctypes as C

import numpy as np
import pytest

from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3
NOALLOC_BYTES = 8 << 20  # G4_MOE_NOALLOC_SCRATCH_BYTES in include/g4.h


def _call(g4, ctx, layer, x, n, out, idx, prob):
    import torch

    rc = g4.lib().g4_moe_layer_noalloc(ctx.handle, C.byref(layer.w), C.c_void_p(x.data_ptr()),
                                       C.c_void_p(out.data_ptr()), n, C.c_void_p(idx.data_ptr()),
                                       C.c_void_p(prob.data_ptr()),
                                       C.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc


def test_noalloc_matches_moe_layer_twice(g4, ctx):
    import torch
    from gemma4_kt_b200 import synth

    d = synth.MoeLayerData(seed=3, n_expert=32)
    layer = g4.MoeLayer.upload(ctx, d)
    for call, n in enumerate((16, 5)):
        x = torch.from_numpy(d.tokens(n, seed=10 + call)).cuda()
        ref_out = torch.empty((n, d.dim), dtype=torch.float32, device="cuda")
        ref_idx = torch.empty((n, d.n_used), dtype=torch.int32, device="cuda")
        ref_prob = torch.empty((n, d.n_used), dtype=torch.float32, device="cuda")
        layer.forward(x, ref_out, n, topk_idx=ref_idx, topk_prob=ref_prob)
        out = torch.full((n, d.dim), float("nan"), dtype=torch.float32, device="cuda")
        idx = torch.full((n, d.n_used), -1, dtype=torch.int32, device="cuda")
        prob = torch.zeros((n, d.n_used), dtype=torch.float32, device="cuda")
        rc = _call(g4, ctx, layer, x, n, out, idx, prob)
        assert rc == 0, ctx.last_error()
        ctx.sync()
        assert np.array_equal(idx.cpu().numpy(), ref_idx.cpu().numpy())
        assert rel_l2(prob.cpu().numpy(), ref_prob.cpu().numpy()) < 1e-6
        for t in range(n):
            assert rel_l2(out[t].cpu().numpy(), ref_out[t].cpu().numpy()) < TOL


def test_noalloc_rejects_batches_beyond_the_fixed_array(g4, ctx):
    import torch
    from gemma4_kt_b200 import synth

    d = synth.MoeLayerData(seed=3, n_expert=32)
    layer = g4.MoeLayer.upload(ctx, d)
    # about 135 KB of work memory per token at this geometry: 100 tokens do not fit
    n = 100
    x = torch.zeros((n, d.dim), dtype=torch.float32, device="cuda")
    out = torch.zeros((n, d.dim), dtype=torch.float32, device="cuda")
    idx = torch.zeros((n, d.n_used), dtype=torch.int32, device="cuda")
    prob = torch.zeros((n, d.n_used), dtype=torch.float32, device="cuda")
    rc = _call(g4, ctx, layer, x, n, out, idx, prob)
    assert rc == -1  # G4_E_ARG
    assert "work memory" in ctx.last_error()
    ctx.sync()
