"""GPU parity of g4_ffn_moe_block, the whole FFN half of a MoE layer in one
call (Llama.kt:226-353 and the layer output scale, Llama.kt:393-397): the
shared MLP (ffn_norm, gate / up / down, post_ffw_norm_1), the expert half
(g4_moe_layer) and the merge (post_ffw_norm, x += xb), against the oracle's
composition of the reference's steps.  Device and host-buffer entry points,
one and several tokens; the change of the residual stream must be within
1e-3 relative L2 of the oracle's for every token."""
import numpy as np
import pytest

from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3
_BLOCKS = {}


def _block(g4, ctx, gate_type):
    from gemma4_kt_b200 import synth
    from oracle import oracle

    key = int(gate_type)
    if key not in _BLOCKS:
        d = synth.MoeLayerData(seed=4, n_expert=32)
        sh = synth.SharedMlpData(d.dim, 2112, seed=4, gate_type=gate_type)
        moe = g4.MoeLayer.upload(ctx, d)
        _BLOCKS[key] = (d, sh, g4.FfnMoeBlock.upload(ctx, moe, sh), oracle.MoeOracle(d, int(d.expert_type),
                                                                                   int(d.expert_type)))
    return _BLOCKS[key]


@pytest.mark.parametrize("gate_type", ["Q8_0", "Q4_K"])
@pytest.mark.parametrize("n", [1, 3])
def test_ffn_moe_block_vs_oracle(g4, ctx, gate_type, n):
    import torch

    from oracle import oracle

    d, sh, blk, orc = _block(g4, ctx, getattr(g4.GGMLType, gate_type))
    x0 = d.tokens(n, seed=40 + n)
    ref = np.stack([oracle.ffn_moe_block(x0[t], orc, sh, d.eps) for t in range(n)])
    xd = torch.from_numpy(x0.copy()).cuda()
    blk.forward(xd, n)
    ctx.sync()
    got = xd.cpu().numpy()
    xh = x0.copy()
    blk.forward(xh, n)
    for t in range(n):
        e = rel_l2(got[t] - x0[t], ref[t] - x0[t])
        assert e < TOL, (t, e)
        assert rel_l2(xh[t] - x0[t], ref[t] - x0[t]) < TOL
        assert rel_l2(got[t], ref[t]) < TOL


def test_ffn_moe_block_rejects_bad_weights(g4, ctx):
    import ctypes as C

    d, sh, blk, _ = _block(g4, ctx, g4.GGMLType.Q8_0)
    w = g4._lib.FfnMoeWeightsStruct.from_buffer_copy(blk.w)
    w.ff = sh.ff + 1  # the shared tensors no longer match
    x = np.zeros((1, d.dim), np.float32)
    rc = g4.lib().g4_ffn_moe_block_host(ctx.handle, C.byref(w), x.ctypes.data_as(C.c_void_p), 1)
    assert rc == -1 and "shared MLP" in ctx.last_error()
