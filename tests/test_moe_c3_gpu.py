"""The MoE layer at the benchmark geometry (hidden 2816, 128 experts, top-8,
expert ff 704, Q4_K experts, F32 router, seed 2) at every batch size of the
benchmark, T = 1, 16, 256 and 4096, through g4_moe_layer (Llama.kt:247-346).

T <= 256: every token against the CPU oracle.  T = 4096 (tensor-core path):
every token against the fp32 CUDA-core kernels (G4_MOE_TC=0, themselves
pinned to the oracle at T <= 256) and 256 tokens against the oracle.  The
per-token relative L2 of the tensor-core path is printed as max / p99 (run
with -s to see it) and must stay within the 1e-3 bar.
"""
import numpy as np
import pytest

from oracle import oracle
from tests.conftest import rel_l2
from tests.test_moe_gpu import near_tie

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.fixture(scope="module")
def c3(g4, ctx):
    from gemma4_kt_b200 import synth

    d = synth.MoeLayerData(seed=2)
    layer = g4.MoeLayer.upload(ctx, d)
    orc = oracle.MoeOracle(d, int(d.expert_type), int(d.expert_type))
    return d, layer, orc


def _run(ctx, layer, d, x):
    import torch

    n = x.shape[0]
    out = torch.empty((n, d.dim), dtype=torch.float32, device="cuda")
    idx = torch.empty((n, d.n_used), dtype=torch.int32, device="cuda")
    prob = torch.empty((n, d.n_used), dtype=torch.float32, device="cuda")
    layer.forward(torch.from_numpy(x).cuda(), out, n, topk_idx=idx, topk_prob=prob)
    ctx.sync()
    return out.cpu().numpy(), idx.cpu().numpy(), prob.cpu().numpy()


def _vs_oracle(orc, x, out, idx, prob, tokens):
    errs, flips = [], 0
    for t in tokens:
        o, oi, op, ol = orc.token(x[t])
        if not np.array_equal(idx[t], oi):
            assert near_tie(ol, idx[t], oi), f"token {t}: {idx[t]} vs {oi}"
            flips += 1
            continue
        assert rel_l2(prob[t], op) < 1e-5, t
        errs.append(rel_l2(out[t], o))
    errs = np.array(errs)
    assert flips <= max(1, len(tokens) // 50), flips
    return errs


@pytest.mark.parametrize("T", [1, 16, 256])
def test_c3_every_token_vs_oracle(g4, ctx, c3, T):
    d, layer, orc = c3
    x = d.tokens(T)
    out, idx, prob = _run(ctx, layer, d, x)
    errs = _vs_oracle(orc, x, out, idx, prob, list(range(T)))
    print(f"\nC3 T={T}: per-token rel L2 vs oracle max {errs.max():.2e} p99 {np.percentile(errs, 99):.2e}")
    assert errs.max() < TOL


def test_c3_4096_tensor_cores(g4, ctx, c3, monkeypatch):
    d, layer, orc = c3
    T = 4096
    x = d.tokens(T)
    monkeypatch.setenv("G4_MOE_TC", "0")
    ref, ridx, rprob = _run(ctx, layer, d, x)
    monkeypatch.delenv("G4_MOE_TC")
    out, idx, prob = _run(ctx, layer, d, x)
    # the routing is computed by the same front kernels on both paths
    assert np.array_equal(idx, ridx)
    np.testing.assert_array_equal(prob, rprob)
    errs = np.array([rel_l2(out[t], ref[t]) for t in range(T)])
    print(f"\nC3 T=4096 tensor-core vs fp32 CUDA-core: per-token rel L2 max {errs.max():.2e} "
          f"p99 {np.percentile(errs, 99):.2e} mean {errs.mean():.2e}")
    assert errs.max() < TOL
    sample = list(range(0, T, 16))  # 256 tokens
    e_tc = _vs_oracle(orc, x, out, idx, prob, sample)
    e_cc = _vs_oracle(orc, x, ref, ridx, rprob, sample)
    print(f"C3 T=4096 vs oracle (256 tokens): tensor-core max {e_tc.max():.2e} p99 {np.percentile(e_tc, 99):.2e}; "
          f"CUDA-core max {e_cc.max():.2e}")
    assert e_tc.max() < TOL and e_cc.max() < TOL
