"""GPU tests of g4_moe_layer_noalloc, the MoE entry point that allocates no
device memory.  It exists for hosts that cannot let the library call
cudaMalloc once they are running: a host that hands all free HBM to its own
pool at start-up (a later cudaMalloc would fail), or a decode loop that must
not stall on the device-wide synchronisation a cudaMalloc/cudaFree can cause.

Each case calls the entry point through the C ABI twice in a row, with
different tokens, and checks every token against the CPU oracle (the
reference's MoE arithmetic) and against g4_moe_layer: same top-k selection,
outputs within the 1e-3 relative L2 tolerance of the other MoE tests.  The
cases reach every kernel path of the entry point: the decode kernels (one
token, and two with G4_MOE_DEC=1), the CUDA-core rows kernels (5 and 16
tokens) and the generic expert kernel (BF16 experts).  Further tests check
that a call made after the first allocates nothing (free device memory is
unchanged), that the fixed array comes into being when the context is created
even under lazy module loading, and that a batch larger than the array is
refused with an error.  Kept in a file of its own, collected last.
"""
import ctypes as C
import os

import numpy as np
import pytest

from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3
NOALLOC_BYTES = 8 << 20  # G4_MOE_NOALLOC_SCRATCH_BYTES in include/g4.h


def _call(g4, ctx, layer, x, n, out, idx, prob):
    import torch

    return g4.lib().g4_moe_layer_noalloc(ctx.handle, C.byref(layer.w), C.c_void_p(x.data_ptr()),
                                         C.c_void_p(out.data_ptr()), n, C.c_void_p(idx.data_ptr()),
                                         C.c_void_p(prob.data_ptr()),
                                         C.c_void_p(torch.cuda.current_stream().cuda_stream))


def _buffers(n, d, device="cuda"):
    import torch

    out = torch.full((n, d.dim), float("nan"), dtype=torch.float32, device=device)
    idx = torch.full((n, d.n_used), -1, dtype=torch.int32, device=device)
    prob = torch.zeros((n, d.n_used), dtype=torch.float32, device=device)
    return out, idx, prob


_LAYERS = {}


def _layer(g4, ctx, expert_type):
    """One uploaded 32-expert layer per expert format (host data, device layer, oracle)."""
    from gemma4_kt_b200 import synth
    from oracle import oracle

    key = int(expert_type)
    if key not in _LAYERS:
        d = synth.MoeLayerData(seed=3, n_expert=32, expert_type=expert_type)
        _LAYERS[key] = (d, g4.MoeLayer.upload(ctx, d), oracle.MoeOracle(d, key, key))
    return _LAYERS[key]


CASES = [
    # (expert format, token counts of the two calls, G4_MOE_DEC)
    ("Q4_K", (1, 1), None),    # decode kernels
    ("Q4_K", (2, 2), "1"),     # decode kernels up to two tokens
    ("Q4_K", (16, 5), None),   # CUDA-core rows kernels
    ("BF16", (3, 4), None),    # generic expert kernel
]


@pytest.mark.parametrize("fmt,ns,dec", CASES, ids=[f"{c[0]}-{c[1][0]}x{c[1][1]}-dec{c[2]}" for c in CASES])
def test_noalloc_matches_oracle_and_moe_layer_twice(g4, ctx, fmt, ns, dec, monkeypatch):
    import torch

    if dec is not None:
        monkeypatch.setenv("G4_MOE_DEC", dec)  # read by the library at every call
    d, layer, orc = _layer(g4, ctx, getattr(g4.GGMLType, fmt))
    for call, n in enumerate(ns):
        x_h = d.tokens(n, seed=10 + call + 7 * n)
        x = torch.from_numpy(x_h).cuda()
        ref_out, ref_idx, ref_prob = _buffers(n, d)
        layer.forward(x, ref_out, n, topk_idx=ref_idx, topk_prob=ref_prob)
        out, idx, prob = _buffers(n, d)
        rc = _call(g4, ctx, layer, x, n, out, idx, prob)
        assert rc == 0, ctx.last_error()
        ctx.sync()
        assert np.array_equal(idx.cpu().numpy(), ref_idx.cpu().numpy())
        assert rel_l2(prob.cpu().numpy(), ref_prob.cpu().numpy()) < 1e-6
        o, i_, p_ = out.cpu().numpy(), idx.cpu().numpy(), prob.cpu().numpy()
        r = ref_out.cpu().numpy()
        for t in range(n):
            assert rel_l2(o[t], r[t]) < TOL
            oo, oi, op, _ = orc.token(x_h[t])
            assert np.array_equal(i_[t], oi), (t, i_[t], oi)
            assert rel_l2(p_[t], op) < 1e-5
            assert rel_l2(o[t], oo) < TOL, (t, rel_l2(o[t], oo))


def test_noalloc_allocates_nothing(g4, ctx, monkeypatch):
    """After a first call of each kernel path (which loads the kernels' code
    under lazy module loading), further calls leave free device memory
    unchanged: the entry point allocates nothing."""
    import torch

    bufs = []
    for fmt, ns, dec in CASES:
        d, layer, _ = _layer(g4, ctx, getattr(g4.GGMLType, fmt))
        for n in ns:
            x = torch.from_numpy(d.tokens(n, seed=99 + n)).cuda()
            bufs.append((layer, x, n, dec, *_buffers(n, d)))
    torch.cuda.synchronize()

    def run_all():
        for layer, x, n, dec, out, idx, prob in bufs:
            if dec is None:
                monkeypatch.delenv("G4_MOE_DEC", raising=False)
            else:
                monkeypatch.setenv("G4_MOE_DEC", dec)
            assert _call(g4, ctx, layer, x, n, out, idx, prob) == 0, ctx.last_error()
        ctx.sync()

    run_all()  # first calls: kernel code loads
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        run_all()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)


def _lazy_child(q):
    os.environ["CUDA_MODULE_LOADING"] = "LAZY"
    import torch

    import __graft_entry__

    g4 = __graft_entry__.load_package()
    torch.cuda.init()
    torch.zeros(1, device="cuda")  # the CUDA context exists before the library is used
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    ctx = g4.Context(0)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    ctx.close()
    q.put(free0 - free1)


def test_noalloc_array_exists_after_context_creation():
    """Under lazy module loading, creating the context already reserves the
    fixed array on the device (free memory drops by at least its size), so a
    host can reserve the remaining HBM for itself right after g4_init.  Runs
    in a fresh child process, killed if it ever hangs."""
    import multiprocessing as mp

    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    p = mpc.Process(target=_lazy_child, args=(q,))
    p.start()
    try:
        drop = q.get(timeout=300)
    finally:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert p.exitcode == 0
    assert drop >= NOALLOC_BYTES, drop


def test_noalloc_rejects_batches_beyond_the_fixed_array(g4, ctx):
    import torch

    d, layer, _ = _layer(g4, ctx, g4.GGMLType.Q4_K)
    # about 135 KB of work memory per token at this geometry: 100 tokens do not fit
    n = 100
    x = torch.zeros((n, d.dim), dtype=torch.float32, device="cuda")
    out, idx, prob = _buffers(n, d)
    rc = _call(g4, ctx, layer, x, n, out, idx, prob)
    assert rc == -1  # G4_E_ARG
    assert "work memory" in ctx.last_error()
    ctx.sync()
