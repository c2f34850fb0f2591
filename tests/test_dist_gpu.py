"""g4_matmul_sharded on 2 GPUs: each rank uploads its output-row slice
(g4_tensor_upload_rows), computes it and all-gathers y over NCCL; every rank's
y is compared with the unsharded CPU oracle (the checker) within the GEMV
tolerance.  Needs two GPUs in one box; skipped otherwise."""
import os
import socket

import numpy as np
import pytest

import __graft_entry__

g4 = __graft_entry__.load_package()

pytestmark = pytest.mark.gpu

TOL = 1e-3  # relative L2, fp32 outputs


def _gpus() -> int:
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, cases, q):
    import datetime

    import torch
    import torch.distributed as dist

    from gemma4_kt_b200 import synth

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    # gloo only carries the 128-byte NCCL id; the data path is the library's own NCCL communicator
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        torch.cuda.set_device(rank)
        ctx = g4.Context(rank)
        obj = [g4.Context.dist_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ctx.dist_init(rank, world, obj[0])
        res = []
        for t, rows, cols, seed in cases:
            raw, x = synth.gemv_case(t, rows, cols, seed=seed)
            begin, per = g4.row_shard(rows, world, rank)
            w = g4.FloatTensorFactory.create_rows(ctx, t, raw, cols, begin, per)
            xd = torch.from_numpy(x).cuda()
            yd = torch.full((rows,), float("nan"), device="cuda")
            w.matmul_sharded(xd, yd, rows, cols)
            torch.cuda.synchronize()
            res.append(yd.cpu().numpy())
            w.free()
        q.put((rank, res))
        dist.barrier()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_matmul_sharded_two_gpus():
    import multiprocessing as mp

    from gemma4_kt_b200 import synth
    from oracle import oracle

    T = g4.GGMLType
    cases = [(T.Q4_K, 4096, 1536, 1), (T.Q8_0, 2048, 2048, 0), (T.Q6_K, 1536, 1536, 1), (T.BF16, 6144, 1536, 1)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, cases, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for i, (t, rows, cols, seed) in enumerate(cases):
        raw, x = synth.gemv_case(t, rows, cols, seed=seed)
        ref = oracle.matmul(int(t), raw, x, rows, cols)
        for r in range(2):
            y = got[r][i]
            err = np.linalg.norm(y - ref) / np.linalg.norm(ref)
            assert err < TOL, (t.name, r, err)


def _ep_rank_main(rank, world, port, q):
    import datetime

    import torch
    import torch.distributed as dist

    from gemma4_kt_b200 import synth

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        torch.cuda.set_device(rank)
        ctx = g4.Context(rank)
        obj = [g4.Context.dist_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ctx.dist_init(rank, world, obj[0])
        d = synth.MoeLayerData(seed=2, n_expert=32)
        full = g4.MoeLayer.upload(ctx, d)
        ep = g4.MoeLayer.upload_shard(ctx, d, rank, world)
        res = []
        for t_per_rank in ((48, 48), (40, 0)):  # the second call leaves rank 1 without tokens
            T = t_per_rank[rank]
            x_all = d.tokens(sum(t_per_rank))
            x = torch.from_numpy(x_all[sum(t_per_rank[:rank]):sum(t_per_rank[:rank]) + T].copy()).cuda()
            out = torch.empty((T, d.dim), device="cuda")
            idx = torch.empty((T, d.n_used), dtype=torch.int32, device="cuda")
            ep.forward_ep(x, out, T, topk_idx=idx)
            torch.cuda.synchronize()
            ref = torch.empty((T, d.dim), device="cuda")
            ridx = torch.empty((T, d.n_used), dtype=torch.int32, device="cuda")
            if T:
                full.forward(x, ref, T, topk_idx=ridx)
            torch.cuda.synchronize()
            res.append((out.cpu().numpy(), ref.cpu().numpy(), idx.cpu().numpy(), ridx.cpu().numpy()))
        q.put((rank, res))
        dist.barrier()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_moe_expert_parallel_two_gpus():
    """g4_moe_layer_ep over 2 GPUs (16 of 32 experts each) equals the
    single-GPU layer on the same tokens (same routing, outputs within 1e-3)."""
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(2):
        for out, ref, idx, ridx in got[r]:
            assert np.array_equal(idx, ridx)
            for t in range(out.shape[0]):
                err = np.linalg.norm(out[t] - ref[t]) / np.linalg.norm(ref[t])
                assert err < TOL, (r, t, err)


def _lonely_rank_main(q):
    """Rank 0 of a 2-rank communicator whose peer never joins."""
    import time

    import torch

    from gemma4_kt_b200 import synth

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(0)
    ctx = g4.Context(0)
    uid = g4.Context.dist_unique_id()
    t0 = time.monotonic()
    msg = ""
    try:
        ctx.dist_init(0, 2, uid, timeout_ms=3000)
        joined = True
    except g4.G4Error as e:
        joined, msg = False, str(e)
    waited = time.monotonic() - t0
    # the context is single-GPU again and still computes
    raw, x = synth.gemv_case(g4.GGMLType.Q8_0, 256, 2048, seed=0)
    w = g4.FloatTensorFactory.create(ctx, g4.GGMLType.Q8_0, raw, 256 * 2048)
    y = np.zeros(256, dtype=np.float32)
    w.matmul(x, y, 256, 2048)
    q.put((joined, msg, waited, y, raw, x))
    w.free()
    ctx.close()


def test_dist_init_gives_up_when_a_peer_never_joins():
    """A rank whose peer never joins gets G4_E_DIST after the timeout (the
    communicator is created non-blocking and aborted on expiry) instead of
    hanging; the context keeps working on one GPU.  The failure is made on
    the host (no second rank is started); runs in a child process that is
    killed if it ever hangs."""
    if _gpus() < 1:
        pytest.skip("no CUDA device")
    import multiprocessing as mp

    from oracle import oracle

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_rank_main, args=(q,))
    p.start()
    try:
        joined, msg, waited, y, raw, x = q.get(timeout=180)
    finally:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert p.exitcode == 0
    assert not joined
    assert "timed out" in msg and "G4_E_DIST" in msg, msg
    assert 2.5 < waited < 60, waited
    ref = oracle.matmul(int(g4.GGMLType.Q8_0), raw, x, 256, 2048)
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < TOL


def _batch_ep_rank_main(rank, world, port, q):
    import datetime

    import torch
    import torch.distributed as dist

    from gemma4_kt_b200 import synth
    from tests.test_decode_gpu import SPECS

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        torch.cuda.set_device(rank)
        ctx = g4.Context(rank)
        obj = [g4.Context.dist_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ctx.dist_init(rank, world, obj[0])
        m = synth.SynthDecoder(SPECS["moe"], seed=39)
        model = g4.DecoderModel(ctx, g4.TensorSource.from_synth(m))
        n_seq, steps = 3, 16
        ep = model.new_batch(n_seq, steps)
        ep.expert_parallel()
        local = model.new_batch(n_seq, steps)  # the same sequences, every expert on this GPU
        prompts = np.stack([np.concatenate([[2], m.prompt(steps, seed=500 + 10 * rank + i)]) for i in range(n_seq)])
        res = []
        for p in range(steps):
            tok = prompts[:, p].astype(np.int32)
            pos = np.full(n_seq, p, np.int32)
            lg_ep, nt_ep = ep.step(tok, pos)
            lg_lo, nt_lo = local.step(tok, pos)
            res.append((lg_ep, nt_ep, lg_lo, nt_lo))
        q.put((rank, res))
        dist.barrier()
        ep.free()
        local.free()
        model.free()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_batch_expert_parallel_two_gpus():
    """Batched decode with data-parallel sequences and expert-parallel MoE
    layers (g4_batch_expert_parallel, 8 of 16 experts per GPU): every rank's
    logits and argmax equal those of a batch that runs all experts on the
    rank's own GPU for the same sequences (teacher-forced prompt tokens)."""
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_batch_ep_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(2):
        for step, (lg_ep, nt_ep, lg_lo, nt_lo) in enumerate(got[r]):
            for i in range(lg_ep.shape[0]):
                err = np.linalg.norm(lg_ep[i] - lg_lo[i]) / np.linalg.norm(lg_lo[i])
                assert err < 1e-5, (r, step, i, err)
            assert np.array_equal(nt_ep, nt_lo), (r, step)
