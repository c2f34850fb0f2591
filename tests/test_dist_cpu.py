"""Row-sharded GEMV across ranks, host side, on CPU with gloo (world size 2).

The GPU path (g4_matmul_sharded) computes each rank's output rows
[row_shard(rows, world, rank)] and all-gathers them in rank order with NCCL.
Here every rank computes its slice with the CPU oracle (the checker) from the
row range that row_shard assigns and the same all-gather runs over gloo; the
assembled y must equal the unsharded oracle result bit for bit, because a
row's dot product does not depend on which rank computes it.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import __graft_entry__

g4 = __graft_entry__.load_package()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, cases, q):
    from gemma4_kt_b200 import synth
    from oracle import oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = []
        for t, rows, cols, seed in cases:
            raw, x = synth.gemv_case(t, rows, cols, seed=seed)
            begin, per = g4.row_shard(rows, world, rank)
            off = begin * cols
            mine = oracle.matmul(int(t), raw, x, per, cols, this_offset=off)
            full = torch.empty(rows, dtype=torch.float32)
            dist.all_gather_into_tensor(full, torch.from_numpy(np.ascontiguousarray(mine, dtype=np.float32)))
            out.append(full.numpy().copy())
        if rank == 0:
            q.put(out)
    finally:
        dist.destroy_process_group()


def test_row_shard_ranges():
    assert g4.row_shard(262144, 8, 3) == (98304, 32768)
    assert g4.row_shard(1536, 1, 0) == (0, 1536)
    spans = [g4.row_shard(6144, 4, r) for r in range(4)]
    assert [b for b, _ in spans] == [0, 1536, 3072, 4608] and {n for _, n in spans} == {1536}
    with pytest.raises(ValueError):
        g4.row_shard(1537, 2, 0)
    with pytest.raises(ValueError):
        g4.row_shard(1536, 2, 2)


def test_sharded_gemv_gloo_world2():
    from gemma4_kt_b200 import synth
    from oracle import oracle

    T = g4.GGMLType
    cases = [(T.Q4_K, 512, 1536, 1), (T.Q8_0, 256, 2048, 0), (T.Q6_K, 128, 1536, 1), (T.BF16, 64, 1536, 1)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, cases, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for (t, rows, cols, seed), y in zip(cases, got):
        raw, x = synth.gemv_case(t, rows, cols, seed=seed)
        ref = oracle.matmul(int(t), raw, x, rows, cols)
        np.testing.assert_array_equal(y, ref)
