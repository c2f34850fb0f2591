"""Expert-parallel MoE, host side, on CPU with gloo (world size 2).

Restates what g4_moe_layer_ep does across ranks, with the CPU oracle as the
arithmetic: every rank routes its own tokens, sends each routed slot's moe_in
row to the rank that owns the slot's expert (experts split by
MoeLayer.expert_shard), that rank evaluates its expert on the row
(gate_up matmul at the expert's offset in its own weight slice, gelu*up,
down matmul), the products return to the token's rank and are combined in
selection order with the post-norm.  The result must equal the unsharded
oracle layer (Llama.kt:247-346) for every token.
"""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import __graft_entry__

g4 = __graft_entry__.load_package()

T_PER_RANK = 3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rmsnorm(x, w, eps):
    # Llama.kt:27-37: sequential float sum of squares, 1/sqrt in double
    ss = np.float32(0)
    for v in x.astype(np.float32):
        ss = np.float32(ss + np.float32(v * v))
    m = np.float32(np.float32(ss / np.float32(x.size)) + np.float32(eps))
    s = np.float32(1.0 / np.sqrt(np.float64(m)))
    return (w.astype(np.float32) * (s * x.astype(np.float32))).astype(np.float32)


def _rank_main(rank, world, port, q):
    from gemma4_kt_b200 import synth
    from oracle import oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        d = synth.MoeLayerData(seed=2, n_expert=16)
        e0, ne = g4.MoeLayer.expert_shard(d.n_expert, world, rank)
        t = g4.GGMLType(int(d.expert_type))
        gu_n, dn_n = 2 * d.ff * d.dim, d.dim * d.ff
        gu_b, dn_b = t.byte_size_for(gu_n), t.byte_size_for(dn_n)
        my_gu = np.ascontiguousarray(d.gate_up.view(np.uint8)[e0 * gu_b:(e0 + ne) * gu_b])
        my_dn = np.ascontiguousarray(d.down.view(np.uint8)[e0 * dn_b:(e0 + ne) * dn_b])
        orc = oracle.MoeOracle(d, int(t), int(t))
        x = d.tokens(world * T_PER_RANK)[rank * T_PER_RANK:(rank + 1) * T_PER_RANK]
        # route this rank's tokens
        slots = []  # (token, k, expert, prob, moe_in row)
        for i in range(T_PER_RANK):
            _, idx, prob, _ = orc.token(x[i], threads=1)
            mi = _rmsnorm(x[i], d.pre_norm, d.eps)
            for k in range(d.n_used):
                slots.append((i, k, int(idx[k]), np.float32(prob[k]), mi))
        # dispatch: every rank sees every slot and evaluates the ones it owns
        gathered = [None] * world
        dist.all_gather_object(gathered, [(rank, i, k, e, row) for (i, k, e, _, row) in slots])
        products = {}
        for src in gathered:
            for (r0, i, k, e, row) in src:
                if e0 <= e < e0 + ne:
                    le = e - e0
                    h = oracle.matmul(int(t), my_gu, row, 2 * d.ff, d.dim, this_offset=le * gu_n, threads=1)
                    g = np.array([oracle.gelu(float(h[j])) for j in range(d.ff)], np.float32) * h[d.ff:]
                    products[(r0, i, k)] = oracle.matmul(int(t), my_dn, g.astype(np.float32), d.dim, d.ff,
                                                         this_offset=le * dn_n, threads=1)
        back = [None] * world
        dist.all_gather_object(back, products)
        mine = {}
        for part in back:
            mine.update({key[1:]: v for key, v in part.items() if key[0] == rank})
        # combine in selection order (saxpyInPlace: product rounded, then added), then the post-norm
        outs = []
        for i in range(T_PER_RANK):
            acc = np.zeros(d.dim, np.float32)
            for (ti, k, e, p, _) in slots:
                if ti == i:
                    fw = np.float32(p * np.float32(d.down_scale[e]))
                    acc = (acc + (fw * mine[(i, k)]).astype(np.float32)).astype(np.float32)
            outs.append(_rmsnorm(acc, d.post_norm, d.eps))
        ref = [orc.token(x[i], threads=1)[0] for i in range(T_PER_RANK)]
        q.put((rank, outs, ref))
    finally:
        dist.destroy_process_group()


def test_expert_shard_ranges():
    assert g4.MoeLayer.expert_shard(128, 8, 3) == (48, 16)
    assert g4.MoeLayer.expert_shard(128, 1, 0) == (0, 128)
    with pytest.raises(ValueError):
        g4.MoeLayer.expert_shard(128, 3, 0)


def test_expert_parallel_dispatch_combine_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, outs, ref in res:
        for o, r in zip(outs, ref):
            err = np.linalg.norm(o.astype(np.float64) - r) / np.linalg.norm(r)
            assert err < 1e-5, (rank, err)
