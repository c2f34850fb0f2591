"""Host-side mirror of gemma4.kt's MoE block, backed by libg4b200.

The reference inlines the block in Llama.forward (Llama.kt:226-353) and keeps
its weights in LlamaWeights (LlamaWeights.kt:50-65: ffnGateInp,
ffnGateInpScale, ffnGateUpExps, ffnDownExps, ffnDownExpsScale, preFfwNorm2,
ffnPostNorm2).  `MoeLayer.forward` runs the expert half (Llama.kt:247-346)
for a batch of tokens in one call of g4_moe_layer; `FfnMoeBlock.forward` the
whole FFN half of the layer (shared MLP, experts, merge: Llama.kt:226-353) in
one call of g4_ffn_moe_block.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import FfnMoeWeightsStruct, MoeWeightsStruct, check, lib
from .floattensor import Context, CudaFloatTensor, FloatTensorFactory, GGMLType, _is_torch, _stream_ptr


class MoeLayer:
    def __init__(self, ctx: Context, *, dim: int, n_expert: int, n_used: int, expert_ff: int, eps: float,
                 gate_inp: CudaFloatTensor, gate_inp_scale: CudaFloatTensor, gate_up_exps: CudaFloatTensor,
                 down_exps: CudaFloatTensor, down_exps_scale: CudaFloatTensor, pre_ffw_norm_2: CudaFloatTensor,
                 post_ffw_norm_2: CudaFloatTensor | None):
        self.ctx = ctx
        self.dim, self.n_expert, self.n_used, self.expert_ff = dim, n_expert, n_used, expert_ff
        self._tensors = [gate_inp, gate_inp_scale, gate_up_exps, down_exps, down_exps_scale, pre_ffw_norm_2,
                         post_ffw_norm_2]
        self.w = MoeWeightsStruct(dim, n_expert, n_used, expert_ff, eps, gate_inp.handle, gate_inp_scale.handle,
                                  gate_up_exps.handle, down_exps.handle, down_exps_scale.handle,
                                  pre_ffw_norm_2.handle, post_ffw_norm_2.handle if post_ffw_norm_2 else None)

    @staticmethod
    def upload(ctx: Context, data, post_norm: bool = True) -> "MoeLayer":
        """Upload a synth.MoeLayerData (or anything with the same fields)."""
        f32 = GGMLType.F32
        up = FloatTensorFactory.create
        return MoeLayer(
            ctx, dim=data.dim, n_expert=data.n_expert, n_used=data.n_used, expert_ff=data.ff, eps=data.eps,
            gate_inp=up(ctx, f32, data.gate_inp, data.n_expert * data.dim),
            gate_inp_scale=up(ctx, f32, data.gate_inp_scale, data.dim),
            gate_up_exps=up(ctx, data.expert_type, data.gate_up, data.n_expert * 2 * data.ff * data.dim),
            down_exps=up(ctx, data.expert_type, data.down, data.n_expert * data.dim * data.ff),
            down_exps_scale=up(ctx, f32, data.down_scale, data.n_expert),
            pre_ffw_norm_2=up(ctx, f32, data.pre_norm, data.dim),
            post_ffw_norm_2=up(ctx, f32, data.post_norm, data.dim) if post_norm else None,
        )

    @staticmethod
    def expert_shard(n_expert: int, world: int, rank: int) -> tuple[int, int]:
        """Experts [begin, begin + count) that `rank` of `world` holds in the
        expert-parallel layer (contiguous, equal shares)."""
        if world < 1 or not 0 <= rank < world:
            raise ValueError(f"bad rank {rank} of world {world}")
        if n_expert % world:
            raise ValueError(f"{n_expert} experts do not split evenly over {world} GPUs")
        per = n_expert // world
        return rank * per, per

    @staticmethod
    def upload_shard(ctx: Context, data, rank: int, world: int, post_norm: bool = True) -> "MoeLayer":
        """Upload the expert-parallel share of rank `rank`: its experts' slices
        of ffn_gate_up_exps / ffn_down_exps (whole experts are contiguous in the
        GGUF block stream), everything else replicated."""
        e0, ne = MoeLayer.expert_shard(data.n_expert, world, rank)
        t = GGMLType(int(data.expert_type))
        gu_n, dn_n = 2 * data.ff * data.dim, data.dim * data.ff  # elements per expert
        gu_b, dn_b = t.byte_size_for(gu_n), t.byte_size_for(dn_n)
        raw_gu = np.frombuffer(data.gate_up, np.uint8) if not isinstance(data.gate_up, np.ndarray) else data.gate_up.view(np.uint8).reshape(-1)
        raw_dn = np.frombuffer(data.down, np.uint8) if not isinstance(data.down, np.ndarray) else data.down.view(np.uint8).reshape(-1)
        f32 = GGMLType.F32
        up = FloatTensorFactory.create
        return MoeLayer(
            ctx, dim=data.dim, n_expert=data.n_expert, n_used=data.n_used, expert_ff=data.ff, eps=data.eps,
            gate_inp=up(ctx, f32, data.gate_inp, data.n_expert * data.dim),
            gate_inp_scale=up(ctx, f32, data.gate_inp_scale, data.dim),
            gate_up_exps=up(ctx, t, raw_gu[e0 * gu_b:(e0 + ne) * gu_b], ne * gu_n),
            down_exps=up(ctx, t, raw_dn[e0 * dn_b:(e0 + ne) * dn_b], ne * dn_n),
            down_exps_scale=up(ctx, f32, data.down_scale, data.n_expert),
            pre_ffw_norm_2=up(ctx, f32, data.pre_norm, data.dim),
            post_ffw_norm_2=up(ctx, f32, data.post_norm, data.dim) if post_norm else None,
        )

    def forward_ep(self, x, out, n_tokens: int, topk_idx=None, topk_prob=None, stream=None) -> None:
        """Expert-parallel forward (g4_moe_layer_ep) of this rank's n_tokens
        tokens; every rank of the communicator must call it at the same time.
        x, out: torch CUDA tensors [n_tokens, dim] (may be empty)."""
        p = lambda t: C.c_void_p(t.data_ptr()) if t is not None and t.numel() else None
        rc = lib().g4_moe_layer_ep(self.ctx.handle, C.byref(self.w), p(x), p(out), n_tokens, p(topk_idx),
                                   p(topk_prob), C.c_void_p(_stream_ptr(stream)))
        check(rc, self.ctx.handle, "g4_moe_layer_ep")

    def forward(self, x, out, n_tokens: int, topk_idx=None, topk_prob=None, stream=None) -> None:
        """x, out: [n_tokens, dim]; topk_idx (int32) / topk_prob: [n_tokens, n_used] or None.
        torch CUDA tensors run asynchronously on `stream`; numpy arrays synchronously."""
        if _is_torch(x):
            p = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None
            rc = lib().g4_moe_layer(self.ctx.handle, C.byref(self.w), p(x), p(out), n_tokens, p(topk_idx),
                                    p(topk_prob), C.c_void_p(_stream_ptr(stream)))
            check(rc, self.ctx.handle, "g4_moe_layer")
        else:
            xa = np.ascontiguousarray(x, dtype=np.float32)
            p = lambda a: a.ctypes.data_as(C.c_void_p) if a is not None else None
            rc = lib().g4_moe_layer_host(self.ctx.handle, C.byref(self.w), p(xa), p(out), n_tokens, p(topk_idx),
                                         p(topk_prob))
            check(rc, self.ctx.handle, "g4_moe_layer_host")


class FfnMoeBlock:
    """The FFN half of a MoE layer (Llama.kt:226-353): the shared MLP
    (ffn_norm, ffn_gate / ffn_up / ffn_down, post_ffw_norm_1), the expert half
    (a MoeLayer) and the merge (post_ffw_norm), plus the layer output scale."""

    def __init__(self, moe: MoeLayer, ff: int, ffn_gate: CudaFloatTensor, ffn_up: CudaFloatTensor,
                 ffn_down: CudaFloatTensor, ffn_norm: CudaFloatTensor, post_ffw_norm_1: CudaFloatTensor,
                 post_ffw_norm: CudaFloatTensor, layer_output_scale: float = 1.0):
        self.moe, self.ctx, self.ff = moe, moe.ctx, ff
        self._tensors = [ffn_gate, ffn_up, ffn_down, ffn_norm, post_ffw_norm_1, post_ffw_norm]
        self.w = FfnMoeWeightsStruct(C.pointer(moe.w), ff, ffn_gate.handle, ffn_up.handle, ffn_down.handle,
                                     ffn_norm.handle, post_ffw_norm_1.handle, post_ffw_norm.handle,
                                     float(layer_output_scale))

    @staticmethod
    def upload(ctx: Context, moe: MoeLayer, shared) -> "FfnMoeBlock":
        """shared: an object with ff, gate_type, ffn_gate / ffn_up / ffn_down (block bytes), ffn_norm,
        post_ffw_norm_1, post_ffw_norm (F32) and layer_output_scale (synth.SharedMlpData)."""
        up = FloatTensorFactory.create
        dim, ff, t, f32 = moe.dim, shared.ff, GGMLType(int(shared.gate_type)), GGMLType.F32
        return FfnMoeBlock(moe, ff, up(ctx, t, shared.ffn_gate, ff * dim), up(ctx, t, shared.ffn_up, ff * dim),
                           up(ctx, t, shared.ffn_down, dim * ff), up(ctx, f32, shared.ffn_norm, dim),
                           up(ctx, f32, shared.post_ffw_norm_1, dim), up(ctx, f32, shared.post_ffw_norm, dim),
                           shared.layer_output_scale)

    def forward(self, x, n_tokens: int, stream=None) -> None:
        """x: [n_tokens, dim] residual stream, updated in place (torch CUDA
        tensor: asynchronous on `stream`; numpy array: synchronous)."""
        if _is_torch(x):
            rc = lib().g4_ffn_moe_block(self.ctx.handle, C.byref(self.w), C.c_void_p(x.data_ptr()), n_tokens,
                                        C.c_void_p(_stream_ptr(stream)))
            check(rc, self.ctx.handle, "g4_ffn_moe_block")
        else:
            if not (isinstance(x, np.ndarray) and x.dtype == np.float32 and x.flags.c_contiguous):
                raise TypeError("x must be a C-contiguous float32 array (updated in place)")
            rc = lib().g4_ffn_moe_block_host(self.ctx.handle, C.byref(self.w), x.ctypes.data_as(C.c_void_p),
                                             n_tokens)
            check(rc, self.ctx.handle, "g4_ffn_moe_block_host")


def topk(ctx: Context, logits, n_tokens: int, n_expert: int, k: int, idx_out, prob_out, stream=None) -> None:
    """Softmax + iterative top-k on given router logits (Llama.kt:273-293)."""
    rc = lib().g4_moe_topk(ctx.handle, C.c_void_p(logits.data_ptr()), n_tokens, n_expert, k,
                           C.c_void_p(idx_out.data_ptr()), C.c_void_p(prob_out.data_ptr()),
                           C.c_void_p(_stream_ptr(stream)))
    check(rc, ctx.handle, "g4_moe_topk")
