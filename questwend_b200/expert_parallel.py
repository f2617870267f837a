"""Expert-parallel MoE layer over N GPUs: one process per GPU, torch.distributed (NCCL).

QuestWend's own multi-GPU plan is a pipeline-style layer split (core/runtime.cpp:1551-1724);
this module adds expert parallelism for the MoE layer built by build_moe
(core/runtime.cpp:2743-2816).  Tokens are data-parallel: every rank holds T tokens (the
same T on every rank).  Rank r owns experts [lo_r, lo_r + n_r) of the layer (shard_range).
Per layer:

  1. prepare on the rank's own tokens (rms_norm * ffn_norm, router, top-k) and quantize
     the normalised rows to the gate/up weights' vec_dot type (qwb_moe_ep_prepare);
  2. all-gather the packed rows, selected expert ids and routing weights (one collective:
     the three are laid side by side in one byte row per token);
  3. run the SwiGLU expert FFN of the rank's experts over all N*T tokens
     (qwb_moe_ep_experts), producing f32 partial sums;
  4. reduce-scatter (sum) the partial sums back to the token owners and add the residual.

Quantization is per row, so the gathered bytes equal a single-GPU run's; only the f32
summation order of the weighted expert outputs differs from qwb_moe_ffn.  The compute steps
go through a backend object (``prepare`` / ``experts``), the CUDA library by default, so the
partition and exchange logic can also run on CPU ranks (gloo) with another backend.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import ops


def shard_range(n_expert: int, world: int, rank: int):
    """Experts [lo, lo + n) owned by `rank` of `world` (contiguous, sizes differ by <= 1)."""
    lo = rank * n_expert // world
    hi = (rank + 1) * n_expert // world
    return lo, hi - lo


@dataclass
class ExpertShard:
    """One rank's slice of a layer's expert matrices (ggml [H, F, n], [H, F, n], [F, H, n])."""
    gate: object
    up: object
    down: object
    lo: int
    n: int


class CudaBackend:
    """The compute steps on this process's GPU (libqwb.so)."""

    def prepare(self, x, router_w, n_used, norm_w, norm_eps, act_type):
        return ops.moe_ep_prepare(x, router_w, n_used, norm_w=norm_w, norm_eps=norm_eps, act_type=act_type)

    def experts(self, xq, selected, weights, shard: ExpertShard, n_expert: int):
        return ops.moe_ep_experts(xq, selected, weights, shard.gate, shard.up, shard.down, shard.lo, n_expert)


def _all_gather(t: torch.Tensor, group) -> torch.Tensor:
    world = dist.get_world_size(group)
    if world == 1:
        return t
    t = t.contiguous()
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t, group=group)
        return out
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t, group=group)
    return torch.cat(parts, 0)


def _reduce_scatter(t: torch.Tensor, group) -> torch.Tensor:
    world = dist.get_world_size(group)
    if world == 1:
        return t
    t = t.contiguous()
    rows = t.shape[0] // world
    if dist.get_backend(group) == "nccl":
        out = torch.empty((rows,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.reduce_scatter_tensor(out, t, op=dist.ReduceOp.SUM, group=group)
        return out
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    rank = dist.get_rank(group)
    return t[rank * rows:(rank + 1) * rows].clone()


def _gather_routed(xq: torch.Tensor, sel: torch.Tensor, w: torch.Tensor, group):
    """All-gather (xq, sel, w) of every rank as one byte tensor [T, xq bytes + 8 n_used]."""
    T = xq.shape[0]
    if dist.get_world_size(group) == 1:
        return xq, sel, w
    row = torch.cat([xq.reshape(T, -1).view(torch.uint8), sel.view(torch.uint8), w.view(torch.uint8)], 1)
    allr = _all_gather(row, group)
    nb = row.shape[1] - sel.shape[1] * 8
    xq_all = allr[:, :nb].contiguous().view(xq.dtype).reshape((allr.shape[0],) + tuple(xq.shape[1:]))
    sel_all = allr[:, nb:nb + 4 * sel.shape[1]].contiguous().view(torch.int32)
    w_all = allr[:, nb + 4 * sel.shape[1]:].contiguous().view(torch.float32)
    return xq_all, sel_all, w_all


def moe_layer(x: torch.Tensor, router_w: torch.Tensor, shard: ExpertShard, n_used: int, n_expert: int,
              group=None, norm_w=None, norm_eps: float = 1e-6, residual: bool = True, act_type: int = ops.Q8_K,
              backend=None):
    """One expert-parallel MoE layer.  x (T, H) f32: this rank's tokens (same T on every
    rank).  Returns (out (T, H), selected (T, n_used), weights (T, n_used)) for this rank's
    tokens; out = build_moe(rms_norm(x) * norm_w) (+ x when residual)."""
    backend = backend or CudaBackend()
    xq, sel, w = backend.prepare(x, router_w, n_used, norm_w, norm_eps, act_type)
    xq_all, sel_all, w_all = _gather_routed(xq, sel, w, group)
    part = backend.experts(xq_all, sel_all, w_all, shard, n_expert)
    out = _reduce_scatter(part, group)
    if residual:
        out = out + x
    return out, sel, w
