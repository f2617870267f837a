"""Expert-parallel MoE layer over N GPUs: one process per GPU, torch.distributed (NCCL).

QuestWend's own multi-GPU plan is a pipeline-style layer split (core/runtime.cpp:1551-1724);
this module adds expert parallelism for the MoE layer built by build_moe
(core/runtime.cpp:2743-2816).  Rank r owns experts [lo_r, lo_r + n_r) of every layer
(shard_range) and every rank holds the hidden states of all T tokens (identical copies).
Per layer:

  1. every rank routes all T tokens (the router is replicated, so the ids and weights are
     the same everywhere) and runs the SwiGLU expert FFN of its own experts over the
     pairs routed to them, writing per token the weighted sum of those experts' outputs;
     rank 0 adds the residual (qwb_moe_ep_layer: one library call);
  2. one all-reduce (sum) of the (T, H) partial outputs: every rank then holds the layer's
     output for all tokens, the next layer's input.  For decode-sized messages the
     peer-memory all-reduce (PeerAllReduce, one kernel) replaces NCCL's.

Quantization is per row, so every rank's activation bytes equal a single-GPU run's; only
the f32 summation order of the weighted expert outputs differs from qwb_moe_ffn.  The
compute step goes through a backend object (``layer``), the CUDA library by default, so
the partition and exchange logic can also run on CPU ranks (gloo) with another backend.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _lib as L
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


class PeerAllReduce:
    """The layer's all-reduce over peer memory (qwb_ep_comm: CUDA IPC mappings of every
    GPU's exchange buffer, one kernel per call; the GPUs' sums are added in rank order, so
    every GPU holds the same bits).  Collective construction: every rank of `group`
    creates its buffer, the IPC handles are all-gathered, every rank maps its peers'.
    max_bytes bounds the message of one call."""

    def __init__(self, group=None, max_bytes: int = 1 << 20):
        self.lib = L.lib()
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        hs = self.lib.qwb_ep_comm_handle_size()
        handle = (C.c_char * hs)()
        ptr = C.c_void_p()
        L.check("qwb_ep_comm_create", self.lib.qwb_ep_comm_create(world, rank, max_bytes, C.byref(ptr), handle))
        self.ptr = ptr
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        allh = b"".join(handles)
        L.check("qwb_ep_comm_connect", self.lib.qwb_ep_comm_connect(self.ptr, allh))
        dist.barrier(group)

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        """In place: t (contiguous f32, numel % 4 == 0) = the sum of every rank's t."""
        L.check("qwb_ep_allreduce_f32", self.lib.qwb_ep_allreduce_f32(
            self.ptr, t.data_ptr(), t.data_ptr(), t.numel(), ops.status_block().data_ptr(),
            C.c_void_p(torch.cuda.current_stream().cuda_stream)))
        return t

    def close(self):
        """After every call has completed (synchronize first)."""
        if self.ptr:
            self.lib.qwb_ep_comm_destroy(self.ptr)
            self.ptr = None


class CudaBackend:
    """The compute step on this process's GPU (libqwb.so)."""

    def layer(self, x, router_w, shard: ExpertShard, n_used, norm_w, norm_eps, residual, out=None, shexp=None):
        return ops.moe_ep_layer(x, router_w, shard.gate, shard.up, shard.down, shard.lo, n_used, residual=residual,
                                norm_w=norm_w, norm_eps=norm_eps, out=out, shexp=shexp)


def moe_layer(x: torch.Tensor, router_w: torch.Tensor, shard: ExpertShard, n_used: int, group=None,
              norm_w=None, norm_eps: float = 1e-6, residual: bool = True, backend=None, out=None, shexp=None,
              comm: PeerAllReduce = None):
    """One expert-parallel MoE layer.  x (T, H) f32: all tokens (the same on every rank).
    shexp: the layer's shared expert (as in ops.moe_ffn), computed on rank 0.  comm: the
    peer-memory all-reduce (else torch.distributed's, NCCL or gloo).  Returns
    (out (T, H), selected (T, n_used), weights (T, n_used)), the same on every rank:
    out = build_moe(rms_norm(x) * norm_w) (+ the shared expert) (+ x when residual)."""
    backend = backend or CudaBackend()
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    res = x if (residual and rank == 0) else None
    kw = {"shexp": shexp} if (shexp is not None and rank == 0) else {}
    part, sel, w = backend.layer(x, router_w, shard, n_used, norm_w, norm_eps, res, out=out, **kw)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        if comm is not None:
            comm.all_reduce(part)
        else:
            dist.all_reduce(part, op=dist.ReduceOp.SUM, group=group)
    return part, sel, w
