"""Data parallelism for MorphoAttention: batch-sharded ranks, one all-reduce of the weight
gradients per step.

Every (batch, head) pair is independent in the forward and backward, so ranks shard the
batch and exchange nothing but the projection-weight gradients (``dW_phi``, ``dW_V``,
``d_gate_q``, ``d_gate_k``), which are summed over the batch.  They travel as one flat
fp32 bucket (one collective per step, NCCL over NVLink for CUDA tensors, gloo for CPU).
The reference has no multi-GPU code; this is the only collective of the path.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

PARAM_ORDER = ("W_phi", "W_V", "gate_q", "gate_k")


def allreduce_bucket(bucket: torch.Tensor, group=None, average: bool = True) -> torch.Tensor:
    """All-reduce a flat fp32 weight-gradient bucket in place (the layout of the C ABI's
    ``dweights_f32``); divides by the world size when ``average``."""
    dist.all_reduce(bucket, op=dist.ReduceOp.SUM, group=group)
    if average:
        bucket.div_(dist.get_world_size(group))
    return bucket


def allreduce_weight_grads(module, group=None, average: bool = True) -> None:
    """All-reduce ``module``'s parameter gradients (a ``MorphoAttention``) through one fp32
    bucket and write them back in their own dtype.  Parameters without a gradient take
    part as zeros so that every rank issues the same collective."""
    params = [getattr(module, n) for n in PARAM_ORDER]
    flat = torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).float().reshape(-1) for p in params])
    allreduce_bucket(flat, group=group, average=average)
    off = 0
    for p in params:
        n = p.numel()
        g = flat[off:off + n].view_as(p).to(p.dtype)
        if p.grad is None:
            p.grad = g
        else:
            p.grad.copy_(g)
        off += n
