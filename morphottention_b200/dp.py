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


_COMM_STREAMS: dict = {}


def _comm_stream(device) -> torch.cuda.Stream:
    idx = torch.device(device).index
    if idx is None:
        idx = torch.cuda.current_device()
    if idx not in _COMM_STREAMS:
        _COMM_STREAMS[idx] = torch.cuda.Stream(device=idx)
    return _COMM_STREAMS[idx]


def backward_allreduce(p, grad_out, saved, X, W_phi, gate_q, gate_k, W_V, out, lse, dX, dW_phi, d_gate_q, d_gate_k,
                       dW_V, bucket, group=None, average: bool = True, timing: list | None = None) -> None:
    """``capi.backward_saved`` for a data-parallel rank, with the weight-gradient all-reduce
    overlapped with the dX GEMM: the library fills the fp32 ``bucket`` first and records an
    event; a communication stream waits for it and all-reduces the bucket while dX runs on
    the current stream, which then waits for the collective and writes the fp16 weight
    gradients (divided by the world size when ``average``).  After the call ``bucket`` holds
    the sum over the ranks.  ``timing`` (a list) receives a ``(start, end)`` pair of timing
    events recorded on the communication stream around the all-reduce."""
    from . import capi
    cur = torch.cuda.current_stream(X.device)
    comm = _comm_stream(X.device)
    ready = torch.cuda.Event()
    capi.backward_saved_dp(p, grad_out, saved, X, W_phi, gate_q, gate_k, W_V, out, lse, dX, bucket,
                           bucket_ready=ready)
    with torch.cuda.stream(comm):
        comm.wait_event(ready)
        if timing is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record(comm)
        dist.all_reduce(bucket, op=dist.ReduceOp.SUM, group=group)
        if timing is not None:
            ev[1].record(comm)
            timing.append(ev)
    cur.wait_stream(comm)
    bucket.record_stream(comm)
    alpha = 1.0 / dist.get_world_size(group) if average else 1.0
    capi.finalize_weight_grads(p, bucket, alpha, dW_phi, d_gate_q, d_gate_k, dW_V)


class _DataParallelFunction(torch.autograd.Function):
    """MorphoAttention whose backward all-reduces the weight gradients, overlapped with dX."""

    @staticmethod
    def forward(ctx, x, W_phi, gate_q, gate_k, W_V, H: int, cube_m: int, scale: float, causal: bool, group):
        from ._ops import ops
        if not x.is_cuda:
            raise ValueError("MorphoAttention expects a CUDA tensor")
        x = x.contiguous()
        from .autograd import current_options
        # every option (the gradient mode included) as this forward ran, for its backward
        ctx.options = current_options()
        _g, proj, mdiag, score, tau = ctx.options
        out, lse, saved = ops.forward_save(x, W_phi, gate_q, gate_k, W_V, H, cube_m, scale, causal, proj, mdiag,
                                           score, tau)
        ctx.save_for_backward(x, W_phi, gate_q, gate_k, W_V, out, lse, saved)
        ctx.H, ctx.cube_m, ctx.scale, ctx.causal, ctx.group = H, cube_m, scale, causal, group
        return out

    @staticmethod
    def backward(ctx, grad_out):
        from . import capi
        x, W_phi, gate_q, gate_k, W_V, out, lse, saved = ctx.saved_tensors
        grad_out = grad_out.contiguous()
        B, N, D = x.shape
        gmode, proj, mdiag, score, tau = ctx.options
        p = capi.problem(B, N, D, ctx.H, ctx.cube_m, ctx.scale, ctx.causal, grad_mode=gmode, projection=proj,
                         mask_diag=mdiag, score=score, tau=tau)
        dX = torch.empty_like(x)
        grads = [torch.empty_like(t) for t in (W_phi, gate_q, gate_k, W_V)]
        bucket = torch.empty(capi.weight_grad_elems(p), dtype=torch.float32, device=x.device)
        backward_allreduce(p, grad_out, saved, x, W_phi, gate_q, gate_k, W_V, out, lse, dX, *grads, bucket,
                           group=ctx.group)
        return (dX, *grads, None, None, None, None, None)


class DataParallelAttention(torch.nn.Module):
    """Wraps a ``MorphoAttention`` for batch-sharded data parallelism: its parameter
    gradients come out of ``backward`` already averaged over ``group`` (one fp32 bucket per
    step, all-reduced while the dX GEMM runs), as ``DistributedDataParallel`` would give
    them.  Every rank must hold the same weights."""

    def __init__(self, module, group=None) -> None:
        super().__init__()
        self.module = module
        self.group = group

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        m = self.module
        return _DataParallelFunction.apply(x, m.W_phi, m.gate_q, m.gate_k, m.W_V, m.num_heads, m.cube_m, m.scale,
                                           m.causal, self.group)
