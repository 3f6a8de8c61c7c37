"""Data parallelism for MorphoAttention: batch-sharded ranks, one all-reduce of the weight
gradients per step.

Every (batch, head) pair is independent in the forward and backward, so ranks shard the
batch and exchange nothing but the projection-weight gradients (``dW_phi``, ``dW_V``,
``d_gate_q``, ``d_gate_k``), which are summed over the batch.  They travel as one flat
fp32 bucket, one collective per step: by default the library's own peer-memory all-reduce
(``PeerExchange``: one kernel that reads the other GPUs' buckets over NVLink, sums them in
rank order and writes the fp16 gradients, running beside the dX GEMM), else NCCL's
all-reduce followed by the finalize kernel (``set_collective("nccl")``, or GPUs without
peer access), and gloo for CPU tensors.  The reference has no multi-GPU code; this is the
only collective of the path.
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
_COLLECTIVE = ["peer"]
_EXCHANGES: dict = {}


def set_collective(kind: str) -> None:
    """``"peer"`` (default): the weight-gradient all-reduce runs as the library's peer-memory
    kernel where every pair of the group's GPUs has peer access; ``"nccl"``: NCCL's all-reduce
    and a separate finalize kernel.  Every rank must use the same setting."""
    if kind not in ("peer", "nccl"):
        raise ValueError(f"collective must be 'peer' or 'nccl', not {kind!r}")
    _COLLECTIVE[0] = kind


def get_collective() -> str:
    return _COLLECTIVE[0]


class PeerExchange:
    """This rank's side of the peer-memory all-reduce of a ``elems``-element fp32 bucket
    (``morpho_sm100_peer_*``).  Collective: every rank of ``group`` constructs it at the same
    point; the ranks exchange their regions' IPC handles through ``group`` and map each other's
    memory.  Raises ``RuntimeError`` on every rank when any pair of the ranks' GPUs has no peer
    access (then use NCCL).  ``bucket()`` is the buffer the next backward writes (it alternates
    between two), ``allreduce_finalize`` sums the buckets of all ranks (the same bits on every
    rank) and writes the fp16 gradients; ``close()`` (collective) frees the region."""

    def __init__(self, elems: int, group=None, device=None):
        from . import capi
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.elems = int(elems)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        # two exchange rounds, each ending with every rank knowing every rank's outcome, so that all
        # ranks take the same path (a rank that gave up alone would leave the others waiting)
        self._g, handle, pci, err = None, None, None, None
        try:
            self._g, handle, pci = capi.peer_create(self.rank, self.world, self.elems)
        except capi.MorphoError as e:
            err = str(e)
        gathered = [None] * self.world
        dist.all_gather_object(gathered, (handle, pci, err), group=group)
        errs = [g[2] for g in gathered if g[2] is not None]
        if not errs:
            try:
                capi.peer_connect(self._g, [g[0] for g in gathered], [g[1] for g in gathered])
            except capi.MorphoError as e:
                err = str(e)
            outcome = [None] * self.world
            dist.all_gather_object(outcome, err, group=group)
            errs = [e for e in outcome if e is not None]
        if errs:
            if self._g is not None:
                capi.peer_destroy(self._g)
                self._g = None
            raise RuntimeError("peer all-reduce unavailable: " + "; ".join(errs))

    def bucket(self) -> torch.Tensor:
        from . import capi
        return capi.peer_bucket(self._g, self.elems, self.device)

    def allreduce_finalize(self, p, alpha, dW_phi, d_gate_q, d_gate_k, dW_V, stream=None) -> None:
        from . import capi
        capi.peer_allreduce_finalize(self._g, p, alpha, dW_phi, d_gate_q, d_gate_k, dW_V, stream=stream)

    def close(self) -> None:
        if self._g is not None:
            from . import capi
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            capi.peer_destroy(self._g)
            self._g = None


def peer_exchange(elems: int, group=None, device=None):
    """The cached ``PeerExchange`` of (group, bucket size, device), created on first use
    (collectively); None when the collective is NCCL or the GPUs have no peer access."""
    if _COLLECTIVE[0] != "peer":
        return None
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    key = (id(group), int(elems), dev.index)
    if key not in _EXCHANGES:
        try:
            _EXCHANGES[key] = PeerExchange(elems, group=group, device=dev)
        except RuntimeError:
            _EXCHANGES[key] = None
    return _EXCHANGES[key]


def close_exchanges() -> None:
    """Free every cached exchange (collective: call on every rank, e.g. before
    ``destroy_process_group``)."""
    for key in sorted(_EXCHANGES, key=lambda k: (k[1], k[2])):
        ex = _EXCHANGES.pop(key)
        if ex is not None:
            ex.close()


def _comm_stream(device) -> torch.cuda.Stream:
    idx = torch.device(device).index
    if idx is None:
        idx = torch.cuda.current_device()
    if idx not in _COMM_STREAMS:
        _COMM_STREAMS[idx] = torch.cuda.Stream(device=idx)
    return _COMM_STREAMS[idx]


def backward_allreduce(p, grad_out, saved, X, W_phi, gate_q, gate_k, W_V, out, lse, dX, dW_phi, d_gate_q, d_gate_k,
                       dW_V, bucket, group=None, average: bool = True, timing: list | None = None,
                       exchange: PeerExchange | None = None) -> None:
    """``capi.backward_saved`` for a data-parallel rank, with the weight-gradient all-reduce
    overlapped with the dX GEMM: the library fills the fp32 ``bucket`` first and records an
    event; a communication stream waits for it and all-reduces the bucket while dX runs on
    the current stream, which then waits for the collective.  With an ``exchange``
    (``bucket`` must be ``exchange.bucket()``) the all-reduce is its one peer-memory kernel,
    which also writes the fp16 weight gradients; without, NCCL's all-reduce and then the
    finalize kernel (divided by the world size when ``average``).  After the call ``bucket``
    holds the sum over the ranks.  ``timing`` (a list) receives a ``(start, end)`` pair of
    timing events recorded on the communication stream around the all-reduce."""
    from . import capi
    cur = torch.cuda.current_stream(X.device)
    comm = _comm_stream(X.device)
    ready = torch.cuda.Event()
    alpha = 1.0 / dist.get_world_size(group) if average else 1.0
    capi.backward_saved_dp(p, grad_out, saved, X, W_phi, gate_q, gate_k, W_V, out, lse, dX, bucket,
                           bucket_ready=ready)
    with torch.cuda.stream(comm):
        comm.wait_event(ready)
        if timing is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record(comm)
        if exchange is not None:
            exchange.allreduce_finalize(p, alpha, dW_phi, d_gate_q, d_gate_k, dW_V, stream=comm)
        else:
            dist.all_reduce(bucket, op=dist.ReduceOp.SUM, group=group)
        if timing is not None:
            ev[1].record(comm)
            timing.append(ev)
    cur.wait_stream(comm)
    if exchange is None:
        bucket.record_stream(comm)
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
        n = capi.weight_grad_elems(p)
        ex = peer_exchange(n, group=ctx.group, device=x.device) if dist.get_world_size(ctx.group) > 1 else None
        bucket = ex.bucket() if ex is not None else torch.empty(n, dtype=torch.float32, device=x.device)
        backward_allreduce(p, grad_out, saved, x, W_phi, gate_q, gate_k, W_V, out, lse, dX, *grads, bucket,
                           group=ctx.group, exchange=ex)
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
