"""The ViT-B-like encoder that calls MorphoAttention: the caller of the attention path in the
reference benchmark (``attn-bench/src/layers/encoder.py:7-40``, ``layers/mlp.py:5-30``).

A pre-norm block is ``x + attn(LN(x))`` then ``x + MLP(LN(x))`` with a GELU MLP of
``mlp_ratio * dim`` hidden units; dropout is 0 in the benchmark and left out.  The reference's
attention wrapper (``layers/attention/morpho_attention.py:31-41``) adds an output ``Linear``
after MorphoAttention; the benchmark configuration measured here has none (``out_proj=False``,
the default), and ``out_proj=True`` restores it.  Everything is fp16, like the attention layer.

``attention`` (optional) builds each block's attention layer from ``(dim, num_heads, cube_m,
scale=, causal=, dtype=, device=)``; the default is this package's ``MorphoAttention``.  A CPU
checker passes its own layer, and then this module needs nothing else from the package.
"""

from __future__ import annotations

import torch
from torch import nn


def _morpho_attention(dim, num_heads, cube_m, **kw):
    from .autograd import MorphoAttention
    return MorphoAttention(dim, num_heads, cube_m, **kw)


class MLP(nn.Module):
    def __init__(self, dim: int, hidden: int, dtype=torch.float16, device=None) -> None:
        super().__init__()
        self.fc1 = nn.Linear(dim, hidden, dtype=dtype, device=device)
        self.act = nn.GELU()
        self.fc2 = nn.Linear(hidden, dim, dtype=dtype, device=device)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.fc2(self.act(self.fc1(x)))


class EncoderBlock(nn.Module):
    def __init__(self, dim: int, num_heads: int, cube_m: int, *, mlp_ratio: float = 4.0, scale: float = 1.0,
                 causal: bool = False, out_proj: bool = False, dtype=torch.float16, device=None,
                 attention=None) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(dim, dtype=dtype, device=device)
        make = attention or _morpho_attention
        self.attn = make(dim, num_heads, cube_m, scale=scale, causal=causal, dtype=dtype, device=device)
        self.proj = nn.Linear(dim, dim, dtype=dtype, device=device) if out_proj else None
        self.norm2 = nn.LayerNorm(dim, dtype=dtype, device=device)
        self.mlp = MLP(dim, int(dim * mlp_ratio), dtype=dtype, device=device)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        a = self.attn(self.norm1(x))
        if self.proj is not None:
            a = self.proj(a)
        x = x + a
        return x + self.mlp(self.norm2(x))


class Encoder(nn.Module):
    """``depth`` pre-norm blocks (ViT-B: depth 12, dim 768, 12 heads, MLP 3072)."""

    def __init__(self, depth: int = 12, dim: int = 768, num_heads: int = 12, cube_m: int = 16, *,
                 mlp_ratio: float = 4.0, scale: float = 1.0, causal: bool = False, out_proj: bool = False,
                 dtype=torch.float16, device=None, attention=None) -> None:
        super().__init__()
        self.blocks = nn.ModuleList(
            EncoderBlock(dim, num_heads, cube_m, mlp_ratio=mlp_ratio, scale=scale, causal=causal, out_proj=out_proj,
                         dtype=dtype, device=device, attention=attention) for _ in range(depth))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for blk in self.blocks:
            x = blk(x)
        return x


class GraphedTrainingStep:
    """One training step (forward, loss, backward, optimizer step) captured once as a CUDA graph
    and replayed per batch, so the step's several hundred launches (LayerNorm, GELU, cuBLAS MLP
    GEMMs, this library's attention kernels, the foreach optimizer update) cost one graph launch
    on the host instead of one Python dispatch each.

    ``step = GraphedTrainingStep(model, loss_fn, optimizer, x, target)`` runs ``warmup`` ordinary
    training steps on ``(x, target)`` on a side stream (real updates: they create the optimizer's
    state, the cuBLAS handles and this library's per-device state before capture, as CUDA graph
    capture requires), then captures ``loss_fn(model(x), target); loss.backward();
    optimizer.step()`` with the gradients unset at capture, so every replay assigns them afresh
    like ``zero_grad(set_to_none=True)`` before an eager step.  ``step(x_batch, target_batch)``
    copies the batch into the captured input buffers on the current stream, replays, and returns
    the loss tensor (the same storage every call: copy it out before the next call).

    Parameters, gradients and optimizer state live at fixed addresses from then on; changing the
    learning rate needs a tensor ``lr`` in the optimizer or a new capture.  The model must not
    change between calls (no new parameters, no shape change of the batch)."""

    def __init__(self, model: nn.Module, loss_fn, optimizer: torch.optim.Optimizer, x: torch.Tensor,
                 target: torch.Tensor, warmup: int = 3) -> None:
        if not x.is_cuda:
            raise ValueError("GraphedTrainingStep needs CUDA inputs")
        self.model, self.loss_fn, self.optimizer = model, loss_fn, optimizer
        self.x = x.detach().clone()
        self.target = target.detach().clone()
        side = torch.cuda.Stream(device=x.device)
        side.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                optimizer.zero_grad(set_to_none=True)
                loss_fn(model(self.x), self.target).backward()
                optimizer.step()
        torch.cuda.current_stream(x.device).wait_stream(side)
        optimizer.zero_grad(set_to_none=True)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.loss = loss_fn(model(self.x), self.target)
            self.loss.backward()
            optimizer.step()

    def __call__(self, x: torch.Tensor | None = None, target: torch.Tensor | None = None) -> torch.Tensor:
        if x is not None:
            self.x.copy_(x, non_blocking=True)
        if target is not None:
            self.target.copy_(target, non_blocking=True)
        self.graph.replay()
        return self.loss.detach()
