"""The ViT-B-like encoder that calls MorphoAttention: the caller of the attention path in the
reference benchmark (``attn-bench/src/layers/encoder.py:7-40``, ``layers/mlp.py:5-30``).

A pre-norm block is ``x + attn(LN(x))`` then ``x + MLP(LN(x))`` with a GELU MLP of
``mlp_ratio * dim`` hidden units; dropout is 0 in the benchmark and left out.  The reference's
attention wrapper (``layers/attention/morpho_attention.py:31-41``) adds an output ``Linear``
after MorphoAttention; the benchmark configuration measured here has none (``out_proj=False``,
the default), and ``out_proj=True`` restores it.  Everything is fp16, like the attention layer.
"""

from __future__ import annotations

import torch
from torch import nn

from .autograd import MorphoAttention


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
                 causal: bool = False, out_proj: bool = False, dtype=torch.float16, device=None) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(dim, dtype=dtype, device=device)
        self.attn = MorphoAttention(dim, num_heads, cube_m, scale=scale, causal=causal, dtype=dtype, device=device)
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
                 dtype=torch.float16, device=None) -> None:
        super().__init__()
        self.blocks = nn.ModuleList(
            EncoderBlock(dim, num_heads, cube_m, mlp_ratio=mlp_ratio, scale=scale, causal=causal, out_proj=out_proj,
                         dtype=dtype, device=device) for _ in range(depth))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for blk in self.blocks:
            x = blk(x)
        return x
