"""Benchmark / parity configurations and their seeded synthetic inputs.

The five configurations are the ones the MorphoAttention hot path is measured on.
The reference ships no dataset-backed benchmark for the layer, so every input is
synthetic: ``x ~ N(0, 1)`` and the module's own default initialisation
(``W ~ N(0, D**-0.5)`` drawn in fp32, gates = 1; reference
``torch-ext/morphottention/autograd.py:129-135``).

Inputs are drawn on the CPU with a seeded ``torch.Generator`` in the fixed order
``W_phi, W_V, x`` (then optional random gates, then an optional ``grad_out``), cast to
fp16, and only then moved to the device, so a CPU checker and the GPU path see
bit-identical fp16 inputs.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import torch


@dataclass(frozen=True)
class MorphoConfig:
    name: str
    B: int
    N: int
    D: int
    H: int
    cube_m: int
    scale: float = 1.0
    causal: bool = False
    seed: int = 0

    @property
    def head_dim(self) -> int:
        return self.D // self.H

    @property
    def tokens(self) -> int:
        return self.B * self.N

    def with_(self, **kw) -> "MorphoConfig":
        return replace(self, **kw)

    # ---- algorithmic work of one forward + backward (formulas of the measurement plan)
    def pairs(self) -> float:
        """Score elements per forward pass: ``B*H*N^2`` (halved when causal)."""
        nn = float(self.B) * self.H * self.N * self.N
        return nn * 0.5 if self.causal else nn

    def tensor_flops_fwd_bwd(self) -> float:
        """Dense contraction FLOPs of fwd + bwd, recompute excluded:
        projection fwd + the two backward GEMMs, S and PV forward, and S, dP, dV, dq, dk
        backward."""
        m, hd = self.cube_m, self.head_dim
        proj = 3.0 * 2.0 * self.tokens * self.D * (self.H * m + self.D)
        nn = self.pairs()
        return proj + 2.0 * nn * (m + hd) + 2.0 * nn * (3 * m + 2 * hd)

    def exps_fwd_bwd(self) -> float:
        return 2.0 * self.pairs()

    def min_hbm_bytes(self) -> float:
        return (2.0 * self.tokens * self.D * 6 + 8.0 * self.B * self.H * self.N
                + 6.0 * self.D * (self.H * self.cube_m + self.D))


CONFIGS = {
    "c1": MorphoConfig("c1_readme", 2, 128, 256, 8, 16, 1.0, False, 0),
    "c2": MorphoConfig("c2_causal", 8, 1024, 512, 8, 16, 1.0, True, 1),
    "c3": MorphoConfig("c3_long", 4, 4096, 1024, 16, 32, 0.5, False, 2),
    "c4": MorphoConfig("c4_vit_layer", 64, 197, 768, 12, 16, 1.0, False, 3),
    "c5": MorphoConfig("c5_dp_rank", 8, 8192, 2048, 16, 64, 1.0, True, 4),
}


def make_inputs(cfg: MorphoConfig, device="cpu", random_gates: bool = False, with_grad_out: bool = False,
                dtype=torch.float16):
    """Seeded synthetic inputs for ``cfg``.  Returns a dict of tensors on ``device``:
    ``x, W_phi, gate_q, gate_k, W_V`` (and ``grad_out`` when asked)."""
    g = torch.Generator(device="cpu").manual_seed(cfg.seed)
    D, H, m = cfg.D, cfg.H, cfg.cube_m
    std = D ** -0.5
    W_phi = torch.empty(D, H * m, dtype=torch.float32).normal_(0.0, std, generator=g)
    W_V = torch.empty(D, D, dtype=torch.float32).normal_(0.0, std, generator=g)
    x = torch.empty(cfg.B, cfg.N, D, dtype=torch.float32).normal_(0.0, 1.0, generator=g)
    if random_gates:
        gate_q = 1.0 + 0.5 * torch.empty(H, m, dtype=torch.float32).normal_(0.0, 1.0, generator=g)
        gate_k = 1.0 + 0.5 * torch.empty(H, m, dtype=torch.float32).normal_(0.0, 1.0, generator=g)
    else:
        gate_q = torch.ones(H, m, dtype=torch.float32)
        gate_k = torch.ones(H, m, dtype=torch.float32)
    out = {"x": x, "W_phi": W_phi, "gate_q": gate_q, "gate_k": gate_k, "W_V": W_V}
    if with_grad_out:
        out["grad_out"] = torch.empty(cfg.B, cfg.N, D, dtype=torch.float32).normal_(0.0, 1.0, generator=g)
    return {k: v.to(dtype).to(device) for k, v in out.items()}
