"""Parity of the sm_100a kernels (called through the C ABI) against the fp32 oracle on
identical seeded fp16 inputs.  Tolerances: rel-L2 <= 1e-3 for out and lse, <= 5e-3 for
every gradient.

Cases cover each supported (cube_m, head_dim) pair, causal and non-causal, sequence
lengths that are not a multiple of the 128-row tile (197, 1, 15, 129), a single tile,
random gates, random grad_out, and both gradient modes.  The LONG cases have at least 16
query tiles, where the backward kernel runs its two softmax warpgroups half a tile apart
(every head shape whose shared-memory budget holds two dS tiles), causal ones included so
that the last key tiles see one or two query tiles.
"""

import pytest
import torch

from morphottention_b200.configs import CONFIGS, MorphoConfig

from .helpers import compare, gate_tolerance, inputs, run_cuda, run_oracle

pytestmark = pytest.mark.gpu

SMALL = [
    CONFIGS["c1"],                                                     # README shape, m16 hd32
    MorphoConfig("vit_narrow", 2, 197, 128, 2, 16, 1.0, False, 3),     # ragged N, m16 hd64
    MorphoConfig("causal_m16", 2, 256, 128, 2, 16, 1.0, True, 1),      # causal, two tiles
    MorphoConfig("m32_hd64", 1, 300, 256, 4, 32, 0.5, False, 2),       # m32, ragged
    MorphoConfig("m32_causal", 1, 333, 128, 2, 32, 0.5, True, 5),      # causal + ragged
    MorphoConfig("m64_hd128", 1, 256, 256, 2, 64, 1.0, True, 4),       # c5-like head shape
    MorphoConfig("m64_hd64", 2, 130, 256, 4, 64, 0.7, False, 6),       # N = tile + 2
    MorphoConfig("m16_hd128", 1, 64, 384, 3, 16, 1.0, False, 7),       # N < tile, odd H
    MorphoConfig("n1", 3, 1, 64, 2, 16, 1.0, False, 8),                # single token
    MorphoConfig("n15_causal", 2, 15, 64, 2, 32, 2.0, True, 9),        # tiny causal
    MorphoConfig("hd32_m64", 1, 129, 128, 4, 64, 1.0, False, 10),      # hd 32 with m 64
]

LONG = [
    MorphoConfig("long_m16_hd64_causal", 1, 2100, 128, 2, 16, 1.0, True, 11),   # ragged last tile
    MorphoConfig("long_m32_hd64", 1, 2048, 128, 2, 32, 0.5, False, 12),         # c3 head shape
    MorphoConfig("long_m64_hd64_causal", 1, 2200, 128, 2, 64, 1.0, True, 13),
    MorphoConfig("long_m16_hd128", 1, 2049, 128, 1, 16, 1.0, False, 14),        # one row past 16 tiles
    MorphoConfig("long_m32_hd32_causal", 2, 2304, 64, 2, 32, 0.7, True, 15),
    MorphoConfig("long_m64_hd128_causal", 1, 2048, 256, 2, 64, 1.0, True, 16),  # one dS tile: lockstep
]


@pytest.mark.parametrize("cfg", SMALL, ids=lambda c: c.name)
@pytest.mark.parametrize("random_gates", [False, True], ids=["gates1", "gatesR"])
def test_parity_small(cuda, cfg, random_gates):
    inp = inputs(cfg, cuda, random_gates=random_gates, with_grad_out=random_gates)
    g = inp.pop("grad_out", None)
    ours = run_cuda(cfg, inp, grad_out=g)
    ref = run_oracle(cfg, {k: v.cpu() for k, v in inp.items()}, grad_out=None if g is None else g.cpu())
    compare(ours, ref, tol_gate=gate_tolerance(cfg))


@pytest.mark.parametrize("cfg", LONG, ids=lambda c: c.name)
def test_parity_long(cuda, cfg):
    inp = inputs(cfg, cuda, random_gates=True, with_grad_out=True)
    g = inp.pop("grad_out")
    ours = run_cuda(cfg, inp, grad_out=g)
    ref = run_oracle(cfg, {k: v.cpu() for k, v in inp.items()}, grad_out=g.cpu())
    compare(ours, ref, tol_gate=gate_tolerance(cfg))


@pytest.mark.parametrize("cfg", [SMALL[0], SMALL[2], SMALL[3]], ids=lambda c: c.name)
def test_parity_reference_grad_mode(cuda, cfg):
    """grad_mode=reference reproduces the reference kernel's gradient semantics."""
    inp = inputs(cfg, cuda, random_gates=True)
    ours = run_cuda(cfg, inp, grad_mode="reference")
    ref = run_oracle(cfg, {k: v.cpu() for k, v in inp.items()}, grad_mode="reference")
    compare(ours, ref)


def test_deterministic(cuda):
    """No fp16 global atomics: two runs give bit-identical out/lse/weight grads (dX goes
    through fp32 dq atomics, whose summation order may vary, so it is compared loosely)."""
    cfg = SMALL[3]
    inp = inputs(cfg, cuda, random_gates=True)
    a = run_cuda(cfg, inp)
    b = run_cuda(cfg, inp)
    for k in ("out", "lse", "dW_V"):
        assert torch.equal(a[k], b[k]), k
    for k in ("dX", "dW_phi", "d_gate_q", "d_gate_k"):
        assert (a[k].float() - b[k].float()).abs().max().item() <= 1e-2 * a[k].float().abs().max().item() + 1e-6, k
