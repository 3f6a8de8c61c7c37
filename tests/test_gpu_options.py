"""The reference's compile-time variants as run-time options: the HardTanh01 and Identity
hypercube projections (reference csrc/cuda/morfology/cube.cuh:10-45) and the diagonal
mask (MORPHO_MASK_DIAG, csrc/cuda/utils/declarations.cuh:79-82, attention.cu:131, :363),
through the C ABI and through the module API, against the fp32 oracle with the same
tolerances as the default path (rel-L2 <= 1e-3 out / lse, <= 5e-3 gradients)."""

import pytest
import torch

import morphottention_b200 as M
from morphottention_b200.configs import MorphoConfig
from oracle import morpho_oracle as O

from .helpers import compare, gate_tolerance, inputs, run_cuda, run_oracle

pytestmark = pytest.mark.gpu

# The HardTanh01 and Identity codes spread wider than the sigmoid's, so at cube_m = 64 the
# self-score S_ii = 2 scale |phi_i - 1/2|^2 dominates every row at scale 1: the softmax
# saturates, the weight gradients through it vanish (~1e-5 of their usual size) and a
# relative error of them measures fp16 noise only.  The m = 64 case uses scale 0.2 (and 0.03
# for the unbounded Identity codes, whose |phi - 1/2|^2 is about 1.25 per column).
CASES = [
    MorphoConfig("m16_hd64", 2, 197, 128, 2, 16, 1.0, False, 31),
    MorphoConfig("m32_causal", 1, 300, 256, 4, 32, 0.5, True, 32),
    MorphoConfig("m64_hd128", 1, 256, 256, 2, 64, 0.2, False, 33),
]


@pytest.mark.parametrize("cfg", CASES, ids=lambda c: c.name)
@pytest.mark.parametrize("projection", ["hardtanh01", "identity"])
def test_projection_parity(cuda, cfg, projection):
    if projection == "identity" and cfg.cube_m == 64:
        cfg = cfg.with_(scale=0.03)
    inp = inputs(cfg, cuda, random_gates=True, with_grad_out=True)
    g = inp.pop("grad_out")
    ours = run_cuda(cfg, inp, grad_out=g, projection=projection)
    ref = run_oracle(cfg, {k: v.cpu() for k, v in inp.items()}, grad_out=g.cpu(), projection=projection)
    compare(ours, ref, tol_gate=gate_tolerance(cfg))


def _compare_masked(ours, ref, cfg):
    """lse of rows without any key is -FLT_MAX on both sides; compare the others."""
    dead = ref["lse"] <= O.FLT_LOWEST / 2
    assert torch.equal(dead, ours["lse"].cpu() <= O.FLT_LOWEST / 2)
    live = {k: v for k, v in ours.items() if k != "lse"}
    errs = compare(live, ref, keys=[k for k in live], tol_gate=gate_tolerance(cfg))
    lse_err = O.rel_l2(ours["lse"].cpu()[~dead].double(), ref["lse"][~dead].double())
    assert lse_err <= 1e-3, lse_err
    if dead.any():
        assert torch.all(ours["out"].float().view(cfg.B, cfg.N, cfg.H, -1).permute(0, 2, 1, 3)
                         .reshape(cfg.B * cfg.H, cfg.N, -1)[dead.to(ours["out"].device)] == 0)
    return errs


@pytest.mark.parametrize("cfg", CASES + [MorphoConfig("n15_causal", 2, 15, 64, 2, 32, 2.0, True, 34),
                                         # hd 128 forward (P over S, two K/V stages): causal, ragged,
                                         # three key tiles, a dead first row
                                         MorphoConfig("hd128_causal", 1, 290, 256, 2, 32, 0.5, True, 39)],
                         ids=lambda c: c.name)
def test_mask_diag_parity(cuda, cfg):
    inp = inputs(cfg, cuda, random_gates=True, with_grad_out=True)
    g = inp.pop("grad_out")
    ours = run_cuda(cfg, inp, grad_out=g, mask_diag=True)
    ref = run_oracle(cfg, {k: v.cpu() for k, v in inp.items()}, grad_out=g.cpu(), mask_diag=True)
    _compare_masked(ours, ref, cfg)


def test_options_through_module(cuda):
    """attention_options() reaches the torch ops: the module matches the oracle with a
    non-default projection and the diagonal mask, and the settings are restored after."""
    cfg = MorphoConfig("mod", 2, 160, 128, 4, 16, 0.8, True, 35)
    inp = inputs(cfg, cuda, random_gates=True)
    mod = M.MorphoAttention(cfg.D, cfg.H, cfg.cube_m, scale=cfg.scale, causal=cfg.causal, device=cuda)
    with torch.no_grad():
        for n in ("W_phi", "W_V", "gate_q", "gate_k"):
            getattr(mod, n).copy_(inp[n])
    x = inp["x"].clone().requires_grad_(True)
    with M.attention_options(projection="hardtanh01", mask_diag=True):
        assert M.get_cube_projection() == "hardtanh01" and M.get_mask_diag()
        out = mod(x)
        out.float().sum().backward()
    assert M.get_cube_projection() == "sigmoid" and not M.get_mask_diag()
    ref = run_oracle(cfg, {k: v.cpu() for k, v in inp.items()}, projection="hardtanh01", mask_diag=True)
    ours = {"out": out.detach(), "dX": x.grad, "dW_phi": mod.W_phi.grad, "d_gate_q": mod.gate_q.grad,
            "d_gate_k": mod.gate_k.grad, "dW_V": mod.W_V.grad}
    compare(ours, ref, tol_gate=gate_tolerance(cfg))


def test_invalid_options_are_rejected(cuda):
    from morphottention_b200 import capi
    with pytest.raises(ValueError):
        M.set_cube_projection("relu")
    p = capi.problem(1, 128, 128, 2, 16, projection=7)
    x = torch.zeros(1, 128, 128, dtype=torch.float16, device=cuda)
    w = torch.zeros(128, 32, dtype=torch.float16, device=cuda)
    gq = torch.ones(2, 16, dtype=torch.float16, device=cuda)
    with pytest.raises(capi.MorphoError, match="projection"):
        capi.forward(p, x, w, gq, gq, torch.zeros(128, 128, dtype=torch.float16, device=cuda), torch.empty_like(x),
                     torch.empty(2, 128, device=cuda))


def _module_with(cfg, inp, cuda):
    mod = M.MorphoAttention(cfg.D, cfg.H, cfg.cube_m, scale=cfg.scale, causal=cfg.causal, device=cuda)
    with torch.no_grad():
        for n in ("W_phi", "W_V", "gate_q", "gate_k"):
            getattr(mod, n).copy_(inp[n])
    return mod


@pytest.mark.parametrize("opts", [{"score": "dilation", "tau": 0.9}, {"projection": "hardtanh01"},
                                  {"mask_diag": True}], ids=["dilation", "hardtanh01", "mask_diag"])
def test_backward_outside_the_options_block(cuda, opts):
    """The loss is built inside attention_options() and differentiated after the block has
    restored the defaults: the backward must differentiate the variant the forward ran (the
    autograd Function captured the options with the forward), matching the oracle's gradients
    of that variant."""
    cfg = MorphoConfig("late_bwd", 2, 150, 128, 4, 16, 0.7, True, 36)
    inp = inputs(cfg, cuda, random_gates=True, with_grad_out=True)
    g = inp.pop("grad_out")
    mod = _module_with(cfg, inp, cuda)
    x = inp["x"].clone().requires_grad_(True)
    with M.attention_options(**opts):
        out = mod(x)
        loss = (out.float() * g.float()).sum()
    assert M.get_score()[0] == "softmax" and M.get_cube_projection() == "sigmoid" and not M.get_mask_diag()
    loss.backward()
    t = {k: v.cpu() for k, v in inp.items()}
    if "score" in opts:
        ref = O.soft_morph_forward_backward(t["x"], t["W_phi"], t["gate_q"], t["gate_k"], t["W_V"], cfg.H,
                                            cfg.cube_m, cfg.scale, cfg.causal, opts["score"], opts["tau"],
                                            grad_out=g.cpu())
    else:
        ref = run_oracle(cfg, t, grad_out=g.cpu(), projection=opts.get("projection", "sigmoid"),
                         mask_diag=opts.get("mask_diag", False))
    ours = {"out": out.detach(), "dX": x.grad, "dW_phi": mod.W_phi.grad, "d_gate_q": mod.gate_q.grad,
            "d_gate_k": mod.gate_k.grad, "dW_V": mod.W_V.grad}
    if opts.get("mask_diag"):  # causal + diagonal mask: query 0 has no key (out 0, no gradient there)
        assert torch.all(out[:, 0] == 0)
    compare(ours, ref, tol_gate=gate_tolerance(cfg))


def test_two_modules_with_different_options_in_one_graph(cuda):
    """A sigmoid-projection layer feeding a HardTanh01 + diagonal-mask layer, one backward over
    both after the options block has closed: each layer's gradients are those of its own
    variant (checked against each layer run alone under its own options)."""
    cfg = MorphoConfig("two_mods", 1, 128, 128, 2, 16, 0.8, False, 37)
    inp = inputs(cfg, cuda, random_gates=True)
    a = _module_with(cfg, inp, cuda)
    b = _module_with(cfg, inp, cuda)
    x = inp["x"].clone().requires_grad_(True)
    h = a(x)
    with M.attention_options(projection="hardtanh01", mask_diag=True):
        y = b(h)
    y.float().sum().backward()
    grads = {n: getattr(b, n).grad.clone() for n in ("W_phi", "W_V", "gate_q", "gate_k")}
    # the second layer alone on the same input, differentiated inside its block
    b.zero_grad(set_to_none=True)
    h2 = h.detach().clone().requires_grad_(True)
    with M.attention_options(projection="hardtanh01", mask_diag=True):
        b(h2).float().sum().backward()
    for n, gr in grads.items():
        assert torch.equal(gr, getattr(b, n).grad), n


def test_grad_mode_is_bound_to_the_forward(cuda):
    """grad_mode("reference") around the forward only: the backward still uses the reference
    semantics (the query path dropped), matching the oracle's reference mode."""
    cfg = MorphoConfig("late_mode", 2, 130, 128, 2, 16, 1.0, False, 38)
    inp = inputs(cfg, cuda, random_gates=True)
    mod = _module_with(cfg, inp, cuda)
    x = inp["x"].clone().requires_grad_(True)
    with M.grad_mode("reference"):
        out = mod(x)
    assert M.get_grad_mode() == "full"
    out.float().sum().backward()
    ref = run_oracle(cfg, {k: v.cpu() for k, v in inp.items()}, grad_mode="reference")
    ours = {"out": out.detach(), "dX": x.grad, "dW_phi": mod.W_phi.grad, "d_gate_q": mod.gate_q.grad,
            "d_gate_k": mod.gate_k.grad, "dW_V": mod.W_V.grad}
    compare(ours, ref, tol_gate=gate_tolerance(cfg))
