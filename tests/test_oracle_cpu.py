"""Self-checks of the CPU oracle (no GPU).  The reference ships no tests, golden vectors
or eager formulation, so the oracle is pinned by (a) fp64 gradcheck of its own autograd,
(b) the algebraic identities of the score, (c) the known behaviour of the reference
backward (query-side gradients dropped) and (d) the committed golden fixtures produced by
the reference kernel itself (``tests/golden``)."""

import torch

from morphottention_b200.configs import CONFIGS, MorphoConfig, make_inputs
from oracle import morpho_oracle as O

TINY = MorphoConfig("tiny", 2, 9, 8, 2, 3, 0.7, False, 0)


def _inputs(cfg, dtype=torch.float64, gates=True):
    inp = make_inputs(cfg, random_gates=gates, dtype=torch.float32)
    return {k: v.to(dtype) for k, v in inp.items()}


def test_gradcheck_fp64():
    for causal in (False, True):
        cfg = TINY.with_(causal=causal)
        inp = _inputs(cfg)
        args = [inp[k].clone().requires_grad_(True) for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")]

        def f(*a):
            out, lse = O.forward(*a, cfg.H, cfg.cube_m, cfg.scale, cfg.causal)
            return out, lse

        assert torch.autograd.gradcheck(f, args, eps=1e-6, atol=1e-6)


def test_score_is_soft_hamming():
    cfg = TINY
    inp = _inputs(cfg)
    phi, q, k, qb, cb, _ = O.project(inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], cfg.H,
                                     cfg.cube_m)
    dot = cfg.scale * (2 * q @ k.transpose(-1, -2) - qb.unsqueeze(-1) - cb.unsqueeze(-2))
    gq = inp["gate_q"].view(1, cfg.H, 1, cfg.cube_m)
    gk = inp["gate_k"].view(1, cfg.H, 1, cfg.cube_m)
    ham = O.soft_hamming_score(phi, phi, gq.unsqueeze(-2), gk.unsqueeze(-2), cfg.scale)
    assert torch.allclose(dot, ham, atol=1e-12)


def test_query_bias_gradient_is_zero():
    """dL/dqbias_i = -scale * sum_j dS_ij = 0 exactly (softmax is shift-invariant per row);
    the kernels use this identity instead of accumulating the query-bias gradient."""
    cfg = TINY.with_(causal=True)
    inp = _inputs(cfg)
    _, q, k, qb, cb, v = O.project(inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], cfg.H,
                                   cfg.cube_m)
    qb = qb.detach().requires_grad_(True)
    o, lse = O._attend(q.detach(), k.detach(), qb, cb.detach(), v.detach(), cfg.scale, cfg.causal)
    g = torch.randn_like(o)
    (dqb,) = torch.autograd.grad((o * g).sum(), qb)
    assert dqb.abs().max().item() < 1e-12


def test_lse_is_log2_domain():
    cfg = TINY
    inp = _inputs(cfg)
    _, q, k, qb, cb, v = O.project(inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], cfg.H,
                                   cfg.cube_m)
    s = cfg.scale * (2 * q @ k.transpose(-1, -2) - qb.unsqueeze(-1) - cb.unsqueeze(-2)) * O.LOG2E
    m = s.max(-1).values
    lse_ref = m + torch.log2(torch.exp2(s - m.unsqueeze(-1)).sum(-1))  # attention.cu:186
    _, lse = O.forward(inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], cfg.H, cfg.cube_m,
                       cfg.scale, cfg.causal)
    assert torch.allclose(lse, lse_ref.reshape(cfg.B * cfg.H, cfg.N), atol=1e-12)


def test_reference_grad_mode_differs_only_on_query_path():
    cfg = CONFIGS["c1"].with_(B=1, N=32)
    inp = _inputs(cfg, dtype=torch.float64)
    full = O.forward_backward(*(inp[k] for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")), cfg.H, cfg.cube_m,
                              dtype=torch.float64)
    ref = O.forward_backward(*(inp[k] for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")), cfg.H, cfg.cube_m,
                             grad_mode="reference", dtype=torch.float64)
    for k in ("out", "lse", "dW_V", "d_gate_k"):
        assert O.rel_l2(ref[k], full[k]) < 1e-10, k
    for k in ("dX", "dW_phi", "d_gate_q"):
        assert O.rel_l2(ref[k], full[k]) > 1e-3, k


def test_causal_first_row_attends_to_itself():
    cfg = TINY.with_(causal=True)
    inp = _inputs(cfg)
    out, _ = O.forward(inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], cfg.H, cfg.cube_m,
                       cfg.scale, True)
    v = (inp["x"] @ inp["W_V"])
    assert torch.allclose(out[:, 0], v[:, 0], atol=1e-12)


def test_chunked_forward_matches():
    cfg = MorphoConfig("chunk", 1, 40, 64, 4, 16, 0.5, True, 5)
    inp = _inputs(cfg, dtype=torch.float32)
    a = O.forward(*(inp[k] for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")), cfg.H, cfg.cube_m, cfg.scale,
                  cfg.causal)
    b = O.forward_chunked(*(inp[k] for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")), cfg.H, cfg.cube_m,
                          cfg.scale, cfg.causal, heads_per_chunk=3)
    assert O.rel_l2(b[0], a[0]) < 1e-6 and O.rel_l2(b[1], a[1]) < 1e-6


def test_seeded_inputs_are_deterministic():
    a = make_inputs(CONFIGS["c1"], random_gates=True, with_grad_out=True)
    b = make_inputs(CONFIGS["c1"], random_gates=True, with_grad_out=True)
    for k in a:
        assert torch.equal(a[k], b[k])
        assert a[k].dtype == torch.float16


def test_gradcheck_projections_and_diagonal_mask_fp64():
    """Autograd of the oracle with the HardTanh01 / Identity projections and the diagonal
    mask matches finite differences (the kinks of HardTanh01 at z = +-1 are not hit)."""
    for projection, causal, mask_diag in (("hardtanh01", False, False), ("identity", True, False),
                                          ("sigmoid", False, True), ("hardtanh01", True, True)):
        cfg = TINY.with_(causal=causal)
        inp = _inputs(cfg)
        args = [inp[k].clone().requires_grad_(True) for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")]

        def f(*a):
            out, lse = O.forward(*a, cfg.H, cfg.cube_m, cfg.scale, cfg.causal, projection=projection,
                                 mask_diag=mask_diag)
            return out, lse.clamp_min(-1e30)

        assert torch.autograd.gradcheck(f, args, eps=1e-6, atol=1e-6), (projection, causal, mask_diag)


def test_hardtanh01_gradient_is_strict():
    """Gradient 1/2 strictly inside -1 < z < 1, 0 at and beyond the ends (cube.cuh:33-35)."""
    z = torch.tensor([-2.0, -1.0, -0.5, 0.0, 0.999, 1.0, 3.0], dtype=torch.float64, requires_grad=True)
    phi = O.cube_project(z, "hardtanh01")
    phi.sum().backward()
    assert torch.equal(phi.detach(), torch.tensor([0.0, 0.0, 0.25, 0.5, 0.9995, 1.0, 1.0], dtype=torch.float64))
    assert torch.equal(z.grad, torch.tensor([0.0, 0.0, 0.5, 0.5, 0.5, 0.0, 0.0], dtype=torch.float64))


def test_diagonal_mask_rows():
    """With the diagonal mask every query loses its own key; with causal masking as well,
    query 0 has no key left: out = 0, lse = -FLT_MAX, and it passes no gradient."""
    cfg = TINY.with_(causal=True)
    inp = _inputs(cfg)
    r = O.forward_backward(inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], cfg.H, cfg.cube_m,
                           cfg.scale, True, dtype=torch.float64, mask_diag=True)
    lse = r["lse"].view(cfg.B, cfg.H, cfg.N)
    assert torch.all(lse[:, :, 0] == O.FLT_LOWEST)
    assert torch.all(torch.isfinite(lse[:, :, 1:]))
    assert torch.all(r["out"][:, 0] == 0)
    # query 1 attends to key 0 only: its output is head-wise V of token 0
    v = (inp["x"] @ inp["W_V"])
    assert torch.allclose(r["out"][:, 1], v[:, 0], atol=1e-12)
    for k in ("dX", "dW_phi", "d_gate_q", "d_gate_k", "dW_V"):
        assert torch.all(torch.isfinite(r[k]))
