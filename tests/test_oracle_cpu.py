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


def _split_soft_morph(x, W_phi, gate_q, gate_k, W_V, H, cube_m, scale, score, tau, dtype):
    """The soft-morphology aggregation through the split the CUDA path uses (log2 units):
    sum_j 2^(x_ij + y_jc) = 2^(m_i + R_c) (E_S . E_V)_ic with E_S = 2^(x - m), E_V = 2^(y - R),
    m_i the row maximum of x, R_c the column maximum of y; returns out and the accumulators."""
    sgn = 1.0 if score == "dilation" else -1.0
    B, N, D = x.shape
    _, q, k, qbias, cbias, v = O.project(x, W_phi, gate_q, gate_k, W_V, H, cube_m)
    s = scale * (2.0 * (q @ k.transpose(-1, -2)) - qbias.unsqueeze(-1) - cbias.unsqueeze(-2))
    log2e = 1.4426950408889634
    xs = (sgn * s * log2e / tau).to(dtype)
    ys = (sgn * v * log2e / tau).to(dtype)
    m = xs.amax(dim=-1, keepdim=True)
    R = ys.amax(dim=-2, keepdim=True)
    acc = torch.exp2(xs - m) @ torch.exp2(ys - R)
    t = m + R + torch.log2(acc)
    out = sgn * tau * 0.6931471805599453 * t
    return out.permute(0, 2, 1, 3).reshape(B, N, D), acc


def test_soft_morph_split_identity():
    """The split of the exponential (softmorph_tc.cu, softmorph_tc_bwd.cu) reproduces the
    direct log-sum-exp of the oracle: in float64 to 1e-12 relative, in float32 to 1e-5."""
    cfg = MorphoConfig("split", 1, 48, 64, 2, 16, 0.7, False, 21)
    inp = {k: v.double() for k, v in make_inputs(cfg, device="cpu", random_gates=True).items()}
    args = (inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], cfg.H, cfg.cube_m)
    for score, tau in (("dilation", 1.0), ("erosion", 0.4)):
        ref = O.soft_morph_forward(*args, scale=cfg.scale, score=score, tau=tau)
        out64, _ = _split_soft_morph(*args, cfg.scale, score, tau, torch.float64)
        assert O.rel_l2(out64, ref) < 1e-12
        out32, acc32 = _split_soft_morph(*args, cfg.scale, score, tau, torch.float32)
        assert O.rel_l2(out32.double(), ref) < 1e-5
        assert acc32.min() >= 2.0 ** -90  # the guard's floor holds: the split path is taken


def test_soft_morph_split_guard_floor():
    """With tau small enough that a dominant term lies more than 90 log2 units below its two
    stabilisers, the float32 accumulator falls below 2^-90 (or to 0): the CUDA path's guard
    then hands the problem to the exact kernels."""
    cfg = MorphoConfig("guard", 1, 48, 64, 2, 16, 1.0, False, 22)
    inp = {k: v.double() for k, v in make_inputs(cfg, device="cpu", random_gates=True).items()}
    args = (inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], cfg.H, cfg.cube_m)
    _, acc32 = _split_soft_morph(*args, cfg.scale, "dilation", 0.005, torch.float32)
    assert acc32.min() < 2.0 ** -90


def test_soft_morph_tau_gradient_pinned():
    """dL/dtau of the soft-morphology score: the oracle's autograd value against a central finite
    difference in float64, and the decomposition the kernels use,
    tau dL/dtau = sum dO.out - sum_ij S_ij dL/dS_ij - sum_jc V_jc dL/dV_jc
    (dL/dS and dL/dV by autograd through S and V), for dilation and erosion, causal."""
    import torch

    from morphottention_b200.configs import MorphoConfig, make_inputs
    from oracle import morpho_oracle as O
    cfg = MorphoConfig("tau", 1, 24, 32, 2, 16, 0.7, True, 61)
    inp = {k: v.double() for k, v in make_inputs(cfg, random_gates=True, with_grad_out=True).items()}
    g = inp.pop("grad_out")
    args = [inp[k] for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")]
    for score, tau in (("dilation", 0.8), ("erosion", 1.3)):
        r = O.soft_morph_forward_backward(*args, cfg.H, cfg.cube_m, cfg.scale, cfg.causal, score, tau, grad_out=g,
                                          dtype=torch.float64, tau_grad=True)
        h = 1e-5
        fp = (O.soft_morph_forward(*args, cfg.H, cfg.cube_m, cfg.scale, cfg.causal, score, tau + h) * g).sum()
        fm = (O.soft_morph_forward(*args, cfg.H, cfg.cube_m, cfg.scale, cfg.causal, score, tau - h) * g).sum()
        fd = float((fp - fm) / (2 * h))
        assert abs(float(r["d_tau"]) - fd) <= 1e-6 * max(1.0, abs(fd)), (score, float(r["d_tau"]), fd)
        # the decomposition through the score and value gradients
        sgn = 1.0 if score == "dilation" else -1.0
        B, N, D = args[0].shape
        _, q, k, qbias, cbias, v = O.project(*args, cfg.H, cfg.cube_m)
        s = (cfg.scale * (2.0 * (q @ k.transpose(-1, -2)) - qbias.unsqueeze(-1) - cbias.unsqueeze(-2))).detach()
        v = v.detach()
        s.requires_grad_(True)
        v.requires_grad_(True)
        a = sgn * (s.unsqueeze(-1) + v.unsqueeze(-3)) / tau
        mask = torch.ones(N, N, dtype=torch.bool).triu(1)
        a = a.masked_fill(mask.unsqueeze(-1), float("-inf"))
        out = (sgn * tau * torch.logsumexp(a, dim=-2)).permute(0, 2, 1, 3).reshape(B, N, D)
        gs, gv = torch.autograd.grad(out, (s, v), grad_outputs=g)
        decomposed = ((g * out).sum() - (s.masked_fill(mask, 0.0) * gs).sum() - (v * gv).sum()) / tau
        assert abs(float(decomposed) - float(r["d_tau"])) <= 1e-9 * max(1.0, abs(fd)), score
