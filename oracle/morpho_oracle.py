"""CPU oracle for the MorphoAttention forward and backward.

TEST INFRASTRUCTURE ONLY.  This module is the checker for the CUDA product path.
Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl
reference`` legs of ``bench.py`` may import it.  The product package never does.

It is an fp32 (or fp64) eager restatement of the reference algorithm.  The reference
ships no eager formulation: its only implementation is the WMMA CUDA kernel pair, so
every step below cites the line of that kernel it restates.  Paths are relative to
the reference project root (``packages/morphottention/...``).

Math, per head ``h`` with token features ``x`` [N, D]:

* ``z = x @ W_phi[:, h*m:(h+1)*m]`` and ``phi = sigmoid(z)``
  (``csrc/cuda/sm120/project.cuh:26-34``, ``csrc/cuda/morfology/cube.cuh:12-14``), or
  the reference's other compile-time projections ``hardtanh01(z) = min(1, max(0, (z+1)/2))``
  with gradient 1/2 on ``-1 < z < 1`` only, and ``identity`` (``cube.cuh:15-45``)
* ``q = gate_q[h] * phi``, ``k = gate_k[h] * phi`` (``project.cuh:36-37``)
* ``qbias_i = sum_c gate_k[c] q_ic`` and ``cbias_j = sum_c gate_q[c] k_jc``
  (``project.cuh:39-44``; called with swapped gates at ``attention.cu:78-79``, ``:102-103``)
* ``S_ij = scale * (2 q_i.k_j - qbias_i - cbias_j)`` (``attention.cu:125``), causal mask
  ``j > i`` (``attention.cu:129-130``), optional diagonal mask ``j == i``
  (``MORPHO_MASK_DIAG``, ``attention.cu:131-132``), softmax over j (``attention.cu:138-158``).
  A row with every key masked (causal plus diagonal mask at i = 0) is defined here as
  ``out = 0``, ``lse = -FLT_MAX`` and no gradient; the reference kernel's forward instead
  turns such a row into a uniform average (all its scores are ``-FLT_MAX``)
* ``V = x @ W_V[:, h*hd:(h+1)*hd]`` (``attention.cu:106-111``) and
  ``out[:, :, h*hd:(h+1)*hd] = P @ V`` (``attention.cu:163-183``)
* ``lse[b*H+h, i]`` in the log2 domain: ``max_j(s_ij) + log2(sum_j 2^(s_ij - max))``
  with ``s = S * log2(e)`` (``attention.cu:186``), i.e. ``logsumexp(S_i) * log2(e)``.

Gradient modes:

* ``"full"``: true autograd of the math above.  This is the accuracy target.
* ``"reference"``: the reference backward kernel's semantics.  That kernel
  accumulates the query-side code gradient (``attention.cu:447-451``) and the
  query-bias gradient (``attention.cu:425``) but never propagates them: no
  ``project_phi_bwd`` runs for the query rows and the query-row ``dX`` accumulator
  stays zero (``attention.cu:265-267``, ``:473-482``).  So ``dX``, ``dW_phi``,
  ``d_gate_q`` and ``d_gate_k`` miss every term that flows through ``q`` and
  ``qbias``.  Detaching ``q`` and ``qbias`` reproduces that exactly; ``out``, ``lse``
  and ``dW_V`` are the same in both modes.
"""

from __future__ import annotations

import torch

LOG2E = 1.4426950408889634  # csrc/cuda/utils/declarations.cuh:7

GRAD_MODES = ("full", "reference")
PROJECTIONS = ("sigmoid", "hardtanh01", "identity")
FLT_LOWEST = -3.4028234663852886e38


class _HardTanh01(torch.autograd.Function):
    """``min(1, max(0, (z+1)/2))`` with the reference's gradient: 1/2 strictly inside
    ``-1 < z < 1``, else 0 (``cube.cuh:15-17``, ``:33-35``)."""

    @staticmethod
    def forward(ctx, z):
        ctx.save_for_backward(z)
        return (0.5 * (z + 1.0)).clamp(0.0, 1.0)

    @staticmethod
    def backward(ctx, g):
        (z,) = ctx.saved_tensors
        return g * ((z > -1.0) & (z < 1.0)).to(g.dtype) * 0.5


def cube_project(z, projection: str = "sigmoid"):
    if projection == "sigmoid":
        return torch.sigmoid(z)
    if projection == "hardtanh01":
        return _HardTanh01.apply(z)
    if projection == "identity":
        return z
    raise ValueError(f"projection must be one of {PROJECTIONS}")


def project(x, W_phi, gate_q, gate_k, W_V, H: int, cube_m: int, projection: str = "sigmoid"):
    """Per-head hypercube codes, biases and values.

    Restates ``project_phi`` (``csrc/cuda/sm120/project.cuh:16-47``) and the value
    projection (``csrc/cuda/attention/attention.cu:106-111``).
    Returns ``phi, q, k, qbias, cbias, v`` with shapes
    ``[B,H,N,m] x3, [B,H,N] x2, [B,H,N,hd]``.
    """
    B, N, _ = x.shape
    hd = W_V.shape[1] // H
    z = (x @ W_phi).view(B, N, H, cube_m).permute(0, 2, 1, 3)  # [B,H,N,m]
    phi = cube_project(z, projection)
    gq = gate_q.view(1, H, 1, cube_m)
    gk = gate_k.view(1, H, 1, cube_m)
    q = gq * phi
    k = gk * phi
    qbias = (gk * q).sum(-1)
    cbias = (gq * k).sum(-1)
    v = (x @ W_V).view(B, N, H, hd).permute(0, 2, 1, 3)  # [B,H,N,hd]
    return phi, q, k, qbias, cbias, v


def _attend(q, k, qbias, cbias, v, scale: float, causal: bool, mask_diag: bool = False):
    """Score, mask, softmax and P.V; ``attention.cu:113-188``."""
    N = q.shape[2]
    s = scale * (2.0 * (q @ k.transpose(-1, -2)) - qbias.unsqueeze(-1) - cbias.unsqueeze(-2))
    mask = None
    if causal:
        mask = torch.ones(N, N, dtype=torch.bool, device=q.device).triu(1)
    if mask_diag:
        eye = torch.eye(N, dtype=torch.bool, device=q.device)
        mask = eye if mask is None else (mask | eye)
    if mask is None:
        p = torch.softmax(s, dim=-1)
        lse2 = torch.logsumexp(s, dim=-1) * LOG2E  # [B,H,N], log2 domain
    else:
        s = s.masked_fill(mask, float("-inf"))
        dead = mask.all(dim=-1)  # rows without any key
        s_safe = s.masked_fill(dead.unsqueeze(-1), 0.0)
        p = torch.softmax(s_safe, dim=-1).masked_fill(dead.unsqueeze(-1), 0.0)
        lse2 = (torch.logsumexp(s_safe, dim=-1) * LOG2E).masked_fill(dead, FLT_LOWEST)
    o = p @ v  # [B,H,N,hd]
    return o, lse2


def forward(x, W_phi, gate_q, gate_k, W_V, H: int, cube_m: int, scale: float = 1.0,
            causal: bool = False, grad_mode: str = "full", projection: str = "sigmoid", mask_diag: bool = False):
    """Eager forward.  Returns ``(out [B,N,D], lse [B*H,N])`` like ``morphottention::forward``
    (``csrc/cuda/binder.cpp:7-8``, ``csrc/cuda/attention/attention.cpp:40-56``).

    ``grad_mode="reference"`` detaches the query codes and the query bias so that a
    later ``backward`` matches the reference kernel's gradient semantics.
    """
    if grad_mode not in GRAD_MODES:
        raise ValueError(f"grad_mode must be one of {GRAD_MODES}")
    B, N, D = x.shape
    _, q, k, qbias, cbias, v = project(x, W_phi, gate_q, gate_k, W_V, H, cube_m, projection)
    if grad_mode == "reference":
        q = q.detach()
        qbias = qbias.detach()
    o, lse2 = _attend(q, k, qbias, cbias, v, scale, causal, mask_diag)
    out = o.permute(0, 2, 1, 3).reshape(B, N, D)
    return out, lse2.reshape(B * H, N)


def forward_backward(x, W_phi, gate_q, gate_k, W_V, H: int, cube_m: int, scale: float = 1.0,
                     causal: bool = False, grad_out=None, grad_mode: str = "full",
                     dtype=torch.float32, projection: str = "sigmoid", mask_diag: bool = False):
    """Forward plus the backward of ``sum(out * grad_out)`` (``out.sum()`` when
    ``grad_out`` is None).  Returns a dict with ``out, lse, dX, dW_phi, d_gate_q,
    d_gate_k, dW_V`` in ``dtype`` on the inputs' device.
    """
    leaves = [t.detach().to(dtype).clone().requires_grad_(True) for t in (x, W_phi, gate_q, gate_k, W_V)]
    with torch.enable_grad():
        out, lse = forward(*leaves, H, cube_m, scale, causal, grad_mode, projection, mask_diag)
        g = torch.ones_like(out) if grad_out is None else grad_out.detach().to(dtype)
        grads = torch.autograd.grad(out, leaves, grad_outputs=g)
    names = ("dX", "dW_phi", "d_gate_q", "d_gate_k", "dW_V")
    res = {"out": out.detach(), "lse": lse.detach()}
    res.update({n: gr.detach() for n, gr in zip(names, grads)})
    return res


def forward_chunked(x, W_phi, gate_q, gate_k, W_V, H: int, cube_m: int, scale: float = 1.0,
                    causal: bool = False, heads_per_chunk: int = 1):
    """Forward only, looping over heads so that the ``N x N`` score matrix of one head is
    the largest temporary.  Used for CPU timing at long sequence lengths."""
    B, N, D = x.shape
    hd = D // H
    out = torch.empty(B, N, D, dtype=x.dtype)
    lse = torch.empty(B * H, N, dtype=torch.float32)
    for h0 in range(0, H, heads_per_chunk):
        h1 = min(H, h0 + heads_per_chunk)
        cols = slice(h0 * cube_m, h1 * cube_m)
        sub_phi = W_phi[:, cols]
        sub_v = W_V[:, h0 * hd:h1 * hd]
        _, q, k, qb, cb, v = project(x, sub_phi, gate_q[h0:h1], gate_k[h0:h1], sub_v, h1 - h0, cube_m)
        o, l2 = _attend(q, k, qb, cb, v, scale, causal)
        out[:, :, h0 * hd:h1 * hd] = o.permute(0, 2, 1, 3).reshape(B, N, (h1 - h0) * hd)
        lse.view(B, H, N)[:, h0:h1] = l2
    return out, lse


def rel_l2(a, b) -> float:
    """Relative L2 error ``||a - b|| / ||b||`` in fp64 (``b`` is the reference)."""
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    den = b.norm().item()
    num = (a - b).norm().item()
    if den == 0.0:
        return num
    return num / den


def soft_hamming_score(phi_i, phi_j, gate_q, gate_k, scale: float):
    """Closed form of the score as a gated soft-Hamming (XOR) distance:
    ``-scale * sum_c gq_c gk_c (phi_ic (1 - phi_jc) + phi_jc (1 - phi_ic))``.
    Used by the tests to check the dot-product form of ``attention.cu:125``."""
    w = gate_q * gate_k
    a = phi_i.unsqueeze(-2)
    b = phi_j.unsqueeze(-3)
    return -scale * (w * (a * (1 - b) + b * (1 - a))).sum(-1)


__all__ = ["LOG2E", "GRAD_MODES", "project", "forward", "forward_backward", "forward_chunked",
           "rel_l2", "soft_hamming_score"]


SCORES = ("softmax", "dilation", "erosion")


def soft_morph_forward(x, W_phi, gate_q, gate_k, W_V, H: int, cube_m: int, scale: float = 1.0,
                       causal: bool = False, score: str = "dilation", tau: float = 1.0,
                       projection: str = "sigmoid", mask_diag: bool = False):
    """The soft-morphology score of ``csrc/cuda/morfology/soft_morph.cuh:10-77`` (dead code in
    the reference: no kernel calls it) in place of softmax . V:
    ``out[i, c] = sgn * tau * logsumexp_j(sgn * (S_ij + V_jc) / tau)``, a soft max-plus
    (``dilation``, sgn = +1) or min-plus (``erosion``, sgn = -1) aggregation of the values
    over the keys (``morph_accumulate`` / ``lse_finalize``, ``:33-61``), with the
    morphological score ``S_ij = scale * (2 q_i.k_j - qbias_i - cbias_j)`` of the attention
    path.  Masked keys (causal, diagonal, padding) are left out; a row without keys gives 0.
    Returns ``out [B,N,D]``.  The gradient w.r.t. S and V is ``P_ijc = exp(sgn (S_ij + V_jc -
    out_ic) / tau)`` (``morph_weight``, ``:63-67``); ``tau`` is a fixed hyper-parameter here.
    """
    if score not in ("dilation", "erosion"):
        raise ValueError("score must be 'dilation' or 'erosion'")
    sgn = 1.0 if score == "dilation" else -1.0
    B, N, D = x.shape
    _, q, k, qbias, cbias, v = project(x, W_phi, gate_q, gate_k, W_V, H, cube_m, projection)
    s = scale * (2.0 * (q @ k.transpose(-1, -2)) - qbias.unsqueeze(-1) - cbias.unsqueeze(-2))  # [B,H,N,N]
    a = sgn * (s.unsqueeze(-1) + v.unsqueeze(-3)) / tau  # [B,H,N(i),N(j),hd]
    mask = None
    if causal:
        mask = torch.ones(N, N, dtype=torch.bool, device=x.device).triu(1)
    if mask_diag:
        eye = torch.eye(N, dtype=torch.bool, device=x.device)
        mask = eye if mask is None else (mask | eye)
    if mask is not None:
        a = a.masked_fill(mask.unsqueeze(-1), float("-inf"))
        dead = mask.all(dim=-1)  # [N]
        a = a.masked_fill(dead.view(N, 1, 1), 0.0)
        o = sgn * tau * torch.logsumexp(a, dim=-2)
        o = o.masked_fill(dead.view(N, 1), 0.0)
    else:
        o = sgn * tau * torch.logsumexp(a, dim=-2)  # [B,H,N,hd]
    return o.permute(0, 2, 1, 3).reshape(B, N, D)


def soft_morph_forward_backward(x, W_phi, gate_q, gate_k, W_V, H: int, cube_m: int, scale: float = 1.0,
                                causal: bool = False, score: str = "dilation", tau: float = 1.0, grad_out=None,
                                dtype=torch.float32, projection: str = "sigmoid", mask_diag: bool = False,
                                tau_grad: bool = False):
    """Forward plus the backward of ``sum(out * grad_out)`` for :func:`soft_morph_forward`.  With
    ``tau_grad`` the temperature is a leaf too and ``res["d_tau"]`` is ``dL/dtau``, the sum over
    (i, c) of ``grad_out_ic (out_ic - sum_j P_ijc (S_ij + V_jc)) / tau``
    (``csrc/cuda/morfology/soft_morph.cuh:67-77``), here by autograd."""
    leaves = [t.detach().to(dtype).clone().requires_grad_(True) for t in (x, W_phi, gate_q, gate_k, W_V)]
    tau_t = torch.tensor(float(tau), dtype=dtype, requires_grad=True) if tau_grad else tau
    with torch.enable_grad():
        out = soft_morph_forward(*leaves, H, cube_m, scale, causal, score, tau_t, projection, mask_diag)
        g = torch.ones_like(out) if grad_out is None else grad_out.detach().to(dtype)
        grads = torch.autograd.grad(out, leaves + ([tau_t] if tau_grad else []), grad_outputs=g)
    names = ("dX", "dW_phi", "d_gate_q", "d_gate_k", "dW_V") + (("d_tau",) if tau_grad else ())
    res = {"out": out.detach()}
    res.update({n: gr.detach() for n, gr in zip(names, grads)})
    return res


def soft_morph_dtau_terms(x, W_phi, gate_q, gate_k, W_V, H: int, cube_m: int, scale: float = 1.0,
                          causal: bool = False, score: str = "dilation", tau: float = 1.0, grad_out=None,
                          mask_diag: bool = False, dtype=torch.float64):
    """The three sums whose difference is ``tau * dL/dtau`` (``soft_morph.cuh:67-77`` regrouped):
    ``(sum dO.out, sum_ij S_ij dL/dS_ij, sum_jc V_jc dL/dV_jc)``, by autograd through the score
    and the values.  Tests judge a computed ``dL/dtau`` against the size of these terms, since
    they cancel (sigmoid projection)."""
    sgn = 1.0 if score == "dilation" else -1.0
    args = [t.detach().to(dtype) for t in (x, W_phi, gate_q, gate_k, W_V)]
    B, N, D = args[0].shape
    _, q, k, qbias, cbias, v = project(*args, H, cube_m)
    s = (scale * (2.0 * (q @ k.transpose(-1, -2)) - qbias.unsqueeze(-1) - cbias.unsqueeze(-2))).detach()
    v = v.detach()
    s.requires_grad_(True)
    v.requires_grad_(True)
    mask = torch.zeros(N, N, dtype=torch.bool)
    if causal:
        mask |= torch.ones(N, N, dtype=torch.bool).triu(1)
    if mask_diag:
        mask |= torch.eye(N, dtype=torch.bool)
    g = torch.ones(B, N, D, dtype=dtype) if grad_out is None else grad_out.detach().to(dtype)
    with torch.enable_grad():
        a = sgn * (s.unsqueeze(-1) + v.unsqueeze(-3)) / tau
        a = a.masked_fill(mask.unsqueeze(-1), float("-inf"))
        dead = mask.all(dim=-1)
        a = a.masked_fill(dead.view(N, 1, 1), 0.0)
        o = (sgn * tau * torch.logsumexp(a, dim=-2)).masked_fill(dead.view(N, 1), 0.0)
        out = o.permute(0, 2, 1, 3).reshape(B, N, D)
        gs, gv = torch.autograd.grad(out, (s, v), grad_outputs=g)
    return (float((g * out).sum()), float((s.masked_fill(mask, 0.0) * gs).sum()), float((v * gv).sum()))
