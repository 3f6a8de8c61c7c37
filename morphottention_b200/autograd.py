"""Autograd wrapper and ``nn.Module`` around the sm_100a MorphoAttention kernels.

Drop-in for the reference's ``torch-ext/morphottention/autograd.py``: the same
``MorphoAttention`` constructor (``:101-135``), the same ``MorphoAttentionFunction``
(``:34-88``) and ``morpho_attention`` (``:143-162``), calling the same
``torch.ops.morphottention.forward/backward`` schemas.  Additions: a fake (meta)
implementation for ``backward``, :func:`set_grad_mode`, and -- when a gradient is needed --
the ``forward_save`` / ``backward_saved`` op pair, which keeps the forward's projection
(codes, values, biases, phi) for the backward instead of recomputing it.  Gradients are
bit-identical either way; the kept buffer costs ``morpho_sm100_saved_bytes`` of memory per
call until the backward runs.

The variant options (gradient mode, cube projection, diagonal mask, score and tau) are
process-wide settings, read once when a forward runs: the autograd Function stores them with
the forward and passes them explicitly to its backward, so a backward that runs after the
settings changed (outside an :func:`attention_options` block, say) still differentiates the
forward that ran.
"""

from __future__ import annotations

import contextlib

import torch
from torch import nn

from ._ops import add_op_namespace_prefix, ops

GRAD_MODES = {"full": 0, "reference": 1}


@torch.library.register_fake(add_op_namespace_prefix("forward"))
def _morpho_forward_fake(X, W_phi, gate_q, gate_k, W_V, H: int, cube_m: int, scale: float, causal: bool):
    B, N, _D = X.shape
    out = torch.empty_like(X)
    lse = X.new_empty((B * H, N), dtype=torch.float32)
    return [out, lse]


@torch.library.register_fake(add_op_namespace_prefix("backward"))
def _morpho_backward_fake(grad_out, X, W_phi, gate_q, gate_k, W_V, out, lse, H: int, cube_m: int, scale: float,
                          causal: bool):
    return [torch.empty_like(X), torch.empty_like(W_phi), torch.empty_like(gate_q), torch.empty_like(gate_k),
            torch.empty_like(W_V)]


@torch.library.register_fake(add_op_namespace_prefix("forward_save"))
def _morpho_forward_save_fake(X, W_phi, gate_q, gate_k, W_V, H: int, cube_m: int, scale: float, causal: bool,
                              projection: int, mask_diag: int, score: int, tau: float):
    from . import capi
    B, N, D = X.shape
    nbytes = capi.saved_bytes(capi.problem(B, N, D, H, cube_m, scale, causal, projection=projection,
                                           mask_diag=mask_diag, score=score, tau=tau))
    return [torch.empty_like(X), X.new_empty((B * H, N), dtype=torch.float32),
            X.new_empty((nbytes,), dtype=torch.uint8)]


@torch.library.register_fake(add_op_namespace_prefix("backward_saved"))
def _morpho_backward_saved_fake(grad_out, saved, X, W_phi, gate_q, gate_k, W_V, out, lse, H: int, cube_m: int,
                                scale: float, causal: bool, grad_mode: int, projection: int, mask_diag: int,
                                score: int, tau: float):
    return [torch.empty_like(X), torch.empty_like(W_phi), torch.empty_like(gate_q), torch.empty_like(gate_k),
            torch.empty_like(W_V)]


@torch.library.register_fake(add_op_namespace_prefix("backward_saved_tau"))
def _morpho_backward_saved_tau_fake(grad_out, saved, X, W_phi, gate_q, gate_k, W_V, out, lse, H: int, cube_m: int,
                                    scale: float, causal: bool, grad_mode: int, projection: int, mask_diag: int,
                                    score: int, tau: float):
    return [torch.empty_like(X), torch.empty_like(W_phi), torch.empty_like(gate_q), torch.empty_like(gate_k),
            torch.empty_like(W_V), X.new_empty((), dtype=torch.float32)]


def set_grad_mode(mode: str) -> str:
    """Select the backward's gradient semantics process-wide and return the previous one.

    ``"full"`` (default): the true gradient of the forward.  ``"reference"``: the
    reference kernel's semantics, which never propagate the query-code and query-bias
    gradients (reference ``csrc/cuda/attention/attention.cu:447-451``, ``:473-482``), so
    ``dX``, ``dW_phi`` and the gate gradients lack every term through the query side.
    """
    if mode not in GRAD_MODES:
        raise ValueError(f"grad mode must be one of {sorted(GRAD_MODES)}")
    prev = int(ops.set_grad_mode(GRAD_MODES[mode]))
    return {v: k for k, v in GRAD_MODES.items()}[prev]


def get_grad_mode() -> str:
    return {v: k for k, v in GRAD_MODES.items()}[int(ops.get_grad_mode())]


CUBE_PROJECTIONS = {"sigmoid": 0, "hardtanh01": 1, "identity": 2}


def set_cube_projection(proj: str) -> str:
    """Select the hypercube projection phi = proj(x @ W_phi) for subsequent calls:
    ``"sigmoid"`` (default), ``"hardtanh01"`` (``min(1, max(0, (z + 1) / 2))``) or
    ``"identity"``.  The reference picks one at compile time
    (``csrc/cuda/morfology/cube.cuh:10-45``).  Process-wide; returns the previous one."""
    if proj not in CUBE_PROJECTIONS:
        raise ValueError(f"cube projection must be one of {tuple(CUBE_PROJECTIONS)}")
    prev = int(ops.set_cube_projection(CUBE_PROJECTIONS[proj]))
    return {v: k for k, v in CUBE_PROJECTIONS.items()}[prev]


def get_cube_projection() -> str:
    return {v: k for k, v in CUBE_PROJECTIONS.items()}[int(ops.get_cube_projection())]


def set_mask_diag(on: bool) -> bool:
    """Also mask key j == query i (the reference's compile-time ``MORPHO_MASK_DIAG``,
    ``csrc/cuda/utils/declarations.cuh:79-82``) in subsequent calls.  A query row left
    without any key gets ``out = 0``, ``lse = -FLT_MAX`` and no gradient.  Process-wide;
    returns the previous setting."""
    return bool(ops.set_mask_diag(1 if on else 0))


def get_mask_diag() -> bool:
    return bool(ops.get_mask_diag())


SCORES = {"softmax": 0, "dilation": 1, "erosion": 2}


def set_score(score: str, tau: float = 1.0) -> tuple:
    """Select how the keys are aggregated for subsequent calls: ``"softmax"`` (attention,
    the default), or the soft-morphology score of the reference's
    ``csrc/cuda/morfology/soft_morph.cuh`` (unused there): ``"dilation"``,
    ``out_ic = tau * logsumexp_j((S_ij + V_jc) / tau)``, and ``"erosion"``, its min-plus mirror.
    ``tau`` is a fixed temperature (no gradient).  Process-wide; returns the previous
    ``(score, tau)``."""
    if score not in SCORES:
        raise ValueError(f"score must be one of {tuple(SCORES)}")
    prev = get_score()
    ops.set_score(SCORES[score], float(tau))
    return prev


def get_score() -> tuple:
    return {v: k for k, v in SCORES.items()}[int(ops.get_score())], float(ops.get_score_tau())


def current_options() -> tuple:
    """The settings the next forward runs with, as the integer codes of the C ABI:
    ``(grad_mode, projection, mask_diag, score, tau)``."""
    g, p, m, sc, tau = ops.get_options()
    return int(g), int(p), int(m), int(sc), float(tau)


@contextlib.contextmanager
def attention_options(projection: str | None = None, mask_diag: bool | None = None, score: str | None = None,
                      tau: float = 1.0):
    """Scoped :func:`set_cube_projection` / :func:`set_mask_diag` / :func:`set_score`."""
    prev_p = set_cube_projection(projection) if projection is not None else None
    prev_m = set_mask_diag(mask_diag) if mask_diag is not None else None
    prev_s = set_score(score, tau) if score is not None else None
    try:
        yield
    finally:
        if prev_p is not None:
            set_cube_projection(prev_p)
        if prev_m is not None:
            set_mask_diag(prev_m)
        if prev_s is not None:
            set_score(*prev_s)


@contextlib.contextmanager
def grad_mode(mode: str):
    prev = set_grad_mode(mode)
    try:
        yield
    finally:
        set_grad_mode(prev)


class MorphoAttentionFunction(torch.autograd.Function):
    """``torch.autograd.Function`` over the torch ops: the forward keeps what the backward
    reads (the projection buffer, out, lse, and the variant options of this call), the
    backward returns the five gradients followed by ``None`` for the four non-tensor arguments."""

    @staticmethod
    def forward(ctx, x, W_phi, gate_q, gate_k, W_V, H: int, cube_m: int, scale: float, causal: bool):
        if not x.is_cuda:
            raise ValueError("MorphoAttention expects a CUDA tensor")
        x = x.contiguous()
        if any(ctx.needs_input_grad[:5]):
            # the variant this forward runs is the one its backward differentiates
            ctx.options = current_options()
            _g, proj, mdiag, score, tau = ctx.options
            out, lse, saved = ops.forward_save(x, W_phi, gate_q, gate_k, W_V, H, cube_m, scale, causal, proj, mdiag,
                                               score, tau)
            ctx.save_for_backward(x, W_phi, gate_q, gate_k, W_V, out, lse, saved)
        else:
            out, lse = ops.forward(x, W_phi, gate_q, gate_k, W_V, H, cube_m, scale, causal)
        ctx.H = H
        ctx.cube_m = cube_m
        ctx.scale = scale
        ctx.causal = causal
        return out

    @staticmethod
    def backward(ctx, grad_out):
        x, W_phi, gate_q, gate_k, W_V, out, lse, saved = ctx.saved_tensors
        grad_out = grad_out.contiguous()
        dX, dW_phi, d_gate_q, d_gate_k, dW_V = ops.backward_saved(
            grad_out, saved, x, W_phi, gate_q, gate_k, W_V, out, lse, ctx.H, ctx.cube_m, ctx.scale, ctx.causal,
            *ctx.options)
        return dX, dW_phi, d_gate_q, d_gate_k, dW_V, None, None, None, None


class MorphoAttention(nn.Module):
    """Attention layer whose query-key score is a gated soft-Hamming distance between per-head
    sigmoid codes in the unit hypercube (no output projection inside the layer).

    :param dim: width ``D`` of the token features; ``num_heads`` must divide it.
    :param num_heads: head count ``H``; each head's values span ``D / H`` features.
    :param cube_m: code length ``m`` of each head (16, 32 or 64): ``W_phi`` maps ``D`` to
        ``H * m`` codes.
    :param scale: factor applied to the score before the softmax.
    :param causal: drop keys that come after the query.
    :param dtype: parameter dtype (the kernels take float16).
    :param device: where the parameters live.
    """

    def __init__(self, dim: int, num_heads: int, cube_m: int, *, scale: float = 1.0, causal: bool = False,
                 dtype: torch.dtype = torch.float16, device=None) -> None:
        super().__init__()
        if dim % num_heads != 0:
            raise ValueError(f"dim ({dim}) must be divisible by num_heads ({num_heads})")
        self.dim = dim
        self.num_heads = num_heads
        self.cube_m = cube_m
        self.scale = scale
        self.causal = causal
        head_dim_v = dim // num_heads
        self.W_phi = nn.Parameter(torch.empty(dim, num_heads * cube_m, dtype=dtype, device=device))
        self.gate_q = nn.Parameter(torch.empty(num_heads, cube_m, dtype=dtype, device=device))
        self.gate_k = nn.Parameter(torch.empty(num_heads, cube_m, dtype=dtype, device=device))
        self.W_V = nn.Parameter(torch.empty(dim, num_heads * head_dim_v, dtype=dtype, device=device))
        self.reset_parameters()

    def reset_parameters(self) -> None:
        std = self.dim ** -0.5
        with torch.no_grad():
            for w in (self.W_phi, self.W_V):
                w.copy_(torch.empty(w.shape, dtype=torch.float32, device=w.device).normal_(0.0, std))
            self.gate_q.fill_(1.0)
            self.gate_k.fill_(1.0)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return MorphoAttentionFunction.apply(
            x, self.W_phi, self.gate_q, self.gate_k, self.W_V, self.num_heads, self.cube_m, self.scale, self.causal)


def morpho_attention(x, W_phi, gate_q, gate_k, W_V, num_heads: int, cube_m: int, *, scale: float = 1.0,
                     causal: bool = False):
    """Functional form of :class:`MorphoAttention` with the parameters passed in.

    :param x: float16 CUDA tensor ``[B, N, D]``.
    :returns: ``[B, N, D]``; gradients flow to ``x``, ``W_phi``, ``gate_q``, ``gate_k`` and ``W_V``.
    """
    return MorphoAttentionFunction.apply(x, W_phi, gate_q, gate_k, W_V, num_heads, cube_m, scale, causal)


class SoftMorphAttentionFunction(torch.autograd.Function):
    """The soft-morphology score (dilation or erosion) with the temperature as a tensor input, so
    that ``tau`` can be learned: its gradient ``dL/dtau`` comes from the same backward pass
    (reference ``csrc/cuda/morfology/soft_morph.cuh:67-77``, ``morph_dtau_term``).  The kernels take
    the temperature's value when the forward runs (read on the host: a CUDA ``tau`` costs one
    device-to-host copy per call).  The cube projection and diagonal mask are the process-wide
    settings at forward time, as for :class:`MorphoAttentionFunction`."""

    @staticmethod
    def forward(ctx, x, W_phi, gate_q, gate_k, W_V, tau, H: int, cube_m: int, scale: float, causal: bool,
                score: str):
        if not x.is_cuda:
            raise ValueError("MorphoAttention expects a CUDA tensor")
        if score not in ("dilation", "erosion"):
            raise ValueError("score must be 'dilation' or 'erosion'")
        tau_value = float(tau)
        if not tau_value > 0.0:
            raise ValueError("tau must be positive")
        x = x.contiguous()
        _g, proj, mdiag, _score, _tau = current_options()
        ctx.options = (GRAD_MODES["full"], proj, mdiag, SCORES[score], tau_value)
        out, lse, saved = ops.forward_save(x, W_phi, gate_q, gate_k, W_V, H, cube_m, scale, causal, proj, mdiag,
                                           SCORES[score], tau_value)
        ctx.save_for_backward(x, W_phi, gate_q, gate_k, W_V, out, lse, saved)
        ctx.H, ctx.cube_m, ctx.scale, ctx.causal = H, cube_m, scale, causal
        ctx.tau_meta = (tau.dtype, tau.device) if isinstance(tau, torch.Tensor) else None
        return out

    @staticmethod
    def backward(ctx, grad_out):
        x, W_phi, gate_q, gate_k, W_V, out, lse, saved = ctx.saved_tensors
        grad_out = grad_out.contiguous()
        args = (grad_out, saved, x, W_phi, gate_q, gate_k, W_V, out, lse, ctx.H, ctx.cube_m, ctx.scale, ctx.causal,
                *ctx.options)
        d_tau = None
        if ctx.needs_input_grad[5] and ctx.tau_meta is not None:
            dX, dW_phi, d_gate_q, d_gate_k, dW_V, dt = ops.backward_saved_tau(*args)
            dtype, device = ctx.tau_meta
            d_tau = dt.to(device=device, dtype=dtype)
        else:
            dX, dW_phi, d_gate_q, d_gate_k, dW_V = ops.backward_saved(*args)
        return dX, dW_phi, d_gate_q, d_gate_k, dW_V, d_tau, None, None, None, None, None


def soft_morph_attention(x, W_phi, gate_q, gate_k, W_V, tau, num_heads: int, cube_m: int, *,
                         score: str = "dilation", scale: float = 1.0, causal: bool = False):
    """:func:`morpho_attention` with the soft-morphology aggregation in place of softmax . V:
    ``out_ic = sgn * tau * logsumexp_j(sgn * (S_ij + V_jc) / tau)`` (``sgn`` = +1 for
    ``"dilation"``, -1 for ``"erosion"``).  ``tau`` may be a float or a scalar tensor; a tensor that
    requires grad receives ``dL/dtau``."""
    return SoftMorphAttentionFunction.apply(x, W_phi, gate_q, gate_k, W_V, tau, num_heads, cube_m, scale, causal,
                                            score)


class SoftMorphAttention(MorphoAttention):
    """:class:`MorphoAttention` aggregating with the soft-morphology score and a learnable
    temperature ``tau`` (an fp32 scalar parameter; ``learn_tau=False`` keeps it fixed)."""

    def __init__(self, dim: int, num_heads: int, cube_m: int, *, score: str = "dilation", tau: float = 1.0,
                 learn_tau: bool = True, scale: float = 1.0, causal: bool = False,
                 dtype: torch.dtype = torch.float16, device=None) -> None:
        super().__init__(dim, num_heads, cube_m, scale=scale, causal=causal, dtype=dtype, device=device)
        if score not in ("dilation", "erosion"):
            raise ValueError("score must be 'dilation' or 'erosion'")
        self.score = score
        self.tau = nn.Parameter(torch.tensor(float(tau), dtype=torch.float32, device=device),
                                requires_grad=learn_tau)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return SoftMorphAttentionFunction.apply(x, self.W_phi, self.gate_q, self.gate_k, self.W_V, self.tau,
                                                self.num_heads, self.cube_m, self.scale, self.causal, self.score)
