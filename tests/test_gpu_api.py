"""The drop-in surface on the GPU: module / functional autograd path against the oracle,
the reference's error messages, gradient modes, streams, and that the native library is
what runs (no fallback)."""

import pytest
import torch

import morphottention_b200 as M
from morphottention_b200 import capi
from morphottention_b200.configs import CONFIGS, MorphoConfig, make_inputs
from oracle import morpho_oracle as O

from .helpers import TOL_GRAD, TOL_OUT

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _device_status_clean(cuda):
    """Every kernel's bounded waits must have finished in time."""
    yield
    torch.cuda.synchronize()
    assert capi.device_status(reset=True) == 0


def _module(cfg, inp, dev):
    m = M.MorphoAttention(cfg.D, cfg.H, cfg.cube_m, scale=cfg.scale, causal=cfg.causal, device=dev)
    with torch.no_grad():
        for name in ("W_phi", "gate_q", "gate_k", "W_V"):
            getattr(m, name).copy_(inp[name])
    return m


@pytest.mark.parametrize("cfg", [CONFIGS["c1"], MorphoConfig("vit_narrow", 2, 197, 128, 2, 16, 1.0, True, 3)],
                         ids=lambda c: c.name)
def test_module_autograd(cuda, cfg):
    inp = make_inputs(cfg, device=cuda, random_gates=True, with_grad_out=True)
    m = _module(cfg, inp, cuda)
    x = inp["x"].clone().requires_grad_(True)
    out = m(x)
    out.backward(inp["grad_out"])
    ref = O.forward_backward(*(inp[k].cpu() for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")), cfg.H, cfg.cube_m,
                             cfg.scale, cfg.causal, grad_out=inp["grad_out"].cpu())
    assert O.rel_l2(out.float(), ref["out"]) < TOL_OUT
    assert O.rel_l2(x.grad.float(), ref["dX"]) < TOL_GRAD
    for name, key in (("W_phi", "dW_phi"), ("gate_q", "d_gate_q"), ("gate_k", "d_gate_k"), ("W_V", "dW_V")):
        assert O.rel_l2(getattr(m, name).grad.float(), ref[key]) < TOL_GRAD, name


def test_functional_matches_module(cuda):
    cfg = CONFIGS["c1"]
    inp = make_inputs(cfg, device=cuda)
    m = _module(cfg, inp, cuda)
    a = m(inp["x"])
    b = M.morpho_attention(inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], cfg.H, cfg.cube_m,
                           scale=cfg.scale, causal=cfg.causal)
    assert torch.equal(a, b)
    assert capi.last_launch_count() == 2  # projection GEMM + attention


def test_causal_flag_is_honoured(cuda):
    cfg = CONFIGS["c1"].with_(causal=False)
    inp = make_inputs(cfg, device=cuda)
    args = (inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], cfg.H, cfg.cube_m)
    a = M.morpho_attention(*args, causal=False)
    b = M.morpho_attention(*args, causal=True)
    assert not torch.allclose(a, b)
    # the first query attends only to itself under the causal mask
    v = (inp["x"].float() @ inp["W_V"].float())
    assert O.rel_l2(b[:, 0].float(), v[:, 0]) < 2e-3


def test_reference_grad_mode_through_ops(cuda):
    cfg = MorphoConfig("m32", 1, 300, 256, 4, 32, 0.5, False, 2)
    inp = make_inputs(cfg, device=cuda, random_gates=True)
    with M.grad_mode("reference"):
        m = _module(cfg, inp, cuda)
        m(inp["x"]).sum(dtype=torch.float32).backward()
    ref = O.forward_backward(*(inp[k].cpu() for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")), cfg.H, cfg.cube_m,
                             cfg.scale, cfg.causal, grad_mode="reference")
    assert O.rel_l2(m.W_phi.grad.float(), ref["dW_phi"]) < TOL_GRAD
    assert O.rel_l2(m.gate_q.grad.float(), ref["d_gate_q"]) < TOL_GRAD
    assert M.get_grad_mode() == "full"


def test_non_default_stream(cuda):
    cfg = CONFIGS["c1"]
    inp = make_inputs(cfg, device=cuda)
    ref, _ = torch.ops.morphottention.forward(inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"],
                                              cfg.H, cfg.cube_m, cfg.scale, cfg.causal)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        out, _ = torch.ops.morphottention.forward(inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"],
                                                  cfg.H, cfg.cube_m, cfg.scale, cfg.causal)
    torch.cuda.current_stream().wait_stream(s)
    assert torch.equal(out, ref)


def _args(cfg, inp):
    return [inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], cfg.H, cfg.cube_m, cfg.scale, cfg.causal]


@pytest.mark.parametrize("mutate,msg", [
    (lambda a: a.__setitem__(0, a[0].float()), "X must be float16"),
    (lambda a: a.__setitem__(1, a[1].t().contiguous().t()), "W_phi must be contiguous"),
    (lambda a: a.__setitem__(1, a[1][:, :64].contiguous()), r"W_phi must be \[D, H\*cube_m\]"),
    (lambda a: a.__setitem__(4, a[4][:, :128].contiguous()), r"W_V must be \[D, H\*head_dim_v\]"),
    (lambda a: a.__setitem__(2, a[2][:4].contiguous()), r"gate_q must be \[H, cube_m\]"),
    (lambda a: a.__setitem__(5, 3), "D must be divisible by H"),
    (lambda a: a.__setitem__(0, a[0][0]), r"X must be \[B, N, D\]"),
])
def test_forward_error_messages(cuda, mutate, msg):
    cfg = CONFIGS["c1"]
    a = _args(cfg, make_inputs(cfg, device=cuda))
    mutate(a)
    with pytest.raises(RuntimeError, match=msg):
        torch.ops.morphottention.forward(*a)


def test_unsupported_shape_is_a_clean_error(cuda):
    cfg = MorphoConfig("bad", 1, 16, 64, 2, 24, 1.0, False, 0)  # cube_m 24
    inp = make_inputs(cfg, device=cuda)
    with pytest.raises(RuntimeError, match="cube_m"):
        torch.ops.morphottention.forward(*_args(cfg, inp))
    assert capi.device_status(reset=True) == 0


def test_backward_error_messages(cuda):
    cfg = CONFIGS["c1"]
    inp = make_inputs(cfg, device=cuda)
    out, lse = torch.ops.morphottention.forward(*_args(cfg, inp))
    g = torch.ones_like(out)
    base = [g, inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], out, lse, cfg.H, cfg.cube_m,
            cfg.scale, cfg.causal]
    bad = list(base)
    bad[7] = lse[:, :10].contiguous()
    with pytest.raises(RuntimeError, match=r"lse must be \[B\*H, N\]"):
        torch.ops.morphottention.backward(*bad)
    bad = list(base)
    bad[7] = lse.half()
    with pytest.raises(RuntimeError, match="lse must be float32"):
        torch.ops.morphottention.backward(*bad)
    bad = list(base)
    bad[0] = g[:, :64].contiguous()
    with pytest.raises(RuntimeError, match=r"grad_out must match X shape"):
        torch.ops.morphottention.backward(*bad)
    bad = list(base)
    bad[0] = g.cpu()
    with pytest.raises(RuntimeError, match="Gradient output and X must be a CUDA tensors"):
        torch.ops.morphottention.backward(*bad)


def test_native_library_is_loaded(cuda):
    cfg = CONFIGS["c1"]
    inp = make_inputs(cfg, device=cuda)
    torch.ops.morphottention.forward(*_args(cfg, inp))
    maps = open("/proc/self/maps").read()
    assert "libmorpho_sm100.so" in maps and "morphottention_b200/_C.so" in maps


@pytest.mark.parametrize("cfg", [CONFIGS["c1"], MorphoConfig("saved_causal", 2, 300, 256, 4, 32, 0.7, True, 5),
                                 MorphoConfig("saved_m64", 1, 256, 512, 4, 64, 1.0, False, 6)],
                         ids=lambda c: c.name)
def test_saved_pair_matches_recompute(cuda, cfg):
    """forward_save + backward_saved (projection kept) give bit-identical results to
    forward + backward (projection recomputed), through the C ABI and the torch ops."""
    inp = make_inputs(cfg, device=cuda, random_gates=True, with_grad_out=True)
    p = capi.problem(cfg.B, cfg.N, cfg.D, cfg.H, cfg.cube_m, cfg.scale, cfg.causal)
    args = [inp[k] for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")]

    def run(saved_path):
        out = torch.empty_like(inp["x"])
        lse = torch.empty(cfg.B * cfg.H, cfg.N, dtype=torch.float32, device=cuda)
        grads = [torch.empty_like(t) for t in args]
        if saved_path:
            saved = capi.forward_save(p, *args, out, lse)
            assert saved.numel() == capi.saved_bytes(p)
            capi.backward_saved(p, inp["grad_out"], saved, *args, out, lse, *grads)
        else:
            capi.forward(p, *args, out, lse)
            capi.backward(p, inp["grad_out"], *args, out, lse, *grads)
        torch.cuda.synchronize()
        return [out, lse] + grads

    a, b = run(False), run(True)
    for name, u, v in zip(("out", "lse", "dX", "dW_phi", "d_gate_q", "d_gate_k", "dW_V"), a, b):
        assert torch.equal(u, v), name
    opts = (0, 0, 0, 1.0)  # projection sigmoid, no diagonal mask, softmax score, tau
    o, l, s = torch.ops.morphottention.forward_save(*args, cfg.H, cfg.cube_m, cfg.scale, cfg.causal, *opts)
    assert torch.equal(o, a[0]) and s.dtype == torch.uint8
    g = torch.ops.morphottention.backward_saved(inp["grad_out"], s, *args, o, l, cfg.H, cfg.cube_m, cfg.scale,
                                                cfg.causal, 0, *opts)
    for name, u, v in zip(("dX", "dW_phi", "d_gate_q", "d_gate_k", "dW_V"), a[2:], g):
        assert torch.equal(u, v), name


def test_saved_buffer_size_is_checked(cuda):
    cfg = CONFIGS["c1"]
    inp = make_inputs(cfg, device=cuda, with_grad_out=True)
    p = capi.problem(cfg.B, cfg.N, cfg.D, cfg.H, cfg.cube_m, cfg.scale, cfg.causal)
    args = [inp[k] for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")]
    out = torch.empty_like(inp["x"])
    lse = torch.empty(cfg.B * cfg.H, cfg.N, dtype=torch.float32, device=cuda)
    small = torch.empty(capi.saved_bytes(p) - 4096, dtype=torch.uint8, device=cuda)
    with pytest.raises(capi.MorphoError, match="saved buffer too small"):
        capi.forward_save(p, *args, out, lse, saved=small)
