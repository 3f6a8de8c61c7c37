"""Data-parallel paths on one GPU (a single-rank NCCL group): the overlapped backward
(`morpho_sm100_backward_saved_dp`, weight-gradient bucket all-reduced on a communication
stream while dX runs) and the `DataParallelAttention` wrapper give bit-identical results to
the plain backward."""

import os
import socket

import pytest
import torch
import torch.distributed as dist

from morphottention_b200 import MorphoAttention, capi, dp
from morphottention_b200.configs import MorphoConfig, make_inputs

pytestmark = pytest.mark.gpu

CFG = MorphoConfig("dp1", 2, 300, 256, 4, 32, 0.7, True, 21)


@pytest.fixture(scope="module")
def nccl_group():
    if dist.is_initialized():
        yield None
        return
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda:0"))
    try:
        yield None
    finally:
        torch.cuda.synchronize()
        dist.destroy_process_group()


def test_backward_saved_dp_matches_bucket_backward(nccl_group):
    inp = make_inputs(CFG, device="cuda:0", random_gates=True)
    args = [inp[k] for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")]
    x = args[0]
    p = capi.problem(CFG.B, CFG.N, CFG.D, CFG.H, CFG.cube_m, CFG.scale, CFG.causal)
    out = torch.empty_like(x)
    lse = torch.empty(CFG.B * CFG.H, CFG.N, dtype=torch.float32, device=x.device)
    saved = capi.forward_save(p, *args, out, lse)
    g = torch.randn(x.shape, generator=torch.Generator().manual_seed(5)).half().to(x.device)
    n = capi.weight_grad_elems(p)

    dX0 = torch.empty_like(x)
    b0 = torch.empty(n, dtype=torch.float32, device=x.device)
    capi.backward_saved(p, g, saved, *args, out, lse, dX0, None, None, None, None, dweights_f32=b0)
    w0 = [torch.empty_like(t) for t in args[1:]]  # W_phi, gate_q, gate_k, W_V
    capi.finalize_weight_grads(p, b0, 1.0, w0[0], w0[1], w0[2], w0[3])

    dX1 = torch.empty_like(x)
    b1 = torch.empty(n, dtype=torch.float32, device=x.device)
    w1 = [torch.empty_like(t) for t in args[1:]]
    dp.backward_allreduce(p, g, saved, *args, out, lse, dX1, w1[0], w1[1], w1[2], w1[3], b1)
    torch.cuda.synchronize()
    assert capi.device_status(reset=True) == 0
    assert torch.equal(dX0, dX1)
    assert torch.equal(b0, b1)
    for a, b in zip(w0, w1):
        assert torch.equal(a, b)


def test_backward_saved_dp_needs_a_bucket(nccl_group):
    inp = make_inputs(CFG, device="cuda:0")
    args = [inp[k] for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")]
    x = args[0]
    p = capi.problem(CFG.B, CFG.N, CFG.D, CFG.H, CFG.cube_m, CFG.scale, CFG.causal)
    out = torch.empty_like(x)
    lse = torch.empty(CFG.B * CFG.H, CFG.N, dtype=torch.float32, device=x.device)
    saved = capi.forward_save(p, *args, out, lse)
    with pytest.raises(capi.MorphoError):
        capi.backward_saved_dp(p, torch.ones_like(x), saved, *args, out, lse, torch.empty_like(x), None)


def test_data_parallel_module_matches_module(nccl_group):
    inp = make_inputs(CFG, device="cuda:0", random_gates=True)
    ref = MorphoAttention(CFG.D, CFG.H, CFG.cube_m, scale=CFG.scale, causal=CFG.causal, device="cuda:0")
    mod = MorphoAttention(CFG.D, CFG.H, CFG.cube_m, scale=CFG.scale, causal=CFG.causal, device="cuda:0")
    with torch.no_grad():
        for m in (ref, mod):
            m.W_phi.copy_(inp["W_phi"])
            m.W_V.copy_(inp["W_V"])
            m.gate_q.copy_(inp["gate_q"])
            m.gate_k.copy_(inp["gate_k"])
    wrapped = dp.DataParallelAttention(mod)
    x0 = inp["x"].clone().requires_grad_(True)
    x1 = inp["x"].clone().requires_grad_(True)
    g = torch.randn(x0.shape, generator=torch.Generator().manual_seed(6)).half().to(x0.device)
    o0 = ref(x0)
    o1 = wrapped(x1)
    o0.backward(g)
    o1.backward(g)
    torch.cuda.synchronize()
    assert torch.equal(o0, o1)
    assert torch.equal(x0.grad, x1.grad)
    for n in dp.PARAM_ORDER:
        assert torch.equal(getattr(ref, n).grad, getattr(mod, n).grad), n
