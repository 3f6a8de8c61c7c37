"""The allocation-free forward entry point (``morpho_sm100_forward_noalloc``).

It exists for callers that cannot allocate device memory where they run the forward
(memory-pressure callbacks, servers with a frozen memory plan, hosts without an
allocator binding): its scratch is a fixed array inside the library.  Checked through
the C ABI against the regular entry point, bit for bit (both run the same kernels on the
same inputs), on two calls in a row with different problems -- the softmax score and then
the soft-morphology score, whose range flag lives in the shared scratch -- so that state
left by one call in the shared array cannot leak into the next.  Also checked: a call after
the first one on a device reserves no device memory, and problems beyond the array's size
are rejected.  This file is collected last on purpose."""

import pytest
import torch

from morphottention_b200 import capi
from morphottention_b200.configs import CONFIGS, MorphoConfig, make_inputs

pytestmark = pytest.mark.gpu

# (configuration, score, tau): a causal softmax problem, then a soft dilation of another shape
CASES = [(MorphoConfig("vit_narrow", 2, 197, 128, 2, 16, 1.0, True, 3), "softmax", 1.0),
         (MorphoConfig("dilation", 1, 300, 256, 4, 32, 0.5, False, 5), "dilation", 0.8),
         (CONFIGS["c1"], "softmax", 1.0)]


def _problem(cfg, score, tau):
    return capi.problem(cfg.B, cfg.N, cfg.D, cfg.H, cfg.cube_m, cfg.scale, cfg.causal, score=score, tau=tau)


def _run(cfg, score, tau, inp, noalloc: bool):
    p = _problem(cfg, score, tau)
    out = torch.empty_like(inp["x"])
    lse = torch.empty(cfg.B * cfg.H, cfg.N, dtype=torch.float32, device=inp["x"].device)
    fn = capi.forward_noalloc if noalloc else capi.forward
    fn(p, inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], out, lse)
    torch.cuda.synchronize()
    assert capi.device_status(reset=True) == 0
    return out, lse


def test_noalloc_matches_regular_forward_twice(cuda):
    inputs = [make_inputs(cfg, device=cuda, random_gates=True) for cfg, _, _ in CASES]
    refs = [_run(cfg, score, tau, inp, noalloc=False) for (cfg, score, tau), inp in zip(CASES, inputs)]
    for _ in range(2):  # every case twice over, one after the other, through the one shared array
        for (cfg, score, tau), inp, (ref_out, ref_lse) in zip(CASES, inputs, refs):
            out, lse = _run(cfg, score, tau, inp, noalloc=True)
            assert torch.equal(out, ref_out), (cfg.name, score)
            assert torch.equal(lse, ref_lse), (cfg.name, score)


def test_noalloc_reserves_no_memory_after_the_first_call(cuda):
    cfg, score, tau = CASES[1]
    inp = make_inputs(cfg, device=cuda, random_gates=True)
    p = _problem(cfg, score, tau)
    out = torch.empty_like(inp["x"])
    lse = torch.empty(cfg.B * cfg.H, cfg.N, dtype=torch.float32, device=cuda)
    args = (p, inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], out, lse)
    capi.forward_noalloc(*args)  # the first call on the device does the set-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    torch0 = torch.cuda.memory_allocated()
    for _ in range(3):
        capi.forward_noalloc(*args)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert torch.cuda.memory_allocated() == torch0
    assert free1 == free0, (free0, free1)
    assert capi.device_status(reset=True) == 0


def test_noalloc_rejects_problems_beyond_its_scratch(cuda):
    cfg = CONFIGS["c3"]  # forward scratch of c3 is ~66 MB > 32 MiB
    p = capi.problem(cfg.B, cfg.N, cfg.D, cfg.H, cfg.cube_m, cfg.scale, cfg.causal)
    x = torch.empty(cfg.B, cfg.N, cfg.D, dtype=torch.float16, device=cuda)
    w = torch.empty(cfg.D, cfg.H * cfg.cube_m, dtype=torch.float16, device=cuda)
    g = torch.empty(cfg.H, cfg.cube_m, dtype=torch.float16, device=cuda)
    wv = torch.empty(cfg.D, cfg.D, dtype=torch.float16, device=cuda)
    lse = torch.empty(cfg.B * cfg.H, cfg.N, dtype=torch.float32, device=cuda)
    with pytest.raises(capi.MorphoError) as e:
        capi.forward_noalloc(p, x, w, g, g, wv, torch.empty_like(x), lse)
    assert e.value.code == capi.MORPHO_ERR_WORKSPACE
    assert capi.forward_noalloc_max_scratch() == 32 << 20
