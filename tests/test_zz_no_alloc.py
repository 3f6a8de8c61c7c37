"""The allocation-free forward entry point (``morpho_sm100_forward_noalloc``).

It exists for callers that cannot allocate device memory where they run the forward
(memory-pressure callbacks, servers with a frozen memory plan, hosts without an
allocator binding): its scratch is a fixed array inside the library.  Checked through
the C ABI against the regular entry point, on two calls in a row with different
problems (the shared scratch must not leak state from one call into the next), plus the
size limit.  This file is collected last on purpose."""

import pytest
import torch

from morphottention_b200 import capi
from morphottention_b200.configs import CONFIGS, MorphoConfig, make_inputs
from oracle import morpho_oracle as O

pytestmark = pytest.mark.gpu

TOL_OUT = 1e-3


def _run(cfg, dev, noalloc: bool):
    inp = make_inputs(cfg, device=dev, random_gates=True)
    p = capi.problem(cfg.B, cfg.N, cfg.D, cfg.H, cfg.cube_m, cfg.scale, cfg.causal)
    out = torch.empty_like(inp["x"])
    lse = torch.empty(cfg.B * cfg.H, cfg.N, dtype=torch.float32, device=dev)
    fn = capi.forward_noalloc if noalloc else capi.forward
    fn(p, inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], out, lse)
    torch.cuda.synchronize()
    assert capi.device_status(reset=True) == 0
    return out, lse


def test_noalloc_matches_regular_forward_twice(cuda):
    cases = [MorphoConfig("vit_narrow", 2, 197, 128, 2, 16, 1.0, True, 3), CONFIGS["c1"]]
    for cfg in cases:  # two calls in a row, different shapes, same shared scratch
        ref_out, ref_lse = _run(cfg, cuda, noalloc=False)
        out, lse = _run(cfg, cuda, noalloc=True)
        assert O.rel_l2(out.float(), ref_out.float()) <= TOL_OUT
        assert O.rel_l2(lse, ref_lse) <= TOL_OUT


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
