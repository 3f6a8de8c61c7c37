"""The half2 CUDA-core score probe (`morpho_sm100_score_probe_half2`, the alternative the
attention kernels' tcgen05 score was measured against) computes what it claims: the row maxima of
qc . k^T over every key, within fp16-accumulation error, for ragged N and each cube_m."""

import pytest
import torch

from morphottention_b200 import capi
from morphottention_b200.configs import MorphoConfig

from .helpers import inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg", [MorphoConfig("m32", 1, 512, 256, 4, 32, 0.5, False, 71),
                                 MorphoConfig("m16_ragged", 2, 197, 128, 2, 16, 1.0, False, 72),
                                 MorphoConfig("m64_odd", 1, 129, 256, 2, 64, 1.0, False, 73)], ids=lambda c: c.name)
def test_score_probe_row_maxima(cuda, cfg):
    inp = inputs(cfg, cuda, random_gates=True)
    p = capi.problem(cfg.B, cfg.N, cfg.D, cfg.H, cfg.cube_m, cfg.scale, cfg.causal)
    o = capi.project(p, inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], with_phi=False)
    rowmax = torch.empty(cfg.B * cfg.H, cfg.N, dtype=torch.float32, device=cuda)
    capi.score_probe_half2(o["qc"], o["kc"], rowmax)
    torch.cuda.synchronize()
    ref = (o["qc"].float() @ o["kc"].float().transpose(1, 2)).amax(-1)
    err = (rowmax - ref).abs().max().item()
    assert err <= 2e-2 * max(1.0, ref.abs().max().item()), err
