"""The projection GEMM + epilogue (codes, biases, V, phi) against the oracle's
``project`` on identical fp16 inputs."""

import pytest
import torch

from morphottention_b200 import capi
from morphottention_b200.configs import CONFIGS, MorphoConfig, make_inputs
from oracle import morpho_oracle as O

pytestmark = pytest.mark.gpu

CASES = [
    CONFIGS["c1"],
    MorphoConfig("hp_pad", 2, 197, 128, 2, 16, 1.0, False, 3),   # H*m = 32 -> padded to 64
    MorphoConfig("m32", 1, 300, 256, 4, 32, 0.5, False, 2),
    MorphoConfig("m64_hd128", 1, 256, 256, 2, 64, 1.0, True, 4),
    MorphoConfig("vit", 2, 197, 768, 12, 16, 1.0, False, 3),      # H*m = 192: BN 64 tiles
    MorphoConfig("odd_h", 1, 64, 384, 3, 16, 1.0, False, 7),
]


@pytest.mark.parametrize("cfg", CASES, ids=lambda c: c.name)
def test_project(cuda, cfg):
    inp = make_inputs(cfg, device=cuda, random_gates=True)
    p = capi.problem(cfg.B, cfg.N, cfg.D, cfg.H, cfg.cube_m, cfg.scale, cfg.causal)
    o = capi.project(p, inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"])
    torch.cuda.synchronize()
    assert capi.device_status(reset=True) == 0
    c = {k: v.cpu().float() for k, v in inp.items()}
    phi, q, k, qb, cb, v = O.project(c["x"], c["W_phi"], c["gate_q"], c["gate_k"], c["W_V"], cfg.H, cfg.cube_m)
    BH, N = cfg.B * cfg.H, cfg.N
    cl = cfg.scale * O.LOG2E
    assert O.rel_l2(o["phi"].cpu(), phi.reshape(BH, N, -1)) < 1e-5
    gq = c["gate_q"].view(1, cfg.H, 1, cfg.cube_m)
    qc = (q - 0.5 * gq).reshape(BH, N, -1)  # centered query codes
    assert O.rel_l2(o["qc"].cpu().float(), qc) < 2e-3
    assert O.rel_l2(o["kc"].cpu().float(), k.reshape(BH, N, -1)) < 1e-3
    assert O.rel_l2(o["v"].cpu().float(), v.reshape(BH, N, -1)) < 1e-3
    assert O.rel_l2(o["qb"][:, :N].cpu(), cl * qb.reshape(BH, N)) < 1e-5
    assert O.rel_l2(o["cb"][:, :N].cpu(), cl * cb.reshape(BH, N)) < 1e-5
