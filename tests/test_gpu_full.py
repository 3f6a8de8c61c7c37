"""Full-size configurations against the fp32 oracle evaluated on the GPU (torch fp32,
TF32 off), plus size-independent properties: finite outputs, batch independence, and
bitwise-stable forward outputs across runs."""

import pytest
import torch

from morphottention_b200.configs import CONFIGS
from oracle import morpho_oracle as O

from .helpers import compare, inputs, run_cuda

pytestmark = pytest.mark.gpu


def _oracle_gpu(cfg, inp, grad_mode="full"):
    torch.backends.cuda.matmul.allow_tf32 = False
    r = O.forward_backward(*(inp[k] for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")), cfg.H, cfg.cube_m,
                           cfg.scale, cfg.causal, grad_mode=grad_mode)
    return r


@pytest.mark.parametrize("name", ["c2", "c3", "c4"])
def test_full_size_config(cuda, name):
    cfg = CONFIGS[name]
    inp = inputs(cfg, cuda)
    ours = run_cuda(cfg, inp)
    ref = _oracle_gpu(cfg, inp)
    errs = compare(ours, ref)
    print(name, {k: f"{v:.2e}" for k, v in errs.items()})
    del ref
    torch.cuda.empty_cache()


def test_c5_one_sequence_and_batch_independence(cuda):
    """c5 (N=8192, D=2048, H=16, m=64, hd=128, causal) on one sequence against the oracle;
    then the full per-rank batch of 8: sequence 0 must reproduce the single-sequence
    forward exactly (batches are independent)."""
    cfg1 = CONFIGS["c5"].with_(B=1)
    inp = inputs(cfg1, cuda)
    ours = run_cuda(cfg1, inp)
    ref = _oracle_gpu(cfg1, inp)
    compare(ours, ref)
    del ref
    torch.cuda.empty_cache()
    cfg8 = CONFIGS["c5"]
    inp8 = inputs(cfg8, cuda)
    inp8["x"][0].copy_(inp["x"][0])
    for k in ("W_phi", "W_V", "gate_q", "gate_k"):
        inp8[k] = inp[k]
    big = run_cuda(cfg8, inp8)
    for k in big:
        assert torch.isfinite(big[k].float()).all(), k
    assert torch.equal(big["out"][0], ours["out"][0])
    assert torch.equal(big["lse"][: cfg8.H], ours["lse"])
