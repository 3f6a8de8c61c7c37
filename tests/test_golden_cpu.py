"""Pins the CPU oracle against golden outputs of the reference's own CUDA kernels.

``tests/golden/*.npz`` were produced on a B200 by ``tests/golden/make_golden.py`` from the
unmodified reference ``attention.cu`` (compiled per variant by ``oracle/build_ref.py``).
The inputs are regenerated here from their seeds.  Expected agreement:

* ``out`` and ``lse``: within the fp16 rounding of the reference (rel-L2 <= 1e-3);
* ``dW_V`` (the only gradient the reference propagates completely): <= 5e-3 against
  either oracle mode;
* ``dX``, ``dW_phi``, ``d_gate_q``, ``d_gate_k``: <= 1.5e-2 against the oracle's
  ``grad_mode="reference"`` (query-side terms detached, as the reference kernel drops
  them; the reference sums its gradients with fp16 atomics, hence the looser bound), and
  clearly different from the full gradient (which the reference does not compute).
"""

import json
import os

import numpy as np
import pytest
import torch

from morphottention_b200.configs import MorphoConfig, make_inputs
from oracle import morpho_oracle as O

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
META = json.load(open(os.path.join(HERE, "golden_meta.json")))


@pytest.mark.parametrize("name", sorted(META))
def test_oracle_matches_reference_kernel(name):
    m = META[name]
    cfg = MorphoConfig(**m["config"])
    inp = make_inputs(cfg, random_gates=m["random_gates"])
    gold = {k: torch.from_numpy(v) for k, v in np.load(os.path.join(HERE, f"{name}.npz")).items()}
    args = [inp[k] for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")]
    ref_mode = O.forward_backward(*args, cfg.H, cfg.cube_m, cfg.scale, cfg.causal, grad_mode="reference")
    full = O.forward_backward(*args, cfg.H, cfg.cube_m, cfg.scale, cfg.causal, grad_mode="full")
    assert O.rel_l2(gold["out"].float(), ref_mode["out"]) <= 1e-3
    assert O.rel_l2(gold["lse"], ref_mode["lse"]) <= 1e-3
    assert O.rel_l2(gold["dW_V"].float(), ref_mode["dW_V"]) <= 5e-3
    for k in ("dX", "dW_phi", "d_gate_q", "d_gate_k"):
        assert O.rel_l2(gold[k].float(), ref_mode[k]) <= 1.5e-2, k
    # the reference kernel really omits the query-side terms
    for k in ("dX", "dW_phi", "d_gate_q"):
        assert O.rel_l2(gold[k].float(), full[k]) > 2e-2, k
