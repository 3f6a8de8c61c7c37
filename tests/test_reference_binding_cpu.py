"""The reference's own Python package on this library's op shim, without a GPU.

The reference package directory (``packages/morphottention/torch-ext/morphottention/``:
``__init__.py``, ``autograd.py``, ``_cmake_ops.py``) is copied as it is into a temporary
directory next to this repository's ``_C.so`` and ``libmorpho_sm100.so``, and imported in a
fresh process (the ``morphottention`` op namespace can be registered only once per process).
Checked there: the reference loader (``_cmake_ops.py:15-28``) finds and loads ``_C.so``, the
ops carry the reference schemas, and the reference's own ``MorphoAttention`` -- its constructor,
initialisation and autograd Function (``autograd.py:34-162``) -- runs a forward and a backward
through them under fake CUDA tensors with the shapes the reference expects (the Function's own
``forward`` and ``backward`` are called directly with a minimal context: autograd's engine would
need a real device).  Needs the
reference sources, so it runs only where they are present (``oracle.build_ref.REF_ROOT``,
set by ``MORPHO_REFERENCE_ROOT``); the numerics of the same ops are covered by the
GPU tests of this package's own module."""

import json
import os
import shutil
import subprocess
import sys

import pytest

from oracle.build_ref import PY_PKG as REF_PKG

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "morphottention_b200")

PROBE = r"""
import json, sys
sys.path.insert(0, sys.argv[1])
import torch
import morphottention as R
from morphottention import _cmake_ops
res = {"file": R.__file__, "loaded": [l.split()[-1] for l in open('/proc/self/maps') if '_C.so' in l][:1],
       "fwd": str(torch.ops.morphottention.forward.default._schema),
       "bwd": str(torch.ops.morphottention.backward.default._schema)}

# the reference registers a fake only for `forward`; the backward's is this probe's own
@torch.library.register_fake("morphottention::backward")
def _bwd_fake(grad_out, X, W_phi, gate_q, gate_k, W_V, out, lse, H, cube_m, scale, causal):
    return [torch.empty_like(X), torch.empty_like(W_phi), torch.empty_like(gate_q), torch.empty_like(gate_k),
            torch.empty_like(W_V)]

class Ctx:  # what autograd hands the Function (the engine itself needs a real device)
    def save_for_backward(self, *t):
        self.saved_tensors = t

from torch._subclasses.fake_tensor import FakeTensorMode
with FakeTensorMode():
    m = R.MorphoAttention(256, 8, 16, scale=0.5, causal=True, device="cuda")
    x = torch.empty(2, 128, 256, dtype=torch.float16, device="cuda")
    res["module_out"] = list(m(x).shape)
    ctx = Ctx()
    out = R.MorphoAttentionFunction.forward(ctx, x, m.W_phi, m.gate_q, m.gate_k, m.W_V, m.num_heads, m.cube_m,
                                            m.scale, m.causal)
    grads = R.MorphoAttentionFunction.backward(ctx, torch.ones_like(out))
    res["out"] = list(out.shape)
    res["grads"] = [list(t.shape) for t in grads[:5]] + [g is None for g in grads[5:]]
    res["params"] = [n for n, _ in m.named_parameters()]
print("PROBE " + json.dumps(res))
"""


@pytest.mark.skipif(not os.path.isdir(REF_PKG), reason="reference sources not present")
def test_reference_package_binds_to_this_op_shim(tmp_path):
    dst = tmp_path / "morphottention"
    dst.mkdir()
    for name in ("__init__.py", "autograd.py", "_cmake_ops.py"):
        shutil.copy(os.path.join(REF_PKG, name), dst / name)
    for lib in ("_C.so", "libmorpho_sm100.so"):
        os.symlink(os.path.join(PKG, lib), dst / lib)
    r = subprocess.run([sys.executable, "-c", PROBE, str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    res = json.loads(r.stdout.split("PROBE ", 1)[1])
    assert res["file"].startswith(str(dst))
    assert res["loaded"] and res["loaded"][0].endswith("_C.so")
    assert res["fwd"] == ("morphottention::forward(Tensor X, Tensor W_phi, Tensor gate_q, Tensor gate_k, "
                          "Tensor W_V, int H, int cube_m, float scale, bool causal) -> Tensor[]")
    assert res["bwd"].startswith("morphottention::backward(Tensor grad_out, Tensor X, Tensor W_phi")
    assert res["out"] == res["module_out"] == [2, 128, 256]
    assert res["grads"] == [[2, 128, 256], [256, 128], [8, 16], [8, 16], [256, 256], True, True, True, True]
    assert res["params"] == ["W_phi", "gate_q", "gate_k", "W_V"]
