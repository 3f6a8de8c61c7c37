"""The Python surface mirrors the reference package (no GPU needed for these checks)."""

import inspect

import pytest
import torch

import morphottention_b200 as M


def test_exports():
    for name in ("MorphoAttention", "MorphoAttentionFunction", "morpho_attention"):
        assert hasattr(M, name)
    assert hasattr(torch.ops.morphottention, "forward")
    assert hasattr(torch.ops.morphottention, "backward")


def test_schemas_match_reference():
    fwd = str(torch.ops.morphottention.forward.default._schema)
    bwd = str(torch.ops.morphottention.backward.default._schema)
    assert fwd == ("morphottention::forward(Tensor X, Tensor W_phi, Tensor gate_q, Tensor gate_k, Tensor W_V, "
                   "int H, int cube_m, float scale, bool causal) -> Tensor[]")
    assert bwd == ("morphottention::backward(Tensor grad_out, Tensor X, Tensor W_phi, Tensor gate_q, Tensor gate_k, "
                   "Tensor W_V, Tensor out, Tensor lse, int H, int cube_m, float scale, bool causal) -> Tensor[]")


def test_module_constructor_and_init():
    torch.manual_seed(0)
    m = M.MorphoAttention(256, 8, 16, scale=0.5, causal=True)
    assert m.W_phi.shape == (256, 128) and m.W_V.shape == (256, 256)
    assert m.gate_q.shape == (8, 16) and m.gate_k.shape == (8, 16)
    assert m.W_phi.dtype == torch.float16
    assert torch.all(m.gate_q == 1) and torch.all(m.gate_k == 1)
    std = m.W_V.float().std().item()
    assert abs(std - 256 ** -0.5) < 0.1 * 256 ** -0.5
    assert [n for n, _ in m.named_parameters()] == ["W_phi", "gate_q", "gate_k", "W_V"]
    assert m.scale == 0.5 and m.causal is True


def test_constructor_signature():
    sig = inspect.signature(M.MorphoAttention.__init__)
    assert list(sig.parameters) == ["self", "dim", "num_heads", "cube_m", "scale", "causal", "dtype", "device"]
    assert sig.parameters["scale"].kind is inspect.Parameter.KEYWORD_ONLY
    fsig = inspect.signature(M.morpho_attention)
    assert list(fsig.parameters)[:7] == ["x", "W_phi", "gate_q", "gate_k", "W_V", "num_heads", "cube_m"]


def test_dim_not_divisible():
    with pytest.raises(ValueError, match="must be divisible"):
        M.MorphoAttention(100, 3, 16)


def test_cpu_input_rejected():
    m = M.MorphoAttention(64, 2, 16)
    with pytest.raises(ValueError, match="expects a CUDA tensor"):
        m(torch.randn(1, 4, 64, dtype=torch.float16))


def test_fake_kernels():
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        x = torch.empty(2, 5, 64, dtype=torch.float16, device="cuda")
        wp = torch.empty(64, 32, dtype=torch.float16, device="cuda")
        g = torch.empty(2, 16, dtype=torch.float16, device="cuda")
        wv = torch.empty(64, 64, dtype=torch.float16, device="cuda")
        out, lse = torch.ops.morphottention.forward(x, wp, g, g, wv, 2, 16, 1.0, False)
        assert out.shape == x.shape and lse.shape == (4, 5) and lse.dtype == torch.float32
        grads = torch.ops.morphottention.backward(out, x, wp, g, g, wv, out, lse, 2, 16, 1.0, False)
        assert [t.shape for t in grads] == [x.shape, wp.shape, g.shape, g.shape, wv.shape]


def test_training_pair_takes_options_explicitly():
    """forward_save / backward_saved carry every variant option as an argument (the autograd
    Function passes the settings captured when its forward ran), and get_options reports the
    process-wide settings in the C ABI's codes."""
    fs = str(torch.ops.morphottention.forward_save.default._schema)
    bs = str(torch.ops.morphottention.backward_saved.default._schema)
    assert fs.endswith("bool causal, int projection, int mask_diag, int score, float tau) -> Tensor[]")
    assert bs.endswith("bool causal, int grad_mode, int projection, int mask_diag, int score, float tau) -> Tensor[]")
    from morphottention_b200.autograd import current_options
    assert current_options() == (0, 0, 0, 0, 1.0)
    with M.attention_options(projection="identity", mask_diag=True, score="erosion", tau=0.25):
        with M.grad_mode("reference"):
            assert current_options() == (1, 2, 1, 2, 0.25)
    assert current_options() == (0, 0, 0, 0, 1.0)
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        x = torch.empty(2, 5, 64, dtype=torch.float16, device="cuda")
        wp = torch.empty(64, 32, dtype=torch.float16, device="cuda")
        g = torch.empty(2, 16, dtype=torch.float16, device="cuda")
        wv = torch.empty(64, 64, dtype=torch.float16, device="cuda")
        out, lse, saved = torch.ops.morphottention.forward_save(x, wp, g, g, wv, 2, 16, 1.0, False, 1, 1, 1, 0.5)
        assert saved.dtype == torch.uint8 and saved.dim() == 1
        grads = torch.ops.morphottention.backward_saved(out, saved, x, wp, g, g, wv, out, lse, 2, 16, 1.0, False,
                                                        0, 1, 1, 1, 0.5)
        assert [t.shape for t in grads] == [x.shape, wp.shape, g.shape, g.shape, wv.shape]


def test_grad_mode_switch():
    assert M.get_grad_mode() == "full"
    with M.grad_mode("reference"):
        assert M.get_grad_mode() == "reference"
    assert M.get_grad_mode() == "full"
    with pytest.raises(ValueError):
        M.set_grad_mode("bogus")


def test_bench_rejects_score_outside_single_layer_ours():
    """`bench.py --score` times the soft-morphology score on the single-layer configurations of
    this library only: with the reference arm or the encoder step it stops before any work."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for extra in (["--impl", "reference"], ["--config", "c4vit"]):
        r = subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--score", "dilation", *extra],
                           capture_output=True, text=True, timeout=120)
        assert r.returncode != 0
        assert "--score applies to the single-layer configurations" in r.stderr


def test_graphed_training_step_needs_cuda_inputs():
    import torch

    from morphottention_b200.encoder import GraphedTrainingStep

    lin = torch.nn.Linear(4, 4)
    opt = torch.optim.SGD(lin.parameters(), lr=0.1)
    with pytest.raises(ValueError, match="CUDA"):
        GraphedTrainingStep(lin, torch.nn.functional.mse_loss, opt, torch.zeros(2, 4), torch.zeros(2, 4))


@pytest.mark.parametrize("config", ["c1", "c4vit"])
def test_reference_arm_loads_no_native_library_of_this_repo(config):
    """`bench.py --impl reference` times the CPU formulation only: it must not import this
    package (whose __init__ loads _C.so and libmorpho_sm100.so) nor map either library."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    probe = (
        "import runpy, sys, json\n"
        f"sys.argv = ['bench.py', '--impl', 'reference', '--config', '{config}', '--steps', '1', '--warmup', '0']\n"
        f"runpy.run_path({os.path.join(root, 'bench.py')!r}, run_name='__main__')\n"
        "mods = [m for m in sys.modules if m.startswith('morphottention_b200')]\n"
        "maps = [l for l in open('/proc/self/maps') if 'libmorpho_sm100' in l or '_C.so' in l]\n"
        "print('PROBE', json.dumps({'mods': mods, 'maps': len(maps)}))\n")
    r = subprocess.run([sys.executable, "-c", probe], capture_output=True, text=True, timeout=600, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    import json
    line = json.loads(r.stdout.splitlines()[0])
    assert line["impl"] == "reference" and line["value"] > 0
    probe_out = json.loads(r.stdout.split("PROBE", 1)[1])
    assert probe_out == {"mods": [], "maps": 0}, probe_out
