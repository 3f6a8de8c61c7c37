"""The ViT-style encoder around MorphoAttention (the caller of the attention path): a small
fp16 encoder on the GPU against the same encoder in fp32 on the CPU with the oracle as its
attention, same weights and inputs, MSE-loss training step.  LayerNorm, the MLP and the
residual stream also run in fp16 on the GPU, so the model-level tolerances (rel-L2 3e-3 for
the output, 1.5e-2 for every parameter gradient) are looser than the attention layer's own."""

import pytest
import torch
from torch import nn

from morphottention_b200.encoder import Encoder, GraphedTrainingStep
from oracle import morpho_oracle as O

pytestmark = pytest.mark.gpu


class OracleAttention(nn.Module):
    def __init__(self, ref) -> None:
        super().__init__()
        self.num_heads, self.cube_m, self.scale, self.causal = ref.num_heads, ref.cube_m, ref.scale, ref.causal
        for n in ("W_phi", "gate_q", "gate_k", "W_V"):
            setattr(self, n, nn.Parameter(getattr(ref, n).detach().float().cpu().clone()))

    def forward(self, x):
        out, _ = O.forward(x, self.W_phi, self.gate_q, self.gate_k, self.W_V, self.num_heads, self.cube_m, self.scale,
                           self.causal)
        return out


@pytest.mark.parametrize("out_proj", [False, True])
def test_encoder_step_matches_oracle_model(cuda, out_proj):
    torch.manual_seed(3)
    gpu = Encoder(depth=2, dim=128, num_heads=2, cube_m=16, scale=0.5, out_proj=out_proj, device=cuda)
    cpu = Encoder(depth=2, dim=128, num_heads=2, cube_m=16, scale=0.5, out_proj=out_proj, dtype=torch.float32,
                  device="cpu")
    cpu.load_state_dict({k: v.float().cpu() for k, v in gpu.state_dict().items()})
    for bg, bc in zip(gpu.blocks, cpu.blocks):
        bc.attn = OracleAttention(bg.attn)
    g = torch.Generator().manual_seed(4)
    x = torch.randn(2, 50, 128, generator=g).half()
    target = torch.randn(2, 50, 128, generator=g)

    out_g = gpu(x.to(cuda))
    loss_g = nn.functional.mse_loss(out_g.float(), target.to(cuda))
    loss_g.backward()
    out_c = cpu(x.float())
    loss_c = nn.functional.mse_loss(out_c, target)
    loss_c.backward()
    torch.cuda.synchronize()

    assert O.rel_l2(out_g.float().cpu(), out_c.detach()) <= 3e-3
    assert abs(loss_g.item() - loss_c.item()) <= 3e-3 * abs(loss_c.item())
    params_c = dict(cpu.named_parameters())
    for name, p in gpu.named_parameters():
        pc = params_c[name]
        assert p.grad is not None and pc.grad is not None, name
        err = O.rel_l2(p.grad.float().cpu(), pc.grad)
        assert err <= 1.5e-2, f"{name}: {err:.2e}"


class OracleAttention16(nn.Module):
    """The fp32 oracle attention inside an fp16 model: fp16 parameters and activations at the
    layer boundary, everything inside in fp32 (autograd through the oracle)."""

    def __init__(self, dim, num_heads, cube_m, scale=1.0, causal=False, dtype=None, device=None) -> None:
        super().__init__()
        self.num_heads, self.cube_m, self.scale, self.causal = num_heads, cube_m, scale, causal
        self.W_phi = nn.Parameter(torch.zeros(dim, num_heads * cube_m, dtype=dtype, device=device))
        self.gate_q = nn.Parameter(torch.ones(num_heads, cube_m, dtype=dtype, device=device))
        self.gate_k = nn.Parameter(torch.ones(num_heads, cube_m, dtype=dtype, device=device))
        self.W_V = nn.Parameter(torch.zeros(dim, dim, dtype=dtype, device=device))

    def forward(self, x):
        out, _ = O.forward(x.float(), self.W_phi.float(), self.gate_q.float(), self.gate_k.float(),
                           self.W_V.float(), self.num_heads, self.cube_m, self.scale, self.causal)
        return out.to(x.dtype)


def test_encoder_step_attention_at_layer_tolerances(cuda):
    """The same fp16 encoder twice on the GPU, differing only in its attention: this library's
    kernels against the fp32 oracle attention (rounded to fp16 at the layer boundary).  LayerNorm,
    the MLP and the residual stream run the same fp16 torch code on both sides, so what differs is
    the attention path, held to the layer's tolerances: output rel-L2 <= 1e-3 and every parameter
    gradient <= 5e-3.  (Against an fp32 model -- the test above -- the fp16 LayerNorm / MLP / GELU
    arithmetic itself moves the result by a few 1e-3, which is why that test is looser.)"""
    prev_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        torch.manual_seed(5)
        ours = Encoder(depth=2, dim=128, num_heads=2, cube_m=16, scale=0.5, device=cuda)
        ref = Encoder(depth=2, dim=128, num_heads=2, cube_m=16, scale=0.5, device=cuda, attention=OracleAttention16)
        ref.load_state_dict(ours.state_dict())
        g = torch.Generator().manual_seed(6)
        x = torch.randn(2, 50, 128, generator=g).half().to(cuda)
        target = torch.randn(2, 50, 128, generator=g).to(cuda)
        losses, outs = [], []
        for model in (ours, ref):
            out = model(x)
            loss = nn.functional.mse_loss(out.float(), target)
            loss.backward()
            losses.append(loss.item())
            outs.append(out.float())
        torch.cuda.synchronize()
        assert O.rel_l2(outs[0], outs[1]) <= 1e-3
        assert abs(losses[0] - losses[1]) <= 1e-3 * abs(losses[1])
        ref_params = dict(ref.named_parameters())
        for name, p in ours.named_parameters():
            err = O.rel_l2(p.grad.float(), ref_params[name].grad.float())
            assert err <= 5e-3, f"{name}: {err:.2e}"
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev_tf32


def test_graphed_training_step_matches_eager(cuda):
    """GraphedTrainingStep (the training step captured once as a CUDA graph, attention kernels
    included) against eager steps from the same initial weights: after its 3 warm-up steps and
    after 3 replays on new batches, every parameter's change from the initial weights matches the
    eager model's to 2 fp16 ulps of the weight plus 1 % of the change (the dq accumulation order
    differs from run to run), and so does each replay's loss (1e-3)."""
    torch.manual_seed(5)
    kw = dict(depth=2, dim=128, num_heads=2, cube_m=16, scale=0.5, device=cuda)
    eager = Encoder(**kw)
    graphed = Encoder(**kw)
    graphed.load_state_dict(eager.state_dict())
    init = {k: v.detach().float().clone() for k, v in eager.named_parameters()}
    opt_e = torch.optim.SGD(eager.parameters(), lr=0.05, foreach=True)
    opt_g = torch.optim.SGD(graphed.parameters(), lr=0.05, foreach=True)

    def loss_fn(out, t):
        return nn.functional.mse_loss(out.float(), t)

    def eager_step(x, t):
        loss = loss_fn(eager(x), t)
        opt_e.zero_grad(set_to_none=True)
        loss.backward()
        opt_e.step()
        return loss.detach()

    def check():
        pe = dict(eager.named_parameters())
        moved = 0.0
        for name, p in graphed.named_parameters():
            a, b = pe[name].detach().float(), p.detach().float()
            moved = max(moved, (a - init[name]).abs().max().item())
            # two fp16 ulps of the weight: an update near a rounding boundary may round either way
            tol = 2.0 ** -9 * a.abs() + 1e-2 * (a - init[name]).abs() + 1e-7
            assert ((a - b).abs() <= tol).all(), name
        assert moved > 0

    g = torch.Generator().manual_seed(6)
    batches = [(torch.randn(2, 50, 128, generator=g).half().to(cuda), torch.randn(2, 50, 128, generator=g).to(cuda))
               for _ in range(4)]
    step = GraphedTrainingStep(graphed, loss_fn, opt_g, *batches[0], warmup=3)
    for _ in range(3):
        eager_step(*batches[0])
    torch.cuda.synchronize()
    check()
    for x, t in batches[1:]:
        le = eager_step(x, t)
        lg = step(x, t)
        torch.cuda.synchronize()
        assert abs(lg.item() - le.item()) <= 1e-3 * abs(le.item())
    check()
