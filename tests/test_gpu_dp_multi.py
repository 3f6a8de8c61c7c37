"""Data parallelism across GPUs: each rank runs `DataParallelAttention` on its own batch shard
(one process per GPU, NCCL), and the averaged weight gradients times the world size must equal
one GPU's gradients over the concatenated batch; each rank's output and input gradient must
equal that run's rows for its shard bit for bit (sequences are independent in both passes).
Runs on 2 GPUs (skipped with fewer): the ranks are child processes with a short process-group
timeout, so a rank that fails ends the others' collectives with an error instead of a hang."""

import datetime
import os
import socket

import pytest
import torch

from morphottention_b200.configs import MorphoConfig, make_inputs

pytestmark = pytest.mark.gpu

WORLD = 2
CFG = MorphoConfig("dp_multi", 2 * WORLD, 300, 256, 4, 32, 0.7, True, 23)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _module(inp, dev):
    from morphottention_b200 import MorphoAttention
    m = MorphoAttention(CFG.D, CFG.H, CFG.cube_m, scale=CFG.scale, causal=CFG.causal, device=dev)
    with torch.no_grad():
        for n in ("W_phi", "W_V", "gate_q", "gate_k"):
            getattr(m, n).copy_(inp[n])
    return m


def _worker(rank, world, port, outdir):
    import torch.distributed as dist

    from morphottention_b200 import dp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        inp = make_inputs(CFG, device=dev, random_gates=True, with_grad_out=True)
        per = CFG.B // world
        shard = slice(rank * per, (rank + 1) * per)
        model = dp.DataParallelAttention(_module(inp, dev))
        x = inp["x"][shard].clone().requires_grad_(True)
        out = model(x)
        (out.float() * inp["grad_out"][shard].float()).sum().backward()
        m = model.module
        res = {"out": out.detach().cpu(), "dX": x.grad.cpu(),
               **{n: getattr(m, n).grad.cpu() for n in ("W_phi", "W_V", "gate_q", "gate_k")}}
        torch.cuda.synchronize()
        torch.save(res, os.path.join(outdir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_data_parallel_matches_one_gpu_over_the_whole_batch(cuda, tmp_path):
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, str(tmp_path))) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    # one GPU over the concatenated batch
    inp = make_inputs(CFG, device=cuda, random_gates=True, with_grad_out=True)
    m = _module(inp, cuda)
    x = inp["x"].clone().requires_grad_(True)
    out = m(x)
    (out.float() * inp["grad_out"].float()).sum().backward()
    per = CFG.B // WORLD
    ranks = [torch.load(os.path.join(tmp_path, f"rank{r}.pt")) for r in range(WORLD)]
    for r, res in enumerate(ranks):
        shard = slice(r * per, (r + 1) * per)
        assert torch.equal(res["out"], out.detach()[shard].cpu()), r
        assert torch.equal(res["dX"], x.grad[shard].cpu()), r
    for n in ("W_phi", "W_V", "gate_q", "gate_k"):
        full = getattr(m, n).grad.float().cpu()
        assert torch.equal(ranks[0][n], ranks[1][n]), n  # every rank holds the same averaged gradient
        dp_sum = ranks[0][n].float() * WORLD
        err = float((dp_sum - full).norm() / full.norm())
        assert err <= 1e-3, (n, err)  # two fp16 roundings of the same fp32 sum
