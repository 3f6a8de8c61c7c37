"""Data parallelism across GPUs: each rank runs `DataParallelAttention` on its own batch shard
(one process per GPU, NCCL), and the averaged weight gradients times the world size must equal
one GPU's gradients over the concatenated batch; each rank's output and input gradient must
equal that run's rows for its shard bit for bit (sequences are independent in both passes).
Both weight-gradient collectives are covered: the library's peer-memory all-reduce (the default)
and NCCL's.  A second test checks the peer all-reduce kernel itself over three steps (both of its
alternating buckets): every rank's result must equal the rank-order fp32 sum of the ranks'
buckets bit for bit, and its fp16 gradients the rounded, scaled sum.
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


def _worker(rank, world, port, outdir, collective):
    import torch.distributed as dist

    from morphottention_b200 import dp
    dp.set_collective(collective)
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
               **{n: getattr(m, n).grad.cpu() for n in ("W_phi", "W_V", "gate_q", "gate_k")},
               "peer": any(v is not None for v in dp._EXCHANGES.values())}
        torch.cuda.synchronize()
        torch.save(res, os.path.join(outdir, f"rank{rank}.pt"))
    finally:
        dp.close_exchanges()
        dist.destroy_process_group()


def _run_ranks(target, args, tmp_path):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, WORLD, port, str(tmp_path)) + args) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


@pytest.mark.parametrize("collective", ["peer", "nccl"])
def test_data_parallel_matches_one_gpu_over_the_whole_batch(cuda, tmp_path, collective):
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    _run_ranks(_worker, (collective,), tmp_path)
    # one GPU over the concatenated batch
    inp = make_inputs(CFG, device=cuda, random_gates=True, with_grad_out=True)
    m = _module(inp, cuda)
    x = inp["x"].clone().requires_grad_(True)
    out = m(x)
    (out.float() * inp["grad_out"].float()).sum().backward()
    per = CFG.B // WORLD
    ranks = [torch.load(os.path.join(tmp_path, f"rank{r}.pt")) for r in range(WORLD)]
    for r, res in enumerate(ranks):
        assert res["peer"] == (collective == "peer"), r  # B200s of one box have peer access
        shard = slice(r * per, (r + 1) * per)
        assert torch.equal(res["out"], out.detach()[shard].cpu()), r
        assert torch.equal(res["dX"], x.grad[shard].cpu()), r
    for n in ("W_phi", "W_V", "gate_q", "gate_k"):
        full = getattr(m, n).grad.float().cpu()
        assert torch.equal(ranks[0][n], ranks[1][n]), n  # every rank holds the same averaged gradient
        dp_sum = ranks[0][n].float() * WORLD
        err = float((dp_sum - full).norm() / full.norm())
        assert err <= 1e-3, (n, err)  # two fp16 roundings of the same fp32 sum


def _peer_worker(rank, world, port, outdir):
    import torch.distributed as dist

    from morphottention_b200 import capi, dp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    ex = None
    try:
        p = capi.problem(2, 64, 256, 4, 32)
        D, Hm = 256, 4 * 32
        n = capi.weight_grad_elems(p)
        ex = dp.PeerExchange(n, device=dev)
        res = []
        for step in range(3):
            b = ex.bucket()
            g = torch.Generator(device=dev).manual_seed(100 * step + rank)
            b.copy_(torch.randn(n, generator=g, device=dev))
            local = b.clone()
            dW_phi = torch.empty(D, Hm, dtype=torch.float16, device=dev)
            dW_V = torch.empty(D, D, dtype=torch.float16, device=dev)
            dgq = torch.empty(Hm, dtype=torch.float16, device=dev)
            dgk = torch.empty(Hm, dtype=torch.float16, device=dev)
            ex.allreduce_finalize(p, 1.0 / world, dW_phi, dgq, dgk, dW_V)
            torch.cuda.synchronize()
            res.append({"local": local.cpu(), "sum": b.clone().cpu(), "dW_phi": dW_phi.cpu(), "dW_V": dW_V.cpu(),
                        "gate_q": dgq.cpu(), "gate_k": dgk.cpu(), "status": capi.device_status(reset=True)})
        torch.save(res, os.path.join(outdir, f"peer{rank}.pt"))
    finally:
        if ex is not None:
            ex.close()
        dist.destroy_process_group()


def test_peer_allreduce_sums_in_rank_order(cuda, tmp_path):
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    _run_ranks(_peer_worker, (), tmp_path)
    ranks = [torch.load(os.path.join(tmp_path, f"peer{r}.pt")) for r in range(WORLD)]
    D, Hm = 256, 128
    for step in range(3):
        want = ranks[0][step]["local"].clone()
        for r in range(1, WORLD):
            want += ranks[r][step]["local"]
        scaled = (want / WORLD).half()
        segs = {"dW_phi": scaled[:D * Hm].view(D, Hm), "dW_V": scaled[D * Hm:D * Hm + D * D].view(D, D),
                "gate_q": scaled[D * Hm + D * D:D * Hm + D * D + Hm],
                "gate_k": scaled[D * Hm + D * D + Hm:D * Hm + D * D + 2 * Hm]}
        for r in range(WORLD):
            res = ranks[r][step]
            assert res["status"] == 0, (r, step)
            assert torch.equal(res["sum"], want), (r, step)
            for k, v in segs.items():
                assert torch.equal(res[k], v), (r, step, k)
