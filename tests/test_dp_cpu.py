"""Data-parallel host logic on CPU with gloo ranks (world size 2): sharding the batch and
all-reducing the weight gradients equals one rank over the whole batch.  The per-rank
gradients come from the CPU oracle (no GPU here)."""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from morphottention_b200 import dp
from morphottention_b200.configs import MorphoConfig, make_inputs
from oracle import morpho_oracle as O

CFG = MorphoConfig("dp", 4, 24, 64, 2, 16, 0.5, True, 13)


class _Params(torch.nn.Module):
    def __init__(self, inp):
        super().__init__()
        for n in dp.PARAM_ORDER:
            setattr(self, n, torch.nn.Parameter(inp[n].float().clone()))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        inp = make_inputs(CFG, random_gates=True, dtype=torch.float32)
        per = CFG.B // world
        x = inp["x"][rank * per:(rank + 1) * per]
        r = O.forward_backward(x, inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], CFG.H, CFG.cube_m,
                               CFG.scale, CFG.causal)
        m = _Params(inp)
        for n, k in (("W_phi", "dW_phi"), ("W_V", "dW_V"), ("gate_q", "d_gate_q"), ("gate_k", "d_gate_k")):
            getattr(m, n).grad = r[k].clone()
        dp.allreduce_weight_grads(m, average=False)
        # max-over-ranks timing reduction used by bench.py
        t = torch.tensor([float(rank + 1)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            q.put({n: getattr(m, n).grad.clone() for n in dp.PARAM_ORDER} | {"tmax": t.item()})
    finally:
        dist.destroy_process_group()


def test_dp_allreduce_equals_full_batch():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    inp = make_inputs(CFG, random_gates=True, dtype=torch.float32)
    full = O.forward_backward(inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], CFG.H, CFG.cube_m,
                              CFG.scale, CFG.causal)
    for n, k in (("W_phi", "dW_phi"), ("W_V", "dW_V"), ("gate_q", "d_gate_q"), ("gate_k", "d_gate_k")):
        assert O.rel_l2(got[n], full[k]) < 1e-5, n
    assert got["tmax"] == float(world)
