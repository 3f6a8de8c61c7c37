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


def _peer_setup_worker(rank, world, port, q, mode):
    """Peer-exchange set-up where it cannot work: every rank must give up together (the same
    RuntimeError everywhere, no rank left waiting in an exchange round)."""
    from morphottention_b200 import capi
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        destroyed = []
        if mode == "rank1_fails":  # rank 0's region is created, rank 1's is not
            def create(r, w, n):
                if r == 1:
                    raise capi.MorphoError(capi.MORPHO_ERR_CUDA, "fake: no device memory")
                return 1234, b"h" * capi.PEER_HANDLE_BYTES, b"p" * capi.PEER_PCI_ID_BYTES
            capi.peer_create = create
            capi.peer_destroy = destroyed.append
        elif mode == "connect_fails":  # both regions exist, rank 0 cannot map rank 1's
            capi.peer_create = lambda r, w, n: (100 + r, b"h" * capi.PEER_HANDLE_BYTES, b"p" * capi.PEER_PCI_ID_BYTES)

            def connect(g, handles, ids):
                assert len(handles) == world and len(ids) == world
                if g == 100:
                    raise capi.MorphoError(capi.MORPHO_ERR_UNSUPPORTED, "fake: no peer access")
            capi.peer_connect = connect
            capi.peer_destroy = destroyed.append
        err = None
        try:
            dp.PeerExchange(1000, device="cuda:0")
        except RuntimeError as e:
            err = str(e)
        cached = dp.peer_exchange(1000, device="cuda:0")
        dp.set_collective("nccl")
        off = dp.peer_exchange(1000, device="cuda:0")
        dp.set_collective("peer")
        t = torch.ones(1)
        dist.all_reduce(t)  # the ranks are still in step
        q.put((rank, err, cached, off, t.item(), destroyed))
    finally:
        dist.destroy_process_group()


def test_peer_exchange_setup_fails_on_every_rank_together():
    world = 2
    ctx = mp.get_context("spawn")
    for mode in ("no_gpu", "rank1_fails", "connect_fails"):
        q = ctx.Queue()
        port = _free_port()
        procs = [ctx.Process(target=_peer_setup_worker, args=(r, world, port, q, mode)) for r in range(world)]
        for p in procs:
            p.start()
        got = sorted(q.get(timeout=120) for _ in range(world))
        for p in procs:
            p.join(timeout=60)
        assert all(p.exitcode == 0 for p in procs), (mode, [p.exitcode for p in procs])
        for rank, err, cached, off, total, destroyed in got:
            assert err is not None and err.startswith("peer all-reduce unavailable"), (mode, rank, err)
            assert cached is None and off is None, (mode, rank)
            assert total == world, (mode, rank)
            # two set-ups per rank (direct, then through the cache): each frees what it created
            if mode == "rank1_fails":
                assert destroyed == ([1234, 1234] if rank == 0 else []), (mode, rank, destroyed)
            if mode == "connect_fails":
                assert destroyed == [100 + rank] * 2, (mode, rank, destroyed)


def test_set_collective_rejects_unknown_names():
    import pytest
    with pytest.raises(ValueError):
        dp.set_collective("mpi")
    assert dp.get_collective() == "peer"
