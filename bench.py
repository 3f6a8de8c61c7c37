#!/usr/bin/env python
"""Benchmark of the fused MorphoAttention forward + backward on B200.

Default workload: the long-sequence layer (B=4, N=4096, D=1024, H=16, cube_m=32,
scale=0.5, non-causal; fp16), one forward plus the backward of ``out.sum()`` per step.
With ``--gpus N`` (launched under torchrun) every rank runs that per-rank batch on its own
batch shard (weak scaling) and the fp32 weight-gradient bucket is all-reduced with NCCL.

Prints ONE JSON line on rank 0.  ``--impl reference`` times the reference path's CPU
formulation instead (the oracle restatement; the reference itself ships only CUDA code)
on the host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "fused fwd+bwd tokens/sec per B200 and whole-box at 1/2/4/8 GPUs; % of roofline"
UNIT = "tokens/s"


def _load_source(name, relpath):
    """Import one source file by path, outside its package.  The reference arm and the CPU
    baseline need the workload configurations (and the encoder's layout) but must not run
    ``morphottention_b200/__init__.py``, which loads this repository's CUDA libraries."""
    import importlib.util
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, relpath))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod  # dataclasses look their module up while the class is built
    spec.loader.exec_module(mod)
    return mod


def _configs():
    """``morphottention_b200/configs.py`` (configurations, seeded inputs), loaded by path."""
    return _load_source("_morpho_bench_configs", os.path.join("morphottention_b200", "configs.py"))


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p["bf16_tflops_sustained"]), "sm_max_mhz": float(p["sm_max_mhz"]),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "sm_max_mhz": 1965.0,
                "source": "fallback"}


class ClockSampler:
    """nvidia-smi sampler running during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline(cfg, seconds: float = 12.0, max_reps: int = 5):
    """Time the fp32 CPU oracle (a restatement of the reference path) on one sequence of
    the workload: forward + backward of out.sum(), all host threads."""
    import torch

    from oracle import morpho_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    one = cfg.with_(B=1)
    inp = _configs().make_inputs(one)
    times = []
    t_start = time.perf_counter()
    while len(times) < max_reps and (time.perf_counter() - t_start) < seconds or len(times) < 2:
        t0 = time.perf_counter()
        O.forward_backward(inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], one.H, one.cube_m,
                           one.scale, one.causal)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times[1:]) if len(times) > 2 else times[-1]
    return {"value": one.N / t, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"1 of {cfg.B} sequences (N={cfg.N}, all {cfg.H} heads), fwd+bwd, fp32 torch CPU, "
                      f"median of {len(times) - 1 if len(times) > 2 else 1} timed reps",
            "seconds_per_sequence": t}


def run_reference(args):
    """--impl reference: the CPU formulation of the reference path on the host cores."""
    import torch

    from oracle import morpho_oracle as O
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    C = _configs()
    cfg = C.CONFIGS[args.config]
    one = cfg.with_(B=1)
    torch.set_num_threads(os.cpu_count() or 1)
    inp = C.make_inputs(one)

    def step():
        O.forward_backward(inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], one.H, one.cube_m,
                           one.scale, one.causal)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    value = one.N * args.steps / dt
    cores = torch.get_num_threads()
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: x~N(0,1) seeded, module default init",
            "config": _config_dict(cfg, args.gpus, per_step_note="each step = 1 sequence of the workload"),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": f"1 of {cfg.B} sequences per step (N={cfg.N}, all {cfg.H} heads), fwd+bwd"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _config_dict(cfg, world, per_step_note=None, score="softmax", tau=1.0):
    d = {"workload": f"{cfg.name}: single MorphoAttention layer fwd + backward(out.sum())"
                     + ("" if score == "softmax" else f", soft-morphology score {score} (tau {tau})"),
         "B_per_gpu": cfg.B, "N": cfg.N, "D": cfg.D, "H": cfg.H, "cube_m": cfg.cube_m, "head_dim": cfg.head_dim,
         "scale": cfg.scale, "causal": cfg.causal, "global_batch": cfg.B * world, "seq_len": cfg.N,
         "parallelism": f"dp{world}", "l2": "inputs larger than L2 (>300 MB touched per step), no flush"}
    if per_step_note:
        d["step"] = per_step_note
    if score != "softmax":
        d["score"] = score
        d["tau"] = tau
    return d


def _traffic(kernel, config_name, cfg):
    """DRAM bytes per launch of `kernel` from the committed ncu summary (profiles/traffic.json),
    scaled from the captured batch to this run's batch; None when not captured."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            t = json.load(f).get(kernel)
        if t is None or t.get("config") != config_name:
            return None
        return t["dram_bytes_per_launch"] * cfg.B / _configs().CONFIGS[config_name].B
    except Exception:
        return None


def algorithmic_flops(cfg):
    """Dense-contraction FLOPs per launch of each kernel (recompute included per launch)."""
    m, hd, T = cfg.cube_m, cfg.head_dim, cfg.tokens
    nn = cfg.pairs()
    gemm = 2.0 * T * cfg.D * (cfg.H * m + cfg.D)
    return {"attn_bwd": 2.0 * nn * (3 * m + 2 * hd), "attn_fwd": 2.0 * nn * (m + hd), "proj": gemm,
            "dx_gemm": gemm, "dw_gemm": gemm,
            # soft-morphology split path: S (f16) + E_S.E_V / G.E_V^T, dS.kd / E_S^T.G, dS^T.qc (tf32)
            "soft_morph_tc_fwd": 2.0 * nn * (m + hd), "soft_morph_tc_bwd_q": 2.0 * nn * (2 * m + hd),
            "soft_morph_tc_bwd_k": 2.0 * nn * (2 * m + 2 * hd)}


def reference_kernel_leg(dev):
    """The reference's own CUDA kernel (its ``attention.cu`` compiled unmodified for sm_100a by
    ``oracle/build_ref.py`` into ``oracle/_ref``) timed beside this library on the same GPU, a
    comparator of the baseline leg: the c3 forward (its backward cannot launch at c3: it asks
    for 1,005,056 B of shared memory, 232,448 B are allowed) and forward + backward at
    c3-narrow (B=4, N=4096, D=128, H=2, m=32, scale 0.5), where its backward launches.  CUDA
    events on the current stream after one warm-up call; this library's side in the
    reference's gradient semantics (equal work) and with full gradients."""
    import torch

    from morphottention_b200 import capi
    from oracle import refkernel
    C = _configs()

    def time_ms(fn, reps):
        fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    res = {"source": "reference attention.cu built unmodified (oracle/build_ref.py), CUDA events, same GPU"}
    fwd_cfg = C.CONFIGS["c3"]
    narrow = fwd_cfg.with_(name="c3_narrow", D=128, H=2)
    for cfg in (fwd_cfg, narrow):
        if not refkernel.available(cfg.cube_m, cfg.head_dim, cfg.causal):
            return {"unavailable": "reference kernel not built in oracle/_ref (oracle/build_ref.py)"}
    # c3 forward
    inp = C.make_inputs(fwd_cfg, device=dev)
    args5 = [inp[k] for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")]
    p = capi.problem(fwd_cfg.B, fwd_cfg.N, fwd_cfg.D, fwd_cfg.H, fwd_cfg.cube_m, fwd_cfg.scale, fwd_cfg.causal)
    out = torch.empty_like(inp["x"])
    lse = torch.empty(fwd_cfg.B * fwd_cfg.H, fwd_cfg.N, dtype=torch.float32, device=dev)
    r_ms = time_ms(lambda: refkernel.forward(fwd_cfg, inp), 2)
    o_ms = time_ms(lambda: capi.forward(p, *args5, out, lse), 10)
    res["c3_forward"] = {"reference_ms": r_ms, "ours_ms": o_ms, "reference_tokens_per_s": fwd_cfg.tokens / r_ms * 1e3,
                         "ours_tokens_per_s": fwd_cfg.tokens / o_ms * 1e3, "speedup": r_ms / o_ms,
                         "ours_api": "morpho_sm100_forward (projection + attention forward)"}
    res["c3_backward"] = "reference cannot launch: 1,005,056 B dynamic shared memory > 232,448 B"
    del inp, args5, out, lse
    # c3-narrow forward + backward
    inp = C.make_inputs(narrow, device=dev)
    args5 = [inp[k] for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")]
    g = torch.ones_like(inp["x"])
    out = torch.empty_like(inp["x"])
    lse = torch.empty(narrow.B * narrow.H, narrow.N, dtype=torch.float32, device=dev)
    grads = [torch.empty_like(t) for t in args5]

    def ours(mode):
        q = capi.problem(narrow.B, narrow.N, narrow.D, narrow.H, narrow.cube_m, narrow.scale, narrow.causal, mode)
        saved = torch.empty(capi.saved_bytes(q), dtype=torch.uint8, device=dev)

        def run():
            capi.forward_save(q, *args5, out, lse, saved=saved)
            capi.backward_saved(q, g, saved, *args5, out, lse, *grads)
        return run

    def ref():
        o, l_ = refkernel.forward(narrow, inp)
        refkernel.backward(narrow, inp, o, l_, g)

    r_ms = time_ms(ref, 2)
    o_ms = time_ms(ours(capi.MORPHO_GRAD_REFERENCE), 10)
    f_ms = time_ms(ours(capi.MORPHO_GRAD_FULL), 10)
    res["c3_narrow_fwd_bwd"] = {"shape": "B=4, N=4096, D=128, H=2, cube_m=32, scale 0.5", "reference_ms": r_ms,
                                "ours_ms": o_ms, "ours_full_gradient_ms": f_ms,
                                "reference_tokens_per_s": narrow.tokens / r_ms * 1e3,
                                "ours_tokens_per_s": narrow.tokens / o_ms * 1e3, "speedup": r_ms / o_ms,
                                "ours_api": "forward_save + backward_saved, grad_mode reference (the reference "
                                            "kernel's semantics); full-gradient time beside it"}
    return res


def dp_leg(args, world, rank, dev, barrier):
    """The data-parallel configuration c5 (per rank B=8, N=8192, D=2048, H=16, cube_m=64,
    causal, scale 1.0; global batch 8 x ranks, weak scaling): the training pair on each rank's
    own batch shard, the fp32 weight-gradient bucket all-reduced with NCCL on a communication
    stream overlapped with the dX GEMM, timed on the device as the max over ranks, with the
    all-reduce's own duration per rank (CUDA events on the communication stream).  Then, once,
    the collective is checked: every rank's unreduced bucket is all-gathered and their fp64 sum
    compared with the all-reduced bucket."""
    import torch
    import torch.distributed as dist

    from morphottention_b200 import capi, dp
    from morphottention_b200.configs import CONFIGS, make_inputs
    cfg = CONFIGS["c5"]
    # weights from the configuration's seed (drawn before x, so independent of B and N);
    # each rank's shard of x from its own seeded device generator
    w = {k: v.to(dev) for k, v in make_inputs(cfg.with_(B=1, N=1), device="cpu").items() if k != "x"}
    gen = torch.Generator(device=dev).manual_seed(cfg.seed * 1000 + rank)
    x = torch.randn(cfg.B, cfg.N, cfg.D, generator=gen, device=dev, dtype=torch.float32).half()
    args5 = [x, w["W_phi"], w["gate_q"], w["gate_k"], w["W_V"]]
    p = capi.problem(cfg.B, cfg.N, cfg.D, cfg.H, cfg.cube_m, cfg.scale, cfg.causal)
    grad = torch.ones_like(x)
    out, dX = torch.empty_like(x), torch.empty_like(x)
    lse = torch.empty(cfg.B * cfg.H, cfg.N, dtype=torch.float32, device=dev)
    grads = [torch.empty_like(t) for t in args5[1:]]  # W_phi, gate_q, gate_k, W_V
    saved = torch.empty(capi.saved_bytes(p), dtype=torch.uint8, device=dev)
    n_bucket = capi.weight_grad_elems(p)
    exchange = dp.peer_exchange(n_bucket, device=dev) if world > 1 else None
    own_bucket = torch.empty(n_bucket, dtype=torch.float32, device=dev) if exchange is None else None
    timing = []

    def step(rec=None):
        """One training step; returns the bucket that holds the all-reduced sum (world > 1)."""
        capi.forward_save(p, *args5, out, lse, saved=saved)
        if world > 1:
            b = exchange.bucket() if exchange is not None else own_bucket
            dp.backward_allreduce(p, grad, saved, *args5, out, lse, dX, grads[0], grads[1], grads[2], grads[3],
                                  b, timing=rec, exchange=exchange)
            return b
        capi.backward_saved(p, grad, saved, *args5, out, lse, dX, grads[0], grads[1], grads[2], grads[3])
        return None

    for _ in range(max(3, args.warmup)):
        step()
    steps = args.steps
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step(timing)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    ms = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    ar_ms = (sum(a.elapsed_time(b) for a, b in timing) / len(timing)) if timing else 0.0
    per_rank = torch.tensor([ms.item() / steps, ar_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        gathered = [torch.empty_like(per_rank) for _ in range(world)]
        dist.all_gather(gathered, per_rank)
    else:
        gathered = [per_rank]
    ms_step = float(ms.item()) / steps
    check = None
    if world > 1:
        bucket = step()  # the sum over ranks
        torch.cuda.synchronize()
        local = torch.empty(n_bucket, dtype=torch.float32, device=dev)
        capi.forward_save(p, *args5, out, lse, saved=saved)
        capi.backward_saved(p, grad, saved, *args5, out, lse, dX, None, None, None, None, dweights_f32=local)
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local)
        want = torch.stack(parts).double().sum(0)
        check = {"rel_l2": float((bucket.double() - want).norm() / want.norm()),
                 "what": "all-reduced fp32 bucket vs the fp64 sum of every rank's unreduced bucket (all-gathered; "
                         "recomputed, so it differs from the step's own in the last bits: dq is accumulated by "
                         "TMA reduce-adds in no fixed order)",
                 "bucket_elems": n_bucket}
        del parts, want, local, bucket
    peaks = _peaks()
    tokens = cfg.tokens * world
    res = {"workload": "c5_dp: causal MorphoAttention layer, per rank B=8, N=8192, D=2048, H=16, cube_m=64, "
                       "scale 1.0; fwd + backward(out.sum()), "
                       + ("weight-gradient bucket all-reduced (peer-memory kernel over NVLink)" if exchange is not None
                          else "weight-gradient bucket all-reduced (NCCL)" if world > 1
                          else "one GPU: no all-reduce"),
           "B_per_gpu": cfg.B, "global_batch": cfg.B * world, "n_gpus": world, "steps": steps,
           "ms_per_step": ms_step, "value": tokens / (ms_step / 1000.0), "unit": UNIT, "scaling": "weak",
           "timing": "CUDA events around the steps on each rank, max over ranks",
           "step_roofline_frac": cfg.tensor_flops_fwd_bwd() / (peaks["bf16_tflops_sustained"] * 1e12)
           / (ms_step / 1000.0),
           "per_rank_ms_per_step": [float(t[0]) for t in gathered],
           "allreduce_ms_per_rank": [float(t[1]) for t in gathered] if world > 1 else None,
           "allreduce_bytes": n_bucket * 4 if world > 1 else 0, "dp_check": check}
    del x, out, dX, grad, saved, own_bucket, grads, args5
    torch.cuda.empty_cache()
    return res


def run_ours(args):
    import datetime

    import torch
    import torch.distributed as dist

    import morphottention_b200 as M
    from morphottention_b200 import capi, dp
    from morphottention_b200.configs import CONFIGS, make_inputs

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 under torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    cfg = CONFIGS[args.config]
    if args.batch is not None:
        cfg = cfg.with_(B=args.batch)
    w = make_inputs(cfg, device="cpu")  # weights: identical on every rank
    if world > 1:
        g = torch.Generator().manual_seed(cfg.seed * 1000 + rank)
        w["x"] = torch.empty(cfg.B, cfg.N, cfg.D).normal_(0.0, 1.0, generator=g).half()
    t = {k: v.to(dev) for k, v in w.items()}
    x, W_phi, gq, gk, W_V = t["x"], t["W_phi"], t["gate_q"], t["gate_k"], t["W_V"]
    p = capi.problem(cfg.B, cfg.N, cfg.D, cfg.H, cfg.cube_m, cfg.scale, cfg.causal, score=args.score, tau=args.tau)
    if args.score != "softmax":  # the module path (e2e) reads the score from the op settings
        M.set_score(args.score, args.tau)
    grad = torch.ones_like(x)  # d out.sum() / d out
    out = torch.empty_like(x)
    lse = torch.empty(cfg.B * cfg.H, cfg.N, dtype=torch.float32, device=dev)
    dX = torch.empty_like(x)
    dW_phi, dW_V = torch.empty_like(W_phi), torch.empty_like(W_V)
    dgq, dgk = torch.empty_like(gq), torch.empty_like(gk)
    # data parallel: the peer-memory all-reduce where the GPUs allow it (else NCCL)
    exchange = dp.peer_exchange(capi.weight_grad_elems(p), device=dev) if world > 1 else None
    bucket = None
    if world > 1 and exchange is None:
        bucket = torch.empty(capi.weight_grad_elems(p), dtype=torch.float32, device=dev)

    # the training pair: the forward keeps its projection for the backward (as the
    # module's autograd Function does)
    saved = torch.empty(capi.saved_bytes(p), dtype=torch.uint8, device=dev)

    ar_timing = []  # (start, end) events of each timed all-reduce, on the communication stream

    def step(rec=None):
        capi.forward_save(p, x, W_phi, gq, gk, W_V, out, lse, saved=saved)
        if world > 1:  # weight-gradient all-reduce overlapped with the dX GEMM
            b = exchange.bucket() if exchange is not None else bucket
            dp.backward_allreduce(p, grad, saved, x, W_phi, gq, gk, W_V, out, lse, dX, dW_phi, dgq, dgk, dW_V,
                                  b, timing=rec, exchange=exchange)
        else:
            capi.backward_saved(p, grad, saved, x, W_phi, gq, gk, W_V, out, lse, dX, dW_phi, dgq, dgk, dW_V)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    status = capi.device_status(reset=True)

    # every kernel's time and launch count over as many steps as the timed region, before it;
    # the timed region then times the dominant kernel alone (events around every launch cost
    # the step about 5 us per launch)
    capi.profile_select(None)
    capi.profile_enable(True)
    for _ in range(args.steps):
        step()
    torch.cuda.synchronize()
    prof = capi.profile_collect()
    dom = max(prof.items(), key=lambda kv: kv[1][0])[0] if prof else None
    capi.profile_select(dom)

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        step(ar_timing)
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    allreduce = None
    if world > 1:
        ar = torch.tensor([sum(a.elapsed_time(b) for a, b in ar_timing) / len(ar_timing)], device=dev,
                          dtype=torch.float64)
        ars = [torch.empty_like(ar) for _ in range(world)]
        dist.all_gather(ars, ar)
        allreduce = {"ms_per_rank": [float(t.item()) for t in ars], "bytes": capi.weight_grad_elems(p) * 4,
                     "collective": "peer_allreduce kernel (NVLink peer loads, fused fp16 finalize)"
                     if exchange is not None else "NCCL all_reduce + finalize kernel",
                     "nccl_max_nchannels": os.environ.get("NCCL_MAX_NCHANNELS"),
                     "timing": "CUDA events around each step's all-reduce on the communication stream"}
    prof_live = capi.profile_collect()
    capi.profile_enable(False)
    capi.profile_select(None)
    ms = ev0.elapsed_time(ev1)
    ms_t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    status |= capi.device_status(reset=True)
    tokens_total = cfg.tokens * world * args.steps
    value = tokens_total / (ms / 1000.0)

    # ---- end to end through the public module API: pinned host x -> device, fwd, bwd, loss.item()
    e2e = None
    if not args.no_e2e:
        mod = M.MorphoAttention(cfg.D, cfg.H, cfg.cube_m, scale=cfg.scale, causal=cfg.causal, device=dev)
        with torch.no_grad():
            mod.W_phi.copy_(W_phi)
            mod.W_V.copy_(W_V)
            mod.gate_q.copy_(gq)
            mod.gate_k.copy_(gk)
        # data parallel: gradients averaged over the ranks inside backward, the all-reduce
        # overlapped with the dX GEMM
        model = dp.DataParallelAttention(mod) if world > 1 else mod
        x_host = x.cpu().pin_memory()
        params = list(mod.parameters())
        # Overlapped form, as a prefetching training loop runs: step k+1's host->device input
        # copy runs on a copy stream while step k computes (two device input buffers), and
        # step k's loss comes back by an asynchronous device->host copy that the host reads
        # once step k+1 is queued.  Every step's copies lie inside the timed region.
        copy_stream = torch.cuda.Stream(device=dev)
        x_dev = [torch.empty_like(x) for _ in range(2)]
        landed = [torch.cuda.Event() for _ in range(2)]
        released = [torch.cuda.Event() for _ in range(2)]
        for ev in released:
            ev.record()
        loss_host = torch.zeros(2, dtype=torch.float32).pin_memory()
        fetched = [torch.cuda.Event() for _ in range(2)]

        def prefetch(k):
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(released[k % 2])
                x_dev[k % 2].copy_(x_host, non_blocking=True)
                landed[k % 2].record(copy_stream)

        def e2e_step(k, n, overlap):
            if overlap:
                if k == 0:
                    prefetch(0)
                if k + 1 < n:
                    prefetch(k + 1)
                torch.cuda.current_stream().wait_event(landed[k % 2])
                xd = x_dev[k % 2]
            else:
                xd = x_host.to(dev, non_blocking=True)
            o = model(xd)
            loss = o.sum(dtype=torch.float32)
            for q in params:
                q.grad = None
            loss.backward()
            if not overlap:
                return loss.item()
            released[k % 2].record()
            loss_host[k % 2].copy_(loss.detach(), non_blocking=True)
            fetched[k % 2].record()
            if k > 0:  # the previous step's loss, read while this step runs
                fetched[(k - 1) % 2].synchronize()
                prev = float(loss_host[(k - 1) % 2])
                assert prev == prev, "loss is NaN"
            if k + 1 == n:
                fetched[k % 2].synchronize()
                return float(loss_host[k % 2])
            return None

        def time_e2e(overlap):
            for k in range(max(2, args.warmup)):
                e2e_step(k, max(2, args.warmup), overlap)
            barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for k in range(args.steps):
                e2e_step(k, args.steps, overlap)
            e1.record()
            torch.cuda.synchronize()
            t = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return tokens_total / (float(t.item()) / 1000.0)

        serial = time_e2e(False)
        e2e = {"value": time_e2e(True), "unit": UNIT,
               "h2d_bytes_per_step": x.numel() * x.element_size(), "d2h_bytes_per_step": 4,
               "api": "morphottention_b200.MorphoAttention(x).sum().backward(), loss back to the host",
               "input_copy": "step k+1's pinned host->device copy on a copy stream during step k",
               "loss_read": "step k's loss copied back asynchronously, read on the host during step k+1",
               "value_serial_copy": serial}

    # the data-parallel configuration on every rank (the collective steps are the same on all)
    dp_res = None
    if not args.no_dp_leg and args.config != "c5" and args.score == "softmax" and args.batch is None:
        dp_res = dp_leg(args, world, rank, dev, barrier)

    if rank != 0:
        if world > 1:
            dp.close_exchanges()
            dist.destroy_process_group()
        return

    peaks = _peaks()
    flops = algorithmic_flops(cfg)
    kernels = {}
    total_ms = sum(v[0] for v in prof.values()) or 1.0
    for name, (kms, cnt) in prof.items():
        kernels[name] = {"ms_per_launch": kms / cnt, "launches_per_step": cnt / args.steps, "share": kms / total_ms}
    roof = None
    if dom is not None and dom in prof_live:
        kernels[dom]["ms_per_launch_timed_region"] = prof_live[dom][0] / prof_live[dom][1]
        per_launch_s = prof_live[dom][0] / prof_live[dom][1] / 1000.0
        achieved = flops.get(dom, 0.0) / per_launch_s / 1e12
        peak = peaks["bf16_tflops_sustained"]
        note = f"{peaks['source']} dense bf16 (sustained, kernel timed inside a step); fp16 rate equal"
        if dom.startswith("soft_morph_tc"):  # mostly kind::tf32 MMAs: half the dense 16-bit rate
            peak /= 2.0
            note = f"half the {peaks['source']} dense bf16 rate (sustained): the tf32 rate"
        roof = {"kernel": dom, "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": _traffic(dom, args.config, cfg), "peak_note": note,
                "timing": "CUDA events around each of its launches in the timed region (the other kernels "
                          "untimed there; their shares from as many profiled steps just before it)",
                "flops_per_launch": flops.get(dom, 0.0)}
        if dom in ("attn_bwd", "attn_fwd"):
            sm_mhz = clocks.get("sm_mhz") or peaks["sm_max_mhz"]
            mufu_peak = torch.cuda.get_device_properties(dev).multi_processor_count * 16 * sm_mhz * 1e6
            exps = cfg.pairs()
            roof["mufu_ex2_per_s"] = exps / per_launch_s
            roof["mufu_frac"] = exps / per_launch_s / mufu_peak
            roof["mufu_peak_note"] = f"{torch.cuda.get_device_properties(dev).multi_processor_count} SMs x 16 ex2/clk x {sm_mhz:.0f} MHz"
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16", "data": "synthetic: x~N(0,1) seeded, module default init",
            "config": _config_dict(cfg, world, score=args.score, tau=args.tau), "roofline": roof, "e2e": e2e,
            "gpu_launches": int(sum(v[1] for v in prof.values())), "clocks": clocks, "kernels": kernels,
            "tensor_tflops_step": cfg.tensor_flops_fwd_bwd() / (ms / args.steps / 1000.0) / 1e12,
            "step_roofline_frac": (cfg.tensor_flops_fwd_bwd() / (peaks["bf16_tflops_sustained"] * 1e12))
            / (ms / args.steps / 1000.0),
            "device_status": status, "dp_config": dp_res, "allreduce": allreduce}
    # baseline legs (rank 0 at N = 1): the fp32 CPU oracle on the host cores, and the
    # reference's own CUDA kernel on this GPU
    if world == 1 and not args.no_cpu_baseline and args.score == "softmax":
        line["cpu_baseline"] = cpu_baseline(cfg)
        if args.config == "c3" and args.batch is None and not args.no_reference_kernel:
            line["reference_kernel"] = reference_kernel_leg(dev)
    elif args.score != "softmax":  # the fp32 oracle materialises [B, H, N, N, hd]: not at these sizes
        line["cpu_baseline"] = None
    print(json.dumps(line), flush=True)
    if world > 1:
        dp.close_exchanges()
        dist.destroy_process_group()


VIT_DEPTH = 12
VIT_MLP_RATIO = 4


def _vit_flops(cfg):
    """Tensor FLOPs of one ViT encoder training step: per block the attention layer's
    (projection GEMMs and attention, fwd + bwd) plus the MLP's two Linear layers, forward and
    the two backward GEMMs: 3 * 2 * 2 * T * D * (4 D)."""
    mlp = 3.0 * 2.0 * 2.0 * cfg.tokens * cfg.D * (VIT_MLP_RATIO * cfg.D)
    return VIT_DEPTH * (cfg.tensor_flops_fwd_bwd() + mlp)


def _oracle_attention(dim, num_heads, cube_m, scale=1.0, causal=False, dtype=None, device=None):
    """CPU attention layer for the reference arm of the encoder workload: the module's
    parameters with its default initialisation, and the fp32 oracle as the forward (autograd
    through the oracle's torch ops)."""
    import torch

    from oracle import morpho_oracle as O

    class OracleAttention(torch.nn.Module):
        def __init__(self):
            super().__init__()
            f32 = dict(dtype=torch.float32, device=device)
            std = dim ** -0.5
            self.W_phi = torch.nn.Parameter(torch.empty(dim, num_heads * cube_m, **f32).normal_(0.0, std))
            self.W_V = torch.nn.Parameter(torch.empty(dim, dim, **f32).normal_(0.0, std))
            self.gate_q = torch.nn.Parameter(torch.ones(num_heads, cube_m, **f32))
            self.gate_k = torch.nn.Parameter(torch.ones(num_heads, cube_m, **f32))

        def forward(self, x):
            return O.forward(x, self.W_phi, self.gate_q, self.gate_k, self.W_V, num_heads, cube_m, scale, causal)[0]

    return OracleAttention()


def _vit_cpu_step_seconds(cfg, steps=2, warmup=1):
    """fp32 CPU encoder (oracle attention) on one sequence: seconds per training step."""
    import torch
    Encoder = _load_source("_morpho_bench_encoder", os.path.join("morphottention_b200", "encoder.py")).Encoder
    torch.set_num_threads(os.cpu_count() or 1)
    torch.manual_seed(cfg.seed)
    model = Encoder(depth=VIT_DEPTH, dim=cfg.D, num_heads=cfg.H, cube_m=cfg.cube_m, mlp_ratio=VIT_MLP_RATIO,
                    scale=cfg.scale, dtype=torch.float32, device="cpu", attention=_oracle_attention)
    g = torch.Generator().manual_seed(cfg.seed)
    x = torch.randn(1, cfg.N, cfg.D, generator=g)
    target = torch.randn(1, cfg.N, cfg.D, generator=g)
    opt = torch.optim.SGD(model.parameters(), lr=1e-4)

    def step():
        loss = torch.nn.functional.mse_loss(model(x), target)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()

    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    return (time.perf_counter() - t0) / steps, torch.get_num_threads()


def _vit_config(cfg, world, graph=False):
    return {"workload": f"c4_vit_train: {VIT_DEPTH}-block pre-norm ViT-B encoder (LayerNorm -> MorphoAttention -> "
                        f"LayerNorm -> GELU MLP {VIT_MLP_RATIO * cfg.D}, residuals), MSE loss, SGD step",
            "B_per_gpu": cfg.B, "N": cfg.N, "D": cfg.D, "H": cfg.H, "cube_m": cfg.cube_m, "head_dim": cfg.head_dim,
            "scale": cfg.scale, "causal": cfg.causal, "depth": VIT_DEPTH, "global_batch": cfg.B * world,
            "seq_len": cfg.N, "parallelism": f"dp{world} (DistributedDataParallel)",
            "l2": "activations of 12 blocks (> 1 GB) per step, no flush",
            "cuda_graph": "the whole training step replayed as one captured CUDA graph "
                          "(morphottention_b200.encoder.GraphedTrainingStep)" if graph else "eager"}


def run_vit(args):
    """--config c4vit: the 12-block ViT-B encoder training step around the attention layers."""
    import datetime

    import torch
    import torch.distributed as dist

    from morphottention_b200 import capi
    from morphottention_b200.configs import CONFIGS
    from morphottention_b200.encoder import Encoder, GraphedTrainingStep

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 under torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    cfg = CONFIGS["c4"]
    if args.batch is not None:
        cfg = cfg.with_(B=args.batch)
    torch.manual_seed(cfg.seed)
    model = Encoder(depth=VIT_DEPTH, dim=cfg.D, num_heads=cfg.H, cube_m=cfg.cube_m, mlp_ratio=VIT_MLP_RATIO,
                    scale=cfg.scale, device=dev)
    if world > 1:
        model = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local])
    opt = torch.optim.SGD(model.parameters(), lr=1e-4, foreach=True)
    g = torch.Generator().manual_seed(cfg.seed * 1000 + rank)
    x_host = torch.randn(cfg.B, cfg.N, cfg.D, generator=g).half().pin_memory()
    target = torch.randn(cfg.B, cfg.N, cfg.D, generator=g).to(dev)
    x = x_host.to(dev)

    def step(xd):
        loss = torch.nn.functional.mse_loss(model(xd).float(), target)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
        return loss

    # one rank: the step captured once as a CUDA graph (DistributedDataParallel's hooks stay eager)
    use_graph = world == 1 and not args.eager
    gstep = None
    if use_graph:
        gstep = GraphedTrainingStep(model, lambda out, t: torch.nn.functional.mse_loss(out.float(), t), opt, x,
                                    target, warmup=args.warmup)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def timed(fn, n):
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for k in range(n):
            fn(k)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        t = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        gstep() if use_graph else step(x)
    torch.cuda.synchronize()
    status = capi.device_status(reset=True)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    capi.profile_enable(not use_graph)
    ms = timed(lambda k: gstep() if use_graph else step(x), args.steps)
    clocks = sampler.stop()
    if use_graph:
        # a graph replay runs the launches captured once, past the library's per-launch timers:
        # the attention kernels' times and count come from 3 eager steps of the same model
        capi.profile_enable(True)
        timed(lambda k: step(x), 3)
        prof_steps = 3
    else:
        prof_steps = args.steps
    prof = capi.profile_collect()
    capi.profile_enable(False)
    status |= capi.device_status(reset=True)
    tokens_total = cfg.tokens * world * args.steps
    value = tokens_total / (ms / 1000.0)
    ours_ms = sum(v[0] for v in prof.values()) / prof_steps
    launches = sum(v[1] for v in prof.values()) / prof_steps

    # end to end: the input copied from pinned host memory every step (next step's copy on a
    # copy stream, two device buffers) and the loss read back one step later
    e2e = None
    if not args.no_e2e:
        copy_stream = torch.cuda.Stream(device=dev)
        x_dev = [torch.empty_like(x) for _ in range(2)]
        landed = [torch.cuda.Event() for _ in range(2)]
        released = [torch.cuda.Event() for _ in range(2)]
        fetched = [torch.cuda.Event() for _ in range(2)]
        loss_host = torch.zeros(2, dtype=torch.float32).pin_memory()
        for ev in released:
            ev.record()

        def prefetch(k):
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(released[k % 2])
                x_dev[k % 2].copy_(x_host, non_blocking=True)
                landed[k % 2].record(copy_stream)

        def e2e_step(k, n):
            if k == 0:
                prefetch(0)
            if k + 1 < n:
                prefetch(k + 1)
            torch.cuda.current_stream().wait_event(landed[k % 2])
            loss = gstep(x_dev[k % 2]) if use_graph else step(x_dev[k % 2])
            released[k % 2].record()
            loss_host[k % 2].copy_(loss.detach(), non_blocking=True)
            fetched[k % 2].record()
            if k > 0:
                fetched[(k - 1) % 2].synchronize()
                assert float(loss_host[(k - 1) % 2]) == float(loss_host[(k - 1) % 2])

        for k in range(2):
            e2e_step(k, 2)
        ems = timed(lambda k: e2e_step(k, args.steps), args.steps)
        e2e = {"value": tokens_total / (ems / 1000.0), "unit": UNIT,
               "h2d_bytes_per_step": x.numel() * x.element_size(), "d2h_bytes_per_step": 4,
               "api": ("morphottention_b200.encoder.GraphedTrainingStep over Encoder (MorphoAttention modules)"
                       if use_graph else "morphottention_b200.encoder.Encoder training step (MorphoAttention modules)"),
               "input_copy": "step k+1's pinned host->device copy on a copy stream during step k"}
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    peaks = _peaks()
    flops = _vit_flops(cfg)
    achieved = flops / (ms / args.steps / 1000.0) / 1e12
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16", "data": "synthetic: x, target ~ N(0,1) seeded, default init",
            "config": _vit_config(cfg, world, use_graph),
            "roofline": {"kernel": "whole training step (torch LayerNorm/GELU/cuBLAS MLP + this library's "
                                   "attention)", "bound": "tensor", "achieved": achieved,
                         "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                         "frac": achieved / peaks["bf16_tflops_sustained"], "traffic": None,
                         "flops_per_step": flops},
            "e2e": e2e, "gpu_launches": int(round(launches)), "clocks": clocks,
            "attention_ms_per_step": ours_ms, "attention_share": ours_ms / (ms / args.steps),
            "kernels": {k: {"ms_per_launch": v[0] / v[1], "launches_per_step": v[1] / prof_steps}
                        for k, v in prof.items()},
            "device_status": status}
    if world == 1 and not args.no_cpu_baseline:
        sec, cores = _vit_cpu_step_seconds(cfg)
        line["cpu_baseline"] = {"value": cfg.N / sec, "unit": UNIT, "cores": cores, "kind": "port",
                                "sample": "1 of %d sequences, fp32 CPU encoder with the oracle attention, "
                                          "training step" % cfg.B, "seconds_per_sequence": sec}
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_vit_reference(args):
    """--impl reference --config c4vit: the fp32 CPU encoder (oracle attention), 1 sequence per step."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = _configs().CONFIGS["c4"]
    sec, cores = _vit_cpu_step_seconds(cfg, steps=args.steps, warmup=args.warmup)
    value = cfg.N / sec
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * sec, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic: x, target ~ N(0,1) seeded",
            "config": _vit_config(cfg, args.gpus),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": f"1 of {cfg.B} sequences per step"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_score_probe(args):
    """--probe score: the design comparison behind running the morphological score on the tensor
    cores.  On the configuration's codes (this library's projection), times the packed-half2
    CUDA-core score probe (every pair's qc . k with HFMA2, row maxima with HMNMX2) and this
    library's forward, whose attention kernel issues the same score as tcgen05 MMAs next to the
    softmax and P.V; prints one JSON line with both rates (not the benchmark contract line)."""
    import torch

    from morphottention_b200 import capi
    from morphottention_b200.configs import CONFIGS, make_inputs
    cfg = CONFIGS[args.config if args.config in CONFIGS else "c3"]
    if args.batch is not None:
        cfg = cfg.with_(B=args.batch)
    dev = torch.device("cuda", 0)
    inp = make_inputs(cfg, device=dev)
    p = capi.problem(cfg.B, cfg.N, cfg.D, cfg.H, cfg.cube_m, cfg.scale, cfg.causal)
    o = capi.project(p, inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], with_phi=False)
    rowmax = torch.empty(cfg.B * cfg.H, cfg.N, dtype=torch.float32, device=dev)
    out = torch.empty_like(inp["x"])
    lse = torch.empty(cfg.B * cfg.H, cfg.N, dtype=torch.float32, device=dev)

    def timed(fn, reps):
        for _ in range(max(1, args.warmup)):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    probe_ms = timed(lambda: capi.score_probe_half2(o["qc"], o["kc"], rowmax), args.steps)
    capi.profile_select("attn_fwd")
    capi.profile_enable(True)
    timed(lambda: capi.forward(p, inp["x"], inp["W_phi"], inp["gate_q"], inp["gate_k"], inp["W_V"], out, lse),
          args.steps)
    prof = capi.profile_collect()
    capi.profile_enable(False)
    capi.profile_select(None)
    fwd_ms = prof["attn_fwd"][0] / prof["attn_fwd"][1]
    pairs = cfg.pairs()
    score_flops = 2.0 * cfg.cube_m * pairs
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    line = {"probe": "score", "config": cfg.name, "B": cfg.B, "N": cfg.N, "H": cfg.H, "cube_m": cfg.cube_m,
            "pairs": pairs,
            "half2_score_probe": {"ms": probe_ms, "score_tflops": score_flops / probe_ms / 1e9,
                                  # HFMA2: 64 thread instructions per clock per SM (ncu's
                                  # sm__sass_thread_inst_executed_op_hfma_pred_on peak), 2 FMAs each
                                  "fp16_cuda_core_peak_tflops": sms * 64 * 2 * 2 * 1.965e9 / 1e12,
                                  "work": "qc . k with HFMA2 (fp16 accumulation) and the row maximum (HMNMX2)"},
            "tcgen05_attn_fwd": {"ms": fwd_ms, "score_tflops": score_flops / fwd_ms / 1e9,
                                 "all_tensor_tflops": 2.0 * (cfg.cube_m + cfg.head_dim) * pairs / fwd_ms / 1e9,
                                 "work": "S = qc . k^T (tcgen05), exact online softmax (ex2), P . V (tcgen05)"},
            "speedup_of_tensor_core_forward_over_half2_score_alone": probe_ms / fwd_ms}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="c3", choices=["c1", "c2", "c3", "c4", "c5", "c4vit"],
                    help="c1..c5: one MorphoAttention layer; c4vit: the 12-block ViT-B encoder training step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-dp-leg", action="store_true",
                    help="skip the data-parallel configuration c5 timed after the main workload")
    ap.add_argument("--no-reference-kernel", action="store_true",
                    help="skip timing the reference's own CUDA kernel beside ours (N = 1, c3)")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the per-GPU batch (small cases for profiler captures)")
    ap.add_argument("--score", choices=["softmax", "dilation", "erosion"], default="softmax",
                    help="the attention score: softmax (the reference's), or the soft-morphology aggregation")
    ap.add_argument("--tau", type=float, default=1.0, help="temperature of the soft-morphology score")
    ap.add_argument("--probe", choices=["score"], default=None,
                    help="score: time the packed-half2 CUDA-core score probe against the tcgen05 forward")
    ap.add_argument("--eager", action="store_true",
                    help="c4vit: run the training step eagerly instead of replaying it as a CUDA graph")
    args = ap.parse_args()
    if args.score != "softmax" and (args.impl == "reference" or args.config == "c4vit"):
        raise SystemExit("--score applies to the single-layer configurations of --impl ours")
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.probe == "score":
        run_score_probe(args)
    elif args.config == "c4vit":
        run_vit_reference(args) if args.impl == "reference" else run_vit(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
