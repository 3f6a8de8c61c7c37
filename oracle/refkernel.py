"""TEST INFRASTRUCTURE ONLY: loader for the reference's own CUDA kernels, built unmodified
from the reference sources by ``oracle/build_ref.py`` into ``oracle/_ref``.

Used by the tests (our kernels against the reference's on identical inputs) and by the
baseline leg of ``bench.py`` (the reference kernel timed beside ours as a comparator).  The
product package never imports it."""

from __future__ import annotations

import ctypes
import os

import torch

REF_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref")

# (cube_m, head_dim, causal) -> variant name (compile-time constants of the reference)
VARIANT_OF = {(16, 32, False): "m16_hd32", (16, 64, False): "m16_hd64", (16, 64, True): "m16_hd64_causal",
              (32, 64, False): "m32_hd64"}
_cache = {}


def available(m, hd, causal) -> bool:
    name = VARIANT_OF.get((m, hd, causal))
    return name is not None and os.path.exists(os.path.join(REF_DIR, f"ref_{name}.so"))


def lib(m, hd, causal):
    name = VARIANT_OF[(m, hd, causal)]
    if name not in _cache:
        L = ctypes.CDLL(os.path.join(REF_DIR, f"ref_{name}.so"))
        vp, i32, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        L.ref_forward.argtypes = [vp] * 7 + [i32] * 6 + [f32, vp, ctypes.c_char_p, i32]
        L.ref_forward.restype = i32
        L.ref_backward.argtypes = [vp] * 13 + [i32] * 6 + [f32, vp, ctypes.c_char_p, i32]
        L.ref_backward.restype = i32
        _cache[name] = L
    return _cache[name]


def forward(cfg, inp):
    L = lib(cfg.cube_m, cfg.head_dim, cfg.causal)
    x = inp["x"]
    out = torch.empty_like(x)
    lse = torch.empty(cfg.B * cfg.H, cfg.N, dtype=torch.float32, device=x.device)
    err = ctypes.create_string_buffer(2048)
    rc = L.ref_forward(x.data_ptr(), inp["W_phi"].data_ptr(), inp["gate_q"].data_ptr(), inp["gate_k"].data_ptr(),
                       inp["W_V"].data_ptr(), out.data_ptr(), lse.data_ptr(), cfg.B, cfg.N, cfg.D, cfg.H,
                       cfg.cube_m, cfg.head_dim, cfg.scale, torch.cuda.current_stream().cuda_stream, err, 2048)
    if rc != 0:
        raise RuntimeError(err.value.decode())
    return out, lse


def backward(cfg, inp, out, lse, grad_out):
    """Reference backward; its outputs must start at zero (the kernel accumulates with
    fp16 atomics, reference attention.cpp:93-98)."""
    L = lib(cfg.cube_m, cfg.head_dim, cfg.causal)
    g = {k: torch.zeros_like(inp[k]) for k in ("x", "W_phi", "gate_q", "gate_k", "W_V")}
    err = ctypes.create_string_buffer(2048)
    rc = L.ref_backward(grad_out.data_ptr(), inp["x"].data_ptr(), inp["W_phi"].data_ptr(), inp["gate_q"].data_ptr(),
                        inp["gate_k"].data_ptr(), inp["W_V"].data_ptr(), out.data_ptr(), lse.data_ptr(),
                        g["x"].data_ptr(), g["W_phi"].data_ptr(), g["gate_q"].data_ptr(), g["gate_k"].data_ptr(),
                        g["W_V"].data_ptr(), cfg.B, cfg.N, cfg.D, cfg.H, cfg.cube_m, cfg.head_dim, cfg.scale,
                        torch.cuda.current_stream().cuda_stream, err, 2048)
    if rc != 0:
        raise RuntimeError(err.value.decode())
    return {"dX": g["x"], "dW_phi": g["W_phi"], "d_gate_q": g["gate_q"], "d_gate_k": g["gate_k"], "dW_V": g["W_V"]}
