"""ctypes binding of the C ABI in ``include/morpho_sm100.h`` (``libmorpho_sm100.so``).

This is the binding a non-torch host (or a test) uses; the torch ops in ``_C.so`` call
the same entry points.  Tensors passed in must be contiguous CUDA tensors on the
current device; the workspace is allocated by the caller (here: torch).
"""

from __future__ import annotations

import ctypes
import os

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIBRARY_PATH = os.path.join(_PKG_DIR, "libmorpho_sm100.so")

MORPHO_OK = 0
MORPHO_ERR_INVALID = 1
MORPHO_ERR_CUDA = 2
MORPHO_ERR_WORKSPACE = 3
MORPHO_ERR_DEVICE = 4
MORPHO_ERR_TIMEOUT = 5
MORPHO_ERR_UNSUPPORTED = 6
PEER_HANDLE_BYTES = 64
PEER_PCI_ID_BYTES = 32
MORPHO_GRAD_FULL = 0
MORPHO_GRAD_REFERENCE = 1
MORPHO_PROJ_SIGMOID = 0
MORPHO_PROJ_HARDTANH01 = 1
MORPHO_PROJ_IDENTITY = 2
PROJECTIONS = {"sigmoid": MORPHO_PROJ_SIGMOID, "hardtanh01": MORPHO_PROJ_HARDTANH01,
               "identity": MORPHO_PROJ_IDENTITY}
MORPHO_SCORE_SOFTMAX = 0
MORPHO_SCORE_DILATION = 1
MORPHO_SCORE_EROSION = 2
SCORES = {"softmax": MORPHO_SCORE_SOFTMAX, "dilation": MORPHO_SCORE_DILATION, "erosion": MORPHO_SCORE_EROSION}

EXPORTED = (
    "morpho_sm100_forward_workspace_size",
    "morpho_sm100_backward_workspace_size",
    "morpho_sm100_forward",
    "morpho_sm100_backward",
    "morpho_sm100_saved_bytes",
    "morpho_sm100_backward_saved_workspace_size",
    "morpho_sm100_forward_save",
    "morpho_sm100_backward_saved",
    "morpho_sm100_backward_saved_dp",
    "morpho_sm100_project",
    "morpho_sm100_forward_noalloc",
    "morpho_sm100_forward_noalloc_max_scratch",
    "morpho_sm100_weight_grad_elems",
    "morpho_sm100_finalize_weight_grads",
    "morpho_sm100_last_error",
    "morpho_sm100_device_status",
    "morpho_sm100_last_launch_count",
    "morpho_sm100_selftest_wait_timeout",
    "morpho_sm100_profile_enable",
    "morpho_sm100_profile_collect",
    "morpho_sm100_profile_select",
    "morpho_sm100_score_probe_half2",
    "morpho_sm100_peer_create",
    "morpho_sm100_peer_connect",
    "morpho_sm100_peer_bucket",
    "morpho_sm100_peer_allreduce_finalize",
    "morpho_sm100_peer_destroy",
)


class MorphoProblem(ctypes.Structure):
    _fields_ = [("B", ctypes.c_int32), ("N", ctypes.c_int32), ("D", ctypes.c_int32), ("H", ctypes.c_int32),
                ("cube_m", ctypes.c_int32), ("scale", ctypes.c_float), ("causal", ctypes.c_int32),
                ("grad_mode", ctypes.c_int32), ("projection", ctypes.c_int32), ("mask_diag", ctypes.c_int32),
                ("score", ctypes.c_int32), ("tau", ctypes.c_float)]


class MorphoError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"morpho_sm100 error {code}: {msg}")
        self.code = code


_lib = None


def lib() -> ctypes.CDLL:
    """Load ``libmorpho_sm100.so`` once and declare the prototypes."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIBRARY_PATH):
        raise ImportError(f"{LIBRARY_PATH} is missing; build it with `python morphottention_b200/build.py`")
    L = ctypes.CDLL(LIBRARY_PATH)
    P = ctypes.POINTER(MorphoProblem)
    vp, sz, i32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
    L.morpho_sm100_forward_workspace_size.argtypes = [P]
    L.morpho_sm100_forward_workspace_size.restype = sz
    L.morpho_sm100_backward_workspace_size.argtypes = [P]
    L.morpho_sm100_backward_workspace_size.restype = sz
    L.morpho_sm100_weight_grad_elems.argtypes = [P]
    L.morpho_sm100_weight_grad_elems.restype = sz
    L.morpho_sm100_forward.argtypes = [P] + [vp] * 7 + [vp, sz, vp]
    L.morpho_sm100_forward.restype = i32
    L.morpho_sm100_backward.argtypes = [P] + [vp] * 14 + [vp, sz, vp]
    L.morpho_sm100_backward.restype = i32
    L.morpho_sm100_saved_bytes.argtypes = [P]
    L.morpho_sm100_saved_bytes.restype = sz
    L.morpho_sm100_backward_saved_workspace_size.argtypes = [P]
    L.morpho_sm100_backward_saved_workspace_size.restype = sz
    L.morpho_sm100_forward_save.argtypes = [P] + [vp] * 7 + [vp, sz, vp]
    L.morpho_sm100_forward_save.restype = i32
    L.morpho_sm100_backward_saved.argtypes = [P, vp, vp, sz] + [vp] * 13 + [vp, sz, vp]
    L.morpho_sm100_backward_saved.restype = i32
    L.morpho_sm100_backward_saved_dp.argtypes = [P, vp, vp, sz] + [vp] * 10 + [vp, sz, vp]
    L.morpho_sm100_backward_saved_dp.restype = i32
    L.morpho_sm100_forward_noalloc.argtypes = [P] + [vp] * 7 + [vp]
    L.morpho_sm100_forward_noalloc.restype = i32
    L.morpho_sm100_forward_noalloc_max_scratch.argtypes = []
    L.morpho_sm100_forward_noalloc_max_scratch.restype = sz
    L.morpho_sm100_project.argtypes = [P] + [vp] * 11 + [vp]
    L.morpho_sm100_project.restype = i32
    L.morpho_sm100_finalize_weight_grads.argtypes = [P, vp, ctypes.c_float, vp, vp, vp, vp, vp]
    L.morpho_sm100_finalize_weight_grads.restype = i32
    L.morpho_sm100_last_error.argtypes = []
    L.morpho_sm100_last_error.restype = ctypes.c_char_p
    L.morpho_sm100_device_status.argtypes = [vp, i32, ctypes.POINTER(ctypes.c_uint32)]
    L.morpho_sm100_device_status.restype = i32
    L.morpho_sm100_last_launch_count.argtypes = []
    L.morpho_sm100_last_launch_count.restype = i32
    L.morpho_sm100_selftest_wait_timeout.argtypes = [ctypes.c_uint32, vp]
    L.morpho_sm100_selftest_wait_timeout.restype = i32
    L.morpho_sm100_profile_enable.argtypes = [i32]
    L.morpho_sm100_profile_enable.restype = None
    L.morpho_sm100_profile_select.argtypes = [ctypes.c_char_p]
    L.morpho_sm100_profile_select.restype = None
    L.morpho_sm100_profile_collect.argtypes = [ctypes.c_char_p, i32, ctypes.POINTER(ctypes.c_float),
                                               ctypes.POINTER(ctypes.c_int), i32]
    L.morpho_sm100_profile_collect.restype = i32
    L.morpho_sm100_score_probe_half2.argtypes = [vp, vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, vp, vp]
    L.morpho_sm100_score_probe_half2.restype = i32
    L.morpho_sm100_peer_create.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, vp, ctypes.c_char_p,
                                           ctypes.POINTER(vp)]
    L.morpho_sm100_peer_create.restype = i32
    L.morpho_sm100_peer_connect.argtypes = [vp, ctypes.c_char_p, ctypes.c_char_p]
    L.morpho_sm100_peer_connect.restype = i32
    L.morpho_sm100_peer_bucket.argtypes = [vp]
    L.morpho_sm100_peer_bucket.restype = vp
    L.morpho_sm100_peer_allreduce_finalize.argtypes = [vp, P, ctypes.c_float, vp, vp, vp, vp, vp]
    L.morpho_sm100_peer_allreduce_finalize.restype = i32
    L.morpho_sm100_peer_destroy.argtypes = [vp]
    L.morpho_sm100_peer_destroy.restype = i32
    _lib = L
    return L


def problem(B, N, D, H, cube_m, scale=1.0, causal=False, grad_mode=MORPHO_GRAD_FULL, projection=MORPHO_PROJ_SIGMOID,
            mask_diag=False, score=MORPHO_SCORE_SOFTMAX, tau=1.0) -> MorphoProblem:
    if isinstance(projection, str):
        projection = PROJECTIONS[projection]
    if isinstance(score, str):
        score = SCORES[score]
    return MorphoProblem(B, N, D, H, cube_m, float(scale), 1 if causal else 0, int(grad_mode), int(projection),
                         1 if mask_diag else 0, int(score), float(tau))


def last_error() -> str:
    return lib().morpho_sm100_last_error().decode()


def _check(rc: int) -> None:
    if rc != MORPHO_OK:
        raise MorphoError(rc, last_error())


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream) -> int:
    import torch
    s = torch.cuda.current_stream() if stream is None else stream
    return s.cuda_stream


def forward(p: MorphoProblem, X, W_phi, gate_q, gate_k, W_V, out, lse, stream=None) -> None:
    """Run the forward through the C ABI, with a torch-allocated workspace."""
    import torch
    L = lib()
    ws_bytes = L.morpho_sm100_forward_workspace_size(ctypes.byref(p))
    if ws_bytes == 0:
        raise MorphoError(MORPHO_ERR_INVALID, last_error())
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=X.device)
    _check(L.morpho_sm100_forward(ctypes.byref(p), _ptr(X), _ptr(W_phi), _ptr(gate_q), _ptr(gate_k), _ptr(W_V),
                                  _ptr(out), _ptr(lse), _ptr(ws), ws_bytes, _stream(stream)))


def forward_noalloc(p: MorphoProblem, X, W_phi, gate_q, gate_k, W_V, out, lse, stream=None) -> None:
    """Forward without any device allocation: the scratch is the library's built-in array
    (see ``morpho_sm100_forward_noalloc`` in include/morpho_sm100.h)."""
    _check(lib().morpho_sm100_forward_noalloc(ctypes.byref(p), _ptr(X), _ptr(W_phi), _ptr(gate_q), _ptr(gate_k),
                                              _ptr(W_V), _ptr(out), _ptr(lse), _stream(stream)))


def forward_noalloc_max_scratch() -> int:
    return int(lib().morpho_sm100_forward_noalloc_max_scratch())


def backward(p: MorphoProblem, grad_out, X, W_phi, gate_q, gate_k, W_V, out, lse, dX, dW_phi, d_gate_q, d_gate_k,
             dW_V, dweights_f32=None, stream=None) -> None:
    """Run the backward through the C ABI, with a torch-allocated workspace."""
    import torch
    L = lib()
    ws_bytes = L.morpho_sm100_backward_workspace_size(ctypes.byref(p))
    if ws_bytes == 0:
        raise MorphoError(MORPHO_ERR_INVALID, last_error())
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=X.device)
    _check(L.morpho_sm100_backward(ctypes.byref(p), _ptr(grad_out), _ptr(X), _ptr(W_phi), _ptr(gate_q),
                                   _ptr(gate_k), _ptr(W_V), _ptr(out), _ptr(lse), _ptr(dX), _ptr(dW_phi),
                                   _ptr(d_gate_q), _ptr(d_gate_k), _ptr(dW_V), _ptr(dweights_f32), _ptr(ws),
                                   ws_bytes, _stream(stream)))


def saved_bytes(p: MorphoProblem) -> int:
    n = int(lib().morpho_sm100_saved_bytes(ctypes.byref(p)))
    if n == 0:
        raise MorphoError(MORPHO_ERR_INVALID, last_error())
    return n


def forward_save(p: MorphoProblem, X, W_phi, gate_q, gate_k, W_V, out, lse, saved=None, stream=None):
    """Forward that keeps the projection outputs for ``backward_saved``; returns the
    ``saved`` uint8 CUDA tensor (allocated here when not given)."""
    import torch
    n = saved_bytes(p)
    if saved is None:
        saved = torch.empty(n, dtype=torch.uint8, device=X.device)
    _check(lib().morpho_sm100_forward_save(ctypes.byref(p), _ptr(X), _ptr(W_phi), _ptr(gate_q), _ptr(gate_k),
                                           _ptr(W_V), _ptr(out), _ptr(lse), _ptr(saved), saved.numel(),
                                           _stream(stream)))
    return saved


def backward_saved(p: MorphoProblem, grad_out, saved, X, W_phi, gate_q, gate_k, W_V, out, lse, dX, dW_phi,
                   d_gate_q, d_gate_k, dW_V, dweights_f32=None, stream=None) -> None:
    """Backward reading the projection ``forward_save`` kept (no projection recompute)."""
    import torch
    L = lib()
    ws_bytes = L.morpho_sm100_backward_saved_workspace_size(ctypes.byref(p))
    if ws_bytes == 0:
        raise MorphoError(MORPHO_ERR_INVALID, last_error())
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=X.device)
    _check(L.morpho_sm100_backward_saved(ctypes.byref(p), _ptr(grad_out), _ptr(saved), saved.numel(), _ptr(X),
                                         _ptr(W_phi), _ptr(gate_q), _ptr(gate_k), _ptr(W_V), _ptr(out), _ptr(lse),
                                         _ptr(dX), _ptr(dW_phi), _ptr(d_gate_q), _ptr(d_gate_k), _ptr(dW_V),
                                         _ptr(dweights_f32), _ptr(ws), ws_bytes, _stream(stream)))


def backward_saved_dp(p: MorphoProblem, grad_out, saved, X, W_phi, gate_q, gate_k, W_V, out, lse, dX,
                      dweights_f32, bucket_ready=None, stream=None) -> None:
    """Data-parallel ``backward_saved``: the weight gradients go to the fp32 bucket, which is
    complete before dX; ``bucket_ready`` (a ``torch.cuda.Event``) is recorded at that point."""
    import torch
    L = lib()
    ws_bytes = L.morpho_sm100_backward_saved_workspace_size(ctypes.byref(p))
    if ws_bytes == 0:
        raise MorphoError(MORPHO_ERR_INVALID, last_error())
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=X.device)
    ev = None
    if bucket_ready is not None:
        if not bucket_ready.cuda_event:  # torch creates the CUDA event on its first record
            bucket_ready.record()
        ev = bucket_ready.cuda_event
    _check(L.morpho_sm100_backward_saved_dp(ctypes.byref(p), _ptr(grad_out), _ptr(saved), saved.numel(), _ptr(X),
                                            _ptr(W_phi), _ptr(gate_q), _ptr(gate_k), _ptr(W_V), _ptr(out),
                                            _ptr(lse), _ptr(dX), _ptr(dweights_f32), ev, _ptr(ws), ws_bytes,
                                            _stream(stream)))


def project(p: MorphoProblem, X, W_phi, gate_q, gate_k, W_V, stream=None, with_phi=True) -> dict:
    """Projection only; returns {qc, kc, v, qb, cb, phi} (layouts of morpho_sm100_project)."""
    import torch
    BH, N, m, hd = p.B * p.H, p.N, p.cube_m, p.D // p.H
    npad = (N + 127) // 128 * 128
    dev = X.device
    o = {"qc": torch.empty(BH, N, m, dtype=torch.float16, device=dev),
         "kc": torch.empty(BH, N, m, dtype=torch.float16, device=dev),
         "v": torch.empty(BH, N, hd, dtype=torch.float16, device=dev),
         "qb": torch.empty(BH, npad, dtype=torch.float32, device=dev),
         "cb": torch.empty(BH, npad, dtype=torch.float32, device=dev),
         "phi": torch.empty(BH, N, m, dtype=torch.float32, device=dev) if with_phi else None}
    _check(lib().morpho_sm100_project(ctypes.byref(p), _ptr(X), _ptr(W_phi), _ptr(gate_q), _ptr(gate_k), _ptr(W_V),
                                      _ptr(o["qc"]), _ptr(o["kc"]), _ptr(o["v"]), _ptr(o["qb"]), _ptr(o["cb"]),
                                      _ptr(o["phi"]), _stream(stream)))
    return o


def finalize_weight_grads(p: MorphoProblem, bucket, alpha, dW_phi, d_gate_q, d_gate_k, dW_V, stream=None) -> None:
    _check(lib().morpho_sm100_finalize_weight_grads(ctypes.byref(p), _ptr(bucket), float(alpha), _ptr(dW_phi),
                                                    _ptr(d_gate_q), _ptr(d_gate_k), _ptr(dW_V), _stream(stream)))


def device_status(reset: bool = True, stream=None) -> int:
    """Read (and by default clear) the device status word; raises on a timed-out wait."""
    v = ctypes.c_uint32(0)
    rc = lib().morpho_sm100_device_status(_stream(stream), 1 if reset else 0, ctypes.byref(v))
    if rc != MORPHO_OK:
        raise MorphoError(rc, last_error())
    return v.value


def last_launch_count() -> int:
    return int(lib().morpho_sm100_last_launch_count())


def weight_grad_elems(p: MorphoProblem) -> int:
    return int(lib().morpho_sm100_weight_grad_elems(ctypes.byref(p)))


def profile_enable(on: bool) -> None:
    """Record a CUDA event pair around every kernel launch of the library."""
    lib().morpho_sm100_profile_enable(1 if on else 0)


def profile_select(kernel_name: str | None) -> None:
    """Time only the launches of ``kernel_name`` (a name profile_collect reports); None: all."""
    lib().morpho_sm100_profile_select(kernel_name.encode() if kernel_name else None)


def profile_collect(max_kernels: int = 32) -> dict:
    """{kernel name: (total ms, launches)} of the launches recorded on this thread."""
    name_len = 64
    names = ctypes.create_string_buffer(name_len * max_kernels)
    ms = (ctypes.c_float * max_kernels)()
    cnt = (ctypes.c_int * max_kernels)()
    n = lib().morpho_sm100_profile_collect(names, name_len, ms, cnt, max_kernels)
    out = {}
    for i in range(n):
        nm = names.raw[i * name_len:(i + 1) * name_len].split(b"\0", 1)[0].decode()
        out[nm] = (float(ms[i]), int(cnt[i]))
    return out


class _DeviceArray:
    """A raw fp32 device buffer seen by torch through the CUDA array interface (no copy)."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 2,
                                         "strides": None, "stream": None}


def peer_create(rank: int, world: int, bucket_elems: int):
    """Create this rank's peer-exchange region; returns (group handle, IPC handle bytes, PCI bus id bytes)."""
    h = ctypes.create_string_buffer(PEER_HANDLE_BYTES)
    pci = ctypes.create_string_buffer(PEER_PCI_ID_BYTES)
    g = ctypes.c_void_p()
    _check(lib().morpho_sm100_peer_create(rank, world, bucket_elems, h, pci, ctypes.byref(g)))
    return g.value, h.raw, pci.raw


def peer_connect(group: int, handles: list, pci_ids: list) -> None:
    """Map every rank's region (``handles`` and ``pci_ids`` in rank order, as peer_create gave them)."""
    _check(lib().morpho_sm100_peer_connect(group, b"".join(handles), b"".join(pci_ids)))


def peer_bucket(group: int, n: int, device) -> torch.Tensor:
    """The fp32 bucket of the group's next all-reduce as a tensor view (``n`` elements)."""
    import torch
    ptr = lib().morpho_sm100_peer_bucket(group)
    return torch.as_tensor(_DeviceArray(ptr, n), device=device)


def peer_allreduce_finalize(group: int, p: MorphoProblem, alpha: float, dW_phi, d_gate_q, d_gate_k, dW_V,
                            stream=None) -> None:
    _check(lib().morpho_sm100_peer_allreduce_finalize(group, ctypes.byref(p), alpha, _ptr(dW_phi), _ptr(d_gate_q),
                                                      _ptr(d_gate_k), _ptr(dW_V), _stream(stream)))


def peer_destroy(group: int) -> None:
    _check(lib().morpho_sm100_peer_destroy(group))


def score_probe_half2(qc, kc, rowmax, stream=None) -> None:
    """Row maxima of qc . k^T over all keys on packed half2 CUDA-core math (the design probe
    ``morpho_sm100_score_probe_half2``); qc, kc fp16 [BH, N, m], rowmax fp32 [BH, N]."""
    BH, N, m = qc.shape
    _check(lib().morpho_sm100_score_probe_half2(_ptr(qc), _ptr(kc), BH, N, m, _ptr(rowmax), _stream(stream)))


def selftest_wait_timeout(limit_us: int = 20000, stream=None) -> None:
    """Launch the failure-path self test (a bounded wait that is made to run out)."""
    _check(lib().morpho_sm100_selftest_wait_timeout(int(limit_us), _stream(stream)))
