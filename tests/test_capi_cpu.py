"""The C ABI library loads, exports every entry point declared in include/*.h, and its
argument validation works without a GPU (no compute call is made here)."""

import ctypes
import glob
import os
import re

import pytest

from morphottention_b200 import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        names.update(re.findall(r"MORPHO_API\s+[\w\s\*]+?\b(morpho_\w+)\s*\(", src))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    assert {"morpho_sm100_forward", "morpho_sm100_backward", "morpho_sm100_project"} <= names
    assert names == set(capi.EXPORTED), names ^ set(capi.EXPORTED)


def test_library_exports_every_declared_symbol():
    L = capi.lib()
    for name in declared_symbols():
        assert hasattr(L, name), name


def test_workspace_sizes():
    L = capi.lib()
    p = capi.problem(4, 4096, 1024, 16, 32, 0.5, False)
    fw = L.morpho_sm100_forward_workspace_size(ctypes.byref(p))
    bw = L.morpho_sm100_backward_workspace_size(ctypes.byref(p))
    assert 0 < fw < bw
    # codes (2 x fp16 [BH,N,m]) + V (fp16 [BH,N,hd]) + two fp32 bias rows
    assert fw >= 2 * 64 * 4096 * 32 * 2 + 64 * 4096 * 64 * 2 + 2 * 64 * 4096 * 4
    assert capi.weight_grad_elems(p) == 1024 * (512 + 1024) + 2 * 512


def test_invalid_problems_rejected():
    L = capi.lib()
    bad = [capi.problem(0, 16, 64, 2, 16), capi.problem(1, 16, 65, 2, 16), capi.problem(1, 16, 96, 2, 16),
           capi.problem(1, 16, 64, 2, 24), capi.problem(1, 16, 64, 2, 16, grad_mode=7),
           capi.problem(1, 16, 64, 2, 16, projection=3), capi.problem(1, 16, 64, 2, 16, projection=-1)]
    bad_mask = capi.problem(1, 16, 64, 2, 16)
    bad_mask.mask_diag = 2
    bad.append(bad_mask)
    # soft-morphology score: unknown score, non-positive tau, reference gradient mode
    bad += [capi.problem(1, 16, 64, 2, 16, score=3), capi.problem(1, 16, 64, 2, 16, score="dilation", tau=0.0),
            capi.problem(1, 16, 64, 2, 16, score="erosion", tau=-2.0),
            capi.problem(1, 16, 64, 2, 16, score="dilation", grad_mode=capi.MORPHO_GRAD_REFERENCE)]
    for p in bad:
        assert L.morpho_sm100_forward_workspace_size(ctypes.byref(p)) == 0
        rc = L.morpho_sm100_forward(ctypes.byref(p), *([None] * 8), 0, None)
        assert rc == capi.MORPHO_ERR_INVALID
        assert capi.last_error()


def test_null_pointer_rejected_before_device_use():
    L = capi.lib()
    p = capi.problem(1, 16, 64, 2, 16)
    rc = L.morpho_sm100_forward(ctypes.byref(p), *([None] * 8), 0, None)
    assert rc == capi.MORPHO_ERR_INVALID
    assert "NULL" in capi.last_error()


def test_misaligned_pointer_rejected():
    L = capi.lib()
    p = capi.problem(1, 16, 64, 2, 16)
    ptrs = [ctypes.c_void_p(0x1000 + 16 * i) for i in range(8)]
    ptrs[0] = ctypes.c_void_p(0x1002)
    rc = L.morpho_sm100_forward(ctypes.byref(p), *ptrs, 1 << 30, None)
    assert rc == capi.MORPHO_ERR_INVALID
    assert "aligned" in capi.last_error()


def test_soft_morph_workspace_keeps_statistics():
    """With the soft-morphology score the training pair's saved buffer also holds the forward's
    m + log2(l) per (row, channel) (fp32 [B*H, N, hd]) and the tensor-core forward's scratch
    (E_V^T fp32 [B*H, hd, Npad], the column maxima R [B*H, hd], per-256-key partial maxima
    [B*H, ceil(N/256), hd], the fallback flag and the row references m [B*H, Npad]); the softmax
    score needs none of it."""
    L = capi.lib()
    a = capi.problem(2, 100, 128, 2, 16)
    b = capi.problem(2, 100, 128, 2, 16, score="dilation", tau=0.5)
    extra = L.morpho_sm100_saved_bytes(ctypes.byref(b)) - L.morpho_sm100_saved_bytes(ctypes.byref(a))
    BH, N, Npad, hd = 4, 100, 128, 64
    need = BH * N * hd * 4 + BH * hd * Npad * 4 + BH * hd * 4 + BH * 1 * hd * 4 + 64 * 4 + BH * Npad * 4
    assert need <= extra <= need + 6 * 256


@pytest.mark.parametrize("H", [4, 2, 1])  # head dims 32, 64, 128 at D = 128
def test_soft_morph_backward_workspace_holds_tensor_core_operands(H):
    """The backward workspace of a soft-morphology problem also holds the fp32 operand layouts of
    its tensor-core kernels (G [B*H, N, hd], G^T and E_V [B*H, hd, Npad], kd^T and qc^T
    [B*H, m, Npad]) for every head dim; the softmax score needs none of them."""
    L = capi.lib()
    B, N, D, m = 2, 100, 128, 16
    a = capi.problem(B, N, D, H, m)
    b = capi.problem(B, N, D, H, m, score="erosion", tau=0.7)
    extra = L.morpho_sm100_backward_workspace_size(ctypes.byref(b)) - L.morpho_sm100_backward_workspace_size(
        ctypes.byref(a))
    BH, hd, Npad = B * H, D // H, 128
    operands = 4 * (BH * N * hd + 2 * BH * hd * Npad + 2 * BH * m * Npad)
    assert extra >= operands


def test_bucket_holds_the_temperature_gradient_for_soft_morphology():
    """The fp32 weight-gradient bucket gains one last element, dL/dtau, for the dilation and
    erosion scores (no device needed: sizes only)."""
    base = capi.weight_grad_elems(capi.problem(2, 64, 128, 2, 16))
    assert base == 128 * (2 * 16 + 128) + 2 * 2 * 16
    for score in ("dilation", "erosion"):
        assert capi.weight_grad_elems(capi.problem(2, 64, 128, 2, 16, score=score, tau=0.5)) == base + 1
