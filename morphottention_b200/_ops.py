"""Op loader: registers ``torch.ops.morphottention.*`` from the in-tree ``_C.so``.

Mirrors the reference loader (``torch-ext/morphottention/_cmake_ops.py:15-34``): the
compiled extension is required, and importing fails loudly when it is missing.  There is
no CPU or eager fallback.
"""

from __future__ import annotations

import os

import torch

_NAMESPACE = "morphottention"
_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIBRARY_PATH = os.path.join(_PKG_DIR, "libmorpho_sm100.so")
SHIM_PATH = os.path.join(_PKG_DIR, "_C.so")


def _load_c_extension() -> None:
    if not os.path.exists(SHIM_PATH) or not os.path.exists(LIBRARY_PATH):
        raise ImportError(
            f"Could not find the compiled morphottention_b200 extension in {_PKG_DIR} "
            "(_C.so and libmorpho_sm100.so). Build it with `python morphottention_b200/build.py`.")
    if not hasattr(torch.ops, _NAMESPACE) or not hasattr(getattr(torch.ops, _NAMESPACE), "forward"):
        torch.ops.load_library(SHIM_PATH)


_load_c_extension()

ops = getattr(torch.ops, _NAMESPACE)


def add_op_namespace_prefix(op_name: str) -> str:
    return f"{_NAMESPACE}::{op_name}"
