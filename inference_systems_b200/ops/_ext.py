"""Loader for the in-tree sm_100a extension (``inference_systems_b200/_C*.so``).

The extension registers its kernels as ``torch.ops.isb.*`` (see
``csrc/ops.cpp``).  It is built in-tree by ``python setup.py build_ext
--inplace`` (or ``__graft_entry__.build()``); nothing is JIT-compiled at run
time, and a CUDA call without the built extension raises.
"""

from __future__ import annotations

import importlib

import torch

_loaded = False


def load_extension() -> None:
    global _loaded
    if _loaded:
        return
    try:
        importlib.import_module("inference_systems_b200._C")
    except ImportError as exc:  # pragma: no cover - exercised on GPU boxes only
        raise RuntimeError(
            "inference_systems_b200._C (the sm_100a kernel library) is not built; "
            "run `python setup.py build_ext --inplace` in the repository root"
        ) from exc
    _loaded = True


def extension_available() -> bool:
    try:
        load_extension()
    except RuntimeError:
        return False
    return True


def cuda_ops():
    load_extension()
    return torch.ops.isb
