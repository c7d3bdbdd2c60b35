"""Strict Hugging Face safetensors loader.

Parity: ``nanovllm/utils/loader.py:9-151`` -- walk every ``*.safetensors``
file, apply checkpoint prefix remapping (``model.language_model.`` ->
``model.``), skip explicit prefixes (``model.visual.``; ``mtp.`` for the
target), include-only prefixes (``mtp.`` for the MTP head), skip ``*_scale_inv``,
alias-aware tied embeddings, a ``LoadReport`` and strict failure on missing or
unexpected tensors.

Design: every packed parameter of a model declares the checkpoint tensors it
is built from and a build function (``checkpoint_plan()``), so the loader pulls
exactly the tensors each parameter needs (lazily, one file handle per shard)
and fills the parameter in one copy, already TP-sharded and packed.
"""

from __future__ import annotations

import glob
import os
import zlib
from dataclasses import dataclass, field
from typing import Callable

import torch
from torch import nn


@dataclass
class LoadReport:
    loaded_parameters: list[str] = field(default_factory=list)
    consumed_tensors: list[str] = field(default_factory=list)
    skipped_tensors: list[str] = field(default_factory=list)
    missing_tensors: list[str] = field(default_factory=list)
    unexpected_tensors: list[str] = field(default_factory=list)

    @property
    def ok(self) -> bool:
        return not self.missing_tensors and not self.unexpected_tensors


def _normalize(name: str, mapping) -> str:
    for src, dst in mapping:
        if name.startswith(src):
            return dst + name[len(src):]
    return name


def _resolve(module: nn.Module, dotted: str) -> nn.Parameter:
    obj = module
    for part in dotted.split("."):
        obj = obj[int(part)] if part.isdigit() else getattr(obj, part)
    return obj


class _Checkpoint:
    """Lazy name -> tensor access over all safetensors shards of a directory."""

    def __init__(self, path: str, mapping):
        from safetensors import safe_open

        files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
        if not files:
            raise FileNotFoundError(f"no *.safetensors files in {path}")
        self._handles = [safe_open(f, framework="pt", device="cpu") for f in files]
        self.index: dict[str, tuple[int, str]] = {}
        for i, h in enumerate(self._handles):
            for raw in h.keys():
                self.index[_normalize(raw, mapping)] = (i, raw)

    def get(self, name: str) -> torch.Tensor:
        i, raw = self.index[name]
        return self._handles[i].get_tensor(raw)


def _fill(param: torch.Tensor, value: torch.Tensor, name: str) -> None:
    if tuple(value.shape) != tuple(param.shape):
        raise ValueError(f"shape mismatch for {name}: checkpoint gives {tuple(value.shape)}, "
                         f"parameter is {tuple(param.shape)}")
    with torch.no_grad():
        param.copy_(value.to(device=param.device, dtype=param.dtype))


def load_model(model: nn.Module, path: str, *, strict: bool = True,
               include_prefixes: tuple[str, ...] | None = None) -> LoadReport:
    mapping = getattr(model, "checkpoint_prefix_mapping", ())
    skipped = tuple(getattr(model, "explicitly_skipped_prefixes", ()))
    include = include_prefixes or tuple(getattr(model, "checkpoint_included_prefixes", ()) or ())
    ckpt = _Checkpoint(path, mapping)
    report = LoadReport()
    available: set[str] = set()
    for name in ckpt.index:
        if name.endswith("_scale_inv"):
            report.skipped_tensors.append(name)
        elif include and not name.startswith(include):
            report.skipped_tensors.append(name)
        elif not include and skipped and name.startswith(skipped):
            report.skipped_tensors.append(name)
        else:
            available.add(name)
    consumed: set[str] = set()
    for pname, (sources, build) in model.checkpoint_plan().items():
        miss = [s for s in sources if s not in available]
        if miss:
            report.missing_tensors.extend(miss)
            continue
        cache: dict[str, torch.Tensor] = {}

        def get(key: str, _cache=cache) -> torch.Tensor:
            if key not in _cache:
                _cache[key] = ckpt.get(key)
            return _cache[key]

        _fill(_resolve(model, pname), build(get), pname)
        consumed.update(sources)
        report.loaded_parameters.append(pname)
    # A tied LM head is an alias of the embedding table.
    if getattr(model, "tied", False) and "lm_head.weight" in available:
        consumed.add("lm_head.weight")
    report.consumed_tensors = sorted(consumed)
    report.unexpected_tensors = sorted(available - consumed)
    report.missing_tensors = sorted(set(report.missing_tensors))
    if strict and not report.ok:
        raise RuntimeError(f"strict checkpoint load failed: missing={report.missing_tensors[:8]} "
                           f"(total {len(report.missing_tensors)}), unexpected={report.unexpected_tensors[:8]} "
                           f"(total {len(report.unexpected_tensors)})")
    return report


def init_dummy(model: nn.Module, hf_cfg, *, seed: int = 0, std: float = 0.02) -> LoadReport:
    """Random-initialise ``model`` through its checkpoint plan (no files).

    Each checkpoint tensor is generated on the parameter's device from a
    seed derived from ``seed`` and the tensor name, with the same init rule as
    ``models.presets.random_state_dict``.
    """
    from inference_systems_b200.models.weights import hf_parameter_shapes

    shapes = hf_parameter_shapes(hf_cfg, include_mtp=True)
    report = LoadReport()
    for pname, (sources, build) in model.checkpoint_plan().items():
        param = _resolve(model, pname)
        dev = param.device

        def get(key: str, _dev=dev, _dtype=param.dtype) -> torch.Tensor:
            shape, kind = shapes[key]
            if kind == "matrix":
                gen = torch.Generator(device=_dev).manual_seed((seed * 1000003 + zlib.crc32(key.encode())) & 0x7FFFFFFF)
                return torch.empty(shape, device=_dev, dtype=torch.float32).normal_(0.0, std, generator=gen).to(_dtype)
            if kind in ("zero_norm", "a_log"):
                return torch.zeros(shape, device=_dev)
            return torch.ones(shape, device=_dev)

        _fill(param, build(get), pname)
        report.loaded_parameters.append(pname)
        report.consumed_tensors.extend(sources)
    return report
