"""Checkpoint sidecars of dense EXL3 linears, delivered to their per-shard parameters.

An EXL3 checkpoint keeps one group of tensors per quantised module
(``<module>.trellis / .suh / .svh / .mcg / .mul1``), while ``EXL3LinearMethod``
registers ``exl3_{i}_{suffix}`` parameters, one set per output shard of the SGLang
linear (which may merge several checkpoint modules).  The routing contract is the
reference's (``src/sglang_exl3/sidecar.py:52-120``); names, return values and error
types are kept so loaders written for it work unchanged:

* ``gate_proj`` / ``up_proj`` fill shards 0 / 1 of ``gate_up_proj``, and
  ``q_a_proj`` / ``kv_a_proj_with_mqa`` shards 0 / 1 of
  ``fused_qkv_a_proj_with_mqa``;
* a ``qkv_proj`` stored as one group (q|k|v along the output axis) is cut into the
  layer's shards along whole 16-wide output tiles, sized by the layer's
  ``_exl3_lin_output_partition_sizes``;
* any other EXL3 module fills shard 0;
* expert sidecars (``.experts.``), names that are parameters themselves and modules
  without EXL3 parameters here are left alone (``False``), so a post-load check still
  sees them.

How it is done here: a name is parsed once into a ``SidecarKey``; a small fold table
says which merged module and shard a checkpoint leaf belongs to; the parameter
dictionary is asked for that module's shard parameters; fused groups are cut with
``torch.split`` on tile counts; every (shard, tensor) delivery goes through the
parameter's own ``weight_loader``.
"""

from __future__ import annotations

import itertools
import re
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Sequence, Tuple

import torch

SIDECAR_SUFFIXES = ("trellis", "suh", "svh", "mcg", "mul1")
TILE = 16

_NAME = re.compile(r"^(?:(?P<parent>.+)\.)?(?P<leaf>[^.]+)\.(?P<suffix>" + "|".join(SIDECAR_SUFFIXES) + r")$")

# checkpoint module leaf -> (leaf of the merged SGLang module, shard it fills)
FOLDED_LEAVES: Dict[str, Tuple[str, int]] = {
    "gate_proj": ("gate_up_proj", 0),
    "up_proj": ("gate_up_proj", 1),
    "q_a_proj": ("fused_qkv_a_proj_with_mqa", 0),
    "kv_a_proj_with_mqa": ("fused_qkv_a_proj_with_mqa", 1),
}

# axis along which a fused group's tensor is cut, and the output columns per unit of it
_CUT_AXIS = {"trellis": (1, TILE), "svh": (0, 1)}


@dataclass(frozen=True)
class SidecarKey:
    parent: str   # module path above the leaf ("" at top level)
    leaf: str
    suffix: str

    @property
    def module(self) -> str:
        return f"{self.parent}.{self.leaf}" if self.parent else self.leaf

    def sibling(self, leaf: str) -> str:
        return f"{self.parent}.{leaf}" if self.parent else leaf


def parse_sidecar(name: str) -> Optional[SidecarKey]:
    m = _NAME.match(name)
    if m is None:
        return None
    return SidecarKey(m.group("parent") or "", m.group("leaf"), m.group("suffix"))


def split_sidecar_name(name: str) -> Optional[Tuple[str, str]]:
    """``"m.trellis" -> ("m", "trellis")``; None for anything that is not a sidecar."""
    key = parse_sidecar(name)
    return None if key is None else (key.module, key.suffix)


def split_fused_group(owner_sizes: Sequence[int], suffix: str, tensor: torch.Tensor) -> List[torch.Tensor]:
    """Cut one fused group into per-shard tensors along the output axis: trellis
    ``[in/16, out/16, 16K]`` by tiles of dim 1, svh ``[out]`` along dim 0; suh and
    the scalar markers belong to every shard.  Sizes that are not whole tiles, or a
    tensor whose output extent disagrees with their sum, raise ValueError."""
    sizes = [int(s) for s in owner_sizes]
    if any(s % TILE for s in sizes):
        raise ValueError(f"EXL3 fused split: output sizes {sizes} are not multiples of {TILE}")
    cut = _CUT_AXIS.get(suffix)
    if cut is None:
        return [tensor] * len(sizes)
    axis, per_unit = cut
    want_dims = 3 if suffix == "trellis" else 1
    if tensor.dim() != want_dims or tensor.shape[axis] * per_unit != sum(sizes):
        raise ValueError(f"EXL3 fused {suffix} shape {tuple(tensor.shape)} does not match out={sum(sizes)}")
    return list(torch.split(tensor, [s // per_unit for s in sizes], dim=axis))


def shard_parameters(params: Dict[str, Any], module: str, suffix: str) -> List[Any]:
    """The ``exl3_{i}_{suffix}`` parameters of ``module``, i = 0, 1, ... while shard i
    has a trellis parameter."""
    out = []
    for i in itertools.count():
        if f"{module}.exl3_{i}_trellis" not in params:
            return out
        out.append(params[f"{module}.exl3_{i}_{suffix}"])


def _deliveries(key: SidecarKey, shards: List[Any], fold_shard: int, tensor: torch.Tensor):
    if key.leaf == "qkv_proj" and len(shards) > 1:
        sizes = [int(s) for s in shards[0]._exl3_owner._exl3_lin_output_partition_sizes]
        if len(sizes) != len(shards):
            raise RuntimeError(f"EXL3 fused qkv {key.module}: {len(shards)} shards but output sizes {sizes}")
        return list(enumerate(split_fused_group(sizes, key.suffix, tensor)))
    if fold_shard >= len(shards):
        raise RuntimeError(f"EXL3 sidecar {key.module}.{key.suffix}: shard {fold_shard} of a module "
                           f"with {len(shards)} shards")
    return [(fold_shard, tensor)]


def route_exl3_sidecar(params: Dict[str, Any], name: str, tensor: torch.Tensor) -> bool:
    """Load one checkpoint tensor into its EXL3 shard parameter(s); True when consumed
    (the caller skips the name), False when it is not a dense EXL3 sidecar here.
    Each target parameter receives ``weight_loader(param, tensor, shard_id=i)``."""
    key = parse_sidecar(name)
    if key is None or ".experts." in name or name in params:
        return False
    target_leaf, fold_shard = FOLDED_LEAVES.get(key.leaf, (key.leaf, 0))
    shards = shard_parameters(params, key.sibling(target_leaf), key.suffix)
    if not shards:
        return False
    for i, part in _deliveries(key, shards, fold_shard, tensor):
        shards[i].weight_loader(shards[i], part, shard_id=i)
    return True
