"""Checkpoint sidecars of dense EXL3 linears routed onto their per-shard parameters.

An EXL3 checkpoint stores one group of tensors per quantised module
(``<module>.trellis / .suh / .svh / .mcg / .mul1``); ``EXL3LinearMethod`` registers
``exl3_{i}_{suffix}`` parameters, one set per output shard of the (possibly merged)
SGLang linear.  Routing rules (reference src/sglang_exl3/sidecar.py:52-120):

* ``gate_proj`` / ``up_proj`` go to shards 0 / 1 of ``gate_up_proj``;
  ``q_a_proj`` / ``kv_a_proj_with_mqa`` to shards 0 / 1 of
  ``fused_qkv_a_proj_with_mqa``;
* a ``qkv_proj`` stored as one group (q|k|v along the output axis) is cut along
  its 16-wide output tiles into the layer's shards, sized by the layer's
  ``_exl3_lin_output_partition_sizes``;
* any other EXL3 module goes to shard 0;
* expert sidecars (``.experts.``), names that are parameters themselves and
  modules with no EXL3 parameters here are not consumed (False), so a post-load
  check still sees them and fails closed.
"""

from __future__ import annotations

from typing import Any, Dict, List, Optional, Tuple

import torch

SIDECAR_SUFFIXES = ("trellis", "suh", "svh", "mcg", "mul1")
TILE = 16

# checkpoint module leaf -> (leaf of the merged SGLang module, its shard index)
MERGED_LEAVES = {
    "gate_proj": ("gate_up_proj", 0),
    "up_proj": ("gate_up_proj", 1),
    "q_a_proj": ("fused_qkv_a_proj_with_mqa", 0),
    "kv_a_proj_with_mqa": ("fused_qkv_a_proj_with_mqa", 1),
}


def split_sidecar_name(name: str) -> Optional[Tuple[str, str]]:
    """``"m.trellis" -> ("m", "trellis")``; None for anything that is not a sidecar."""
    base, dot, suffix = name.rpartition(".")
    if dot and base and suffix in SIDECAR_SUFFIXES:
        return base, suffix
    return None


def split_fused_group(owner_sizes: List[int], suffix: str, tensor: torch.Tensor) -> List[torch.Tensor]:
    """Cut one fused group into per-shard tensors along the output axis.

    trellis ``[in/16, out/16, 16K]`` is cut along dim 1 (in 16-wide tiles), svh
    ``[out]`` along dim 0; suh and the scalar markers belong to every shard.
    Output sizes that are not multiples of 16, or tensors whose output extent
    disagrees with their sum, raise ValueError.
    """
    bad = [s for s in owner_sizes if int(s) % TILE]
    if bad:
        raise ValueError(f"EXL3 fused split: output sizes {owner_sizes} are not multiples of {TILE}")
    total = sum(int(s) for s in owner_sizes)
    bounds = []
    o = 0
    for s in owner_sizes:
        bounds.append((o, o + int(s)))
        o += int(s)
    if suffix == "trellis":
        if tensor.dim() != 3 or tensor.shape[1] * TILE != total:
            raise ValueError(f"EXL3 fused trellis shape {tuple(tensor.shape)} does not match out={total}")
        return [tensor[:, a // TILE:b // TILE, :] for a, b in bounds]
    if suffix == "svh":
        if tensor.dim() != 1 or tensor.shape[0] != total:
            raise ValueError(f"EXL3 fused svh shape {tuple(tensor.shape)} does not match out={total}")
        return [tensor[a:b] for a, b in bounds]
    return [tensor] * len(owner_sizes)


def _shard_count(params: Dict[str, Any], module: str) -> int:
    n = 0
    while f"{module}.exl3_{n}_trellis" in params:
        n += 1
    return n


def route_exl3_sidecar(params: Dict[str, Any], name: str, tensor: torch.Tensor) -> bool:
    """Load one checkpoint tensor into its EXL3 shard parameter(s).

    Returns True when consumed (the caller skips the name), False when the tensor is
    not a dense EXL3 sidecar here.  Each target parameter's ``weight_loader(param,
    tensor, shard_id=i)`` receives it.
    """
    parsed = split_sidecar_name(name)
    if parsed is None or ".experts." in name or name in params:
        return False
    module, suffix = parsed
    parent, _, leaf = module.rpartition(".")
    prefix = parent + "." if parent else ""
    target, shard = module, 0
    if leaf in MERGED_LEAVES:
        merged, shard = MERGED_LEAVES[leaf]
        target = prefix + merged
    n = _shard_count(params, target)
    if n == 0:
        return False
    if leaf == "qkv_proj" and n > 1:
        owner = params[f"{target}.exl3_0_{suffix}"]._exl3_owner
        sizes = [int(s) for s in owner._exl3_lin_output_partition_sizes]
        if len(sizes) != n:
            raise RuntimeError(f"EXL3 fused qkv {target}: {n} shards but output sizes {sizes}")
        for i, part in enumerate(split_fused_group(sizes, suffix, tensor)):
            p = params[f"{target}.exl3_{i}_{suffix}"]
            p.weight_loader(p, part, shard_id=i)
        return True
    if shard >= n:
        raise RuntimeError(f"EXL3 sidecar {name}: shard {shard} but {target} has {n} shards")
    p = params[f"{target}.exl3_{shard}_{suffix}"]
    p.weight_loader(p, tensor, shard_id=shard)
    return True
