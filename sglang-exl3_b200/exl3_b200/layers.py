"""SGLang quant-method surface of the EXL3 backend on the B200 kernels.

Mirrors the reference's plugin classes so a model loads and runs unchanged:

* ``EXL3LinearMethod`` - dense EXL3 linears (``src/sglang_exl3/dense.py:160-408``):
  same parameter names (``exl3_{shard}_{trellis,suh,svh,mcg,mul1}``), loader,
  per-shard codebook markers, fused 2/3-shard paths (gate_up, qkv) now one
  grouped launch, ``apply_kv_only``.  New: tensor-parallel sharding of dense
  layers (column: trellis dim 1 + svh; row: trellis dim 0 + suh, at 128
  multiples), which the reference does not implement (``dense.py:248-264``).
* ``EXL3MoEMethod`` - routed experts (``src/sglang_exl3/exl3.py:1970-2314``): the
  stacked ``w13_*`` / ``w2_*`` layout, the TP / EP loader, marker-based codebook
  detection, device pointer tables, and ``apply`` accepting the dispatcher output
  or ``(x, topk_weights, topk_ids)``.  Routing, experts and the weighted combine
  run in ``exl3b200_moe`` without host synchronisation.
* ``map_topk_to_local`` / ``pin_exl3_expert_map`` - global -> local expert ids,
  invalid ids to the sentinel ``n_local`` (``exl3.py:485-509``).

Without SGLang installed the local base classes below stand in, as in the
reference (``exl3.py:39-67``).
"""

from __future__ import annotations

import itertools
import logging
import math
import os
from typing import Any, Optional

import torch
from torch.nn.parameter import Parameter

from . import moe as _moe
from . import ops as _ops

logger = logging.getLogger("sglang.exl3.b200")

MCG_MARKER_SIGNED_INT32 = -877912083   # 0xCBAC1FED as int32 (exl3.py:92)
MUL1_MARKER_SIGNED_INT32 = -2082680531  # 0x83DCD12D as int32 (exl3.py:94)
SWIGLU_LIMIT_DEFAULT = float("inf")
EXL3_SUFFIXES = ("trellis", "suh", "svh", "mcg", "mul1")

try:  # pragma: no cover - exercised only with SGLang installed
    from sglang.srt.layers.quantization.base_config import FusedMoEMethodBase, LinearMethodBase
except ImportError:
    class QuantizeMethodBase:
        def create_weights(self, layer: torch.nn.Module, *args, **kwargs):
            raise NotImplementedError()

        def apply(self, layer: torch.nn.Module, *args, **kwargs) -> torch.Tensor:
            raise NotImplementedError()

        def process_weights_after_loading(self, layer: torch.nn.Module) -> None:
            pass

    class LinearMethodBase(QuantizeMethodBase):
        pass

    class FusedMoEMethodBase(QuantizeMethodBase):
        runner = None

        def create_moe_runner(self, layer: torch.nn.Module, moe_runner_config: Any):
            self.runner = None


def set_weight_attrs(param: Parameter, extra_attrs: dict) -> None:
    for k, v in extra_attrs.items():
        setattr(param, k, v)


# ---------------------------------------------------------------------------
# tensor-parallel sharding
# ---------------------------------------------------------------------------
# The slice a rank takes of each checkpoint tensor, and the block it must keep whole.
# Column-parallel linears split their output: trellis dim 1 in whole 128-column
# Hadamard blocks (8 tiles) and svh, so each rank's output transform stays local.
# Row-parallel linears split their input: trellis dim 0 and suh, in whole 128-row
# blocks, so each rank's input transform stays local and the partial outputs sum.
# Every other tensor is replicated.  Routed experts are sharded the same way as the
# reference's (exl3.py:347-372); its dense layers have no tensor parallelism.
TP_SPLITS = {
    "column": {"trellis": (1, 8), "svh": (0, 128)},
    "row": {"trellis": (0, 8), "suh": (0, 128)},
}


def tp_shard(tensor: torch.Tensor, suffix: str, kind: str, tp_rank: int, tp_size: int) -> torch.Tensor:
    """This rank's slice of one checkpoint tensor under ``kind`` ("column" or "row")
    parallelism; ValueError unless the extent splits into ``tp_size`` equal slices of
    whole blocks."""
    split = TP_SPLITS[kind].get(suffix)
    if split is None or tp_size <= 1:
        return tensor.contiguous()
    dim, block = split
    extent = int(tensor.shape[dim])
    per_rank, rem = divmod(extent, tp_size)
    if rem or per_rank % block:
        raise ValueError(f"EXL3 TP shard: {suffix} dim {dim} of size {extent} does not split into "
                         f"{tp_size} slices of whole {block}-blocks")
    return tensor.narrow(dim, per_rank * tp_rank, per_rank).contiguous()


def shard_exl3_col(loaded: torch.Tensor, suffix: str, tp_rank: int, tp_size: int) -> torch.Tensor:
    """Column-parallel slice (output tiles of the trellis, svh)."""
    return tp_shard(loaded, suffix, "column", tp_rank, tp_size)


def shard_exl3_row(loaded: torch.Tensor, suffix: str, tp_rank: int, tp_size: int) -> torch.Tensor:
    """Row-parallel slice (input tiles of the trellis, suh)."""
    return tp_shard(loaded, suffix, "row", tp_rank, tp_size)


def _marker_on(t: Optional[torch.Tensor]) -> bool:
    return t is not None and t.numel() > 0 and int(t.reshape(-1)[0]) != 0


_QKV_SHARDS = {"q": 0, "k": 1, "v": 2}


def linear_shard_index(shard_id) -> int:
    """Shard of a dense loader call: None -> 0, "q"/"k"/"v" -> 0/1/2, else an index."""
    if shard_id is None:
        return 0
    key = str(shard_id)
    if key in _QKV_SHARDS:
        return _QKV_SHARDS[key]
    try:
        return int(key)
    except ValueError:
        raise ValueError(f"EXL3 linear shard id {shard_id!r} is neither q/k/v nor an index") from None


class EXL3DenseLinear:
    """One EXL3 linear: trellis, suh, svh, K and codebook (``dense.py:122-157``)."""

    __slots__ = ("trellis", "suh", "svh", "K", "cb", "mcg", "mul1", "in_features", "out_features")

    def __init__(self, trellis, suh, svh, mcg=None, mul1=None):
        self.trellis = trellis.contiguous()
        self.suh = suh.to(torch.float16).contiguous()
        self.svh = svh.to(torch.float16).contiguous()
        self.in_features = int(self.suh.numel())
        self.out_features = int(self.svh.numel())
        K = self.trellis.shape[-1] / 16
        if not float(K).is_integer():
            raise ValueError(f"EXL3 trellis last dim {self.trellis.shape[-1]} is not 16*K")
        self.K = int(K)
        self.mcg = _marker_on(mcg)
        self.mul1 = _marker_on(mul1)
        if self.mcg and self.mul1:
            raise ValueError("EXL3 linear has both mcg and mul1 markers set")
        # no marker = 3INST (cb 0), as exllamav3 does (dense.py:151-157)
        self.cb = _ops.codebook_id(self.mcg, self.mul1)

    def forward(self, x2: torch.Tensor, out_dtype: torch.dtype = torch.float16, out=None) -> torch.Tensor:
        return _ops.matmul(x2, self.trellis, self.suh, self.svh, self.K, self.cb, out_dtype=out_dtype, out=out)


class EXL3LinearMethod(LinearMethodBase):
    """Dense EXL3 linear method (``dense.py:160-408``) on the B200 kernels."""

    def __init__(self, quant_config=None, bits: Optional[int] = None, tp_rank: int = 0, tp_size: int = 1,
                 parallel: str = "none") -> None:
        super().__init__()
        self.quant_config = quant_config
        self.bits = int(bits) if bits is not None else int(getattr(quant_config, "bits", 4))
        self.split_sizes: Optional[list] = None
        self.tp_rank = int(tp_rank)
        self.tp_size = int(tp_size)
        if parallel not in ("none", "column", "row"):
            raise ValueError("parallel must be none, column or row")
        self.parallel = parallel

    def _output_shards(self, output_partition_sizes) -> list:
        """Output sizes of the layer's shards: a merged module whose checkpoint keeps
        separate groups (``split_sizes``, from the quant config) gets one shard each."""
        sizes = [int(s) for s in output_partition_sizes]
        split = self.split_sizes
        if split and len(sizes) == 1 and sum(split) == sizes[0]:
            sizes = [int(s) for s in split]
        return sizes

    def create_weights(self, layer, input_size_per_partition: int, output_partition_sizes: list, input_size: int,
                       output_size: int, params_dtype: torch.dtype, **extra_weight_attrs) -> None:
        """Register the ``exl3_{shard}_{suffix}`` parameters (the checkpoint tensors of
        each output shard land in ``layer._exl3_lin_packs[shard]``) and an empty
        ``weight`` placeholder, which SGLang's model code expects on every linear."""
        sizes = self._output_shards(output_partition_sizes)
        k_in = int(input_size_per_partition)
        if k_in % 16 or any(n % 16 for n in sizes):
            raise ValueError(f"EXL3 trellis tiles are 16-wide; in={k_in} out={sizes}")
        attrs = {k: v for k, v in extra_weight_attrs.items() if k != "weight_loader"}
        layer._exl3_out_dtype = params_dtype or torch.bfloat16
        layer._exl3_lin_packs = [dict.fromkeys(EXL3_SUFFIXES) for _ in sizes]
        layer._exl3_lin_n_shards = len(sizes)
        layer._exl3_lin_input_size_per_partition = k_in
        layer._exl3_lin_output_partition_sizes = sizes
        layer._exl3_linears = None
        if not hasattr(layer, "weight"):
            layer.register_parameter("weight", Parameter(torch.empty(0, dtype=torch.int16), requires_grad=False))
        for shard, suffix in itertools.product(range(len(sizes)), EXL3_SUFFIXES):
            p = Parameter(torch.empty(0), requires_grad=False)
            set_weight_attrs(p, attrs)
            set_weight_attrs(p, {"weight_loader": self._load_linear, "_exl3_owner": layer, "_exl3_shard": shard,
                                 "_exl3_suffix": suffix})
            layer.register_parameter(f"exl3_{shard}_{suffix}", p)

    @staticmethod
    def _shard_index(shard_id) -> int:
        """Shard of a loader call: None -> 0, "q"/"k"/"v" -> 0/1/2, else an index."""
        return linear_shard_index(shard_id)

    def _device_copy(self, src: torch.Tensor, suffix: str) -> torch.Tensor:
        dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else src.device
        if suffix in ("mcg", "mul1") and src.numel() == 1:
            return torch.full((1,), int(src.reshape(())), dtype=torch.int32, device=dev)
        if self.parallel != "none":
            src = tp_shard(src, suffix, self.parallel, self.tp_rank, self.tp_size)
        if suffix in ("suh", "svh"):
            src = src.to(torch.float16)
        return src.to(device=dev).contiguous()

    def _load_linear(self, param, loaded_weight, shard_id=None):
        """weight_loader of every ``exl3_*`` parameter: this rank's slice of the tensor,
        on the current device, into the shard's pack."""
        layer = getattr(param, "_exl3_owner", None)
        suffix = getattr(param, "_exl3_suffix", None)
        if layer is None or suffix is None:
            return
        layer._exl3_lin_packs[linear_shard_index(shard_id)][suffix] = self._device_copy(loaded_weight.detach(), suffix)

    def process_weights_after_loading(self, layer) -> None:
        packs = getattr(layer, "_exl3_lin_packs", None)
        if not packs:
            return
        linears = []
        for i, pack in enumerate(packs):
            if pack.get("trellis") is None:
                raise RuntimeError(f"EXL3 linear shard {i} received no trellis tensor; checkpoint/quantization mismatch?")
            if pack.get("suh") is None or pack.get("svh") is None:
                raise RuntimeError(f"EXL3 linear shard {i} missing suh/svh sign vectors")
            linears.append(EXL3DenseLinear(pack["trellis"], pack["suh"], pack["svh"], pack.get("mcg"), pack.get("mul1")))
        layer._exl3_linears = linears

    def _fusable(self, linears) -> bool:
        l0 = linears[0]
        return all(l.K == l0.K and l.cb == l0.cb and l.in_features == l0.in_features for l in linears)

    def apply(self, layer, x: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        linears = layer._exl3_linears
        if not linears:
            raise RuntimeError("EXL3 linear layers were not built after weight load")
        orig_shape = x.shape
        rows = math.prod(orig_shape[:-1]) if len(orig_shape) > 2 else orig_shape[0]
        scale = None
        if getattr(layer, "_exl3_scale_input", False):  # dense.py:323-336
            x_flat = x.reshape(rows, orig_shape[-1]).float()
            scale = (x_flat.abs().amax(dim=-1, keepdim=True) / 16.0).clamp_min_(1e-6)
            x2 = (x_flat / scale).to(torch.float16).contiguous()
        else:
            x2 = x.reshape(rows, orig_shape[-1])
            if x2.dtype != torch.float16 or not x2.is_contiguous():
                x2 = x2.to(torch.float16).contiguous()
        out_dtype = getattr(layer, "_exl3_out_dtype", x.dtype)
        direct = scale is None and out_dtype in (torch.float16, torch.bfloat16, torch.float32)
        widths = [l.out_features for l in linears]
        y = torch.empty((rows, sum(widths)), dtype=out_dtype if direct else torch.float16, device=x2.device)
        if len(linears) > 1 and self._fusable(linears) and os.environ.get("SGLANG_EXL3_MGEMM", "1") != "0":
            outs, c = [], 0
            for w in widths:
                outs.append(y[:, c:c + w])
                c += w
            _ops.matmul_multi(x2, [(l.trellis, l.suh, l.svh) for l in linears], linears[0].K, linears[0].cb, outs=outs)
        else:
            c = 0
            for l, w in zip(linears, widths):
                l.forward(x2, out=y[:, c:c + w])
                c += w
        if scale is not None:
            y = (y.float() * scale).to(out_dtype)
        elif not direct:
            y = y.to(out_dtype)
        if bias is not None:
            y = y + bias.to(dtype=y.dtype)
        if len(orig_shape) > 2:
            y = y.view(*orig_shape[:-1], y.shape[-1])
        return y

    def apply_kv_only(self, layer, x: torch.Tensor):
        """K and V shards of a 3-shard qkv_proj only (``dense.py:373-408``)."""
        linears = layer._exl3_linears
        if not linears or len(linears) != 3:
            raise RuntimeError("apply_kv_only requires a 3-shard qkv_proj")
        orig_shape = x.shape
        rows = math.prod(orig_shape[:-1]) if len(orig_shape) > 2 else orig_shape[0]
        x2 = x.reshape(rows, orig_shape[-1])
        if x2.dtype != torch.float16 or not x2.is_contiguous():
            x2 = x2.to(torch.float16).contiguous()
        out_dtype = getattr(layer, "_exl3_out_dtype", x.dtype)
        k_lin, v_lin = linears[1], linears[2]
        if self._fusable([k_lin, v_lin]):
            k, v = _ops.matmul_multi(x2, [(k_lin.trellis, k_lin.suh, k_lin.svh), (v_lin.trellis, v_lin.suh, v_lin.svh)],
                                     k_lin.K, k_lin.cb, out_dtype=out_dtype)
        else:
            k, v = k_lin.forward(x2, out_dtype), v_lin.forward(x2, out_dtype)
        if len(orig_shape) > 2:
            k = k.view(*orig_shape[:-1], k.shape[-1])
            v = v.view(*orig_shape[:-1], v.shape[-1])
        return k, v


# ---------------------------------------------------------------------------
# routed experts
# ---------------------------------------------------------------------------

class ExpertIdMap:
    """Global -> local expert ids as one device gather.

    The routing contract is the reference's (``exl3.py:485-509``): an id is replaced by
    its local id when ``expert_map`` (global -> local, -1 elsewhere) gives one in
    ``[0, n_local)``, and by the sentinel ``n_local`` otherwise (negative, past the
    map, or another rank's expert), which the MoE kernels skip.  Here the map is
    folded once into a table of ``n_global + 1`` entries whose last entry is the
    sentinel, and every id outside ``[0, n_global)`` is pointed at it, so a call is a
    ``where`` and a gather, with no host synchronisation (graph-capturable)."""

    def __init__(self, n_local: int, expert_map: Optional[torch.Tensor], device: torch.device):
        if expert_map is None:
            local = torch.arange(n_local, dtype=torch.long, device=device)
        else:
            m = expert_map.to(device=device, dtype=torch.long)
            local = torch.where((m >= 0) & (m < n_local), m, torch.full_like(m, n_local))
        self.table = torch.cat([local, torch.full((1,), n_local, dtype=torch.long, device=device)])
        self.n_global = int(local.numel())
        self.source = expert_map

    def __call__(self, ids: torch.Tensor) -> torch.Tensor:
        ids = ids.to(torch.long)
        inside = (ids >= 0) & (ids < self.n_global)
        return self.table[torch.where(inside, ids, torch.full_like(ids, self.n_global))]


def pin_exl3_expert_map(layer: torch.nn.Module, device: torch.device) -> Optional[torch.Tensor]:
    """Move the layer's ``expert_map`` to ``device`` as int64 (once) and return it."""
    emap = getattr(layer, "expert_map", None)
    if emap is not None and (emap.device != device or emap.dtype != torch.long):
        layer.expert_map = emap = emap.to(device=device, dtype=torch.long)
    return emap


def map_topk_to_local(ids: torch.Tensor, n_local: int, expert_map: Optional[torch.Tensor]) -> torch.Tensor:
    """Global -> local expert ids with the sentinel ``n_local`` for ids that are not
    local (``ExpertIdMap``); ``expert_map`` must already be int64 on the ids' device."""
    if expert_map is not None and (expert_map.device != ids.device or expert_map.dtype != torch.long):
        raise RuntimeError("EXL3 expert_map must be int64 on the hidden-state device: "
                           "call pin_exl3_expert_map before the fused apply")
    return ExpertIdMap(n_local, expert_map, ids.device)(ids)


def _layer_id_map(layer, n_local: int, device: torch.device) -> ExpertIdMap:
    """The layer's cached ``ExpertIdMap``, rebuilt when its expert_map changes."""
    emap = pin_exl3_expert_map(layer, device)
    cached = getattr(layer, "_exl3_id_map", None)
    if cached is None or cached.source is not emap or cached.table.device != device:
        cached = ExpertIdMap(n_local, emap, device)
        layer._exl3_id_map = cached
    return cached


def _suffix_from_mapped_name(weight_name: str) -> str:
    for s in EXL3_SUFFIXES:
        if weight_name.endswith(s):
            return s
    raise ValueError(f"not an EXL3 tensor name: {weight_name}")


class EXL3MoEMethod(FusedMoEMethodBase):
    """Routed-expert EXL3 method (``exl3.py:1970-2314``) on the B200 MoE pipeline."""

    fuse_routed_scaling_factor_in_topk = True

    def __init__(self, quant_config=None, bits: Optional[int] = None, tp_rank: int = 0, tp_size: int = 1) -> None:
        super().__init__()
        self.quant_config = quant_config
        self.bits = int(bits) if bits is not None else int(getattr(quant_config, "bits", 4))
        self.runner = None
        self.tp_rank = int(tp_rank)
        self.tp_size = int(tp_size)

    def create_moe_runner(self, layer, moe_runner_config):
        self.runner = None

    def create_weights(self, layer, num_experts: int, hidden_size: int, intermediate_size_per_partition: int,
                       params_dtype: torch.dtype, **extra_weight_attrs) -> None:
        if hidden_size % 16 or intermediate_size_per_partition % 16:
            raise ValueError("EXL3 trellis tiles are 16-wide; "
                             f"hidden={hidden_size} intermediate_local={intermediate_size_per_partition}")
        k_words = self.bits * 16
        in_tiles = hidden_size // 16
        out_tiles = intermediate_size_per_partition // 16
        extra = {k: v for k, v in extra_weight_attrs.items() if k != "weight_loader"}
        E, H, I = num_experts, hidden_size, intermediate_size_per_partition
        packed = {
            "w13_trellis": torch.empty(E, 2, in_tiles, out_tiles, k_words, dtype=torch.int16),
            "w13_suh": torch.empty(E, 2, H, dtype=torch.float16),
            "w13_svh": torch.empty(E, 2, I, dtype=torch.float16),
            "w13_mcg": torch.zeros((E, 2, 1), dtype=torch.int32),
            "w13_mul1": torch.zeros((E, 2, 1), dtype=torch.int32),
            "w2_trellis": torch.empty(E, out_tiles, in_tiles, k_words, dtype=torch.int16),
            "w2_suh": torch.empty(E, I, dtype=torch.float16),
            "w2_svh": torch.empty(E, H, dtype=torch.float16),
            "w2_mcg": torch.zeros((E, 1), dtype=torch.int32),
            "w2_mul1": torch.zeros((E, 1), dtype=torch.int32),
        }
        for name, t in packed.items():
            p = Parameter(t, requires_grad=False)
            layer.register_parameter(name, p)
            set_weight_attrs(p, extra)
            p.weight_loader = self._load_exl3
            p._exl3_owner = layer
        layer._exl3_hidden_size = H
        layer._exl3_intermediate_local = I
        layer._exl3_k_words = k_words
        layer._exl3_bits = self.bits

    # checkpoint shard id -> (index inside the expert's w13 pair, or None for w2; TP kind)
    EXPERT_SHARDS = {"w1": (0, "column"), "w3": (1, "column"), "w2": (None, "row")}

    def _load_exl3(self, param, loaded_weight, weight_name: str, shard_id: str = "w1", expert_id: int = 0,
                   return_success: bool = False):
        """weight_loader of the stacked expert parameters: this rank's slice of one
        expert tensor into its slot.  An expert that another rank owns is skipped
        (False with ``return_success``); a marker scalar fills its one-element slot."""
        done = True if return_success else None
        owner = getattr(param, "_exl3_owner", None)
        to_local = getattr(owner, "_map_global_expert_id_to_local_expert_id", None)
        if to_local is not None:
            expert_id = to_local(expert_id)
            if expert_id == -1:
                return False if return_success else None
        if shard_id not in self.EXPERT_SHARDS:
            raise ValueError(f"unknown EXL3 shard_id={shard_id}")
        half, kind = self.EXPERT_SHARDS[shard_id]
        suffix = _suffix_from_mapped_name(weight_name)
        src = tp_shard(loaded_weight.detach(), suffix, kind, self.tp_rank, self.tp_size)
        dest = param.data[expert_id] if half is None else param.data[expert_id, half]
        if src.numel() != dest.numel():
            raise RuntimeError(f"EXL3 load shape mismatch {weight_name} shard={shard_id} expert={expert_id}: "
                               f"dest {tuple(dest.shape)} != loaded {tuple(src.shape)}")
        # same element count: the checkpoint's layout of this slot (a 0-d marker, a
        # flattened vector) is taken as the slot's
        dest.copy_(src.reshape(dest.shape))
        return done

    def process_weights_after_loading(self, layer) -> None:
        if not hasattr(layer, "w13_trellis"):
            return
        n_mul1 = int((layer.w13_mul1 != 0).sum() + (layer.w2_mul1 != 0).sum())
        n_mcg = int((layer.w13_mcg != 0).sum() + (layer.w2_mcg != 0).sum())
        cfg_cb = str(getattr(self.quant_config, "codebook", "mcg") or "mcg")
        if n_mul1 > 0 and n_mcg == 0:
            cb = 2
        elif n_mcg > 0 and n_mul1 == 0:
            cb = 1
        else:  # both or none: the reference falls back to the quantization config (exl3.py:2145-2176)
            cb = 2 if cfg_cb == "mul1" else (0 if cfg_cb in ("3inst", "none") else 1)
        layer._exl3_cb = cb
        layer._exl3_use_mul1 = cb == 2
        layer._exl3_use_mcg = cb == 1
        dev = layer.w13_trellis.device
        E = int(layer.w13_trellis.shape[0])

        def ptrs(t: torch.Tensor) -> torch.Tensor:
            return torch.tensor([int(t[e].data_ptr()) for e in range(E)], dtype=torch.int64, device=dev)

        layer._exl3_ptrs = {
            "gate_trellis": ptrs(layer.w13_trellis[:, 0]), "gate_suh": ptrs(layer.w13_suh[:, 0]),
            "gate_svh": ptrs(layer.w13_svh[:, 0]),
            "up_trellis": ptrs(layer.w13_trellis[:, 1]), "up_suh": ptrs(layer.w13_suh[:, 1]),
            "up_svh": ptrs(layer.w13_svh[:, 1]),
            "down_trellis": ptrs(layer.w2_trellis), "down_suh": ptrs(layer.w2_suh), "down_svh": ptrs(layer.w2_svh),
        }
        k13 = int(layer.w13_trellis.shape[-1]) // 16
        k2 = int(layer.w2_trellis.shape[-1]) // 16
        layer._exl3_k_gate = layer._exl3_k_up = k13
        layer._exl3_k_down = k2
        layer._exl3_n_local = E

    @staticmethod
    def _parse_apply_args(args, kwargs):
        d = kwargs.get("dispatch_output")
        if d is None and len(args) >= 1 and hasattr(args[0], "hidden_states") and hasattr(args[0], "topk_output"):
            d = args[0]
        if d is not None:
            tk = d.topk_output
            if not hasattr(tk, "topk_weights") and hasattr(tk, "to_standard"):
                tk = tk.to_standard()
            return d.hidden_states, tk.topk_weights, tk.topk_ids, True
        if len(args) >= 3:
            return args[0], args[1], args[2], False
        if "x" in kwargs and "topk_ids" in kwargs and "topk_weights" in kwargs:
            return kwargs["x"], kwargs["topk_weights"], kwargs["topk_ids"], False
        raise ValueError(f"Unrecognized EXL3MoEMethod.apply arguments: args={args}, kwargs={kwargs}")

    def apply(self, layer, *args, **kwargs):
        x, topk_weights, topk_ids, from_dispatcher = self._parse_apply_args(args, kwargs)
        limit = getattr(getattr(layer, "moe_runner_config", None), "swiglu_limit", None) or SWIGLU_LIMIT_DEFAULT
        out = apply_exl3_experts(x, topk_ids, topk_weights, layer, limit=float(limit))
        if from_dispatcher:
            try:
                from sglang.srt.layers.moe.token_dispatcher.standard import StandardCombineInput
                return StandardCombineInput(hidden_states=out)
            except Exception:
                return (out,)
        return out


def apply_exl3_experts(x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, layer,
                       *, limit: float = SWIGLU_LIMIT_DEFAULT) -> torch.Tensor:
    """Routed experts for ``x [tokens, hidden]``: local ids (``map_topk_to_local``),
    then the device MoE pipeline in chunks of at most 2048 (token, slot) pairs."""
    ptrs = getattr(layer, "_exl3_ptrs", None)
    if not ptrs:
        raise RuntimeError("EXL3 experts were not built after weight load")
    tokens, hidden = x.shape[-2], x.shape[-1]
    x2d = x.reshape(tokens, hidden)
    xh = x2d if (x2d.dtype == torch.float16 and x2d.is_contiguous()) else x2d.to(torch.float16).contiguous()
    n_local = int(layer._exl3_n_local)
    ids = _layer_id_map(layer, n_local, x2d.device)(topk_ids.reshape(tokens, -1)).to(torch.int32)
    w = topk_weights.reshape(tokens, -1).to(torch.float32)
    lim = 0.0 if (limit is None or not math.isfinite(float(limit))) else float(limit)
    topk = ids.shape[1]
    chunk = max(1, _moe.MOE_MAX_PAIRS // topk)
    cap = _moe.workspace_tokens(tokens, chunk)
    out = torch.empty((tokens, hidden), dtype=torch.float32, device=x2d.device)
    for t0 in range(0, tokens, chunk):
        t1 = min(tokens, t0 + chunk)
        _moe.moe_forward(xh[t0:t1], ids[t0:t1], w[t0:t1], ptrs, layer._exl3_k_gate, layer._exl3_k_up,
                         layer._exl3_k_down, layer._exl3_cb, int(layer._exl3_intermediate_local), lim,
                         out=out[t0:t1], max_tokens=cap)
    layer._exl3_last_apply = "b200"
    return out.to(dtype=x.dtype)
