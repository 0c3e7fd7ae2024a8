"""``EXL3Config``: the quantization config that hands SGLang layers to the B200 methods.

Same construction, parsing and per-layer decisions as the reference's config
(src/sglang_exl3/exl3.py:1554-1967): it reads ``quantization_config.json``
(``bits``, ``codebook``, ``scope``, ``layer_bits``, ``non_routed_exl3``,
``tensor_storage``, ``mtp_*``), resolves a module's bits from its stored trellis
width (``trellis[-1] / 16``), splits merged modules stored as separate children
(``gate_up_proj``, ``fused_qkv_a_proj_with_mqa``) and returns, per layer:

* routed-expert layers -> ``EXL3MoEMethod`` (draft / MTP layers too, unless
  ``SGLANG_EXL3_MTP_EXL3=0``; ``mtp_experts="source"`` layers go to the
  non-routed delegate);
* linears stored as EXL3 in a dense scope (or matched by ``non_routed_exl3``, or
  in a draft layer) -> ``EXL3LinearMethod``, column- or row-parallel after the
  SGLang layer class, with the layer's ``tp_rank`` / ``tp_size``;
* attention, embeddings, linears stored as plain weights and everything else ->
  SGLang's own method (its unquantized or FP8 delegate), or None without SGLang.

Differences, by design: the codebook may also be ``"3inst"`` (the B200 kernels
decode all three codebooks; the reference's CUDA path reaches only MCG and
mul1), and ``get_min_capability`` is 100, the only architecture these kernels are
built for.
"""

from __future__ import annotations

import logging
import os
import re
from typing import Any, Dict, List, Optional, Tuple

import torch

from .layers import EXL3LinearMethod, EXL3MoEMethod

logger = logging.getLogger("sglang.exl3.b200")

try:  # pragma: no cover - exercised only with SGLang installed
    from sglang.srt.layers.quantization.base_config import QuantizationConfig
except ImportError:
    class QuantizationConfig:  # stand-in base without SGLang (reference exl3.py:63-67)
        def __init__(self) -> None:
            self.packed_modules_mapping: Dict[str, List[str]] = {}

        def update_packed_modules_mapping(self, mapping: Dict[str, List[str]]) -> None:
            self.packed_modules_mapping.update(mapping)

SUPPORTED_BITS = (2, 3, 4, 5, 6)
SUPPORTED_CODEBOOKS = ("mcg", "mul1", "3inst")

# merged SGLang modules whose checkpoint stores one group per child projection
MERGED_STORAGE_CHILDREN = {
    "gate_up_proj": ("gate_proj", "up_proj"),
    "fused_qkv_a_proj_with_mqa": ("q_a_proj", "kv_a_proj_with_mqa"),
}
_COLUMN_CLASSES = ("ColumnParallelLinear", "MergedColumnParallelLinear", "QKVParallelLinear")
_ROW_CLASSES = ("RowParallelLinear",)
_LAYER_RE = re.compile(r"(?:^|\.)layers\.(\d+)(?:\.|$)")


def _alias(name: str) -> str:
    """Packs record ``model.language_model.layers.N``; SGLang asks for ``model.layers.N``."""
    return name.replace("model.language_model.", "model.", 1)


def _stored(tensor_storage: Any):
    for module, entry in dict(tensor_storage or {}).items():
        yield str(module), dict((entry or {}).get("stored_tensors") or {})


def tensor_storage_kinds(tensor_storage: Any) -> Dict[str, str]:
    """Module prefix -> ``"exl3"`` (stores a ``.trellis``) or ``"native"`` (plain tensors)."""
    kinds: Dict[str, str] = {}
    for module, stored in _stored(tensor_storage):
        if not stored:
            continue
        kind = "exl3" if any(str(t).endswith(".trellis") for t in stored) else "native"
        kinds[module] = kinds[_alias(module)] = kind
    return kinds


def storage_kind_for_prefix(kinds: Dict[str, str], prefix: str) -> Optional[str]:
    """A module's storage kind; a merged module takes its children's common kind.

    Children of different kinds raise RuntimeError (reference exl3.py:1480-1501).
    """
    if prefix in kinds:
        return kinds[prefix]
    parent, _, leaf = prefix.rpartition(".")
    children = MERGED_STORAGE_CHILDREN.get(leaf)
    if not children:
        return None
    base = parent + "." if parent else ""
    found = {kinds[base + c] for c in children if base + c in kinds}
    if len(found) > 1:
        raise RuntimeError(f"EXL3 storage: merged module {prefix} has mixed child kinds {sorted(found)}")
    return found.pop() if found else None


def tensor_storage_out_sizes(tensor_storage: Any) -> Dict[str, int]:
    """Output width of each EXL3 module from its stored trellis ``[in/16, out/16, 16K]``."""
    out: Dict[str, int] = {}
    for module, stored in _stored(tensor_storage):
        for tname, meta in stored.items():
            shape = (meta or {}).get("shape") or []
            if str(tname).endswith(".trellis") and len(shape) == 3:
                out[module] = out[_alias(module)] = int(shape[1]) * 16
    return out


def tensor_storage_bits(tensor_storage: Any) -> Tuple[Dict[str, int], Dict[int, int]]:
    """(bits per module, expert bits per layer) from the stored trellis widths.

    A layer whose experts disagree raises ValueError: the expert kernels take one K
    per layer (reference exl3.py:1522-1551).
    """
    module_bits: Dict[str, int] = {}
    layer_bits: Dict[int, int] = {}
    for module, stored in _stored(tensor_storage):
        for tname, meta in stored.items():
            shape = (meta or {}).get("shape") or []
            if not str(tname).endswith(".trellis") or not shape:
                continue
            if int(shape[-1]) % 16:
                raise ValueError(f"bad trellis shape for {module}: {shape}")
            bits = int(shape[-1]) // 16
            module_bits[module] = module_bits[_alias(module)] = bits
            m = _LAYER_RE.search(module)
            if ".experts." in module and m is not None:
                layer = int(m.group(1))
                if layer_bits.setdefault(layer, bits) != bits:
                    raise ValueError(f"mixed expert bits in layer {layer}: {layer_bits[layer]} vs {bits}")
    return module_bits, layer_bits


def _has_suffix(prefix: str, suffix: str) -> bool:
    return prefix == suffix or prefix.endswith("." + suffix)


def _sglang_unquantized():
    try:  # pragma: no cover - depends on SGLang
        from sglang.srt.layers.quantization.unquant import UnquantizedLinearMethod

        return UnquantizedLinearMethod()
    except Exception:
        return None


class EXL3Config(QuantizationConfig):
    """EXL3 quantization config (``quant_method: exl3``) for the B200 backend."""

    _LAYER_RE = _LAYER_RE

    def __init__(self, bits: int = 4, codebook: str = "mcg", scope: str = "glm53_routed_experts_only",
                 **kwargs: Any) -> None:
        super().__init__()
        self.bits = int(bits)
        self.codebook = str(codebook).lower()
        self.scope = str(scope)
        if self.bits not in SUPPORTED_BITS:
            raise ValueError(f"unsupported EXL3 bits={self.bits}")
        if self.codebook not in SUPPORTED_CODEBOOKS:
            raise ValueError(f"unsupported codebook={codebook!r}; must be one of {SUPPORTED_CODEBOOKS}")
        self.layer_bits: Dict[int, int] = {int(k): int(v) for k, v in dict(kwargs.pop("layer_bits", None) or {}).items()}
        for layer, b in self.layer_bits.items():
            if b not in SUPPORTED_BITS:
                raise ValueError(f"unsupported EXL3 bits={b} for layer {layer}")
        self.non_routed_exl3: Dict[str, Any] = dict(kwargs.pop("non_routed_exl3", None) or {})
        nr_bits = self.non_routed_exl3.get("bits")
        if nr_bits is not None and nr_bits not in SUPPORTED_BITS:
            raise ValueError(f"unsupported non_routed_exl3 bits={nr_bits}")
        if self.non_routed_exl3.get("codebook", "mcg") not in SUPPORTED_CODEBOOKS:
            raise ValueError(f"unsupported non_routed_exl3 codebook={self.non_routed_exl3.get('codebook')!r}")
        self.raw_config = dict(kwargs)
        self.tensor_storage_kinds: Dict[str, str] = {}
        self.tensor_storage_out_sizes: Dict[str, int] = {}
        self.tensor_storage_bits: Dict[str, int] = {}
        self.storage_layer_bits: Dict[int, int] = {}
        self.non_routed_quantization: Optional[dict] = None
        self.non_routed_dtype_policy = ""
        self.mtp_experts = "exl3"
        self.mtp_experts_start_layer: Optional[int] = None
        self.mtp_bits = self.bits

    # -- identity ---------------------------------------------------------------------------
    def get_name(self) -> str:
        return "exl3"

    def get_supported_act_dtypes(self) -> List[torch.dtype]:
        return [torch.bfloat16, torch.float16, torch.float32]

    @classmethod
    def get_min_capability(cls) -> int:
        return 100  # sm_100a kernels only

    @staticmethod
    def get_config_filenames() -> List[str]:
        return ["quantization_config.json"]

    def get_scaled_act_names(self) -> List[str]:
        return []

    def apply_weight_name_mapper(self, hf_to_sglang_mapper: Any) -> None:
        pass

    @classmethod
    def override_quantization_method(cls, hf_quant_cfg: Dict[str, Any], user_quant: Optional[str],
                                     hf_config: Any = None) -> Optional[str]:
        return "exl3" if str((hf_quant_cfg or {}).get("quant_method", "")).lower() == "exl3" else None

    @classmethod
    def from_config(cls, config: Dict[str, Any]) -> "EXL3Config":
        own = {"bits", "codebook", "scope", "quant_method", "tensor_storage", "non_routed_exl3",
               "non_routed_quantization", "mtp_experts", "mtp_experts_start_layer"}
        inst = cls(bits=int(config.get("bits", 4)), codebook=str(config.get("codebook", "mcg")),
                   scope=str(config.get("scope", "glm53_routed_experts_only")),
                   non_routed_exl3=config.get("non_routed_exl3"),
                   **{k: v for k, v in config.items() if k not in own})
        # a config that only says quant_method=exl3 is a dense pack: every linear is EXL3
        if "scope" not in config and str(config.get("quant_method", "")).lower() == "exl3":
            inst.scope = "dense_and_moe"
        storage = config.get("tensor_storage")
        inst.non_routed_quantization = config.get("non_routed_quantization")
        inst.non_routed_dtype_policy = str(config.get("non_routed_dtype_policy", ""))
        inst.mtp_experts = str(config.get("mtp_experts", "exl3"))
        inst.mtp_experts_start_layer = config.get("mtp_experts_start_layer")
        inst.tensor_storage_kinds = tensor_storage_kinds(storage)
        inst.tensor_storage_out_sizes = tensor_storage_out_sizes(storage)
        inst.tensor_storage_bits, inst.storage_layer_bits = tensor_storage_bits(storage)
        mtp = config.get("mtp_bits")
        inst.mtp_bits = int(mtp) if mtp is not None else int(config.get("bits", inst.bits))
        return inst

    # -- per-module facts -------------------------------------------------------------------
    def merged_split_sizes(self, prefix: str) -> Optional[List[int]]:
        """Child output widths of a merged module stored as separate EXL3 children, else None."""
        parent, _, leaf = (prefix or "").rpartition(".")
        children = MERGED_STORAGE_CHILDREN.get(leaf)
        if not children:
            return None
        base = parent + "." if parent else ""
        sizes = [self.tensor_storage_out_sizes.get(base + c) for c in children]
        return None if any(s is None for s in sizes) else [int(s) for s in sizes]

    def bits_for_prefix(self, prefix: str) -> int:
        """Stored trellis width first, then the layer's stored expert bits, then ``layer_bits``."""
        if prefix in self.tensor_storage_bits:
            return self.tensor_storage_bits[prefix]
        m = _LAYER_RE.search(prefix or "")
        if m is None:
            return self.bits
        layer = int(m.group(1))
        if layer in self.storage_layer_bits:
            return self.storage_layer_bits[layer]
        return self.layer_bits.get(layer, self.bits)

    def _matches_non_routed_exl3(self, prefix: str) -> bool:
        nr = self.non_routed_exl3
        if not nr:
            return False
        if prefix in (nr.get("layers") or {}):
            return True
        return any(_has_suffix(prefix, m) for m in nr.get("modules") or [])

    def _bits_for_non_routed(self, prefix: str) -> int:
        nr = self.non_routed_exl3
        if not nr:
            return self.bits
        default = int(nr.get("bits", self.bits))
        layers = nr.get("layers") or {}
        if prefix in layers:
            return int(layers[prefix].get("bits", default))
        for suffix in nr.get("modules") or []:
            if _has_suffix(prefix, suffix):
                per = nr.get("layer_bits") or {}
                return int(per[suffix]) if suffix in per else default
        return default

    def _bf16_shards_for(self, prefix: str) -> List[int]:
        layers = (self.non_routed_exl3 or {}).get("layers") or {}
        return list(layers[prefix].get("bf16_shards", [])) if prefix in layers else []

    @staticmethod
    def is_draft_prefix(prefix: str) -> bool:
        p = (prefix or "").lower()
        return "stages." in p or "mtp" in p or "nextn" in p

    # -- method selection -------------------------------------------------------------------
    def _linear_method(self, layer: torch.nn.Module, bits: int) -> EXL3LinearMethod:
        cls_name = layer.__class__.__name__
        tp_size = int(getattr(layer, "tp_size", 1) or 1)
        tp_rank = int(getattr(layer, "tp_rank", 0) or 0)
        parallel = "none"
        if tp_size > 1:
            if cls_name in _ROW_CLASSES:
                parallel = "row"
            elif cls_name in _COLUMN_CLASSES:
                parallel = "column"
        return EXL3LinearMethod(self, bits=bits, tp_rank=tp_rank, tp_size=tp_size, parallel=parallel)

    def _delegate_method(self, layer: torch.nn.Module, prefix: str, draft: bool):
        d = self._draft_delegate() if draft else self._non_routed_delegate()
        if d is not None and hasattr(d, "get_quant_method"):
            return d.get_quant_method(layer, prefix)
        return None

    def get_quant_method(self, layer: torch.nn.Module, prefix: str):
        cls_name = layer.__class__.__name__
        prefix = prefix or ""
        draft = self.is_draft_prefix(prefix)
        m = _LAYER_RE.search(prefix)
        layer_num = int(m.group(1)) if m else -1

        if ("MoE" in cls_name or "RoutedExperts" in cls_name or hasattr(layer, "num_local_experts")):
            if draft:
                if os.environ.get("SGLANG_EXL3_MTP_EXL3", "1") == "1":
                    return EXL3MoEMethod(self, bits=int(self.mtp_bits or self.bits_for_prefix(prefix)))
                return self._delegate_method(layer, prefix, True)
            if self.mtp_experts == "source":
                start = self.mtp_experts_start_layer if self.mtp_experts_start_layer is not None else 43
                if layer_num >= int(start):
                    return self._delegate_method(layer, prefix, False)
            return EXL3MoEMethod(self, bits=self.bits_for_prefix(prefix))

        if "RadixAttention" in cls_name:
            return self._delegate_method(layer, prefix, draft)

        lm_head = "lm_head" in prefix.lower() or "ParallelLMHead" in cls_name
        if "VocabParallelEmbedding" in cls_name and not lm_head:
            return None  # embedding tables stay bf16
        if not (lm_head or "Linear" in cls_name):
            return None

        nr = self.non_routed_exl3 or {}
        if any(_has_suffix(prefix, mod) for mod in nr.get("bf16_modules") or []):
            return _sglang_unquantized()
        if not draft and self.tensor_storage_kinds and storage_kind_for_prefix(self.tensor_storage_kinds,
                                                                              prefix) != "exl3":
            logger.debug("EXL3 storage: %s stays native", prefix)
            return _sglang_unquantized()
        dense = self.scope in ("dense_and_moe", "dense") or os.environ.get("SGLANG_EXL3_DENSE", "0") == "1"
        if dense and not draft:
            method = self._linear_method(layer, self.bits_for_prefix(prefix))
            method.split_sizes = self.merged_split_sizes(prefix)
            return method
        if not draft and self._matches_non_routed_exl3(prefix):
            return self._linear_method(layer, self._bits_for_non_routed(prefix))
        if draft:
            if os.environ.get("SGLANG_EXL3_MTP_EXL3", "1") == "1":
                bits = (self._bits_for_non_routed(prefix) if self._matches_non_routed_exl3(prefix)
                        else int(self.mtp_bits or self.bits_for_prefix(prefix)))
                return self._linear_method(layer, int(bits))
            return self._delegate_method(layer, prefix, True)
        if (os.environ.get("SGLANG_EXL3_NON_ROUTED_FP8", "0") == "1"
                or self.non_routed_dtype_policy not in ("bf16_as_stored", "official_source_native", "")):
            dm = self._delegate_method(layer, prefix, False)
            if dm is not None:
                return dm
        if self.non_routed_dtype_policy in ("bf16_as_stored", "official_source_native"):
            return _sglang_unquantized()
        dm = self._delegate_method(layer, prefix, False)
        return dm if dm is not None else _sglang_unquantized()

    # -- delegates (SGLang's own quant configs; None without SGLang) --------------------------
    def _draft_delegate(self):
        if not hasattr(self, "_draft_delegate_cached"):
            self._draft_delegate_cached = None
            if os.environ.get("SGLANG_EXL3_MTP_FP8", "1") == "1":
                try:  # pragma: no cover - depends on SGLang
                    from sglang.srt.layers.quantization.fp8 import Fp8Config

                    self._draft_delegate_cached = Fp8Config(is_checkpoint_fp8_serialized=False,
                                                            activation_scheme="dynamic")
                except Exception as exc:
                    logger.debug("no draft FP8 delegate: %s", exc)
        return self._draft_delegate_cached

    def _non_routed_delegate(self):
        if not hasattr(self, "_nr_delegate_cached"):
            self._nr_delegate_cached = None
            nrq = self.non_routed_quantization
            if not (isinstance(nrq, dict) and nrq.get("quant_method")) and \
                    os.environ.get("SGLANG_EXL3_NON_ROUTED_FP8", "0") == "1":
                nrq = {"quant_method": "fp8", "fmt": "e4m3", "weight_block_size": [128, 128],
                       "activation_scheme": "dynamic"}
            if isinstance(nrq, dict) and nrq.get("quant_method"):
                method = str(nrq["quant_method"]).lower()
                try:  # pragma: no cover - depends on SGLang
                    if method == "fp8":
                        from sglang.srt.layers.quantization.fp8 import Fp8Config

                        self._nr_delegate_cached = Fp8Config(
                            is_checkpoint_fp8_serialized=True,
                            activation_scheme=nrq.get("activation_scheme", "dynamic"),
                            ignored_layers=nrq.get("ignored_layers"),
                            weight_block_size=nrq.get("weight_block_size", [128, 128]))
                    else:
                        from sglang.srt.layers.quantization import get_quantization_config

                        qcls = get_quantization_config(method)
                        self._nr_delegate_cached = (qcls.from_config(dict(nrq)) if hasattr(qcls, "from_config")
                                                    else qcls(**dict(nrq)))
                except Exception as exc:
                    logger.warning("no non-routed delegate for %s: %s", method, exc)
        return self._nr_delegate_cached
