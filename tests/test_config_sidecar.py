"""EXL3Config parsing / method selection and checkpoint sidecar routing (CPU).

Cases follow the reference's own tests: tests/test_config.py (bits, layer_bits,
from_config, override, delegation), tests/test_sidecar_routing.py (fused qkv split,
merged gate_up / fused_qkv_a shards, skips, bad sizes, merged split sizes,
storage kinds)."""

import pytest
import torch

from exl3_b200 import layers as L
from exl3_b200.config import EXL3Config, storage_kind_for_prefix, tensor_storage_bits
from exl3_b200.sidecar import route_exl3_sidecar, split_fused_group, split_sidecar_name


# --------------------------------------------------------------------------- config
def test_default_config():
    cfg = EXL3Config(bits=4, codebook="mcg")
    assert cfg.get_name() == "exl3" and cfg.bits == 4 and cfg.codebook == "mcg"
    assert cfg.get_min_capability() == 100
    assert EXL3Config(codebook="3inst").codebook == "3inst"
    with pytest.raises(ValueError):
        EXL3Config(bits=7)
    with pytest.raises(ValueError):
        EXL3Config(codebook="fp8")
    with pytest.raises(ValueError):
        EXL3Config(layer_bits={"3": 9})


def test_mixed_k_layer_bits():
    cfg = EXL3Config(bits=2, layer_bits={"42": 3, "27": 3})
    assert cfg.bits_for_prefix("model.layers.0.mlp.experts") == 2
    assert cfg.bits_for_prefix("model.layers.42.mlp.experts") == 3
    assert cfg.bits_for_prefix("model.layers.27.mlp.experts") == 3


def test_from_config_and_override():
    cfg = EXL3Config.from_config({"quant_method": "exl3", "bits": 3, "codebook": "mcg",
                                  "scope": "glm53_routed_experts_only", "layer_bits": {"10": 4}})
    assert cfg.bits == 3 and cfg.scope == "glm53_routed_experts_only"
    assert cfg.bits_for_prefix("layers.10.mlp.experts") == 4
    assert cfg.bits_for_prefix("layers.5.mlp.experts") == 3
    assert EXL3Config.override_quantization_method({"quant_method": "exl3"}, None) == "exl3"
    assert EXL3Config.override_quantization_method({"quant_method": "fp8"}, None) is None
    # a config that only names quant_method=exl3 is a dense pack
    assert EXL3Config.from_config({"quant_method": "exl3", "bits": 4}).scope == "dense_and_moe"


def test_delegation_fields_without_sglang():
    cfg = EXL3Config.from_config({"quant_method": "exl3", "bits": 2, "non_routed_dtype_policy": "bf16_as_stored",
                                  "non_routed_quantization": {"quant_method": "fp8", "fmt": "e4m3"}})
    assert cfg.non_routed_dtype_policy == "bf16_as_stored"
    assert cfg.non_routed_quantization["quant_method"] == "fp8"
    cfg._non_routed_delegate()
    assert hasattr(cfg, "_nr_delegate_cached")


def test_storage_bits_from_trellis_width():
    ts = {"model.layers.1.mlp.experts.0.gate_proj": {"stored_tensors": {"a.trellis": {"shape": [8, 8, 48]}}},
          "model.layers.1.mlp.experts.1.gate_proj": {"stored_tensors": {"b.trellis": {"shape": [8, 8, 48]}}},
          "model.layers.2.self_attn.o_proj": {"stored_tensors": {"c.trellis": {"shape": [8, 8, 64]}}}}
    cfg = EXL3Config.from_config({"quant_method": "exl3", "bits": 2, "tensor_storage": ts})
    assert cfg.bits_for_prefix("model.layers.2.self_attn.o_proj") == 4
    assert cfg.bits_for_prefix("model.layers.1.mlp.experts") == 3
    ts["model.layers.1.mlp.experts.1.gate_proj"]["stored_tensors"]["b.trellis"]["shape"] = [8, 8, 32]
    with pytest.raises(ValueError):
        tensor_storage_bits(ts)


class ColumnParallelLinear(torch.nn.Module):
    def __init__(self, tp_rank=0, tp_size=1):
        super().__init__()
        self.tp_rank, self.tp_size = tp_rank, tp_size


class RowParallelLinear(ColumnParallelLinear):
    pass


class FusedMoE(torch.nn.Module):
    num_local_experts = 8


class VocabParallelEmbedding(torch.nn.Module):
    pass


def test_get_quant_method_selection():
    ts = {"model.layers.0.mlp.gate_proj": {"stored_tensors": {"x.trellis": {"shape": [4, 8, 48]}}},
          "model.layers.0.mlp.up_proj": {"stored_tensors": {"x.trellis": {"shape": [4, 8, 48]}}},
          "model.layers.0.mlp.down_proj": {"stored_tensors": {"x.trellis": {"shape": [8, 4, 64]}}},
          "model.layers.0.mlp.router": {"stored_tensors": {"x.weight": {"shape": [8, 64]}}}}
    cfg = EXL3Config.from_config({"quant_method": "exl3", "bits": 4, "codebook": "3inst", "tensor_storage": ts})
    gu = cfg.get_quant_method(ColumnParallelLinear(1, 2), "model.layers.0.mlp.gate_up_proj")
    assert isinstance(gu, L.EXL3LinearMethod)
    assert gu.bits == 4 and gu.split_sizes == [128, 128] and gu.parallel == "column" and gu.tp_rank == 1
    down = cfg.get_quant_method(RowParallelLinear(0, 2), "model.layers.0.mlp.down_proj")
    assert isinstance(down, L.EXL3LinearMethod) and down.parallel == "row" and down.bits == 4
    # stored as a plain weight -> not EXL3 (SGLang's unquantized method; None without SGLang)
    assert not isinstance(cfg.get_quant_method(ColumnParallelLinear(), "model.layers.0.mlp.router"),
                          L.EXL3LinearMethod)
    moe = cfg.get_quant_method(FusedMoE(), "model.layers.0.mlp.experts")
    assert isinstance(moe, L.EXL3MoEMethod) and moe.bits == 4
    assert cfg.get_quant_method(VocabParallelEmbedding(), "model.embed_tokens") is None
    # routed-experts-only scope: dense linears are not EXL3
    cfg2 = EXL3Config(bits=3, scope="glm53_routed_experts_only")
    assert not isinstance(cfg2.get_quant_method(ColumnParallelLinear(), "model.layers.0.mlp.gate_up_proj"),
                          L.EXL3LinearMethod)
    assert isinstance(cfg2.get_quant_method(FusedMoE(), "model.layers.3.mlp.experts"), L.EXL3MoEMethod)
    # draft (MTP) layers get EXL3 at mtp bits
    cfg3 = EXL3Config.from_config({"quant_method": "exl3", "bits": 3, "mtp_bits": 4})
    d = cfg3.get_quant_method(ColumnParallelLinear(), "model.mtp.0.proj")
    assert isinstance(d, L.EXL3LinearMethod) and d.bits == 4


# --------------------------------------------------------------------------- sidecar
class _Owner:
    def __init__(self, sizes):
        self._exl3_lin_output_partition_sizes = list(sizes)


class _Param:
    def __init__(self, key, owner, sink):
        self.key, self._exl3_owner, self._sink = key, owner, sink

    def weight_loader(self, param, loaded, shard_id=None):
        self._sink.setdefault(self.key, []).append((shard_id, loaded.clone()))


_ALL = ("trellis", "suh", "svh", "mcg", "mul1")


def _params(base, n, sink, sizes):
    owner = _Owner(sizes)
    return {f"{base}.exl3_{i}_{s}": _Param(f"{base}.exl3_{i}_{s}", owner, sink) for i in range(n) for s in _ALL}


def test_split_sidecar_name():
    assert split_sidecar_name("a.b.trellis") == ("a.b", "trellis")
    assert split_sidecar_name("a.b.weight") is None
    assert split_sidecar_name("trellis") is None


def test_fused_qkv_split_along_output_tiles():
    sizes = [64, 32, 32]
    base = "model.layers.0.self_attn.qkv_proj"
    sink = {}
    params = _params(base, 3, sink, sizes)
    trellis = torch.arange(4 * 8 * 48, dtype=torch.int32).reshape(4, 8, 48).to(torch.int16)
    suh = torch.ones(64, dtype=torch.float16)
    svh = torch.arange(128, dtype=torch.float16)
    mul1 = torch.tensor(1, dtype=torch.int32)
    for name, t in ((base + ".trellis", trellis), (base + ".suh", suh), (base + ".svh", svh), (base + ".mul1", mul1)):
        assert route_exl3_sidecar(params, name, t), name
    assert torch.equal(sink[f"{base}.exl3_0_trellis"][0][1], trellis[:, 0:4])
    assert torch.equal(sink[f"{base}.exl3_1_trellis"][0][1], trellis[:, 4:6])
    assert torch.equal(sink[f"{base}.exl3_2_trellis"][0][1], trellis[:, 6:8])
    assert torch.equal(sink[f"{base}.exl3_1_svh"][0][1], svh[64:96])
    assert torch.equal(sink[f"{base}.exl3_2_svh"][0][1], svh[96:128])
    for i in range(3):
        assert torch.equal(sink[f"{base}.exl3_{i}_suh"][0][1], suh)
        assert sink[f"{base}.exl3_{i}_trellis"][0][0] == i
    assert sink[f"{base}.exl3_0_mul1"][0][1].item() == 1


def test_merged_shards_and_skips():
    sink = {}
    gu = "model.layers.5.mlp.shared_experts.gate_up_proj"
    params = _params(gu, 2, sink, [48, 48])
    t = torch.zeros(4, 3, 48, dtype=torch.int16)
    assert route_exl3_sidecar(params, "model.layers.5.mlp.shared_experts.gate_proj.trellis", t)
    assert route_exl3_sidecar(params, "model.layers.5.mlp.shared_experts.up_proj.trellis", t)
    assert sink[f"{gu}.exl3_0_trellis"][0][0] == 0 and sink[f"{gu}.exl3_1_trellis"][0][0] == 1
    fq = "model.layers.3.self_attn.fused_qkv_a_proj_with_mqa"
    sink2 = {}
    params2 = _params(fq, 2, sink2, [512, 64])
    assert route_exl3_sidecar(params2, "model.layers.3.self_attn.q_a_proj.svh", torch.zeros(512))
    assert route_exl3_sidecar(params2, "model.layers.3.self_attn.kv_a_proj_with_mqa.svh", torch.zeros(64))
    assert sink2[f"{fq}.exl3_0_svh"][0][0] == 0 and sink2[f"{fq}.exl3_1_svh"][0][0] == 1

    o = "model.layers.0.self_attn.o_proj"
    sink3 = {}
    params3 = _params(o, 1, sink3, [64])
    assert route_exl3_sidecar(params3, o + ".trellis", torch.zeros(4, 4, 48, dtype=torch.int16))
    assert sink3[f"{o}.exl3_0_trellis"][0][0] == 0
    assert not route_exl3_sidecar(params3, "model.layers.0.mlp.experts.3.gate_proj.trellis", torch.zeros(1))
    assert not route_exl3_sidecar(params3, o + ".weight", torch.zeros(1))
    assert not route_exl3_sidecar(params3, "model.layers.9.self_attn.nope.trellis", torch.zeros(1))


def test_split_rejects_bad_sizes():
    with pytest.raises(ValueError):
        split_fused_group([24, 16], "svh", torch.zeros(40))
    with pytest.raises(ValueError):
        split_fused_group([32, 32], "trellis", torch.zeros(2, 3, 16))


def test_merged_split_sizes_feed_create_weights():
    def ent(out, in_=4096):
        return {"stored_tensors": {f"x.{out}.trellis": {"shape": [in_ // 16, out // 16, 48]}}}

    ts = {"model.language_model.layers.3.self_attn.q_a_proj": ent(1536),
          "model.language_model.layers.3.self_attn.kv_a_proj_with_mqa": ent(512),
          "model.language_model.layers.5.mlp.shared_experts.gate_proj": ent(1024),
          "model.language_model.layers.5.mlp.shared_experts.up_proj": ent(1024)}
    cfg = EXL3Config.from_config({"bits": 4, "codebook": "mcg", "tensor_storage": ts})
    assert cfg.merged_split_sizes("model.layers.3.self_attn.fused_qkv_a_proj_with_mqa") == [1536, 512]
    assert cfg.merged_split_sizes("model.layers.5.mlp.shared_experts.gate_up_proj") == [1024, 1024]
    assert cfg.merged_split_sizes("model.layers.4.self_attn.o_proj") is None
    method = L.EXL3LinearMethod(cfg, bits=4)
    method.split_sizes = cfg.merged_split_sizes("model.layers.3.self_attn.fused_qkv_a_proj_with_mqa")
    layer = torch.nn.Module()
    method.create_weights(layer, input_size_per_partition=4096, output_partition_sizes=[2048], input_size=4096,
                          output_size=2048, params_dtype=torch.float16)
    assert len(layer._exl3_lin_packs) == 2 and layer._exl3_lin_output_partition_sizes == [1536, 512]
    assert hasattr(layer, "exl3_1_trellis")
    layer2 = torch.nn.Module()
    m2 = L.EXL3LinearMethod(cfg, bits=4)
    m2.split_sizes = [1536, 512]
    m2.create_weights(layer2, 4096, [1024], 4096, 1024, torch.float16)
    assert len(layer2._exl3_lin_packs) == 1


def test_storage_kind_resolves_merged_modules():
    kinds = {"model.layers.5.mlp.shared_experts.gate_proj": "exl3",
             "model.layers.5.mlp.shared_experts.up_proj": "exl3",
             "model.layers.3.self_attn.q_a_proj": "exl3",
             "model.layers.3.self_attn.kv_a_proj_with_mqa": "exl3",
             "model.layers.3.self_attn.indexer.wk": "native"}
    assert storage_kind_for_prefix(kinds, "model.layers.5.mlp.shared_experts.gate_up_proj") == "exl3"
    assert storage_kind_for_prefix(kinds, "model.layers.3.self_attn.fused_qkv_a_proj_with_mqa") == "exl3"
    assert storage_kind_for_prefix(kinds, "model.layers.3.self_attn.indexer.wk") == "native"
    assert storage_kind_for_prefix(kinds, "model.layers.5.mlp.gate_up_proj") is None
    assert storage_kind_for_prefix(kinds, "model.layers.5.self_attn.o_proj") is None
    with pytest.raises(RuntimeError):
        storage_kind_for_prefix({"x.gate_proj": "exl3", "x.up_proj": "native"}, "x.gate_up_proj")


def test_sidecar_into_real_linear_method():
    """Routed sidecars land in EXL3LinearMethod's packs (host tensors, no GPU)."""
    method = L.EXL3LinearMethod(bits=3)
    layer = torch.nn.Module()
    method.create_weights(layer, 128, [128, 128], 128, 256, torch.float16)
    params = dict(layer.named_parameters(prefix="m.gate_up_proj"))
    g = torch.randint(-32768, 32767, (8, 8, 48), dtype=torch.int16)
    u = torch.randint(-32768, 32767, (8, 8, 48), dtype=torch.int16)
    assert route_exl3_sidecar(params, "m.gate_proj.trellis", g)
    assert route_exl3_sidecar(params, "m.up_proj.trellis", u)
    packs = layer._exl3_lin_packs
    assert torch.equal(packs[0]["trellis"].cpu(), g) and torch.equal(packs[1]["trellis"].cpu(), u)


def test_non_routed_modules_bf16_and_mtp_source():
    cfg = EXL3Config.from_config({
        "quant_method": "exl3", "bits": 2, "scope": "glm53_routed_experts_only",
        "non_routed_exl3": {"bits": 4, "modules": ["self_attn.o_proj", "mlp.shared_experts.down_proj"],
                            "layer_bits": {"self_attn.o_proj": 3}, "bf16_modules": ["self_attn.q_proj"]},
        "mtp_experts": "source", "mtp_experts_start_layer": 40})
    o = cfg.get_quant_method(RowParallelLinear(), "model.layers.1.self_attn.o_proj")
    assert isinstance(o, L.EXL3LinearMethod) and o.bits == 3           # per-module bits
    d = cfg.get_quant_method(RowParallelLinear(), "model.layers.1.mlp.shared_experts.down_proj")
    assert isinstance(d, L.EXL3LinearMethod) and d.bits == 4           # non-routed default bits
    assert not isinstance(cfg.get_quant_method(ColumnParallelLinear(), "model.layers.1.self_attn.q_proj"),
                          L.EXL3LinearMethod)                          # bf16 module
    assert isinstance(cfg.get_quant_method(FusedMoE(), "model.layers.39.mlp.experts"), L.EXL3MoEMethod)
    # experts of layers >= mtp_experts_start_layer come from the source checkpoint's delegate
    assert not isinstance(cfg.get_quant_method(FusedMoE(), "model.layers.40.mlp.experts"), L.EXL3MoEMethod)


def test_tensor_parallel_linear_from_layer_class():
    cfg = EXL3Config.from_config({"quant_method": "exl3", "bits": 4})
    col = cfg.get_quant_method(ColumnParallelLinear(3, 4), "model.layers.0.self_attn.qkv_proj")
    row = cfg.get_quant_method(RowParallelLinear(3, 4), "model.layers.0.self_attn.o_proj")
    single = cfg.get_quant_method(ColumnParallelLinear(0, 1), "model.layers.0.self_attn.qkv_proj")
    assert (col.parallel, col.tp_rank, col.tp_size) == ("column", 3, 4)
    assert (row.parallel, row.tp_rank, row.tp_size) == ("row", 3, 4)
    assert single.parallel == "none"


def test_split_fused_group_reassembles():
    """Random 16-multiple output partitions: the shards concatenate back to the fused
    trellis (dim 1) and svh, and suh / markers go to every shard unchanged."""
    from hypothesis import given, settings, strategies as st

    @settings(max_examples=50, deadline=None)
    @given(sizes=st.lists(st.integers(1, 6).map(lambda v: 16 * v), min_size=1, max_size=4),
           k_tiles=st.integers(1, 4))
    def check(sizes, k_tiles):
        total = sum(sizes)
        tr = torch.arange(k_tiles * (total // 16) * 32, dtype=torch.int32).reshape(k_tiles, total // 16, 32)
        sv = torch.arange(total, dtype=torch.float32)
        su = torch.ones(k_tiles * 16)
        assert torch.equal(torch.cat(split_fused_group(sizes, "trellis", tr), dim=1), tr)
        assert torch.equal(torch.cat(split_fused_group(sizes, "svh", sv)), sv)
        assert all(p is su for p in split_fused_group(sizes, "suh", su))
        assert [p.shape[1] * 16 for p in split_fused_group(sizes, "trellis", tr)] == sizes

    check()
