"""Host logic of the plugin-surface mirror (CPU): parameter layout, loaders,
TP sharding, codebook markers, expert-id mapping.  Pins follow the reference's
own CPU tests (tests/test_moe.py, tests/test_dense_marker_codebook.py)."""

import pytest
import torch

from exl3_b200 import layers as L


class _Layer(torch.nn.Module):
    pass


def test_moe_param_shapes_k3():
    """reference tests/test_moe.py:20-49: hidden 4096, inter 2048, K = 3."""
    layer = _Layer()
    m = L.EXL3MoEMethod(bits=3)
    m.create_weights(layer, num_experts=4, hidden_size=4096, intermediate_size_per_partition=2048,
                     params_dtype=torch.float16)
    assert tuple(layer.w13_trellis.shape) == (4, 2, 256, 128, 48)
    assert tuple(layer.w2_trellis.shape) == (4, 128, 256, 48)
    assert tuple(layer.w13_suh.shape) == (4, 2, 4096) and tuple(layer.w13_svh.shape) == (4, 2, 2048)
    assert tuple(layer.w2_suh.shape) == (4, 2048) and tuple(layer.w2_svh.shape) == (4, 4096)
    assert tuple(layer.w13_mcg.shape) == (4, 2, 1) and tuple(layer.w2_mcg.shape) == (4, 1)


def test_moe_rejects_non_tile_sizes():
    with pytest.raises(ValueError):
        L.EXL3MoEMethod(bits=4).create_weights(_Layer(), 2, 4100, 2048, torch.float16)


def test_moe_loader_tp_shards_and_markers():
    layer = _Layer()
    m = L.EXL3MoEMethod(bits=2, tp_rank=1, tp_size=2)
    m.create_weights(layer, 2, 256, 128, torch.float16)  # local inter 128 of global 256
    gate = torch.arange(16 * 16 * 32, dtype=torch.int16).reshape(16, 16, 32)  # [256/16, 256/16, 32]
    m._load_exl3(layer.w13_trellis, gate, "experts.1.gate_proj.trellis", "w1", 1)
    assert torch.equal(layer.w13_trellis[1, 0], gate[:, 8:16])
    down = torch.arange(16 * 16 * 32, dtype=torch.int16).reshape(16, 16, 32)  # [256/16, 256/16]
    m._load_exl3(layer.w2_trellis, down, "experts.0.down_proj.trellis", "w2", 0)
    assert torch.equal(layer.w2_trellis[0], down[8:16])
    svh = torch.arange(256, dtype=torch.float16)
    m._load_exl3(layer.w13_svh, svh, "experts.0.up_proj.svh", "w3", 0)
    assert torch.equal(layer.w13_svh[0, 1], svh[128:])
    m._load_exl3(layer.w13_mcg, torch.tensor(L.MCG_MARKER_SIGNED_INT32), "experts.0.gate_proj.mcg", "w1", 0)
    assert int(layer.w13_mcg[0, 0, 0]) == L.MCG_MARKER_SIGNED_INT32
    with pytest.raises(ValueError):
        m._load_exl3(layer.w13_trellis, gate, "x.trellis", "w9", 0)


def test_moe_codebook_from_markers_and_pointer_tables():
    layer = _Layer()
    m = L.EXL3MoEMethod(bits=2)
    m.create_weights(layer, 3, 128, 128, torch.float16)
    layer.w13_mul1.fill_(L.MUL1_MARKER_SIGNED_INT32)
    layer.w2_mul1.fill_(L.MUL1_MARKER_SIGNED_INT32)
    m.process_weights_after_loading(layer)
    assert layer._exl3_cb == 2 and layer._exl3_use_mul1
    assert set(layer._exl3_ptrs) == {f"{a}_{b}" for a in ("gate", "up", "down") for b in ("trellis", "suh", "svh")}
    t = layer._exl3_ptrs["up_trellis"]
    assert t.dtype == torch.int64 and t.numel() == 3
    assert int(t[2]) == layer.w13_trellis[2, 1].data_ptr()
    assert layer._exl3_k_gate == 2 and layer._exl3_k_down == 2


def test_moe_codebook_fallback_to_config():
    class Cfg:
        codebook = "mcg"

    layer = _Layer()
    m = L.EXL3MoEMethod(Cfg(), bits=2)
    m.create_weights(layer, 1, 128, 128, torch.float16)
    m.process_weights_after_loading(layer)
    assert layer._exl3_cb == 1


def test_map_topk_to_local():
    ids = torch.tensor([[0, 3, 5], [-1, 2, 7]])
    out = L.map_topk_to_local(ids, 4, None)
    assert out.tolist() == [[0, 3, 4], [4, 2, 4]]
    emap = torch.tensor([-1, 0, 1, -1, 2, 3, -1, -1], dtype=torch.long)
    out = L.map_topk_to_local(torch.tensor([[1, 4, 0], [5, 9, -3]]), 4, emap)
    assert out.tolist() == [[0, 2, 4], [3, 4, 4]]
    with pytest.raises(RuntimeError):
        L.map_topk_to_local(ids, 4, emap.to(torch.int32))


def test_dense_marker_codebook():
    """reference tests/test_dense_marker_codebook.py:20-35: no marker = 3INST."""
    tr = torch.zeros((8, 8, 64), dtype=torch.int16)
    s = torch.ones(128, dtype=torch.float16)
    assert L.EXL3DenseLinear(tr, s, s).cb == 0
    assert L.EXL3DenseLinear(tr, s, s, mcg=torch.tensor([L.MCG_MARKER_SIGNED_INT32])).cb == 1
    assert L.EXL3DenseLinear(tr, s, s, mul1=torch.tensor([L.MUL1_MARKER_SIGNED_INT32])).cb == 2
    with pytest.raises(ValueError):
        L.EXL3DenseLinear(tr, s, s, mcg=torch.tensor([1]), mul1=torch.tensor([1]))
    assert L.EXL3DenseLinear(torch.zeros((8, 8, 48), dtype=torch.int16), s, s).K == 3


def test_dense_create_and_load_with_tp():
    layer = _Layer()
    m = L.EXL3LinearMethod(bits=4, tp_rank=0, tp_size=2, parallel="column")
    m.create_weights(layer, 256, [128, 128], 256, 512, torch.bfloat16)
    assert layer._exl3_lin_n_shards == 2 and hasattr(layer, "exl3_1_trellis")
    tr = torch.arange(16 * 16 * 64, dtype=torch.int16).reshape(16, 16, 64)
    m._load_linear(layer.exl3_1_trellis, tr, 1)
    assert torch.equal(layer._exl3_lin_packs[1]["trellis"].cpu(), tr[:, :8])
    m._load_linear(layer.exl3_1_svh, torch.arange(256, dtype=torch.float32), 1)
    assert layer._exl3_lin_packs[1]["svh"].dtype == torch.float16
    assert layer._exl3_lin_packs[1]["svh"].numel() == 128
    with pytest.raises(RuntimeError):
        m.process_weights_after_loading(layer)  # shard 0 has no trellis


def test_row_shard_keeps_hadamard_blocks():
    tr = torch.zeros((24, 8, 32), dtype=torch.int16)  # 384 rows: 3 blocks, not splittable in 2 whole blocks
    with pytest.raises(ValueError):
        L.shard_exl3_row(tr, "trellis", 0, 2)
    assert L.shard_exl3_row(torch.zeros((32, 8, 32), dtype=torch.int16), "trellis", 1, 2).shape == (16, 8, 32)


def test_moe_path_selection(monkeypatch):
    """Host-side choice between the small-M and the tensor-core MoE pipelines."""
    from exl3_b200 import moe

    monkeypatch.delenv("EXL3_B200_MOE_PATH", raising=False)
    assert moe.moe_path(1, 8, 288) == "small"                 # decode: ~0 rows per expert
    assert moe.moe_path(320, 8, 128) == "tc"                  # config 5 verify, batch 64: 20 rows
    assert moe.moe_path(80, 8, 128) == "small"                # config 5 verify, batch 16: 5 rows
    assert moe.moe_path(512, 8, 288) == "tc"                  # config 3, T = 512: 14 rows
    assert moe.moe_path(12, 1, 1) == "tc" and moe.moe_path(11, 1, 1) == "small"
    monkeypatch.setenv("EXL3_B200_MOE_PATH", "small")
    assert moe.moe_path(320, 8, 128) == "small"
    monkeypatch.setenv("EXL3_B200_MOE_PATH", "tc")
    assert moe.moe_path(1, 8, 288) == "tc"
