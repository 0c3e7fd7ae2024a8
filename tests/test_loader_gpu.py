"""Checkpoint loader into HBM (B200): pinned-staging reads, narrowed shard reads, and a
dense EXL3 linear loaded through the sidecar router straight from a shard file,
checked against the CPU oracle."""

import numpy as np
import pytest
import torch
from safetensors.torch import save_file

import exl3_oracle as O
from exl3_b200 import layers as L
from exl3_b200 import loader as LD
from exl3_b200.sidecar import route_exl3_sidecar

pytestmark = pytest.mark.gpu


def test_iterator_into_device_matches_host(tmp_path, cuda_device):
    path = str(tmp_path / "model-00001-of-00001.safetensors")
    tensors = {
        "big.trellis": torch.randint(-32768, 32767, (96, 160, 48), dtype=torch.int16),  # 2.9 MB
        "huge": torch.randint(-32768, 32767, (21 << 20,), dtype=torch.int16),  # 42 MB: several slots per thread
        "bf16": torch.randn(33, 17).to(torch.bfloat16),
        "scalar": torch.tensor(-877912083, dtype=torch.int32),
        "empty": torch.empty(0, 4, dtype=torch.float16),
    }
    save_file(tensors, path)
    for threads in (1, 3):
        got = dict(LD.exl3_mmap_weights_iterator([path], device=cuda_device, num_threads=threads))
        assert set(got) == set(tensors)
        for name, ref in tensors.items():
            assert got[name].device == cuda_device and got[name].dtype == ref.dtype
            assert torch.equal(got[name].cpu(), ref), (threads, name)


@pytest.mark.parametrize("narrow", [(1, 32, 96), (0, 8, 40), None])
def test_narrowed_read_into_device(tmp_path, cuda_device, narrow):
    path = str(tmp_path / "t.safetensors")
    tr = torch.randint(-32768, 32767, (64, 128, 64), dtype=torch.int16)
    save_file({"m.trellis": tr}, path)
    got = LD.read_safetensors_tensor(path, "m.trellis", device=cuda_device, narrow=narrow, threads=2)
    ref = tr if narrow is None else tr.narrow(narrow[0], narrow[1], narrow[2] - narrow[1])
    assert got.is_cuda and torch.equal(got.cpu(), ref)


def test_linear_loaded_from_shard_file(tmp_path, cuda_device):
    """gate/up sidecars read into HBM, routed to a merged gate_up linear, then applied."""
    rng = np.random.default_rng(11)
    k, n, K, cb = 256, 384, 3, 0
    gate = (O.random_trellis(rng, k, n, K), O.random_signs(rng, k), O.random_signs(rng, n))
    up = (O.random_trellis(rng, k, n, K), O.random_signs(rng, k), O.random_signs(rng, n))
    ck = {}
    for leaf, (tr, su, sv) in (("gate_proj", gate), ("up_proj", up)):
        ck[f"model.layers.0.mlp.{leaf}.trellis"] = torch.from_numpy(tr)
        ck[f"model.layers.0.mlp.{leaf}.suh"] = torch.from_numpy(su)
        ck[f"model.layers.0.mlp.{leaf}.svh"] = torch.from_numpy(sv)
    path = str(tmp_path / "model.safetensors")
    save_file(ck, path)

    method = L.EXL3LinearMethod(bits=K)
    layer = torch.nn.Module()
    method.create_weights(layer, k, [n, n], k, 2 * n, torch.float16)
    params = dict(layer.named_parameters(prefix="model.layers.0.mlp.gate_up_proj"))
    for name, t in LD.exl3_mmap_weights_iterator([path], device=cuda_device):
        assert t.is_cuda
        assert route_exl3_sidecar(params, name, t), name
    method.process_weights_after_loading(layer)

    x = rng.standard_normal((3, k)).astype(np.float16)
    y = method.apply(layer, torch.from_numpy(x).to(cuda_device)).float().cpu().numpy()
    ref = np.concatenate([O.gemv_ref(x, *gate, K, cb), O.gemv_ref(x, *up, K, cb)], axis=1)
    assert O.normwise_rel_err(y, ref) < 1e-2  # fp16 output of fp32-accumulated products
