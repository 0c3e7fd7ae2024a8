"""Checkpoint loader on the host (CPU): the native reader into host memory.

Cases follow the reference's tests/test_mmap_loader.py (constants, iterator over
two shards, dtype round trip, unknown dtype fails closed) plus narrowed reads and
a file that ends inside a tensor."""

import json
import os
import struct

import pytest
import torch
from safetensors.torch import save_file

from exl3_b200 import loader as LD


def test_constants_and_platform():
    assert LD.LoadFormatEXL3.EXL3_MMAP == "exl3_mmap" == LD.LOAD_FORMAT_EXL3_MMAP
    assert isinstance(LD.is_unified_memory_platform(), bool)
    line = LD.host_memory_summary()
    assert line.startswith("host_free=") and "device_free=" in line
    assert LD.EXL3MMapModelLoader(load_config=None).load_format == "exl3_mmap"


def test_weights_iterator_two_shards(tmp_path):
    p1, p2 = str(tmp_path / "model-00001-of-00002.safetensors"), str(tmp_path / "model-00002-of-00002.safetensors")
    t1, t2, t3 = torch.randn(64, 128), torch.randn(128, 64), torch.randn(32, 32)
    save_file({"model.layers.0.weight": t1, "model.layers.0.bias": t2}, p1)
    save_file({"model.layers.1.weight": t3}, p2)
    assert isinstance(LD.madvise_file_preload(p1), bool)
    got = dict(LD.exl3_mmap_weights_iterator([p1, p2], device="cpu", num_threads=2, prefetch_shards=2))
    assert set(got) == {"model.layers.0.weight", "model.layers.0.bias", "model.layers.1.weight"}
    assert torch.equal(got["model.layers.0.weight"], t1)
    assert torch.equal(got["model.layers.0.bias"], t2)
    assert torch.equal(got["model.layers.1.weight"], t3)
    assert list(LD.exl3_mmap_weights_iterator([])) == []


def test_pread_roundtrip_dtypes(tmp_path):
    path = str(tmp_path / "model-00001-of-00001.safetensors")
    tensors = {
        "bf16": torch.randn(33, 17).to(torch.bfloat16),
        "f16": torch.randn(8, 16).to(torch.float16),
        "f32": torch.randn(5),
        "i16_trellis": torch.randint(-32768, 32767, (4, 16, 48), dtype=torch.int16),
        "i32": torch.arange(12, dtype=torch.int32).reshape(3, 4),
        "u8": torch.arange(256, dtype=torch.uint8),
        "scalar": torch.tensor(3, dtype=torch.int32),
        "empty": torch.empty(0, 4, dtype=torch.float16),
    }
    save_file(tensors, path)
    got = dict(LD.iter_safetensors_pread(path))
    assert set(got) == set(tensors)
    for name, ref in tensors.items():
        assert got[name].dtype == ref.dtype and tuple(got[name].shape) == tuple(ref.shape), name
        assert torch.equal(got[name], ref), name


def test_large_tensor_spans_many_chunks(tmp_path):
    """A tensor larger than the reader's chunk is split over threads."""
    path = str(tmp_path / "big.safetensors")
    big = torch.randint(-32768, 32767, ((40 << 20) // 2,), dtype=torch.int16)  # 40 MB: 3 host chunks
    save_file({"big": big, "tail": torch.arange(7, dtype=torch.int64)}, path)
    got = dict(LD.iter_safetensors_pread(path, threads=3))
    assert torch.equal(got["big"], big) and torch.equal(got["tail"], torch.arange(7))


def test_unknown_dtype_fails_closed(tmp_path):
    path = str(tmp_path / "bad.safetensors")
    header = json.dumps({"x": {"dtype": "C64", "shape": [2], "data_offsets": [0, 16]}}).encode()
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(header)) + header + bytes(16))
    with pytest.raises(RuntimeError):
        list(LD.iter_safetensors_pread(path))


def test_truncated_file_fails(tmp_path):
    path = str(tmp_path / "trunc.safetensors")
    save_file({"a": torch.arange(1024, dtype=torch.int32)}, path)
    size = os.path.getsize(path)
    with open(path, "r+b") as fh:
        fh.truncate(size - 100)
    with pytest.raises(RuntimeError):  # the header's range now exceeds the file
        list(LD.iter_safetensors_pread(path))


def test_native_reader_reports_short_read(tmp_path):
    """The C reader itself returns EXL3B200_EIO when the file ends inside a range."""
    import ctypes

    from exl3_b200 import _lib

    path = str(tmp_path / "short.bin")
    with open(path, "wb") as fh:
        fh.write(bytes(range(256)) * 4)
    buf = torch.zeros(2048, dtype=torch.uint8)
    fd = os.open(path, os.O_RDONLY)
    try:
        off = (ctypes.c_longlong * 1)(512)
        n = (ctypes.c_longlong * 1)(2048)
        dst = (ctypes.c_void_p * 1)(buf.data_ptr())
        assert _lib.lib().exl3b200_read_ranges(fd, off, n, dst, 1, 0, None, 0, 2, 0, None) == _lib.EIO
        n[0] = 512
        assert _lib.lib().exl3b200_read_ranges(fd, off, n, dst, 1, 0, None, 0, 2, 0, None) == 0
        assert bytes(buf[:512].numpy()) == (bytes(range(256)) * 4)[512:]
        assert _lib.lib().exl3b200_read_ranges(fd, off, n, dst, 1, 0, None, 0, 0, 0, None) == _lib.EBADARG
        assert _lib.lib().exl3b200_read_ranges(fd, off, n, dst, 1, 1, None, 0, 2, 0, None) == _lib.ENULL
    finally:
        os.close(fd)


@pytest.mark.parametrize("narrow", [None, (0, 2, 5), (1, 3, 7), (2, 16, 48), (-1, 0, 48), (1, 4, 4)])
def test_narrowed_read_matches_slice(tmp_path, narrow):
    """Column / row shards of a trellis read only their own bytes."""
    path = str(tmp_path / "t.safetensors")
    tr = torch.randint(-32768, 32767, (8, 10, 48), dtype=torch.int16)
    save_file({"m.trellis": tr, "m.svh": torch.randn(160).half()}, path)
    got = LD.read_safetensors_tensor(path, "m.trellis", narrow=narrow)
    ref = tr if narrow is None else tr.narrow(narrow[0], narrow[1], narrow[2] - narrow[1])
    assert tuple(got.shape) == tuple(ref.shape) and torch.equal(got, ref)
    with pytest.raises(ValueError):
        LD.read_safetensors_tensor(path, "m.trellis", narrow=(1, 5, 11))
    with pytest.raises(KeyError):
        LD.read_safetensors_tensor(path, "nope")


def test_narrow_ranges_property(tmp_path):
    """Random shapes, dtypes and slices: the ranges read equal torch.narrow of the tensor."""
    from hypothesis import given, settings, strategies as st

    path = str(tmp_path / "p.safetensors")

    @settings(max_examples=60, deadline=None)
    @given(shape=st.lists(st.integers(1, 6), min_size=1, max_size=4),
           dtype=st.sampled_from([torch.int16, torch.float32, torch.uint8, torch.bfloat16]),
           data=st.data())
    def check(shape, dtype, data):
        t = (torch.arange(int(torch.tensor(shape).prod())) % 251).to(dtype).reshape(shape)
        save_file({"t": t}, path)
        dim = data.draw(st.integers(0, len(shape) - 1))
        start = data.draw(st.integers(0, shape[dim]))
        stop = data.draw(st.integers(start, shape[dim]))
        got = LD.read_safetensors_tensor(path, "t", narrow=(dim, start, stop))
        assert torch.equal(got, t.narrow(dim, start, stop - start))

    check()
