"""EXL3 checkpoint loading on B200: safetensors shards streamed into HBM.

Same load format and names as the reference's ``exl3_mmap`` loader
(src/sglang_exl3/loader.py): ``LOAD_FORMAT_EXL3_MMAP``, ``iter_safetensors_pread``,
``exl3_mmap_weights_iterator`` and ``EXL3MMapModelLoader``, yielding
``(name, tensor)`` pairs in each shard's file order.  The reference targets a GB10,
whose GPU shares host memory, and only has to keep the page cache from doubling
the footprint.  A B200 keeps its 180 GB of HBM behind PCIe, so here the bytes go
from the file to their device tensor in one pass: reader threads pread() chunks
into a pinned staging buffer and DMA them into the destination
(``exl3b200_read_ranges`` in the C library), and each range is dropped from the
page cache once read.  A tensor can also be read narrowed along one dimension
(``read_safetensors_tensor(..., narrow=...)``), so a tensor-parallel rank reads
only the bytes of its own shard.
"""

from __future__ import annotations

import ctypes
import json
import logging
import os
import struct
import threading
import time
from dataclasses import dataclass
from typing import Any, Dict, Iterator, List, Optional, Sequence, Tuple, Union

import torch

from . import _lib

logger = logging.getLogger("exl3_b200.loader")

LOAD_FORMAT_EXL3_MMAP = "exl3_mmap"


class LoadFormatEXL3:
    EXL3_MMAP = LOAD_FORMAT_EXL3_MMAP


# safetensors header dtype names (the format's own names) -> torch dtypes; the fp8
# kinds only where this torch has them
SAFETENSORS_DTYPES: Dict[str, torch.dtype] = {
    st_name: getattr(torch, attr)
    for st_name, attr in (("BOOL", "bool"), ("U8", "uint8"), ("I8", "int8"), ("I16", "int16"), ("I32", "int32"),
                          ("I64", "int64"), ("F16", "float16"), ("BF16", "bfloat16"), ("F32", "float32"),
                          ("F64", "float64"), ("F8_E4M3", "float8_e4m3fn"), ("F8_E5M2", "float8_e5m2"))
    if hasattr(torch, attr)
}

STAGING_SLOT_BYTES = 8 << 20  # per reader thread
BATCH_BYTES = 1 << 30  # device bytes read per native call by the weights iterator


def is_unified_memory_platform() -> bool:
    """True when the GPU shares coherent memory with the host (GB10, GB200, Grace).

    Same question as the reference's helper (loader.py:31-46), answered from the
    device's own report: an integrated GPU, or a Grace-attached part by name.  A
    discrete B200 (HGX) is not unified although its compute capability is 10.x.
    """
    if not torch.cuda.is_available():
        return False
    try:
        props = torch.cuda.get_device_properties(0)
    except Exception:
        return False
    if getattr(props, "is_integrated", False):
        return True
    name = props.name.lower()
    return any(tag in name for tag in ("gb10", "gb200", "gb300", "grace", "tegra", "spark"))


def madvise_file_preload(file_path: str) -> bool:
    """Map the file read-only and madvise(MADV_WILLNEED) the mapping, so the kernel
    starts reading it ahead; the mapping is dropped again at once (the advice applies
    to the file's page cache).  False where mmap or the advice is unavailable."""
    import mmap

    advice = getattr(mmap, "MADV_WILLNEED", None)
    if advice is None:
        return False
    try:
        with open(file_path, "rb") as fh:
            if os.fstat(fh.fileno()).st_size == 0:
                return False
            with mmap.mmap(fh.fileno(), 0, access=mmap.ACCESS_READ) as mm:
                mm.madvise(advice)
        return True
    except (OSError, ValueError):
        return False


def host_memory_summary(device: Union[str, torch.device, None] = None) -> str:
    """Free host memory (free physical pages) and the CUDA device's free / total
    memory as the driver reports it, for the load-time log line."""
    host_free = float("nan")
    try:
        host_free = os.sysconf("SC_AVPHYS_PAGES") * os.sysconf("SC_PAGE_SIZE") / 2**30
    except (AttributeError, OSError, ValueError):
        pass
    dev_free = dev_total = float("nan")
    if torch.cuda.is_available():
        try:
            dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
            if dev.type == "cuda":
                free_b, total_b = torch.cuda.mem_get_info(dev)
                dev_free, dev_total = free_b / 2**30, total_b / 2**30
        except Exception:  # a log line must not fail the load
            pass
    return f"host_free={host_free:.1f}GiB device_free={dev_free:.1f}/{dev_total:.1f}GiB"


@dataclass(frozen=True)
class TensorEntry:
    """One tensor of a safetensors file: dtype, shape and absolute byte range."""

    name: str
    dtype: torch.dtype
    shape: Tuple[int, ...]
    offset: int  # absolute file offset of the first byte
    nbytes: int


def read_safetensors_header(path: str) -> List[TensorEntry]:
    """Parse a safetensors header; entries in file order.

    Unknown dtypes fail closed with RuntimeError, as the reference's reader does
    (loader.py:139-143); so do ranges that fall outside the file or disagree with
    their shape.
    """
    with open(path, "rb") as fh:
        raw = fh.read(8)
        if len(raw) != 8:
            raise RuntimeError(f"[EXL3 loader] {path}: not a safetensors file (no header length)")
        (hlen,) = struct.unpack("<Q", raw)
        size = os.fstat(fh.fileno()).st_size
        if hlen > size - 8:
            raise RuntimeError(f"[EXL3 loader] {path}: header length {hlen} exceeds the file")
        header = json.loads(fh.read(hlen))
    header.pop("__metadata__", None)
    base = 8 + hlen
    out = []
    for name, info in header.items():
        dt = info.get("dtype")
        if dt not in SAFETENSORS_DTYPES:
            raise RuntimeError(f"[EXL3 loader] unsupported safetensors dtype {dt} for {name} in {path}")
        dtype = SAFETENSORS_DTYPES[dt]
        shape = tuple(int(s) for s in info["shape"])
        start, end = (int(v) for v in info["data_offsets"])
        numel = 1
        for s in shape:
            numel *= s
        nbytes = end - start
        if start < 0 or nbytes != numel * torch.empty((), dtype=dtype).element_size() or base + end > size:
            raise RuntimeError(f"[EXL3 loader] {path}: bad byte range [{start}, {end}) for {name} {shape} {dt}")
        out.append(TensorEntry(name, dtype, shape, base + start, nbytes))
    out.sort(key=lambda e: e.offset)
    return out


def _narrow_ranges(entry: TensorEntry, narrow: Optional[Tuple[int, int, int]]) -> Tuple[Tuple[int, ...], List[Tuple[int, int]]]:
    """(shape, [(file offset, bytes)]) of ``entry`` narrowed along one dimension.

    The tensor is C-contiguous, so a slice [start, stop) of dimension d is one run
    of bytes per index of the dimensions before d.
    """
    shape = entry.shape
    if narrow is None:
        return shape, ([(entry.offset, entry.nbytes)] if entry.nbytes else [])
    dim, start, stop = narrow
    if dim < 0:
        dim += len(shape)
    if not (0 <= dim < len(shape)) or not (0 <= start <= stop <= shape[dim]):
        raise ValueError(f"[EXL3 loader] narrow {narrow} out of range for {entry.name} {shape}")
    item = entry.nbytes // max(1, _numel(shape))
    inner = item * _numel(shape[dim + 1:])
    outer = _numel(shape[:dim])
    run = (stop - start) * inner
    out_shape = shape[:dim] + (stop - start,) + shape[dim + 1:]
    if run == 0 or outer == 0:
        return out_shape, []
    if start == 0 and stop == shape[dim]:
        return out_shape, [(entry.offset, entry.nbytes)]
    first = entry.offset + start * inner
    stride = shape[dim] * inner
    return out_shape, [(first + o * stride, run) for o in range(outer)]


def _numel(shape: Sequence[int]) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n


class _Staging:
    """Pinned host staging buffer, one slot per reader thread, kept across calls.
    ``lock`` serialises the device reads that use it."""

    def __init__(self) -> None:
        self.buf: Optional[torch.Tensor] = None
        self.lock = threading.Lock()

    def get(self, threads: int) -> torch.Tensor:
        need = threads * STAGING_SLOT_BYTES
        if self.buf is None or self.buf.numel() < need:
            self.buf = torch.empty(need, dtype=torch.uint8, pin_memory=True)
        return self.buf


_staging = _Staging()


def _read_into(fd: int, jobs: List[Tuple[torch.Tensor, List[Tuple[int, int]]]], threads: int,
               drop_cache: bool) -> None:
    """Fill each destination tensor (contiguous) from its list of file ranges."""
    offs: List[int] = []
    sizes: List[int] = []
    dsts: List[int] = []
    on_device = None
    for dst, ranges in jobs:
        if not dst.is_contiguous():
            raise ValueError("[EXL3 loader] destination must be contiguous")
        dev = dst.is_cuda
        if on_device is None:
            on_device = dev
        elif on_device != dev:
            raise ValueError("[EXL3 loader] one read targets either host or device memory")
        pos = dst.data_ptr()
        total = 0
        for off, n in ranges:
            offs.append(off)
            sizes.append(n)
            dsts.append(pos + total)
            total += n
        if total != dst.numel() * dst.element_size():
            raise ValueError("[EXL3 loader] ranges do not cover the destination")
    if not offs:
        return
    count = len(offs)
    c_off = (ctypes.c_longlong * count)(*offs)
    c_size = (ctypes.c_longlong * count)(*sizes)
    c_dst = (ctypes.c_void_p * count)(*dsts)
    threads = max(1, min(64, int(threads)))
    L = _lib.lib()
    if on_device:
        with _staging.lock:
            buf = _staging.get(threads)
            rc = L.exl3b200_read_ranges(fd, c_off, c_size, c_dst, count, 1, buf.data_ptr(), buf.numel(), threads,
                                        1 if drop_cache else 0, torch.cuda.current_stream().cuda_stream)
    else:
        rc = L.exl3b200_read_ranges(fd, c_off, c_size, c_dst, count, 0, None, 0, threads, 1 if drop_cache else 0,
                                    None)
    if rc == _lib.EIO:
        raise IOError(f"[EXL3 loader] short read: the file ends inside a tensor's byte range")
    _lib.check(rc, "exl3b200_read_ranges")


def read_safetensors_tensor(path: str, name: str, device: Union[str, torch.device] = "cpu",
                            narrow: Optional[Tuple[int, int, int]] = None, threads: int = 4,
                            drop_cache: bool = True) -> torch.Tensor:
    """Read one tensor (or the slice ``narrow = (dim, start, stop)`` of it) from a shard.

    With a CUDA ``device`` the bytes go from the file to HBM through pinned staging;
    only the slice's bytes are read, so a tensor-parallel rank can load
    ``trellis[:, n0:n1]`` (column shard) or ``trellis[k0:k1]`` (row shard) alone.
    """
    entries = {e.name: e for e in read_safetensors_header(path)}
    if name not in entries:
        raise KeyError(f"[EXL3 loader] {name} not in {path}")
    entry = entries[name]
    shape, ranges = _narrow_ranges(entry, narrow)
    out = torch.empty(shape, dtype=entry.dtype, device=device)
    fd = os.open(path, os.O_RDONLY)
    try:
        _read_into(fd, [(out, ranges)], threads, drop_cache)
    finally:
        os.close(fd)
    return out


def iter_safetensors_pread(path: str, threads: int = 4) -> Iterator[Tuple[str, torch.Tensor]]:
    """Yield every tensor of one shard as a fresh host tensor, in file order.

    Behaviour of the reference's reader (loader.py:121-168): no mmap, each range is
    dropped from the page cache after it is read, unknown dtypes raise
    RuntimeError, a file that ends early raises IOError.
    """
    entries = read_safetensors_header(path)
    fd = os.open(path, os.O_RDONLY)
    try:
        for e in entries:
            t = torch.empty(e.shape, dtype=e.dtype)
            if e.nbytes:
                _read_into(fd, [(t, [(e.offset, e.nbytes)])], threads, True)
            yield e.name, t
            del t
    finally:
        os.close(fd)


def _iter_shard_device(path: str, device: torch.device, threads: int) -> Iterator[Tuple[str, torch.Tensor]]:
    entries = read_safetensors_header(path)
    fd = os.open(path, os.O_RDONLY)
    try:
        i = 0
        while i < len(entries):
            batch, byts = [], 0
            while i < len(entries) and (not batch or byts + entries[i].nbytes <= BATCH_BYTES):
                batch.append(entries[i])
                byts += entries[i].nbytes
                i += 1
            outs = [torch.empty(e.shape, dtype=e.dtype, device=device) for e in batch]
            with torch.cuda.device(device):
                _read_into(fd, [(t, [(e.offset, e.nbytes)] if e.nbytes else []) for t, e in zip(outs, batch)],
                           threads, True)
            for e, t in zip(batch, outs):
                yield e.name, t
            del outs
    finally:
        os.close(fd)


def exl3_mmap_weights_iterator(hf_weights_files: List[str], device: Union[str, torch.device] = "cpu",
                               num_threads: int = 8, prefetch_shards: int = 2,
                               drop_cache_after_load: bool = False) -> Iterator[Tuple[str, torch.Tensor]]:
    """Iterate over the tensors of a checkpoint's shards, in load order.

    Signature of the reference's iterator (loader.py:171-231).  ``device`` "cpu"
    yields host tensors as the reference does; a CUDA device yields tensors already
    in HBM (read by ``num_threads`` threads through pinned staging, up to 1 GiB per
    batch).  ``prefetch_shards`` and ``drop_cache_after_load`` are accepted for API
    compatibility: shards are read in order and the page cache is always released.
    """
    del prefetch_shards, drop_cache_after_load
    if not hf_weights_files:
        return
    dev = torch.device(device)
    t0 = time.perf_counter()
    total_bytes = total = 0
    for idx, path in enumerate(hf_weights_files, start=1):
        it = _iter_shard_device(path, dev, num_threads) if dev.type == "cuda" else iter_safetensors_pread(
            path, threads=max(1, min(8, num_threads)))
        n = 0
        for name, t in it:
            total_bytes += t.numel() * t.element_size()
            total += 1
            n += 1
            yield name, t
        logger.info("[EXL3 loader] shard %d/%d %s tensors=%d %s", idx, len(hf_weights_files),
                    os.path.basename(path), n, host_memory_summary(dev))
    dt = time.perf_counter() - t0
    logger.info("[EXL3 loader] %d tensors (%.2f GiB) from %d shards in %.2f s (%.2f GB/s)", total,
                total_bytes / (1 << 30), len(hf_weights_files), dt, total_bytes / max(dt, 1e-9) / 1e9)


try:  # SGLang is optional: the loader class works without it
    from sglang.srt.model_loader.loader import DefaultModelLoader  # type: ignore

    _HAS_SGLANG_LOADER = True
except ImportError:  # pragma: no cover - depends on the environment
    DefaultModelLoader = object  # type: ignore
    _HAS_SGLANG_LOADER = False


class EXL3MMapModelLoader(DefaultModelLoader):  # type: ignore[misc, valid-type]
    """SGLang model loader for the ``exl3_mmap`` load format (reference loader.py:245-315).

    ``model_loader_extra_config``: ``num_threads`` (reader threads, default 8) and
    ``direct_to_device`` (yield tensors already in HBM on the current CUDA device
    instead of host tensors; default False, matching the reference's host tensors).
    """

    def __init__(self, load_config: Any):
        if _HAS_SGLANG_LOADER:
            super().__init__(load_config)
        else:
            self.load_config = load_config
        self.load_format = LOAD_FORMAT_EXL3_MMAP

    def _prepare_weights(self, model_name_or_path: str, revision: Optional[str], fall_back_to_pt: bool):
        if not _HAS_SGLANG_LOADER:
            raise RuntimeError("EXL3MMapModelLoader._prepare_weights needs SGLang's DefaultModelLoader")
        from sglang.srt.configs.load_config import LoadFormat  # type: ignore

        original = self.load_config.load_format
        self.load_config.load_format = LoadFormat.SAFETENSORS  # shard discovery only knows built-in formats
        try:
            return super()._prepare_weights(model_name_or_path, revision, fall_back_to_pt)
        finally:
            self.load_config.load_format = original

    def _get_weights_iterator(self, source: Any, *, resolved_source: Any = None, **kwargs: Any):
        extra = getattr(self.load_config, "model_loader_extra_config", None) or {}
        threads = int(extra.get("num_threads", 8))
        if resolved_source is None:
            _, files, use_safetensors = self._prepare_weights(source.model_or_path, source.revision,
                                                              source.fall_back_to_pt)
        else:
            files, use_safetensors = list(resolved_source.weight_files), resolved_source.use_safetensors
        if not use_safetensors:
            return super()._get_weights_iterator(source, resolved_source=resolved_source, **kwargs)
        device = "cpu"
        if extra.get("direct_to_device") and torch.cuda.is_available():
            device = torch.device("cuda", torch.cuda.current_device())
        prefix = getattr(source, "prefix", "")
        it = exl3_mmap_weights_iterator(files, device=device, num_threads=threads)
        return ((prefix + name, t) for name, t in it)
