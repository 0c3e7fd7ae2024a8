"""Persistent per-(device, stream) workspaces for the matmul kernels.

The kernels never allocate.  Like the reference's graph-safe workspace cache
(``src/sglang_exl3/dense.py:38-58``), buffers are keyed by (device, stream) and
only grow, so a CUDA graph captured after a warm-up call replays with stable
pointers.  Two kinds:

* state - split-K partial sums and arrival counters.  Zeroed once when
  allocated; every kernel call leaves it zeroed again.
* scratch - per-call temporaries (rotated activations), no initialisation.
"""

from __future__ import annotations

import threading

import torch

_STATE: dict = {}
_SCRATCH: dict = {}
_LOCK = threading.Lock()


def _key(device: torch.device, stream: torch.cuda.Stream):
    return (device.index if device.index is not None else torch.cuda.current_device(), stream.cuda_stream)


def _round_up(n: int) -> int:
    p = 1 << 20
    while p < n:
        p <<= 1
    return p


def state_buffer(device: torch.device, nbytes: int) -> torch.Tensor:
    stream = torch.cuda.current_stream(device)
    key = _key(device, stream)
    with _LOCK:
        buf = _STATE.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(_round_up(nbytes), dtype=torch.uint8, device=device)
            _STATE[key] = buf
        return buf


def scratch_buffer(device: torch.device, nbytes: int) -> torch.Tensor:
    stream = torch.cuda.current_stream(device)
    key = _key(device, stream)
    with _LOCK:
        buf = _SCRATCH.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(_round_up(nbytes), dtype=torch.uint8, device=device)
            _SCRATCH[key] = buf
        return buf


def clear() -> None:
    """Drop every cached buffer (e.g. before tearing down a process group)."""
    with _LOCK:
        _STATE.clear()
        _SCRATCH.clear()
