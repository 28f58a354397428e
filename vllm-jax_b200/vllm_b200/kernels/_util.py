"""Small helpers shared by the torch-facing wrappers of libvjattn."""
from __future__ import annotations

import torch

from .. import _native

_workspaces: dict[tuple[int, str], torch.Tensor] = {}
_retired: list[torch.Tensor] = []


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("vllm_b200 kernels run on CUDA tensors only (no CPU fallback); "
                             f"got a tensor on {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise ValueError("no CUDA tensor given")
    _native.load()
    return dev


def require_dtype(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if t.dtype != dtype:
        raise ValueError(f"The dtype of `{name}` must be {dtype}. Got {t.dtype}")


def workspace(device: torch.device, nbytes: int, tag: str = "decode",
              zeroed: bool = False) -> torch.Tensor:
    """Per-device, per-tag scratch buffer that only grows (256-byte aligned;
    zero-filled when allocated if `zeroed`).

    A buffer that is outgrown is retired, never freed: a CUDA graph captured
    while it was current keeps its address and writes there on every replay."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), tag)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        if buf is not None:
            _retired.append(buf)
        alloc = torch.zeros if zeroed else torch.empty
        buf = alloc(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf
