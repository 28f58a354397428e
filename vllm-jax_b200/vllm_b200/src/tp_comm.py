"""NVLink peer-memory communicator for tensor parallelism.

Each rank allocates one communication region (vj_comm_alloc: flags, then two
partial buffers of [max_rows, hidden] bf16, and for the two-shot reduction
two result buffers), exports it with cudaIpc, and maps
every peer's region (handles exchanged once with all_gather_object). The
model's row-parallel GEMMs (o_proj, down_proj) write their partial products
straight into buffer `site` (0 for o_proj, 1 for down_proj, so consecutive
calls alternate), and vj_allreduce_add_rmsnorm sums all ranks' partials over
NVLink and applies the residual add + RMSNorm in the same kernel. There is
no host synchronisation and no NCCL call on this path, so decode steps under
tensor parallelism can be captured in CUDA graphs.

All ranks must make the same sequence of calls (the engine's replicated
scheduler guarantees it). A peer that stops calling makes the waiting CTAs
time out after 2 s and set the error word (`failed()`), never hang.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from .. import _native


class _DeviceArray:
    """Zero-copy torch view of raw device memory (CUDA array interface)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


def device_view(ptr: int, shape: tuple, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    typestr = {torch.bfloat16: "<i2", torch.int32: "<i4"}[dtype]
    t = torch.as_tensor(_DeviceArray(ptr, tuple(shape), typestr), device=device)
    return t.view(dtype)


class TPComm:

    def __init__(self, group, rank: int, world: int, device: torch.device, max_rows: int,
                 hidden: int, two_shot: bool | None = None):
        if world > 8:
            raise ValueError("at most 8 ranks")
        self.rank, self.world, self.device = rank, world, device
        self.max_rows, self.hidden = max_rows, hidden
        self.group = group
        # one-shot moves (N-1) x the data per rank, two-shot 2 (N-1)/N x plus a
        # second barrier: two-shot from 4 ranks on
        self.two_shot = world > 2 if two_shot is None else bool(two_shot)
        lib = _native.load()
        self.grid = int(lib.vj_tp_grid())
        self.flag_bytes = int(lib.vj_tp_flags_bytes(world))
        self.buf_bytes = (max_rows * hidden * 2 + 4095) // 4096 * 4096
        nbuf = 4 if self.two_shot else 2      # partials x2 (+ results x2)
        total = self.flag_bytes + nbuf * self.buf_bytes
        # every rank must launch the same grid
        grids = [None] * world
        dist.all_gather_object(grids, self.grid, group=group)
        if len(set(grids)) != 1:
            raise RuntimeError(f"ranks disagree on the all-reduce grid: {grids}")
        with torch.cuda.device(device):
            base = ctypes.c_void_p()
            _native.check(lib.vj_comm_alloc(total, ctypes.byref(base)))
            self._base = base.value
            handle = (ctypes.c_char * 64)()
            _native.check(lib.vj_ipc_get_handle(ctypes.c_void_p(self._base), handle))
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
            bases, self._opened = [], []
            for r in range(world):
                if r == rank:
                    bases.append(self._base)
                    continue
                p = ctypes.c_void_p()
                h = (ctypes.c_char * 64).from_buffer_copy(handles[r])
                _native.check(lib.vj_ipc_open_handle(h, ctypes.byref(p)))
                bases.append(p.value)
                self._opened.append(p.value)
        self._flags = (ctypes.c_void_p * world)(*bases)
        self._bufs = [(ctypes.c_void_p * world)(*[b + self.flag_bytes + s * self.buf_bytes
                                                  for b in bases]) for s in (0, 1)]
        self._results = [ctypes.cast((ctypes.c_void_p * world)(
            *[b + self.flag_bytes + (2 + s) * self.buf_bytes for b in bases]), ctypes.c_void_p)
            if self.two_shot else None for s in (0, 1)]
        self.buffers = [device_view(self._base + self.flag_bytes + s * self.buf_bytes,
                                    (max_rows, hidden), torch.bfloat16, device) for s in (0, 1)]
        err_off = (2 * world + 1) * self.grid * 4
        self._error = device_view(self._base + err_off, (1,), torch.int32, device)
        dist.barrier(group=group)

    def buffer(self, site: int, rows: int) -> torch.Tensor:
        """The local partial buffer of call site `site` (0 or 1), first `rows` rows."""
        return self.buffers[site][:rows]

    def allreduce_add_rmsnorm(self, site: int, rows: int, residual: torch.Tensor,
                              weight: torch.Tensor, eps: float):
        """(x = residual + sum of all ranks' buffer(site)[:rows], RMSNorm(x) * weight)."""
        H = self.hidden
        if residual.shape != (rows, H) or not residual.is_contiguous():
            raise ValueError("residual must be a contiguous [rows, hidden] tensor")
        y = torch.empty((rows, H), dtype=torch.bfloat16, device=self.device)
        r_out = torch.empty_like(y)
        _native.call("vj_allreduce_add_rmsnorm", ctypes.cast(self._bufs[site], ctypes.c_void_p),
                     self._results[site], ctypes.cast(self._flags, ctypes.c_void_p),
                     ctypes.c_void_p(self._base), self.rank, self.world, residual.data_ptr(),
                     weight.data_ptr(), r_out.data_ptr(), y.data_ptr(), rows, H, float(eps),
                     torch.cuda.current_stream(self.device).cuda_stream)
        return r_out, y

    def failed(self) -> bool:
        """True if a wait for a peer timed out (synchronises the device)."""
        return bool(self._error.item())

    def close(self) -> None:
        """Unmap the peers' regions and free this rank's (collective)."""
        if self._base is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        lib = _native.load()
        for p in self._opened:
            _native.check(lib.vj_ipc_close_handle(ctypes.c_void_p(p)))
        dist.barrier(group=self.group)
        self.buffers, self._error = [], None
        _native.check(lib.vj_comm_free(ctypes.c_void_p(self._base)))
        self._base = None
