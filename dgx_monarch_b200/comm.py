"""NVLink peer windows bound to one setup generation.

The reference builds its process groups once per setup
(actor/worker_env.py:313-327) and retires the attention implementation bound
to them on invalidate (actor/attention_dispatch.py:383-401).  PeerWindows is
the data-path half of that: each rank allocates one window in its own HBM
(libdgxm_sp.so, cudaMalloc), the CUDA IPC handles are exchanged once over the
torch.distributed group, and every rank maps every peer's window.  Kernels
then store straight into peer memory over NVLink; torch.distributed carries
only the bootstrap.  A window is keyed to its generation and is destroyed,
never reused, when that generation retires.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

_ALIGN = 256


class _RawDevice:
    """A borrowed device byte range, exposed through __cuda_array_interface__."""

    def __init__(self, ptr: int, nbytes: int) -> None:
        self.__cuda_array_interface__ = {
            "shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
            "strides": None,
        }


def device_bytes(ptr: int, nbytes: int, device: torch.device) -> torch.Tensor:
    """A uint8 tensor viewing `nbytes` of device memory at `ptr` (not owned)."""
    with torch.cuda.device(device):
        return torch.as_tensor(_RawDevice(ptr, nbytes), device=device)


def _exchange_handles(handle: bytes, group, device: torch.device) -> bytes:
    import torch.distributed as dist

    world = dist.get_world_size(group)
    mine = torch.tensor(list(handle), dtype=torch.uint8)
    backend = dist.get_backend(group)
    if backend == "nccl":
        mine = mine.to(device)
    bufs = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(bufs, mine, group=group)
    return b"".join(bytes(b.cpu().tolist()) for b in bufs)


class PeerWindows:
    """One window per rank of `group`, mapped into every rank of it."""

    def __init__(self, nbytes: int, *, device: torch.device, group=None, rank: int = 0,
                 world: int = 1, generation: int = 0) -> None:
        import torch.distributed as dist

        if group is not None or (world > 1 and dist.is_initialized()):
            rank = dist.get_rank(group)
            world = dist.get_world_size(group)
        self.rank, self.world, self.device, self.generation = rank, world, device, generation
        self._lib = _lib.load()
        self._handle = ctypes.c_void_p()
        with torch.cuda.device(device):
            _lib.check(self._lib.dgxm_comm_create(rank, world, int(nbytes), generation,
                                                  ctypes.byref(self._handle)), "dgxm_comm_create")
            self.nbytes = int(self._lib.dgxm_comm_bytes(self._handle))
            if world > 1:
                buf = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
                _lib.check(self._lib.dgxm_comm_export(self._handle, buf), "dgxm_comm_export")
                handles = _exchange_handles(buf.raw, group, device)
                _lib.check(self._lib.dgxm_comm_import(self._handle, handles), "dgxm_comm_import")
            self.bases = []
            for r in range(world):
                p = ctypes.c_void_p()
                _lib.check(self._lib.dgxm_comm_window(self._handle, r, ctypes.byref(p)),
                           "dgxm_comm_window")
                self.bases.append(int(p.value))
        self._cursor = 0

    # ---------------------------------------------------------------- carving
    def carve(self, nbytes: int) -> int:
        """Reserve `nbytes` at the same offset in every rank's window."""
        off = self._cursor
        self._cursor = (off + nbytes + _ALIGN - 1) // _ALIGN * _ALIGN
        if self._cursor > self.nbytes:
            raise RuntimeError(f"peer window of {self.nbytes} bytes is too small "
                               f"(needs {self._cursor})")
        return off

    def peer_ptr(self, peer: int, offset: int) -> int:
        return self.bases[peer] + offset

    def local_tensor(self, offset: int, shape, dtype: torch.dtype) -> torch.Tensor:
        n = 1
        for s in shape:
            n *= int(s)
        nbytes = n * torch.empty((), dtype=dtype).element_size()
        raw = device_bytes(self.bases[self.rank] + offset, nbytes, self.device)
        return raw.view(dtype).view(*shape)

    # ---------------------------------------------------------------- sync
    def set_timeout(self, milliseconds: int) -> None:
        """Bound every barrier wait of these windows to about `milliseconds`;
        a wait that runs out sets the device error word and returns."""
        _lib.check(self._lib.dgxm_comm_set_timeout(self._handle, int(milliseconds)), "dgxm_comm_set_timeout")

    def barrier(self, stream: torch.cuda.Stream | None = None) -> None:
        stream = stream or torch.cuda.current_stream(self.device)
        _lib.check(self._lib.dgxm_comm_barrier(self._handle, stream.cuda_stream), "dgxm_comm_barrier")

    def close(self) -> None:
        if self._handle is not None and self._handle.value:
            with torch.cuda.device(self.device):
                rc = self._lib.dgxm_comm_destroy(self._handle)
            self._handle = None
            _lib.check(rc, "dgxm_comm_destroy")

    def __del__(self):  # pragma: no cover - best effort at interpreter exit
        try:
            if self._handle is not None and self._handle.value:
                self._lib.dgxm_comm_destroy(self._handle)
                self._handle = None
        except Exception:
            pass
