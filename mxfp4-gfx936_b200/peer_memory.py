"""Peer-mapped device buffers and a device-side barrier, one process per GPU.

Each rank allocates a buffer through the library (``mxfp4_ipc_alloc``:
cudaMalloc + a CUDA IPC handle), the ranks exchange the 64-byte handles with
``all_gather_object``, and every rank maps every other rank's buffer into its
own device context with peer access enabled (``mxfp4_ipc_open``).  The
library's kernels then read and write peers' memory directly over NVLink.
No NVLink multicast object is created.  The barrier is ``mxfp4_peer_barrier``:
one warp that signals every rank's flag array and waits for theirs, bounded
in time.
"""

from __future__ import annotations

import ctypes
import importlib.util
import sys
from pathlib import Path

import torch
import torch.distributed as dist

_HERE = Path(__file__).resolve().parent
_VPP = ctypes.POINTER(ctypes.c_void_p)


def _soft():
    name = "moe_op_mxfp4_soft"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, _HERE / "moe_op_mxfp4_soft.py")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


def pointer_array(ptrs) -> ctypes.Array:
    """A host array of device pointers for the C ABI (``void* const*``)."""
    arr = (ctypes.c_void_p * max(1, len(ptrs)))()
    for i, p in enumerate(ptrs):
        arr[i] = p
    return arr


_TYPESTR = {torch.int16: "<i2", torch.float16: "<f2", torch.float32: "<f4", torch.int32: "<i4",
            torch.uint8: "|u1"}


class _DeviceArray:
    """A raw device allocation seen through the CUDA array interface."""

    def __init__(self, ptr: int, shape, dtype: torch.dtype):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": _TYPESTR[dtype], "data": (ptr, False),
                                         "version": 2, "strides": None}


def _as_tensor(ptr: int, shape, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    raw_dtype = torch.int16 if dtype == torch.bfloat16 else dtype  # no bf16 typestr: alias as int16
    t = torch.as_tensor(_DeviceArray(ptr, shape, raw_dtype), device=device)
    return t.view(dtype) if raw_dtype != dtype else t


class PeerBuffers:
    """A ``shape``/``dtype`` buffer on every rank of ``group``, each mapped into
    every rank: ``ptrs[j]`` is the address of rank j's buffer in this process
    (``ptrs[rank]`` the local one, also viewed as the tensor ``local``),
    zero-filled at creation.  Collective: every rank of the group
    constructs it with the same shape and dtype.  ``close()`` (or garbage
    collection) unmaps the peers and frees the local allocation; it must not
    run while a kernel still uses the buffer."""

    def __init__(self, shape, dtype: torch.dtype, group=None):
        self._lib = _soft()._load_library()
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device("cuda", torch.cuda.current_device())
        nbytes = max(1, int(torch.Size(shape).numel()) * torch.empty((), dtype=dtype).element_size())
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        _check(self._lib, self._lib.mxfp4_ipc_alloc(nbytes, ctypes.byref(ptr), ctypes.cast(handle, ctypes.c_void_p)))
        self._local_ptr = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.ptrs, self._opened = [], []
        for j, h in enumerate(handles):
            if j == self.rank:
                self.ptrs.append(self._local_ptr)
                continue
            peer = ctypes.c_void_p()
            hb = (ctypes.c_uint8 * 64).from_buffer_copy(h)
            _check(self._lib, self._lib.mxfp4_ipc_open(ctypes.cast(hb, ctypes.c_void_p), ctypes.byref(peer)))
            self.ptrs.append(peer.value)
            self._opened.append(peer.value)
        self.local = _as_tensor(self._local_ptr, shape, dtype, self.device)

    def close(self, group=None, collective: bool = True) -> None:
        """Unmap the peers' buffers, then (after a group barrier, so no peer
        still maps it) free the local one.  Collective unless ``collective``
        is False (process exit)."""
        if getattr(self, "_lib", None) is None:
            return
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            self._lib.mxfp4_ipc_close(ctypes.c_void_p(p))
        self._opened = []
        if collective:
            dist.barrier(group=group)
        if self._local_ptr:
            self._lib.mxfp4_ipc_free(ctypes.c_void_p(self._local_ptr))
            self._local_ptr = 0
        self._lib = None
        self.local = None

    def __del__(self):
        try:
            self.close(collective=False)
        except Exception:
            pass


def _check(lib, rc: int) -> None:
    if rc:
        raise RuntimeError(f"libmxfp4_b200 error {rc}: {lib.mxfp4_last_error().decode(errors='replace')}")


def reset_protocol(quiesce, reset_local, host_barrier) -> None:
    """Collective reset of a device barrier whose epochs may disagree (after a
    bounded wait recorded MXFP4_ERR_TIMEOUT): every rank first waits until its
    own barrier kernels have finished (``quiesce``), a host barrier makes sure
    no rank's kernel can still store into a peer's flags, each rank zeroes its
    own flags and counter (``reset_local``, completed by a second ``quiesce``),
    and a second host barrier keeps every rank from signalling again before
    all have reset."""
    quiesce()
    host_barrier()
    reset_local()
    quiesce()
    host_barrier()


class PeerBarrier:
    """Device-side barrier of the ranks of ``group`` (collective constructor).

    ``timeout_us`` bounds every wait (0: the library default of 2 s); a wait
    that runs out records MXFP4_ERR_TIMEOUT in the device status word.  After
    that, call ``reset()`` on every rank before using the barrier again."""

    def __init__(self, group=None, timeout_us: int = 0):
        self.group = group
        self.flags = PeerBuffers((8,), torch.int32, group)  # zero-filled
        self.counter = torch.zeros(1, dtype=torch.int32, device=self.flags.local.device)
        self.rank, self.world = self.flags.rank, self.flags.world
        self.timeout_us = int(timeout_us)
        self._flag_ptrs = pointer_array(self.flags.ptrs)
        self._lib = _soft()._load_library()

    def __call__(self, stream: torch.cuda.Stream | None = None) -> None:
        s = stream if stream is not None else torch.cuda.current_stream()
        rc = self._lib.mxfp4_peer_barrier_timed(ctypes.cast(self._flag_ptrs, _VPP), self.rank, self.world,
                                                self.counter.data_ptr(), self.timeout_us, s.cuda_stream)
        _check(self._lib, rc)

    def reset(self) -> None:
        """Collective: zero every rank's flags and counter (``reset_protocol``)."""
        device = self.counter.device

        def reset_local():
            _check(self._lib, self._lib.mxfp4_peer_barrier_reset(
                ctypes.c_void_p(self.flags.ptrs[self.rank]), self.world, ctypes.c_void_p(self.counter.data_ptr()),
                torch.cuda.current_stream(device).cuda_stream))

        reset_protocol(lambda: torch.cuda.synchronize(device), reset_local, lambda: dist.barrier(group=self.group))
