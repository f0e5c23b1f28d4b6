"""Column-sharded MXFP4 linear over torch.distributed (tensor parallel).

Each rank holds ``W[n/G, K/2]`` and ``S[n/G, K/32]`` -- a contiguous block of
output features -- and computes its ``y[:, n/G]`` with the B200 linear kernel;
the full ``y[M, n]`` is then assembled on every rank.  This is the dense-layer
partitioning of the reference's serving setup, where vLLM shards the
compressed-tensors linears across TP ranks (the reference runs TP=2,
examples/qwen3_30b_a3b/eval_qwen3_30b_moe_quality.py:107), with every shard
computed by ``linear_mxfp4_soft`` (soft:310-376).

Two ways to assemble the output:

* ``fused=False``: ``all_gather_into_tensor`` (NCCL over NVLink) after the
  shard GEMM, then a column interleave.
* ``fused=True`` (GPUs, one process per GPU): the GEMM epilogue stores every
  output tile into its own buffer and, over NVLink, into the same columns of
  every other rank's buffer, so the transfer overlaps the math tile by tile; a
  device-side barrier (``mxfp4_peer_barrier``) then marks the output complete.
  Two ways to reach the peers: the pusher warps store each tile into every
  peer's buffer, mapped by CUDA IPC (``mxfp4_linear_w4a16_allgather``), or,
  where the GPUs share an NVSwitch multicast object (torch symmetric memory
  reports multicast support), store it once through the multicast address and
  the switch writes it into every rank's buffer
  (``mxfp4_linear_w4a16_allgather_mc``), so a GPU sends its block once instead
  of once per peer.  ``multicast=None`` picks multicast for groups of at least
  ``MULTICAST_MIN_WORLD`` GPUs: measured on B200 (qkv 4096x5120x2048 step) it
  is 5% faster at 8 GPUs and slower at 2 and 4, where the per-peer stores
  move little enough.  The output lives in
  one of two peer-mapped buffers used alternately: the returned tensor stays
  valid until the second call after it (consume it on the current stream
  before then, or copy it).
"""

from __future__ import annotations

import ctypes
import importlib.util
import sys
from pathlib import Path

import torch
import torch.distributed as dist

_HERE = Path(__file__).resolve().parent


def _soft():
    name = "moe_op_mxfp4_soft"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, _HERE / "moe_op_mxfp4_soft.py")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


def _peer_memory():
    name = "mxfp4_peer_memory"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, _HERE / "peer_memory.py")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


MULTICAST_MIN_WORLD = 8


def shard_rows(n: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of the output features owned by ``rank``; n % world == 0."""
    if n % world:
        raise ValueError(f"output features {n} must divide evenly over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


class _SymmBuffer:
    """An output buffer in torch symmetric memory whose ranks share an NVSwitch
    multicast object: ``local`` (this rank's tensor), ``ptrs`` (every rank's
    buffer as mapped in this process) and ``multicast_ptr``."""

    def __init__(self, tensor, handle):
        self.local = tensor
        self._handle = handle  # keeps the mappings alive
        self.ptrs = [int(p) for p in handle.buffer_ptrs]
        self.multicast_ptr = int(handle.multicast_ptr or 0)

    @classmethod
    def create(cls, shape, dtype, device, group):
        """Collective.  None where the group has no multicast support."""
        import torch.distributed._symmetric_memory as symm
        from torch._C._distributed_c10d import _SymmetricMemory

        device = torch.device(device)
        try:
            if not _SymmetricMemory.has_multicast_support(symm.DeviceType.CUDA, device.index):
                return None
            t = symm.empty(*shape, dtype=dtype, device=device)
            h = symm.rendezvous(t, group if group is not None else dist.group.WORLD)
        except (RuntimeError, AttributeError, TypeError):
            return None
        buf = cls(t, h)
        return buf if buf.multicast_ptr else None

    def close(self, group=None, collective: bool = True):
        if self.local is None:
            return
        torch.cuda.synchronize(self.local.device)
        if collective:
            dist.barrier(group=group)  # no rank still reads the old buffers
        self._handle = None
        self.local = None


class _OutputState:
    """The two alternating output buffers of fused column-parallel calls, the
    device barrier that ends each call, and the call count that alternates
    them.  Layers that run one after another in stream order on every rank
    (the linears of a decoder stack) can share one state: a call's result
    stays valid until the second call after it through the same state."""

    def __init__(self):
        self.bufs = None
        self.barrier = None
        self.step = 0


class ColumnParallelLinear:
    def __init__(self, w_shard: torch.Tensor, s_shard: torch.Tensor, n_full: int, rank: int, world: int,
                 group=None, linear_fn=None, fused: bool = False, multicast: bool | None = None,
                 buffer_pool: dict | None = None):
        self.w, self.s = w_shard.contiguous(), s_shard.contiguous()
        self.n_full, self.rank, self.world, self.group = n_full, rank, world, group
        self.linear_fn = linear_fn if linear_fn is not None else _soft().linear_mxfp4_soft
        if self.w.shape[0] * world != n_full:
            raise ValueError("shard rows times world size must equal the output features")
        if fused and linear_fn is not None:
            raise ValueError("the fused all-gather runs the native kernel; linear_fn cannot be injected")
        self.fused = fused and world > 1
        self.multicast = multicast  # None: NVSwitch multicast for groups of >= MULTICAST_MIN_WORLD GPUs
        # output buffers per (output width, dtype): this layer's own, or shared
        # with the other layers given the same pool (same group, same stream order)
        self._pool = buffer_pool if buffer_pool is not None else {}
        self._bufs = None      # the last call's two output buffers [rows, n_full]: _SymmBuffer or PeerBuffers

    @classmethod
    def from_full(cls, w: torch.Tensor, s: torch.Tensor, rank: int, world: int, group=None, linear_fn=None,
                  fused: bool = False, multicast: bool | None = None, buffer_pool: dict | None = None):
        lo, hi = shard_rows(w.shape[0], rank, world)
        return cls(w[lo:hi], s[lo:hi], w.shape[0], rank, world, group, linear_fn, fused, multicast, buffer_pool)

    def _alloc(self, m: int, dtype: torch.dtype, device: torch.device):
        """Two output buffers [m, n_full]; collective over the group."""
        if self.multicast or (self.multicast is None and self.world >= MULTICAST_MIN_WORLD):
            bufs = [_SymmBuffer.create((m, self.n_full), dtype, device, self.group) for _ in range(2)]
            # every rank takes the same path
            ok = torch.tensor([int(all(b is not None for b in bufs))], dtype=torch.int32, device=device)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.group)
            if int(ok.item()):
                return bufs
            if self.multicast:
                raise RuntimeError("NVSwitch multicast is not available for this group")
        pm = _peer_memory()
        return [pm.PeerBuffers((m, self.n_full), dtype, self.group) for _ in range(2)]

    def _fused_call(self, x2: torch.Tensor) -> torch.Tensor:
        soft = _soft()
        pm = _peer_memory()
        m, k = x2.shape
        n_local = self.w.shape[0]
        if x2.dtype not in (torch.bfloat16, torch.float16):
            raise TypeError("x must be BF16 or FP16")
        st = self._pool.setdefault((self.n_full, x2.dtype), _OutputState())
        if st.bufs is None or st.bufs[0].local.shape[0] < m:
            # collective: every rank of a TP group sees the same M
            if st.bufs is not None:
                for b in st.bufs:
                    b.close(self.group)  # collective: every rank reallocates at the same call
            st.bufs = self._alloc(m, x2.dtype, x2.device)
            if st.barrier is None:
                st.barrier = pm.PeerBarrier(self.group)
        self._bufs = st.bufs
        buf = st.bufs[st.step % 2]
        st.step += 1
        esz = x2.element_size()
        col = self.rank * n_local * esz
        peers = [buf.ptrs[j] + col for j in range(self.world) if j != self.rank]
        peer_arr = pm.pointer_array(peers)
        x2 = soft._dense(x2)
        device = x2.device
        backend = soft._backend()
        mode = soft._LINEAR_FUSED if backend in soft._FUSED_BACKENDS else soft._LINEAR_SAFE
        lib = soft._load_library()
        code = soft._DTYPE_CODES[x2.dtype]
        if m:
            ws_bytes = lib.mxfp4_linear_workspace_size(m, n_local, k, code, mode)
            ws = soft._workspace(ws_bytes, device) if ws_bytes else None
            peer_pp = ctypes.cast(peer_arr, ctypes.POINTER(ctypes.c_void_p))
            common = (soft._ptr(x2), code, k, soft._ptr(self.w), k // 2, soft._ptr(self.s), k // 32, None,
                      ctypes.c_void_p(buf.ptrs[self.rank] + col), peer_pp, len(peers))
            tail = (self.n_full, m, n_local, k, mode, soft._ptr(ws), ws_bytes, soft._stream(device))
            with torch.cuda.device(device):
                mc = getattr(buf, "multicast_ptr", 0)
                if mc:
                    soft._check(lib.mxfp4_linear_w4a16_allgather_mc(*common, ctypes.c_void_p(mc + col), *tail))
                else:
                    soft._check(lib.mxfp4_linear_w4a16_allgather(*common, *tail))
        st.barrier()
        return buf.local[:m]

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        if self.fused:
            return self._fused_call(x2).reshape(*lead, self.n_full)
        y_local = self.linear_fn(x2, self.w, self.s)           # [M, n/G]
        if self.world == 1:
            return y_local.reshape(*lead, self.n_full)
        rows, cols = y_local.shape
        gathered = torch.empty((self.world * rows, cols), dtype=y_local.dtype, device=y_local.device)
        dist.all_gather_into_tensor(gathered, y_local.contiguous(), group=self.group)
        y = gathered.view(self.world, rows, cols).permute(1, 0, 2).reshape(rows, self.n_full)
        return y.reshape(*lead, self.n_full)
