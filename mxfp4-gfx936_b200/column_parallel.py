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
  every other rank's buffer (``mxfp4_linear_w4a16_allgather``), so the
  transfer overlaps the math tile by tile; a device-side barrier
  (``mxfp4_peer_barrier``) then marks the output complete.  The output lives in
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


def shard_rows(n: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of the output features owned by ``rank``; n % world == 0."""
    if n % world:
        raise ValueError(f"output features {n} must divide evenly over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


class ColumnParallelLinear:
    def __init__(self, w_shard: torch.Tensor, s_shard: torch.Tensor, n_full: int, rank: int, world: int,
                 group=None, linear_fn=None, fused: bool = False):
        self.w, self.s = w_shard.contiguous(), s_shard.contiguous()
        self.n_full, self.rank, self.world, self.group = n_full, rank, world, group
        self.linear_fn = linear_fn if linear_fn is not None else _soft().linear_mxfp4_soft
        if self.w.shape[0] * world != n_full:
            raise ValueError("shard rows times world size must equal the output features")
        if fused and linear_fn is not None:
            raise ValueError("the fused all-gather runs the native kernel; linear_fn cannot be injected")
        self.fused = fused and world > 1
        self._bufs = None      # two PeerBuffers [rows, n_full]
        self._barrier = None
        self._step = 0

    @classmethod
    def from_full(cls, w: torch.Tensor, s: torch.Tensor, rank: int, world: int, group=None, linear_fn=None,
                  fused: bool = False):
        lo, hi = shard_rows(w.shape[0], rank, world)
        return cls(w[lo:hi], s[lo:hi], w.shape[0], rank, world, group, linear_fn, fused)

    def _fused_call(self, x2: torch.Tensor) -> torch.Tensor:
        soft = _soft()
        pm = _peer_memory()
        m, k = x2.shape
        n_local = self.w.shape[0]
        if x2.dtype not in (torch.bfloat16, torch.float16):
            raise TypeError("x must be BF16 or FP16")
        if self._bufs is None or self._bufs[0].local.shape[0] < m or self._bufs[0].local.dtype != x2.dtype:
            # collective: every rank of a TP group sees the same M
            if self._bufs is not None:
                for b in self._bufs:
                    b.close(self.group)  # collective: every rank reallocates at the same call
            self._bufs = [pm.PeerBuffers((m, self.n_full), x2.dtype, self.group) for _ in range(2)]
            if self._barrier is None:
                self._barrier = pm.PeerBarrier(self.group)
        buf = self._bufs[self._step % 2]
        self._step += 1
        esz = x2.element_size()
        col = self.rank * n_local * esz
        peers = [buf.ptrs[j] + col for j in range(self.world) if j != self.rank]
        peer_arr = pm.pointer_array(peers)
        x2 = soft._dense(x2)
        device = x2.device
        backend = soft._backend()
        mode = soft._LINEAR_FUSED if backend == "fused" else soft._LINEAR_SAFE
        lib = soft._load_library()
        code = soft._DTYPE_CODES[x2.dtype]
        if m:
            ws_bytes = lib.mxfp4_linear_workspace_size(m, n_local, k, code, mode)
            ws = soft._workspace(ws_bytes, device) if ws_bytes else None
            with torch.cuda.device(device):
                soft._check(lib.mxfp4_linear_w4a16_allgather(
                    soft._ptr(x2), code, k, soft._ptr(self.w), k // 2, soft._ptr(self.s), k // 32, None,
                    ctypes.c_void_p(buf.ptrs[self.rank] + col), ctypes.cast(peer_arr, ctypes.POINTER(ctypes.c_void_p)),
                    len(peers), self.n_full, m, n_local, k, mode, soft._ptr(ws), ws_bytes, soft._stream(device)))
        self._barrier()
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
