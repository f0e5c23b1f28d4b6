"""Expert-parallel MXFP4 MoE layer over torch.distributed.

Each of the G ranks owns E/G consecutive experts (global ids
``[rank*E/G, (rank+1)*E/G)``) and its own tokens.  This is the expert-parallel
form of the reference's MoE composition (integration/vllm/vllm_mxfp4_gfx936.py:
233-265), whose only EP-aware code is the rule that routes to non-local
experts produce nothing locally (src/aiter/ops/triton/moe_op_mxfp4_soft.py:
113-115, 478).  Two implementations, both bit-identical to the single-GPU
``moe_layer_mxfp4`` for the rank's tokens:

``fused=True`` (GPUs, one process per GPU; the default on CUDA tensors):
one native call, ``mxfp4_ep_moe_layer``.  The route counts are exchanged
through peer-mapped memory; every rank derives every owner's routed block
layout from the same count matrix; a dispatch kernel writes each route's
activation row straight into the owner's routed-order buffer over NVLink;
the owner runs the grouped gate_up / down GEMMs on the received rows; the
source's combine kernel reads the weighted rows back over NVLink and sums
the top-k rows of each token in FP32 in slot order.  Three device-side
barriers, no NCCL and no host synchronisation.

``fused=False``: torch.distributed collectives (NCCL all-to-all on GPUs,
gloo on CPU ranks, where ``layer_fn`` / ``route_fn`` can be injected):

1. routes ``r = t*top_k + j`` are grouped by destination rank
   ``topk_ids // (E/G)`` (stable);
2. per-destination counts are exchanged, then one all-to-all each carries the
   activation row ``x[r // top_k]``, the local expert id and the route weight;
3. the owner runs the MoE layer on its received routes, one route per row;
4. the weighted rows travel back with the reverse all-to-all and the top-k
   rows of every token are summed in FP32 in slot order and rounded to BF16.
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


def expert_range(num_experts: int, rank: int, world: int) -> tuple[int, int]:
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not divide over {world} ranks")
    per = num_experts // world
    return rank * per, (rank + 1) * per


def sum_topk_rows(rows: torch.Tensor, top_k: int) -> torch.Tensor:
    """out[t] = bf16(sum_j float(rows[t*top_k + j])), FP32 accumulation in j order."""
    t = rows.shape[0] // top_k
    r = rows.view(t, top_k, -1)
    acc = r[:, 0].float()
    for j in range(1, top_k):
        acc = acc + r[:, j].float()
    return acc.to(torch.bfloat16)


class ExpertParallelMoE:
    """One rank's share of an expert-parallel MXFP4 MoE layer.

    ``layer_fn(x, w13, s13, w2, s2, topk_weights, topk_ids)`` computes the
    local layer (default: the native ``moe_layer_mxfp4``); ``route_fn(ids,
    num_groups)`` returns the stable destination order of the routes (default:
    the device routing kernel).  Both are injectable so the exchange logic can
    be tested on CPU ranks.
    """

    def __init__(self, w13_local, s13_local, w2_local, s2_local, num_experts: int, rank: int, world: int,
                 group=None, layer_fn=None, route_fn=None, fused: bool | None = None, max_tokens: int | None = None,
                 buffer_pool: dict | None = None):
        self.w13, self.s13, self.w2, self.s2 = w13_local, s13_local, w2_local, s2_local
        self.num_experts, self.rank, self.world, self.group = num_experts, rank, world, group
        self.lo, self.hi = expert_range(num_experts, rank, world)
        self.per = self.hi - self.lo
        if w13_local.shape[0] != self.per or w2_local.shape[0] != self.per:
            raise ValueError("local weights must hold num_experts / world experts")
        injected = layer_fn is not None or route_fn is not None
        if fused is None:
            fused = w13_local.is_cuda and not injected
        if fused and injected:
            raise ValueError("the fused layer runs the native kernels; layer_fn/route_fn cannot be injected")
        self.fused = fused
        self.max_tokens = max_tokens
        self.layer_fn = layer_fn if layer_fn is not None else _soft().moe_layer_mxfp4
        self.route_fn = route_fn if route_fn is not None else self._device_route
        self._peer = None  # (top_k, capacity, counts, xr, wr, yr, barrier, tables, max_tokens) once allocated
        # peer buffers keyed by (top_k, hidden): this layer's own, or shared with
        # the other layers given the same pool.  Layers that run one after another
        # in stream order on every rank can share them: each call's three device
        # barriers order its buffer uses against the previous call's.
        self._pool = buffer_pool if buffer_pool is not None else {}

    @classmethod
    def from_full(cls, w13, s13, w2, s2, rank: int, world: int, group=None, layer_fn=None, route_fn=None,
                  fused: bool | None = None, max_tokens: int | None = None, buffer_pool: dict | None = None):
        lo, hi = expert_range(w13.shape[0], rank, world)
        return cls(w13[lo:hi].contiguous(), s13[lo:hi].contiguous(), w2[lo:hi].contiguous(),
                   s2[lo:hi].contiguous(), w13.shape[0], rank, world, group, layer_fn, route_fn, fused, max_tokens,
                   buffer_pool)

    # ------------------------------------------------------------------ fused (native) path
    def _peer_buffers(self, t: int, top_k: int, hidden: int):
        """Peer-mapped buffers sized for ``max_tokens`` tokens per rank (set at
        construction, or the largest token count of any rank at the first call:
        one all-reduce).  Collective."""
        if self._peer is not None:
            if self._peer[0] != top_k:
                raise ValueError("top_k changed between calls of a fused expert-parallel layer")
            return self._peer
        shared = self._pool.get((top_k, hidden))
        if shared is not None:
            self._peer = shared
            self.max_tokens = shared[8]
            return shared
        pm = _peer_memory()
        if self.max_tokens is None:
            n = torch.tensor([t], dtype=torch.int64, device=self.w13.device)
            dist.all_reduce(n, op=dist.ReduceOp.MAX, group=self.group)
            self.max_tokens = int(n.item())
        lib = _soft()._load_library()
        cap = int(lib.mxfp4_ep_moe_recv_capacity(self.max_tokens, top_k, self.num_experts, self.world))
        counts = pm.PeerBuffers((self.world * self.num_experts,), torch.int32, self.group)
        xr = pm.PeerBuffers((cap, hidden), torch.bfloat16, self.group)
        wr = pm.PeerBuffers((cap,), torch.float32, self.group)
        yr = pm.PeerBuffers((cap, hidden), torch.bfloat16, self.group)
        barrier = pm.PeerBarrier(self.group)
        tables = [pm.pointer_array(b.ptrs) for b in (counts, xr, wr, yr)]
        self._peer = (top_k, cap, counts, xr, wr, yr, barrier, tables, self.max_tokens)
        self._pool[(top_k, hidden)] = self._peer
        return self._peer

    def _fused_call(self, x, topk_weights, topk_ids):
        soft = _soft()
        pm = _peer_memory()
        t, hidden = x.shape
        top_k = topk_ids.shape[1]
        if x.dtype != torch.bfloat16:
            raise TypeError(f"x must be bf16, got {x.dtype}")
        if topk_ids.shape != topk_weights.shape or topk_ids.shape[0] != t:
            raise ValueError("top-k ids and weights must have matching (M, top_k) shapes")
        top_k_, cap, counts, xr, wr, yr, barrier, tables, _ = self._peer_buffers(t, top_k, hidden)
        if t > self.max_tokens:
            raise ValueError(f"{t} tokens exceed the {self.max_tokens} this expert-parallel layer was sized for")
        inter = self.w13.shape[1] // 2
        lib = soft._load_library()
        device = x.device
        out = torch.empty((t, hidden), dtype=torch.bfloat16, device=device)
        ws_bytes = lib.mxfp4_ep_moe_workspace_size(t, top_k, self.num_experts, inter, cap)
        ws = soft._workspace(ws_bytes, device)
        xs, tw, tid = soft._dense(x), soft._dense(topk_weights), soft._dense(topk_ids)
        vpp = ctypes.POINTER(ctypes.c_void_p)
        with torch.cuda.device(device):
            soft._check(lib.mxfp4_ep_moe_layer(
                soft._ptr(xs), soft._ptr(self.w13), soft._ptr(self.s13), soft._ptr(self.w2), soft._ptr(self.s2),
                soft._ptr(tw), soft._DTYPE_CODES[tw.dtype], soft._ptr(tid), soft._DTYPE_CODES[tid.dtype],
                soft._ptr(out), t, top_k, self.num_experts, hidden, inter, self.rank, self.world,
                ctypes.cast(tables[0], vpp), ctypes.cast(tables[1], vpp), ctypes.cast(tables[2], vpp),
                ctypes.cast(tables[3], vpp), cap, ctypes.cast(barrier._flag_ptrs, vpp), barrier.counter.data_ptr(),
                soft._ptr(ws), ws_bytes, soft._stream(device)))
        return out

    @staticmethod
    def _device_route(dest: torch.Tensor, world: int) -> torch.Tensor:
        sorted_ids, _, post = _soft().moe_route(dest.view(-1, 1), world, block_m=1)
        return sorted_ids[: dest.numel()].long()

    def __call__(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
        if self.fused:
            return self._fused_call(x, topk_weights, topk_ids)
        t, hidden = x.shape
        top_k = topk_ids.shape[1]
        ids = topk_ids.reshape(-1).long()
        dest = (ids // self.per).to(torch.int32)
        order = self.route_fn(dest, self.world)                      # routes grouped by destination
        counts = torch.bincount(dest.long(), minlength=self.world)   # routes per destination
        recv_counts = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        send_sizes = counts.tolist()
        recv_sizes = recv_counts.tolist()
        n_recv = int(sum(recv_sizes))

        # dispatch: activation rows, local expert ids, route weights
        x_send = x.index_select(0, torch.div(order, top_k, rounding_mode="floor"))
        e_send = (ids.index_select(0, order) - dest.long().index_select(0, order) * self.per).to(torch.int32)
        w_send = topk_weights.reshape(-1).float().index_select(0, order)
        x_recv = torch.empty((n_recv, hidden), dtype=x.dtype, device=x.device)
        e_recv = torch.empty((n_recv,), dtype=torch.int32, device=x.device)
        w_recv = torch.empty((n_recv,), dtype=torch.float32, device=x.device)
        dist.all_to_all_single(x_recv, x_send, recv_sizes, send_sizes, group=self.group)
        dist.all_to_all_single(e_recv, e_send, recv_sizes, send_sizes, group=self.group)
        dist.all_to_all_single(w_recv, w_send, recv_sizes, send_sizes, group=self.group)

        # local experts, one route per row (top_k = 1): y = bf16(bf16(h . W2^T) * w)
        if n_recv:
            y_recv = self.layer_fn(x_recv, self.w13, self.s13, self.w2, self.s2, w_recv.view(-1, 1),
                                   e_recv.view(-1, 1))
        else:                                                         # no route chose this rank's experts
            y_recv = torch.empty((0, hidden), dtype=torch.bfloat16, device=x.device)

        # combine: weighted rows back to their origin, unpermute, sum over top-k
        y_send = torch.empty((ids.numel(), hidden), dtype=y_recv.dtype, device=x.device)
        dist.all_to_all_single(y_send, y_recv.contiguous(), send_sizes, recv_sizes, group=self.group)
        y_routes = torch.empty_like(y_send)
        y_routes.index_copy_(0, order, y_send)
        return sum_topk_rows(y_routes, top_k)
