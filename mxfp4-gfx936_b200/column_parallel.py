"""Column-sharded MXFP4 linear over torch.distributed (tensor parallel).

Each rank holds ``W[n/G, K/2]`` and ``S[n/G, K/32]`` -- a contiguous block of
output features -- computes its ``y[:, n/G]`` with the B200 linear kernel and
an all-gather (NCCL over NVLink on GPUs) assembles the full ``y[M, n]``.  This
is the dense-layer partitioning of the reference's serving setup, where vLLM
shards the compressed-tensors linears across TP ranks (the reference runs
TP=2, examples/qwen3_30b_a3b/eval_qwen3_30b_moe_quality.py:107), with every
shard computed by ``linear_mxfp4_soft`` (soft:310-376).
"""

from __future__ import annotations

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


def shard_rows(n: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of the output features owned by ``rank``; n % world == 0."""
    if n % world:
        raise ValueError(f"output features {n} must divide evenly over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


class ColumnParallelLinear:
    def __init__(self, w_shard: torch.Tensor, s_shard: torch.Tensor, n_full: int, rank: int, world: int,
                 group=None, linear_fn=None):
        self.w, self.s = w_shard.contiguous(), s_shard.contiguous()
        self.n_full, self.rank, self.world, self.group = n_full, rank, world, group
        self.linear_fn = linear_fn if linear_fn is not None else _soft().linear_mxfp4_soft
        if self.w.shape[0] * world != n_full:
            raise ValueError("shard rows times world size must equal the output features")

    @classmethod
    def from_full(cls, w: torch.Tensor, s: torch.Tensor, rank: int, world: int, group=None, linear_fn=None):
        lo, hi = shard_rows(w.shape[0], rank, world)
        return cls(w[lo:hi], s[lo:hi], w.shape[0], rank, world, group, linear_fn)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        y_local = self.linear_fn(x2, self.w, self.s)           # [M, n/G]
        if self.world == 1:
            return y_local.reshape(*lead, self.n_full)
        rows, cols = y_local.shape
        gathered = torch.empty((self.world * rows, cols), dtype=y_local.dtype, device=y_local.device)
        dist.all_gather_into_tensor(gathered, y_local.contiguous(), group=self.group)
        y = gathered.view(self.world, rows, cols).permute(1, 0, 2).reshape(rows, self.n_full)
        return y.reshape(*lead, self.n_full)
