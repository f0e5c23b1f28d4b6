"""Multi-rank host logic on CPU (gloo, world size 2): the column-sharded
linear's shard split and all-gather interleave give the unsharded result."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from _paths import PKG, ROOT, load_by_path


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cp = load_by_path("mxfp4_column_parallel", PKG / "column_parallel.py")
        ref = load_by_path("mxfp4_ref_cpu", ROOT / "oracle" / "ref_cpu.py")
        g = torch.Generator().manual_seed(0)
        m, n, k = 6, 256, 256
        x = torch.randn(m, k, generator=g).to(torch.bfloat16)
        w = torch.randint(0, 256, (n, k // 2), generator=g, dtype=torch.uint8)
        s = torch.randint(118, 131, (n, k // 32), generator=g, dtype=torch.uint8)
        layer = cp.ColumnParallelLinear.from_full(w, s, rank, world, linear_fn=ref.linear)
        y = layer(x.reshape(2, 3, k))
        full = ref.linear(x, w, s).reshape(2, 3, n)
        q.put((rank, bool(torch.equal(y.view(torch.int16), full.view(torch.int16)))))
    finally:
        dist.destroy_process_group()


def test_column_parallel_matches_unsharded_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = dict(q.get(timeout=5) for _ in procs)
    assert results == {0: True, 1: True}
    assert all(p.exitcode == 0 for p in procs)


def test_shard_rows_rejects_uneven_split():
    cp = load_by_path("mxfp4_column_parallel", PKG / "column_parallel.py")
    assert cp.shard_rows(5120, 7, 8) == (4480, 5120)
    with pytest.raises(ValueError):
        cp.shard_rows(100, 0, 3)
