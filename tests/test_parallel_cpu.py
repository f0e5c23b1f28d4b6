"""Multi-rank host logic on CPU (gloo, world size 2): the column-sharded
linear's shard split and all-gather interleave give the unsharded result; its
choice between NVSwitch multicast and CUDA IPC output buffers is made by group
size and agreed by every rank; the expert-parallel exchange reproduces the
single layer."""

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


# ---------------------------------------------------------------------------
# expert parallelism: dispatch / combine exchange on CPU ranks
# ---------------------------------------------------------------------------
def _ep_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ep = load_by_path("mxfp4_expert_parallel", PKG / "expert_parallel.py")
        ref = load_by_path("mxfp4_ref_cpu", ROOT / "oracle" / "ref_cpu.py")
        O = load_by_path("mxfp4_oracle", ROOT / "oracle" / "mxfp4_oracle.py")
        g = torch.Generator().manual_seed(3)
        t_local, h, e, k, inter = 12, 256, 8, 2, 128
        x_all = torch.randn(world * t_local, h, generator=g).to(torch.bfloat16)
        w13 = torch.randint(0, 256, (e, 2 * inter, h // 2), generator=g, dtype=torch.uint8)
        s13 = torch.randint(118, 131, (e, 2 * inter, h // 32), generator=g, dtype=torch.uint8)
        w2 = torch.randint(0, 256, (e, h, inter // 2), generator=g, dtype=torch.uint8)
        s2 = torch.randint(114, 127, (e, h, inter // 32), generator=g, dtype=torch.uint8)
        logits = torch.randn(world * t_local, e, generator=g)
        tw_all, tid_all = torch.topk(torch.softmax(logits, -1), k, dim=-1)
        sl = slice(rank * t_local, (rank + 1) * t_local)

        def route_fn(dest, world_):
            return torch.argsort(dest.long(), stable=True)

        layer = ep.ExpertParallelMoE.from_full(w13, s13, w2, s2, rank, world, layer_fn=ref.moe_layer,
                                               route_fn=route_fn)
        y = layer(x_all[sl], tw_all[sl], tid_all[sl])
        full = ref.moe_layer(x_all, w13, s13, w2, s2, tw_all, tid_all)[sl]
        ok = O.check_close(y.float().numpy(), full.float().numpy())[0]
        # one rank's tokens may route only to the other rank's experts and vice versa
        q.put((rank, bool(ok), tuple(y.shape)))
    finally:
        dist.destroy_process_group()


def test_expert_parallel_matches_single_layer_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    results = {r: (ok, shp) for r, ok, shp in (q.get(timeout=5) for _ in procs)}
    assert results == {0: (True, (12, 256)), 1: (True, (12, 256))}
    assert all(p.exitcode == 0 for p in procs)


def test_expert_range_and_topk_sum():
    ep = load_by_path("mxfp4_expert_parallel", PKG / "expert_parallel.py")
    assert ep.expert_range(128, 3, 8) == (48, 64)
    with pytest.raises(ValueError):
        ep.expert_range(10, 0, 4)
    rows = torch.randn(6, 16).to(torch.bfloat16)
    s = ep.sum_topk_rows(rows, 3)
    want = (rows.view(2, 3, 16).float()[:, 0] + rows.view(2, 3, 16).float()[:, 1]
            + rows.view(2, 3, 16).float()[:, 2]).to(torch.bfloat16)
    assert torch.equal(s.view(torch.int16), want.view(torch.int16))


def _multicast_policy_worker(rank, world, port, q):
    # the column-parallel layer's choice between NVSwitch multicast buffers and
    # CUDA IPC peer buffers, with both kinds of buffer faked: the choice is made
    # by group size, and collectively (one rank without multicast -> none use it)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cp = load_by_path("mxfp4_column_parallel", PKG / "column_parallel.py")
        pm = cp._peer_memory()
        made = []

        class FakeIpc:
            def __init__(self, shape, dtype, group):
                made.append("ipc")

        class FakeSymm:
            multicast_ptr = 1

        supported = {"value": True}

        def fake_create(shape, dtype, device, group):
            made.append("symm-try")
            return FakeSymm() if supported["value"] else None

        pm.PeerBuffers = FakeIpc
        cp._SymmBuffer.create = staticmethod(fake_create)
        w = torch.zeros(32, 16, dtype=torch.uint8)
        s = torch.zeros(32, 1, dtype=torch.uint8)
        out = {}
        # group of 2 GPUs, default policy: IPC peer buffers, multicast not tried
        made.clear()
        layer = cp.ColumnParallelLinear(w, s, 32 * world, rank, world, fused=True)
        bufs = layer._alloc(4, torch.bfloat16, "cpu")
        out["two"] = (made.copy(), type(bufs[0]).__name__)
        # a layer of 8 ranks (as it sees its group): multicast buffers
        made.clear()
        layer = cp.ColumnParallelLinear(w, s, 32 * 8, rank, 8, fused=True)
        bufs = layer._alloc(4, torch.bfloat16, "cpu")
        out["eight"] = (made.copy(), type(bufs[0]).__name__)
        # forced multicast, one rank without support: every rank raises
        made.clear()
        supported["value"] = rank == 0
        layer = cp.ColumnParallelLinear(w, s, 32 * world, rank, world, fused=True, multicast=True)
        try:
            layer._alloc(4, torch.bfloat16, "cpu")
            out["forced"] = "no error"
        except RuntimeError:
            out["forced"] = "raised"
        # default policy at 8, one rank without support: every rank falls back to IPC
        made.clear()
        layer = cp.ColumnParallelLinear(w, s, 32 * 8, rank, 8, fused=True)
        bufs = layer._alloc(4, torch.bfloat16, "cpu")
        out["fallback"] = type(bufs[0]).__name__
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_column_parallel_multicast_policy_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_multicast_policy_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    res = dict(q.get(timeout=5) for _ in procs)
    assert all(p.exitcode == 0 for p in procs)
    for rank in (0, 1):
        out = res[rank]
        assert out["two"] == (["ipc", "ipc"], "FakeIpc"), out
        assert out["eight"] == (["symm-try", "symm-try"], "FakeSymm"), out
        assert out["forced"] == "raised", out
        assert out["fallback"] == "FakeIpc", out


def _reset_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    pm = load_by_path("mxfp4_peer_memory", PKG / "peer_memory.py")
    import time
    events = []

    def quiesce():
        events.append(("quiesce", time.monotonic()))

    def reset_local():
        if rank == 1:
            time.sleep(0.3)  # a slow rank: nobody may resume before it has reset
        events.append(("reset", time.monotonic()))

    pm.reset_protocol(quiesce, reset_local, dist.barrier)
    events.append(("resume", time.monotonic()))
    q.put((rank, events))
    dist.destroy_process_group()


def test_barrier_reset_protocol_orders_ranks_gloo():
    # after a timed-out device barrier every rank resets its own flags; no rank
    # may reset while a peer's barrier kernel could still run, and no rank may
    # signal again before every rank has reset
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_reset_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    first_quiesce = [got[r][0] for r in range(2)]
    assert all(e[0] == "quiesce" for e in first_quiesce)
    resets = [next(t for name, t in got[r] if name == "reset") for r in range(2)]
    resumes = [next(t for name, t in got[r] if name == "resume") for r in range(2)]
    assert max(e[1] for e in first_quiesce) <= min(resets)
    assert max(resets) <= min(resumes)
