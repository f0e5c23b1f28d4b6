#!/usr/bin/env python
"""Benchmark of the B200 MXFP4 backend (prints ONE JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Headline workload (the large-prefill dense linear):
qkv_proj M=4096, K=2048, N=5120 through the fused W4A16 backend.  With 16
row blocks of 256 it decodes each weight element once (the decode kernel
into an L2-resident BF16 copy, then the TMA-fed pair GEMM: two launches per
step); ``roofline`` is the GEMM launch's own, timed with CUDA events around
graph replays of that launch alone (``mxfp4_linear_dequantized`` on decoded
weight sets, the second launch of the step).  A "step" is one pass of the
linear over one batch.  ``value`` is the whole-job TFLOP/s (2*M*N*K per step) with the
inputs resident in HBM, timed with CUDA events on the launching stream over
exactly K steps (CUDA-graph replays rotating 4 input sets of 64 MB each, so
the working set of consecutive steps exceeds the 126 MB L2).  ``e2e`` times the
same metric through the public operator call with pinned HOST buffers (the
activation copy in, the output copy out, every step; consecutive steps are
pipelined over upload, compute and download streams).

At N=1 the other BASELINE configurations are measured as ``extra`` entries
(o_proj, the decode sweep, the safe mode, the MoE layer of config 2).  With
N>1 ranks (torchrun, one process per GPU) the headline is the column-sharded
linear: each rank owns N/G output columns and the GEMM epilogue stores every
tile into all ranks' outputs over NVLink (per-peer stores, or NVSwitch
multicast stores from 8 GPUs on), followed by a device barrier (strong
scaling, total work fixed); its ``roofline`` is the shard GEMM's and
``step_roofline`` is the slower of that GEMM at the bf16 peak and the
all-gather bytes at the measured NVLink rate.  The same linear with an NCCL
all-gather, and the expert-parallel MoE layer of config 2 (T/G tokens and E/G
experts per rank; native peer-memory dispatch and combine, and the NCCL
all-to-all path) are ``extra`` entries.

``cpu_baseline`` is the reference's safe path restated with PyTorch CPU ops
(oracle/ref_cpu.py) on the host cores for the headline workload;
``cpu_baselines`` adds configs 0 (M=64 linear), 2 (the MoE layer) and 3 (W4A4,
dequant both + matmul) on bounded samples.  The tensor-core denominators are
measured in the same run by libmxfp4_b200_probe.so (back-to-back BF16 and
block-scaled FP4 MMAs on every SM, ``peaks_probe``); the FP4 fraction of
config 3 is taken against that measured FP4 rate.  At N>1 every rank first
checks the sharded linear and the expert-parallel layer bit for bit against
the single-GPU calls on the same inputs (``parity``); a mismatch fails the run.

``--impl reference`` times the reference's safe path restated with PyTorch CPU
ops (oracle/ref_cpu.py) on this machine's host cores for the same workload; the
reference checkout itself does not exist on the GPU box.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "mxfp4-gfx936_b200"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
METRIC = "MXFP4 GEMM TFLOP/s & MoE-layer tokens/s at 1/2/4/8 B200; % of roofline"
QKV = (4096, 5120, 2048)        # M, N, K
OPROJ = (4096, 2048, 4096)
DECODE_M = (1, 8, 64, 370)
MOE = dict(t=4096, h=2048, e=128, k=8, inter=768)
W4A4 = (8192, 4096, 4096)       # M, N, K
FP4_NOMINAL_TFLOPS = 9000.0     # datasheet dense FP4; not measured on this pool


def _load(name, path):
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(key):
    p = ROOT / "profiles" / "traffic.json"
    if p.is_file():
        return json.loads(p.read_text()).get(key)
    return None


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """Polls SM clock and clock-event reasons through NVML while running."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting"}

    def __init__(self, device_index: int):
        self.samples, self.reasons, self.sm_max = [], set(), None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.h = self._handle_for(pynvml, device_index)
            self.nvml = pynvml
            self.sm_max = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # no NVML: report that, do not fail the bench
            self.nvml, self.error = None, str(exc)

    @staticmethod
    def _handle_for(pynvml, device_index):
        # match the CUDA device to its NVML handle by UUID (CUDA_VISIBLE_DEVICES
        # may renumber devices); fall back to the same index
        try:
            want = str(torch.cuda.get_device_properties(device_index).uuid).lower()
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                u = pynvml.nvmlDeviceGetUUID(h)
                u = (u.decode() if isinstance(u, bytes) else u).lower()
                if u.endswith(want):
                    return h
        except Exception:
            pass
        return pynvml.nvmlDeviceGetHandleByIndex(device_index)

    def _run(self):
        n = self.nvml
        get_r = getattr(n, "nvmlDeviceGetCurrentClocksEventReasons", None) or n.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.samples.append(n.nvmlDeviceGetClockInfo(self.h, n.NVML_CLOCK_SM))
                bits = get_r(self.h)
                for b, name in self.REASONS.items():
                    if bits & b:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def result(self):
        if self.nvml is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "error": self.error}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.sm_max,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ----------------------------------------------------------------------------- helpers
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def make_linear_inputs(m, n, k, seed, device):
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(m, k, generator=g, device=device).to(torch.bfloat16)
    w = torch.randint(0, 256, (n, k // 2), generator=g, device=device, dtype=torch.uint8)
    s = torch.randint(118, 131, (n, k // 32), generator=g, device=device, dtype=torch.uint8)
    return x, w, s


def graphs_for(fn, sets, stream):
    """CUDA graphs for the timed loop: one graph holding one step per input set
    (the whole rotation, replayed as a unit) plus one single-step graph per
    set for a step count that is not a multiple of the rotation."""
    for args in sets:
        fn(*args)  # warm the allocator and one-time attributes outside capture
    torch.cuda.synchronize()
    singles = []
    for args in sets:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            fn(*args)
        singles.append(g)
    rotation = torch.cuda.CUDAGraph()
    with torch.cuda.graph(rotation, stream=stream):
        for args in sets:
            fn(*args)
    torch.cuda.synchronize()
    return {"rotation": rotation, "singles": singles}


def _replay_steps(gs, steps):
    r = len(gs["singles"])
    for _ in range(steps // r):
        gs["rotation"].replay()
    for i in range(steps % r):
        gs["singles"][i].replay()


def time_graphs(gs, steps, warmup, barrier=None, sampler=None):
    """Replay the rotation; returns ms per step measured with CUDA events."""
    stream = torch.cuda.current_stream()
    _replay_steps(gs, warmup)
    torch.cuda.synchronize()
    if barrier:
        barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx = sampler if sampler is not None else _Null()
    with ctx:
        start.record(stream)
        _replay_steps(gs, steps)
        end.record(stream)
        end.synchronize()
    torch.cuda.synchronize()
    if barrier:
        barrier()
    return start.elapsed_time(end) / steps


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def set_backend(name):
    os.environ["MXFP4_GFX936_BACKEND"] = name


# ----------------------------------------------------------------------------- workloads
def bench_linear(soft, shape, steps, warmup, n_sets, backend, device, sampler=None, seed0=0):
    m, n, k = shape
    set_backend(backend)
    sets = [make_linear_inputs(m, n, k, seed0 + i, device) for i in range(n_sets)]
    gs = graphs_for(lambda x, w, s: soft.linear_mxfp4_soft(x, w, s), sets, torch.cuda.Stream())
    ms = time_graphs(gs, steps, warmup, sampler=sampler)
    del gs, sets
    return ms


def bench_decode_kernel(soft, shape, steps, warmup, device):
    """The weight decode kernel alone (the first of the two launches of a
    decode-once fused linear), same rotation of 4 weight sets."""
    m, n, k = shape
    sets = [make_linear_inputs(1, n, k, i, device)[1:] for i in range(4)]
    gs = graphs_for(lambda w, s: soft.dequant_mxfp4(w, s, torch.bfloat16), sets, torch.cuda.Stream())
    ms = time_graphs(gs, steps, warmup)
    del gs, sets
    return ms


def bench_gemm_predecoded(soft, shape, steps, warmup, device):
    """The GEMM launch of a decode-once step on its own: ``linear_dequantized``
    on weights decoded beforehand, 4 rotating sets (x 16 MB, decoded W 21 MB,
    y 42 MB each: the rotation exceeds the L2), CUDA events around replays."""
    m, n, k = shape
    sets = []
    for i in range(4):
        x, w, s = make_linear_inputs(m, n, k, i, device)
        sets.append((x, soft.dequant_mxfp4(w, s, torch.bfloat16)))
        del w, s
    gs = graphs_for(lambda x, wd: soft.linear_dequantized(x, wd), sets, torch.cuda.Stream())
    ms = time_graphs(gs, steps, warmup)
    del gs, sets
    return ms


def probe_peaks():
    """Dense tensor-core rates measured on this GPU by libmxfp4_b200_probe.so:
    MMAs issued back to back from shared-memory operands on every SM (BF16
    kind::f16 and block-scaled FP4 kind::mxf4, M=128 N=256); best of 3."""
    import ctypes
    lib = ctypes.CDLL(str(PKG / "libmxfp4_b200_probe.so"))
    fn = lib.mxfp4_probe_mma_rate
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_double),
                   ctypes.c_void_p]
    out = {}
    stream = torch.cuda.current_stream().cuda_stream
    for kind, name in ((0, "bf16_tflops"), (1, "fp4_tflops")):
        best = 0.0
        for _ in range(4):
            ms, fl = ctypes.c_float(), ctypes.c_double()
            rc = fn(kind, 20000, ctypes.byref(ms), ctypes.byref(fl), ctypes.c_void_p(stream))
            if rc:
                raise RuntimeError(f"tensor-core rate probe failed with status {rc}")
            best = max(best, fl.value / (ms.value * 1e-3) / 1e12)
        out[name] = best
    out["what"] = ("tcgen05 MMAs back to back, operands in shared memory, one CTA per SM, M=128 N=256 "
                   "(kind::f16 BF16 K=16; kind::mxf4.block_scale.block32 K=64), best of 4 x 80000 MMAs per SM")
    return out


DECODE_ONCE_ROW_BLOCKS = 4  # mirrors kDecodeOnceRowBlocks in csrc/capi.cu


def bench_e2e_linear(soft, shape, steps, warmup, device):
    """The public call with host buffers: every step copies its activations in
    from pinned host memory, runs ``linear_mxfp4_soft`` and copies the whole
    result back.  Steps are pipelined over three streams (upload, compute,
    download) the way a serving loop overlaps requests, so step i's download
    runs beside step i+1's upload over the full-duplex host link; events order
    every reuse of the two device input buffers and of the result."""
    m, n, k = shape
    set_backend("fused")
    x, w, s = make_linear_inputs(m, n, k, 123, device)
    x_host = x.cpu().pin_memory()
    y_host = torch.empty(m, n, dtype=torch.bfloat16).pin_memory()
    xd = [torch.empty_like(x), torch.empty_like(x)]
    s_in, s_comp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event(), torch.cuda.Event()]
    ev_used = [torch.cuda.Event(), torch.cuda.Event()]  # the GEMM that read xd[b] is done
    del x

    def step(i):
        b = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_used[b])
            xd[b].copy_(x_host, non_blocking=True)
            ev_in[b].record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(ev_in[b])
            y = soft.linear_mxfp4_soft(xd[b], w, s)
            ev_used[b].record(s_comp)
            done = torch.cuda.Event()
            done.record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(done)
            y_host.copy_(y, non_blocking=True)
            y.record_stream(s_out)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(s_in)
    for i in range(steps):
        step(i)
    s_in.wait_stream(s_out)
    end.record(s_in)
    end.synchronize()
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) * 1e3 / steps
    ms = start.elapsed_time(end) / steps
    return max(ms, wall), x_host.numel() * 2, y_host.numel() * 2


def make_moe_inputs(device, seed=0, **cfg):
    t, h, e, k, inter = cfg["t"], cfg["h"], cfg["e"], cfg["k"], cfg["inter"]
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(t, h, generator=g, device=device).to(torch.bfloat16)
    w13 = torch.randint(0, 256, (e, 2 * inter, h // 2), generator=g, device=device, dtype=torch.uint8)
    s13 = torch.randint(118, 131, (e, 2 * inter, h // 32), generator=g, device=device, dtype=torch.uint8)
    w2 = torch.randint(0, 256, (e, h, inter // 2), generator=g, device=device, dtype=torch.uint8)
    s2 = torch.randint(118, 131, (e, h, inter // 32), generator=g, device=device, dtype=torch.uint8)
    logits = torch.randn(t, e, generator=g, device=device)
    tw, tid = torch.topk(torch.softmax(logits, -1), k, dim=-1)
    tw = tw / tw.sum(-1, keepdim=True)
    return x, w13, s13, w2, s2, tw, tid


def bench_moe(soft, steps, warmup, device, tokens=None):
    cfg = dict(MOE, t=tokens) if tokens else MOE
    sets = [make_moe_inputs(device, seed=i, **cfg) for i in range(2)]
    gs = graphs_for(lambda *a: soft.moe_layer_mxfp4(*a), sets, torch.cuda.Stream())
    ms = time_graphs(gs, steps, warmup)
    del gs, sets
    return ms


def moe_weight_bytes(tid, cfg=MOE):
    """HBM bytes a layer call must read: the packed weights and scales of every
    expert its routes touch (w13 and w2), plus x in and the output."""
    h, inter = cfg["h"], cfg["inter"]
    per_expert = 2 * inter * (h // 2 + h // 32) + h * (inter // 2 + inter // 32)
    experts = int(torch.unique(tid).numel())
    return experts * per_expert + 2 * 2 * tid.shape[0] * h


def moe_kernel_name(routes, experts):
    """The grouped GEMM the MoE layer (BF16) runs at this route count."""
    if routes <= 24:
        return "routed GEMV"
    if routes < 128 * experts:
        return "block-scaled routed GEMM (E2M1 x E4M3 hi/lo, " + ("32" if routes < 48 * experts else "128") + "-route tiles)"
    return "pair GEMM (256-route blocks)"


def bench_moe_decode(soft, device, tokens_list=(1, 8, 64, 256), steps=50, warmup=5):
    """The config-2 layer shape at decode batch sizes (config 4's decode MoE):
    CUDA-graph replays over two input sets with their own weights (426 MB, more
    than L2), so every call reads its experts' weights from HBM."""
    hbm = peaks()[0]["hbm_gbs"]
    out = {}
    for t in tokens_list:
        cfg = dict(MOE, t=t)
        byts = sum(moe_weight_bytes(make_moe_inputs(device, seed=i, **cfg)[6], cfg) for i in range(2)) / 2
        ms = bench_moe(soft, steps, warmup, device, tokens=t)
        out[f"t{t}"] = {"us": ms * 1e3, "tokens_per_s": t / (ms * 1e-3), "hbm_bytes": byts,
                        "gbs": byts / ms / 1e6, "frac_hbm": byts / ms / 1e6 / hbm,
                        "kernel": moe_kernel_name(t * MOE["k"], MOE["e"])}
    return out


def bench_e2e_moe(soft, steps, warmup, device):
    """The MoE layer through its public call with host buffers: each step copies
    x [T, H] BF16 and the routing (top-k weights F32, ids I64) in from pinned
    host memory, runs ``moe_layer_mxfp4`` and copies the whole [T, H] result
    back; steps pipelined over upload, compute and download streams as in the
    linear's e2e."""
    x, w13, s13, w2, s2, tw, tid = make_moe_inputs(device, seed=31, **MOE)
    hosts = [t.cpu().pin_memory() for t in (x, tw, tid)]
    out_host = torch.empty(MOE["t"], MOE["h"], dtype=torch.bfloat16).pin_memory()
    dev_in = [[torch.empty_like(t) for t in (x, tw, tid)] for _ in range(2)]
    del x, tw, tid
    s_in, s_comp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event(), torch.cuda.Event()]
    ev_used = [torch.cuda.Event(), torch.cuda.Event()]

    def step(i):
        b = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_used[b])
            for d, h in zip(dev_in[b], hosts):
                d.copy_(h, non_blocking=True)
            ev_in[b].record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(ev_in[b])
            xd, twd, tidd = dev_in[b]
            y = soft.moe_layer_mxfp4(xd, w13, s13, w2, s2, twd, tidd)
            ev_used[b].record(s_comp)
            done = torch.cuda.Event()
            done.record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(done)
            out_host.copy_(y, non_blocking=True)
            y.record_stream(s_out)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(s_in)
    for i in range(steps):
        step(i)
    s_in.wait_stream(s_out)
    end.record(s_in)
    end.synchronize()
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) * 1e3 / steps
    ms = max(start.elapsed_time(end) / steps, wall)
    h2d = sum(h.numel() * h.element_size() for h in hosts)
    return ms, h2d, out_host.numel() * 2


def bench_router(soft, steps, warmup, device):
    """Device router on config 2's logits (T=4096 x E=128 FP32, top-8, renormalised);
    64 rotating logit sets (128 MB) so consecutive steps miss the L2."""
    g = torch.Generator(device=device).manual_seed(5)
    sets = [(torch.randn(MOE["t"], MOE["e"], generator=g, device=device),) for _ in range(64)]
    gs = graphs_for(lambda lg: soft.moe_router(lg, MOE["k"]), sets, torch.cuda.Stream())
    ms = time_graphs(gs, steps, warmup)
    del gs, sets
    return ms


def bench_w4a4(soft, steps, warmup, device):
    m, n, k = W4A4
    sets = []
    for i in range(2):
        g = torch.Generator(device=device).manual_seed(50 + i)
        xa = torch.randn(m, k, generator=g, device=device).to(torch.bfloat16)
        xb = torch.randn(n, k, generator=g, device=device).to(torch.bfloat16)
        a, sa = soft.quantize_mxfp4(xa)
        b, sb = soft.quantize_mxfp4(xb)
        sets.append((a, sa, b, sb))
        del xa, xb
    gs = graphs_for(lambda *t: soft.gemm_mxfp4_w4a4(*t), sets, torch.cuda.Stream())
    ms = time_graphs(gs, steps, warmup)
    del gs, sets
    return ms


STACK_PREFILL = (8, 2048)        # sequences x tokens
STACK_DECODE_BATCHES = (1, 8, 64, 256)
STACK_DECODE_CTX = 2048          # decode continues 2048-token sequences


def bench_stack_decode(device, steps, warmup, batch, layers):
    """One config-4 decode step (batch tokens, 2048-token context) of a
    ``layers``-layer stack as a replayed CUDA graph (profiling aid)."""
    dsm = _load("mxfp4_decoder_stack", PKG / "decoder_stack.py")
    cfg = dsm.StackConfig(layers=layers)
    full = [dsm.random_layer(cfg, device, seed=1000 + i) for i in range(cfg.layers)]
    stack = dsm.DecoderStack(cfg, full, max_ctx=STACK_DECODE_CTX + 8, max_tokens=max(batch, 1))
    del full
    stack.allocate_cache(batch, STACK_DECODE_CTX + 1)
    hb = torch.randn(batch, cfg.hidden, generator=torch.Generator(device=device).manual_seed(5),
                     device=device).to(torch.bfloat16)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            stack.decode(hb, STACK_DECODE_CTX)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        stack.decode(hb, STACK_DECODE_CTX)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(steps):
        graph.replay()
    en.record()
    en.synchronize()
    return st.elapsed_time(en) / steps


def bench_stack(device, steps, warmup, rank=0, world=1, group=None, barrier=None, layers=48):
    """the Qwen3-30B-A3B-shaped 48-layer stack (random-init
    MXFP4 weights for every linear).  Prefill of 8 x 2048 tokens (eager, CUDA
    events) and decode steps of one token per sequence at batch 1..256 over a
    2048-token KV cache (one CUDA graph per step, replayed); tokens/s of the
    whole job, max over ranks.  On several GPUs: dense linears column-sharded,
    experts expert-parallel, attention sharded by sequence."""
    dsm = _load("mxfp4_decoder_stack", PKG / "decoder_stack.py")
    cfg = dsm.StackConfig(layers=layers)
    full = [dsm.random_layer(cfg, device, seed=1000 + i) for i in range(cfg.layers)]
    stack = dsm.DecoderStack(cfg, full, rank=rank, world=world, group=group,
                             max_ctx=max(STACK_PREFILL[1], STACK_DECODE_CTX) + 8,
                             max_tokens=STACK_PREFILL[0] * STACK_PREFILL[1])
    del full
    torch.cuda.empty_cache()
    sync = barrier if barrier is not None else (lambda: None)
    out = {}
    seqs, seq_len = STACK_PREFILL
    g = torch.Generator(device=device).manual_seed(77)
    h = torch.randn(seqs * seq_len, cfg.hidden, generator=g, device=device).to(torch.bfloat16)
    stack.allocate_cache(seqs, seq_len)
    for _ in range(warmup):
        stack.prefill(h, seqs)
    torch.cuda.synchronize()
    sync()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(steps):
        stack.prefill(h, seqs)
    en.record()
    en.synchronize()
    ms = st.elapsed_time(en) / steps
    if world > 1:
        ms = _max_over_ranks(ms, device)
    tokens = seqs * seq_len
    fl = cfg.layers * cfg.layer_flops(tokens, dsm.attention_ctx_per_token(seq_len, 0))
    out["prefill"] = {"tokens": tokens, "ms": ms, "tokens_per_s": tokens / (ms * 1e-3),
                      "tflops": fl / (ms * 1e-3) / 1e12, "what": f"{seqs} x {seq_len} tokens, {cfg.layers} layers"}
    del h
    for b in STACK_DECODE_BATCHES:
        stack.allocate_cache(b, STACK_DECODE_CTX + 1)
        hb = torch.randn(b, cfg.hidden, generator=g, device=device).to(torch.bfloat16)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                stack.decode(hb, STACK_DECODE_CTX)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            stack.decode(hb, STACK_DECODE_CTX)
        for _ in range(warmup):
            graph.replay()
        torch.cuda.synchronize()
        sync()
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record()
        for _ in range(steps):
            graph.replay()
        en.record()
        en.synchronize()
        ms = st.elapsed_time(en) / steps
        if world > 1:
            ms = _max_over_ranks(ms, device)
        out[f"decode_b{b}"] = {"ms": ms, "tokens_per_s": b / (ms * 1e-3), "context": STACK_DECODE_CTX}
        del graph, hb
        torch.cuda.synchronize()
        sync()
    stack.cache = None
    del stack
    torch.cuda.empty_cache()
    out["config"] = {"layers": cfg.layers, "hidden": cfg.hidden, "heads": cfg.heads, "kv_heads": cfg.kv_heads,
                     "head_dim": cfg.head_dim, "experts": cfg.experts, "top_k": cfg.top_k, "inter": cfg.inter,
                     "attention": "torch SDPA", "parallelism": "single GPU" if world == 1 else
                     f"tp{world} dense (fused all-gather) + ep{world} experts + sequence-sharded attention"}
    return out


def moe_flops(cfg=MOE):
    return 2.0 * cfg["t"] * cfg["k"] * (cfg["h"] * 2 * cfg["inter"] + cfg["inter"] * cfg["h"])


def linear_bytes(m, n, k):
    return 2 * m * k + n * k // 2 + n * k // 32 + 2 * m * n


# ----------------------------------------------------------------------------- CPU side
def cpu_linear_tflops(shape, steps, warmup, budget_s=25.0):
    """The reference's safe linear restated with torch CPU ops, all host threads."""
    ref = _load("mxfp4_ref_cpu", ROOT / "oracle" / "ref_cpu.py")
    torch.set_num_threads(os.cpu_count() or 1)
    m, n, k = shape
    g = torch.Generator().manual_seed(0)
    w = torch.randint(0, 256, (n, k // 2), generator=g, dtype=torch.uint8)
    s = torch.randint(118, 131, (n, k // 32), generator=g, dtype=torch.uint8)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    t0 = time.perf_counter()
    ref.linear(x, w, s)
    one = time.perf_counter() - t0
    m_used = m
    if one * (steps + warmup) > budget_s:  # bounded sample: fewer rows, same weights
        m_used = max(64, int(m * budget_s / (one * (steps + warmup))) // 64 * 64)
        x = x[:m_used].contiguous()
    for _ in range(warmup):
        ref.linear(x, w, s)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        ref.linear(x, w, s)
        times.append(time.perf_counter() - t0)
    best = min(times)
    mean = sum(times) / len(times)
    flops = 2.0 * m_used * n * k
    return {"tflops_best": flops / best / 1e12, "tflops_mean": flops / mean / 1e12, "ms_mean": mean * 1e3,
            "m_used": m_used, "threads": torch.get_num_threads()}


def _time_cpu(fn, budget_s, min_steps=2, max_steps=10):
    fn()  # warm-up
    times = []
    t_all = time.perf_counter()
    while len(times) < max_steps and (len(times) < min_steps or time.perf_counter() - t_all < budget_s):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    return sum(times) / len(times), len(times)


def cpu_baselines(budget_s=8.0):
    """The reference's safe path (torch-CPU port, all host threads) on
    BASELINE configs 0, 2 and 3, each on a bounded sample of its workload."""
    ref = _load("mxfp4_ref_cpu", ROOT / "oracle" / "ref_cpu.py")
    torch.set_num_threads(os.cpu_count() or 1)
    threads = torch.get_num_threads()
    out = {}
    # config 0: the dense safe linear at M=64 (its full size)
    m, n, k = 64, 5120, 2048
    g = torch.Generator().manual_seed(0)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = torch.randint(0, 256, (n, k // 2), generator=g, dtype=torch.uint8)
    s = torch.randint(118, 131, (n, k // 32), generator=g, dtype=torch.uint8)
    sec, steps = _time_cpu(lambda: ref.linear(x, w, s), budget_s)
    out["config0_linear_m64"] = {"value": 2.0 * m * n * k / sec / 1e12, "unit": "TFLOP/s", "ms": sec * 1e3,
                                 "cores": threads, "kind": "port", "sample": f"full config 0 ({m}x{n}x{k}), "
                                 f"{steps} timed calls"}
    # config 2: the MoE layer on a token sample (all 128 experts' weights)
    t = 512
    cfg = dict(MOE, t=t)
    x, w13, s13, w2, s2, tw, tid = make_moe_inputs(torch.device("cpu"), seed=0, **cfg)
    sec, steps = _time_cpu(lambda: ref.moe_layer(x, w13, s13, w2, s2, tw, tid), budget_s, max_steps=4)
    out["config2_moe_layer"] = {"value": t / sec, "unit": "tokens/s", "ms": sec * 1e3, "cores": threads,
                                "kind": "port", "tflops": moe_flops(cfg) / sec / 1e12,
                                "sample": f"{t} of config 2's {MOE['t']} tokens, same experts and routing "
                                          f"distribution, {steps} timed calls"}
    del x, w13, s13, w2, s2, tw, tid
    # config 3: W4A4 as the reference computes it (dequant both operands, BF16 matmul), on a row sample
    m, n, k = 1024, W4A4[1], W4A4[2]
    g = torch.Generator().manual_seed(3)
    a = torch.randint(0, 256, (m, k // 2), generator=g, dtype=torch.uint8)
    sa = torch.randint(118, 131, (m, k // 32), generator=g, dtype=torch.uint8)
    b = torch.randint(0, 256, (n, k // 2), generator=g, dtype=torch.uint8)
    sb = torch.randint(118, 131, (n, k // 32), generator=g, dtype=torch.uint8)

    def w4a4():
        return torch.matmul(ref.dequant(a, sa, torch.bfloat16), ref.dequant(b, sb, torch.bfloat16).T)

    sec, steps = _time_cpu(w4a4, budget_s, max_steps=4)
    out["config3_w4a4"] = {"value": 2.0 * m * n * k / sec / 1e12, "unit": "TFLOP/s", "ms": sec * 1e3,
                           "cores": threads, "kind": "port",
                           "sample": f"{m} of config 3's {W4A4[0]} rows ({m}x{n}x{k}), {steps} timed calls"}
    return out


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    r = cpu_linear_tflops(QKV, args.steps, args.warmup, budget_s=150.0)
    m, n, k = QKV
    sample = f"qkv_proj {r['m_used']}x{n}x{k} (rows sampled from M={m})" if r["m_used"] != m else f"qkv_proj {m}x{n}x{k}"
    line = {
        "impl": "reference", "metric": METRIC, "value": r["tflops_mean"], "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_mean"], "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config1_qkv_prefill", "M": m, "N": n, "K": k},
        "cpu_baseline": {"value": r["tflops_mean"], "unit": "TFLOP/s", "cores": r["threads"], "kind": "port",
                         "sample": sample + "; reference safe path (dequant + torch.matmul) as torch CPU ops"},
        "e2e": {"value": r["tflops_mean"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-extra", action="store_true", help="skip the non-headline configurations")
    ap.add_argument("--decode-m", type=int, default=1, help="rows of x for --workload decode (qkv weights)")
    ap.add_argument("--moe-tokens", type=int, default=None, help="tokens for --workload moe (default: config 2's 4096)")
    ap.add_argument("--stack-layers", type=int, default=48, help="layers for --workload stack-decode")
    ap.add_argument("--workload", default=None, choices=["qkv", "oproj", "safe", "decode", "moe", "w4a4", "stack-decode"],
                    help="run only this configuration (for profiling); prints its timing as JSON")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    soft = _load("moe_op_mxfp4_soft", PKG / "moe_op_mxfp4_soft.py")
    pk, pk_kind = peaks()
    m, n, k = QKV

    if world > 1:
        return run_sharded(args, soft, world, rank, device, pk, pk_kind)
    if args.workload is not None:
        return run_one(args, soft, device)

    sampler = ClockSampler(local)
    ms = bench_linear(soft, QKV, args.steps, args.warmup, 4, "fused", device, sampler=sampler)
    flops = 2.0 * m * n * k
    tflops = flops / (ms * 1e-3) / 1e12
    # decode-once (>= 4 row blocks): two launches per step, the decode kernel then the GEMM;
    # each launch is timed on its own with CUDA events around graph replays of it alone
    decode_once = (m + 255) // 256 >= DECODE_ONCE_ROW_BLOCKS
    dec_ms = bench_decode_kernel(soft, QKV, args.steps, args.warmup, device) if decode_once else 0.0
    gemm_ms = bench_gemm_predecoded(soft, QKV, args.steps, args.warmup, device) if decode_once else ms
    gemm_tflops = flops / (gemm_ms * 1e-3) / 1e12
    probe = probe_peaks()
    e2e_ms, h2d, d2h = bench_e2e_linear(soft, QKV, max(10, args.steps // 4), args.warmup, device)

    line = {
        "metric": METRIC, "value": tflops, "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (BASELINE config-1 distributions, seeded)",
        "config": {"workload": "config1_qkv_prefill", "M": m, "N": n, "K": k, "backend": "fused",
                   "l2": "4 rotating input sets of 64 MB (working set > 126 MB L2)", "timing": "CUDA graph of the 4-set rotation replayed, CUDA events",
                   "parallelism": "single GPU"},
        "roofline": {"bound": "tensor", "achieved": gemm_tflops, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": gemm_tflops / pk["bf16_tflops"], "traffic": profile_traffic("linear_fused_qkv"),
                     "peak_source": f"{pk_kind} bf16 burst",
                     "kernel": "pair GEMM (TMA-fed decoded weights)" if decode_once else "pair GEMM (decode in producer)",
                     "kernel_ms": gemm_ms, "kernel_timing": "the GEMM launch alone: CUDA events around graph "
                     "replays of mxfp4_linear_dequantized over 4 rotating decoded-weight sets",
                     "frac_of_probe": gemm_tflops / probe["bf16_tflops"],
                     "decode_kernel_ms": dec_ms,
                     "decode_kernel_gbs": (n * k // 2 + n * k // 32 + 2 * n * k) / (dec_ms * 1e6) if dec_ms else None,
                     "step_frac": tflops / pk["bf16_tflops"]},
        "e2e": {"value": flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": args.steps * (2 if decode_once else 1),
        "clocks": sampler.result(),
        "peaks_probe": probe,
    }

    if not args.no_extra:
        extra = {}
        ms_o = bench_linear(soft, OPROJ, 100, 10, 4, "fused", device, seed0=10)
        fo = 2.0 * OPROJ[0] * OPROJ[1] * OPROJ[2]
        extra["config1_oproj_fused"] = {"ms": ms_o, "tflops": fo / ms_o / 1e9, "frac_bf16": fo / ms_o / 1e9 / pk["bf16_tflops"]}
        ms_s = bench_linear(soft, QKV, 100, 10, 4, "safe", device, seed0=20)
        extra["config1_qkv_safe"] = {"ms": ms_s, "tflops": flops / ms_s / 1e9}
        for dm in DECODE_M:
            shape = (dm, n, k)
            ms_d = bench_linear(soft, shape, 400, 20, 32, "fused", device, seed0=100 + dm)
            byts = linear_bytes(dm, n, k)
            extra[f"decode_qkv_m{dm}"] = {"ms": ms_d, "us": ms_d * 1e3, "gbs": byts / ms_d / 1e6,
                                          "frac_hbm": byts / ms_d / 1e6 / pk["hbm_gbs"],
                                          "tflops": 2.0 * dm * n * k / ms_d / 1e9}
        ms_m = bench_moe(soft, 20, 3, device)
        fm = moe_flops()
        e2e_m, h2d_m, d2h_m = bench_e2e_moe(soft, 10, 3, device)
        extra["config2_moe_layer"] = {"ms": ms_m, "tokens_per_s": MOE["t"] / (ms_m * 1e-3), "tflops": fm / ms_m / 1e9,
                                      "frac_bf16": fm / ms_m / 1e9 / pk["bf16_tflops"], "launches_per_step": 6,
                                      "e2e": {"value": MOE["t"] / (e2e_m * 1e-3), "unit": "tokens/s", "ms": e2e_m,
                                              "h2d_bytes_per_step": h2d_m, "d2h_bytes_per_step": d2h_m}}
        ms_r = bench_router(soft, 256, 64, device)
        rbytes = MOE["t"] * MOE["e"] * 4 + MOE["t"] * MOE["k"] * 8
        extra["config2_router"] = {"ms": ms_r, "us": ms_r * 1e3, "gbs": rbytes / ms_r / 1e6,
                                   "what": "softmax + top-8 + renormalise over 128 expert logits, 4096 tokens"}
        extra["config4_moe_decode"] = bench_moe_decode(soft, device)
        extra["config4_stack"] = bench_stack(device, 3, 1)
        ms_w = bench_w4a4(soft, 50, 5, device)
        fw = 2.0 * W4A4[0] * W4A4[1] * W4A4[2]
        extra["config3_w4a4"] = {"ms": ms_w, "tflops": fw / ms_w / 1e9,
                                 "frac_fp4_measured": fw / ms_w / 1e9 / probe["fp4_tflops"],
                                 "fp4_peak_measured": probe["fp4_tflops"],
                                 "frac_fp4_nominal": fw / ms_w / 1e9 / FP4_NOMINAL_TFLOPS,
                                 "vs_bf16_peak": fw / ms_w / 1e9 / pk["bf16_tflops"],
                                 "launches_per_step": 3}
        line["extra"] = extra

    cb = cpu_linear_tflops(QKV, 2, 1, budget_s=25.0)
    line["cpu_baseline"] = {"value": cb["tflops_mean"], "unit": "TFLOP/s", "cores": cb["threads"], "kind": "port",
                            "sample": f"qkv_proj {cb['m_used']}x{n}x{k}, 2 timed steps; reference safe path "
                                      "(dequant + torch.matmul) as torch CPU ops (oracle/ref_cpu.py)"}
    if not args.no_extra:
        line["cpu_baselines"] = cpu_baselines()
    status = soft.device_status()
    if status:
        line["device_status"] = status
    print(json.dumps(line), flush=True)
    return 0


def run_one(args, soft, device):
    """One configuration on its own (profiling aid; not the driver's line)."""
    w = args.workload
    if w == "qkv":
        ms = bench_linear(soft, QKV, args.steps, args.warmup, 4, "fused", device)
    elif w == "oproj":
        ms = bench_linear(soft, OPROJ, args.steps, args.warmup, 4, "fused", device, seed0=10)
    elif w == "safe":
        ms = bench_linear(soft, QKV, args.steps, args.warmup, 4, "safe", device, seed0=20)
    elif w == "decode":
        ms = bench_linear(soft, (args.decode_m, QKV[1], QKV[2]), args.steps, args.warmup, 32, "fused", device,
                          seed0=101)
    elif w == "moe":
        ms = bench_moe(soft, args.steps, args.warmup, device, tokens=args.moe_tokens)
    elif w == "stack-decode":
        ms = bench_stack_decode(device, args.steps, args.warmup, args.decode_m, args.stack_layers)
    else:
        ms = bench_w4a4(soft, args.steps, args.warmup, device)
    print(json.dumps({"workload": w, "ms_per_step": ms, "steps": args.steps}), flush=True)
    return 0


NVLINK_GBS = 770.0   # measured peer copy per direction per GPU on this pool (nominal 900)


def _max_over_ranks(v, device):
    import torch.distributed as dist
    t = torch.tensor([v], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def bench_ep_moe(soft, ep_mod, world, rank, device, steps, warmup, barrier, fused=True):
    """Expert-parallel config-2 layer: T tokens in total, T/G per rank, E/G experts per rank.

    The native layer (no host synchronisation inside a call) is timed like the
    single-GPU layer: CUDA-graph replays rotating input sets, each with its own
    weights, enough of them that one rotation's expert weights exceed the L2.
    The NCCL path syncs the host on the route counts, so it is timed eagerly."""
    t_local = MOE["t"] // world
    sl = slice(rank * t_local, (rank + 1) * t_local)
    w_bytes_rank = MOE["e"] // world * 3 * MOE["inter"] * MOE["h"] * (0.5 + 1 / 32)
    n_sets = max(2, -(-int(160e6) // int(w_bytes_rank))) if fused else 1
    sets = []
    for i in range(n_sets):
        x, w13, s13, w2, s2, tw, tid = make_moe_inputs(device, seed=7 + i, **MOE)
        layer = ep_mod.ExpertParallelMoE.from_full(w13, s13, w2, s2, rank, world, fused=fused)
        sets.append((x[sl].contiguous(), tw[sl].contiguous(), tid[sl].contiguous(), layer))
        del w13, s13, w2, s2, x, tw, tid
    # parity before timing: this rank's rows of the expert-parallel layer must
    # equal, bit for bit, the single-GPU layer on the full input (set 0)
    x, w13, s13, w2, s2, tw, tid = make_moe_inputs(device, seed=7, **MOE)
    y_full = soft.moe_layer_mxfp4(x, w13, s13, w2, s2, tw, tid)[sl]
    xs, tws, tids, layer = sets[0]
    y_ep = layer(xs, tws, tids)
    torch.cuda.synchronize()
    parity_ok = bool(torch.equal(y_ep.view(torch.int16), y_full.view(torch.int16)))
    del x, w13, s13, w2, s2, tw, tid, y_full, y_ep
    barrier()
    ms = None
    timing = "eager"
    if fused:
        try:
            gs = graphs_for(lambda xs, tws, tids, layer: layer(xs, tws, tids), sets, torch.cuda.Stream())
            ms = _max_over_ranks(time_graphs(gs, steps, warmup, barrier=barrier), device)
            timing = "graph"
            del gs
        except RuntimeError:  # every rank takes the same path: capture fails alike everywhere
            torch.cuda.synchronize()
            barrier()
    if ms is None:
        xs, tws, tids, layer = sets[0]
        for _ in range(warmup):
            layer(xs, tws, tids)
        torch.cuda.synchronize()
        barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            layer(xs, tws, tids)
        end.record()
        end.synchronize()
        barrier()
        ms = _max_over_ranks(start.elapsed_time(end) / steps, device)
    torch.cuda.synchronize()
    barrier()
    routes_local = t_local * MOE["k"]
    # bytes a rank must receive over NVLink per step: dispatched rows from the
    # other ranks plus their combined rows coming back (uniform routing)
    nv_bytes = 2 * routes_local * (world - 1) / world * MOE["h"] * 2
    return ms, nv_bytes, moe_flops(), timing, parity_ok


def run_sharded(args, soft, world, rank, device, pk, pk_kind):
    """N>1: the column-sharded dense linear (headline) and the expert-parallel
    MoE layer (extra), one process per GPU over NCCL."""
    import datetime

    import torch.distributed as dist

    dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    cp = _load("mxfp4_column_parallel", PKG / "column_parallel.py")
    ep_mod = _load("mxfp4_expert_parallel", PKG / "expert_parallel.py")
    m, n, k = QKV
    set_backend("fused")
    barrier = lambda: dist.barrier(device_ids=[device.index])  # noqa: E731
    sets, shard_sets, nccl_sets = [], [], []
    for i in range(4):
        x, w, s = make_linear_inputs(m, n, k, i, device)  # same full weight on every rank
        layer = cp.ColumnParallelLinear.from_full(w, s, rank, world, fused=True)
        sets.append((x, layer))
        shard_sets.append((x, layer.w, layer.s))
        nccl_sets.append((x, cp.ColumnParallelLinear(layer.w, layer.s, n, rank, world)))
        del w, s
    # parity before timing: the fused sharded linear and the NCCL path against
    # the single-GPU linear on the full weight (set 0), bit for bit, on every rank
    xw, ww, sw = make_linear_inputs(m, n, k, 0, device)
    y_1 = soft.linear_mxfp4_soft(xw, ww, sw)
    y_tp = sets[0][1](xw)
    tp_ok = bool(torch.equal(y_tp.view(torch.int16), y_1.view(torch.int16)))
    y_nccl = nccl_sets[0][1](xw)
    tp_nccl_ok = bool(torch.equal(y_nccl.view(torch.int16), y_1.view(torch.int16)))
    torch.cuda.synchronize()
    del xw, ww, sw, y_1, y_tp, y_nccl
    barrier()
    # the shard GEMM alone (the dominant kernel), then GEMM + all-gather
    gs_local = graphs_for(lambda x, w, s: soft.linear_mxfp4_soft(x, w, s), shard_sets, torch.cuda.Stream())
    ms_gemm = _max_over_ranks(time_graphs(gs_local, args.steps, args.warmup, barrier=barrier), device)
    del gs_local
    gs = graphs_for(lambda x, layer: layer(x), nccl_sets, torch.cuda.Stream())
    ms_nccl = _max_over_ranks(time_graphs(gs, args.steps, args.warmup, barrier=barrier), device)
    del gs, nccl_sets
    gs = graphs_for(lambda x, layer: layer(x), sets, torch.cuda.Stream())
    ag_path = ("NVSwitch multicast stores" if getattr(sets[0][1]._bufs[0], "multicast_ptr", 0)
               else "peer stores over NVLink")
    sampler = ClockSampler(device.index)
    ms = _max_over_ranks(time_graphs(gs, args.steps, args.warmup, barrier=barrier, sampler=sampler), device)
    del gs
    flops = 2.0 * m * n * k
    tflops = flops / (ms * 1e-3) / 1e12
    shard_flops = flops / world
    gemm_tflops = shard_flops / (ms_gemm * 1e-3) / 1e12
    # step roofline: the slower of the shard GEMM at the bf16 peak and the
    # all-gather bytes each GPU must receive at the measured NVLink rate
    ag_bytes = 2.0 * m * n * (world - 1) / world
    t_tensor = shard_flops / (pk["bf16_tflops"] * 1e12)
    t_nvlink = ag_bytes / (NVLINK_GBS * 1e9)
    t_roof = max(t_tensor, t_nvlink)

    # end to end: pinned host activations in on every rank, the gathered output
    # (identical on every rank) read back once, by rank 0.  Steps are pipelined
    # over upload, compute and download streams.  The layer's output buffers
    # alternate and peers write into them, so rank 0's compute of step i+1 waits
    # for its download of step i: the device barrier that ends step i+1 then
    # holds every rank's step i+2 (which writes that buffer again) until the
    # download is done.
    x_host = sets[0][0].cpu().pin_memory()
    y_host = torch.empty(m, n, dtype=torch.bfloat16).pin_memory()
    layer0 = sets[0][1]
    xd = [torch.empty_like(sets[0][0]), torch.empty_like(sets[0][0])]
    s_in, s_comp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event(), torch.cuda.Event()]
    ev_used = [torch.cuda.Event(), torch.cuda.Event()]
    last_d2h = [None]

    def e2e_step(i):
        b = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_used[b])
            xd[b].copy_(x_host, non_blocking=True)
            ev_in[b].record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(ev_in[b])
            if last_d2h[0] is not None:
                s_comp.wait_event(last_d2h[0])
            y = layer0(xd[b])
            ev_used[b].record(s_comp)
            done = torch.cuda.Event()
            done.record(s_comp)
        if rank == 0:
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                y_host.copy_(y, non_blocking=True)
                d2h = torch.cuda.Event()
                d2h.record(s_out)
                last_d2h[0] = d2h

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier()
    e_steps = max(10, args.steps // 4)
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    st.record(s_in)
    for i in range(e_steps):
        e2e_step(i)
    s_in.wait_stream(s_comp)
    s_in.wait_stream(s_out)
    en.record(s_in)
    en.synchronize()
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) * 1e3 / e_steps
    e2e_ms = _max_over_ranks(max(st.elapsed_time(en) / e_steps, wall), device)
    barrier()
    del sets, shard_sets

    # expert-parallel MoE layer (config 2, tokens data-parallel across ranks)
    ep_steps = max(5, min(20, args.steps // 10))
    ms_ep, ep_nv_bytes, fm, ep_timing, ep_ok = bench_ep_moe(soft, ep_mod, world, rank, device, ep_steps,
                                                            args.warmup, barrier)
    ms_ep_nccl, _, _, _, ep_nccl_ok = bench_ep_moe(soft, ep_mod, world, rank, device, ep_steps, args.warmup, barrier,
                                                   fused=False)
    # parity of every rank: the minimum over ranks of each check
    flags = torch.tensor([tp_ok, tp_nccl_ok, ep_ok, ep_nccl_ok], dtype=torch.int32, device=device)
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    parity = {"tp": bool(flags[0]), "tp_nccl": bool(flags[1]), "ep": bool(flags[2]), "ep_nccl": bool(flags[3]),
              "what": "each rank's output vs the single-GPU call on the same inputs, bit for bit, min over ranks"}
    t_ep_roof = max(fm / world / (pk["bf16_tflops"] * 1e12), ep_nv_bytes / (NVLINK_GBS * 1e9))
    stack = bench_stack(device, 3, 1, rank=rank, world=world, barrier=barrier)
    status = soft.device_status()
    status = int(_max_over_ranks(float(status), device))

    if rank == 0:
        line = {
            "metric": METRIC, "value": tflops, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (BASELINE config-1 distributions, seeded)",
            "config": {"workload": "config1_qkv_prefill", "M": m, "N": n, "K": k, "backend": "fused",
                       "parallelism": f"tp{world}: column-sharded W (N/{world} rows per GPU), all-gather fused "
                                      f"into the GEMM epilogue ({ag_path}) + device barrier",
                       "l2": "4 rotating input sets of 64 MB (working set > 126 MB L2)",
                       "timing": "CUDA graph of the 4-set rotation replayed, CUDA events, max over ranks"},
            "roofline": {"bound": "tensor", "achieved": gemm_tflops, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": gemm_tflops / pk["bf16_tflops"], "traffic": None,
                         "kernel": f"shard GEMM {m}x{n // world}x{k}",
                         "peak_source": f"{pk_kind} bf16 burst"},
            "step_roofline": {"bound": "nvlink" if t_nvlink > t_tensor else "tensor",
                              "target_ms": t_roof * 1e3, "frac": t_roof * 1e3 / ms,
                              "allgather_bytes_in_per_gpu": ag_bytes, "nvlink_gbs": NVLINK_GBS,
                              "shard_gemm_ms": ms_gemm},
            "e2e": {"value": flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": x_host.numel() * 2, "d2h_bytes_per_step": y_host.numel() * 2},
            "gpu_launches": args.steps * 3,
            "clocks": sampler.result(),
            "parity": parity,
            "extra": {"tp_nccl_allgather": {"ms": ms_nccl, "tflops": flops / (ms_nccl * 1e-3) / 1e12,
                                            "what": "shard GEMM then NCCL all_gather_into_tensor + interleave"},
                      "config2_moe_layer_ep": {
                "ms": ms_ep, "tokens_per_s": MOE["t"] / (ms_ep * 1e-3), "tflops": fm / ms_ep / 1e9,
                "experts_per_gpu": MOE["e"] // world, "tokens_per_gpu": MOE["t"] // world,
                "roofline_target_ms": t_ep_roof * 1e3, "roofline_frac": t_ep_roof * 1e3 / ms_ep,
                "nvlink_bytes_in_per_gpu": ep_nv_bytes,
                "dispatch_combine": "native: peer-mapped routed buffers over NVLink, device barriers",
                "timing": ("CUDA graph of rotating input sets (expert weights > L2) replayed, CUDA events, "
                           "max over ranks") if ep_timing == "graph" else "CUDA events around eager calls, max over ranks"},
                "config2_moe_layer_ep_nccl": {"ms": ms_ep_nccl, "tokens_per_s": MOE["t"] / (ms_ep_nccl * 1e-3),
                                              "what": "NCCL all-to-all dispatch/combine (host syncs on counts)"},
                "config4_stack": stack},
        }
        if status:
            line["device_status"] = status
        print(json.dumps(line), flush=True)
    barrier()
    dist.destroy_process_group()
    if not all(parity[key] for key in ("tp", "tp_nccl", "ep", "ep_nccl")):
        if rank == 0:
            print("parity check failed: a multi-GPU result differs from the single-GPU call", file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
