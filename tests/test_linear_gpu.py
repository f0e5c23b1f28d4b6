"""K1 dense W4A16 linear vs the reference (golden), the oracle and the
full-size PyTorch restatement.  Tolerance (north star): max|err| <= 2 BF16 ulp
of max|ref| and relative Frobenius error <= 1e-3; fused vs safe: bit-exact."""

import numpy as np
import pytest
import torch

import _gpu_ref as gref
from _paths import bf16_to_f32, fp16_to_f32, golden, oracle, soft_module

pytestmark = pytest.mark.gpu
soft = soft_module()
O = oracle()


def _np(t):
    return t.float().cpu().numpy()


def _run(monkeypatch, backend, *args):
    monkeypatch.setenv("MXFP4_GFX936_BACKEND", backend)
    return soft.linear_mxfp4_soft(*args)


def _inputs(m, n, k, dtype=torch.bfloat16, seed=0, lo=118, hi=130):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(dtype)
    w = torch.randint(0, 256, (n, k // 2), generator=g, dtype=torch.uint8)
    s = torch.randint(lo, hi + 1, (n, k // 32), generator=g, dtype=torch.uint8)
    return x, w, s


@pytest.mark.parametrize("backend", ["safe", "fused"])
@pytest.mark.parametrize("case", range(6))
def test_matches_reference_golden(monkeypatch, backend, case):
    g = golden("linear")
    pre = f"c{case}_"
    dt = str(g[pre + "dtype"])
    tdt = torch.bfloat16 if dt == "bf16" else torch.float16
    x = torch.from_numpy(g[pre + "x"].view(np.int16)).view(tdt).cuda()
    bias = torch.from_numpy(g[pre + "bias"].view(np.int16)).view(tdt).cuda() if pre + "bias" in g.files else None
    y = _run(monkeypatch, backend, x, torch.from_numpy(g[pre + "w"]).cuda(), torch.from_numpy(g[pre + "s"]).cuda(), bias)
    ref = (bf16_to_f32 if dt == "bf16" else fp16_to_f32)(g[pre + "y"])
    ok, err, bound, rel = O.check_close(_np(y), ref)
    assert ok, (err, bound, rel)


SHAPES = [(1, 64, 128), (2, 99, 256), (1, 5120, 2048), (2, 96, 8192), (8, 64, 128), (16, 256, 2048), (16, 128, 24576), (64, 5120, 2048), (130, 384, 256),
          (40, 384, 16384),  # 32 stages per CTA: the few-token kernel's packed ring wraps
          (370, 512, 2048), (300, 1000, 512), (257, 2048, 4096),
          # four-CTA kernel (>= 4 row blocks of 256): odd row-block count, ragged N, K shorter than the ring
          (1100, 1000, 512), (1024, 640, 1024), (2048, 2048, 256)]


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_matches_oracle_and_safe_bit_exact(monkeypatch, m, n, k, dtype):
    x, w, s = _inputs(m, n, k, dtype, seed=m * 7 + n)
    xd, wd, sd = x.cuda(), w.cuda(), s.cuda()
    fused = _run(monkeypatch, "fused", xd, wd, sd)
    safe = _run(monkeypatch, "safe", xd, wd, sd)
    assert fused.dtype == dtype and tuple(fused.shape) == (m, n)
    assert torch.equal(fused.view(torch.int16), safe.view(torch.int16))
    ref = O.linear(_np(x), "bf16" if dtype == torch.bfloat16 else "fp16", w.numpy(), s.numpy())
    ok, err, bound, rel = O.check_close(_np(fused), ref)
    assert ok, (err, bound, rel)


@pytest.mark.parametrize("backend", ["safe", "fused"])
def test_bias_leading_dims_and_views(monkeypatch, backend):
    x, w, s = _inputs(2 * 3 * 5, 320, 512, seed=9)
    bias = torch.randn(320).to(torch.bfloat16)
    x3 = x.reshape(2, 3 * 5, 512)
    y = _run(monkeypatch, backend, x3.cuda(), w.cuda(), s.cuda(), bias.cuda())
    assert tuple(y.shape) == (2, 15, 320)
    ref = O.linear(_np(x), "bf16", w.numpy(), s.numpy(), _np(bias))
    ok, err, bound, rel = O.check_close(_np(y).reshape(30, 320), ref)
    assert ok, (err, bound, rel)
    # FP32 bias takes the reference's promotion (output + bias -> FP32)
    b32 = torch.randn(320)
    y32 = _run(monkeypatch, backend, x.cuda(), w.cuda(), s.cuda(), b32.cuda())
    assert y32.dtype == torch.float32
    # non-contiguous weight view
    wide = torch.cat([w, w], dim=1)
    y2 = _run(monkeypatch, backend, x.cuda(), wide[:, :256].cuda(), s.cuda())
    ref2 = O.linear(_np(x), "bf16", wide[:, :256].numpy(), s.numpy())
    ok, err, bound, rel = O.check_close(_np(y2), ref2)
    assert ok, (err, bound, rel)


def test_edge_scales_nan_inf_subnormal(monkeypatch):
    # scale codes 0 (2^-127), 1, 254 (overflow to inf), 255 (NaN) flow through
    x, w, s = _inputs(4, 256, 256, seed=1)
    s[0, :] = 255
    s[1, :] = 254
    s[2, :] = 0
    s[3, :] = 1
    y = _run(monkeypatch, "fused", x.cuda(), w.cuda(), s.cuda())
    ys = _run(monkeypatch, "safe", x.cuda(), w.cuda(), s.cuda())
    yn, ysn = _np(y), _np(ys)
    assert np.isnan(yn[:, 0]).all()
    assert np.array_equal(np.isnan(yn), np.isnan(ysn))
    ref = O.linear(_np(x), "bf16", w.numpy(), s.numpy())
    fin = np.isfinite(ref) & np.isfinite(yn)
    assert np.array_equal(np.isfinite(ref), np.isfinite(yn))
    ok, err, bound, rel = O.check_close(yn[:, 4:], ref[:, 4:])
    assert ok, (err, bound, rel)
    assert fin[:, 2:4].all()


@pytest.mark.parametrize("name,m,n,k", [("config1_qkv", 4096, 5120, 2048), ("config1_oproj", 4096, 2048, 4096),
                                        ("decode_qkv_m1", 1, 5120, 2048)])
def test_full_size_against_torch_reference(monkeypatch, name, m, n, k):
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    w = torch.randint(0, 256, (n, k // 2), generator=g, device="cuda", dtype=torch.uint8)
    s = torch.randint(118, 131, (n, k // 32), generator=g, device="cuda", dtype=torch.uint8)
    fused = _run(monkeypatch, "fused", x, w, s)
    safe = _run(monkeypatch, "safe", x, w, s)
    assert torch.equal(fused.view(torch.int16), safe.view(torch.int16))
    # the reference's safe path on this GPU: dequant to BF16, BF16 torch.matmul
    ref = gref.linear(x, w, s).float()
    err = (fused.float() - ref).abs()
    ulp = 2.0 ** (torch.floor(torch.log2(ref.abs().max())) - 7)
    assert err.max().item() <= 2 * ulp.item()
    assert (err.norm() / ref.norm()).item() <= 1e-3
    # and against the exact-product FP32 result: within the BF16 output rounding
    exact = gref.linear(x.float(), w, s)
    assert (fused.float() - exact).abs().max().item() <= 2 * ulp.item()
    assert soft.device_status() == 0


@pytest.mark.parametrize("backend", ["safe", "fused"])
def test_bias_many_row_blocks(monkeypatch, backend):
    x, w, s = _inputs(1100, 480, 1024, seed=21)
    bias = torch.randn(480).to(torch.bfloat16)
    y = _run(monkeypatch, backend, x.cuda(), w.cuda(), s.cuda(), bias.cuda())
    ref = O.linear(_np(x), "bf16", w.numpy(), s.numpy(), _np(bias))
    ok, err, bound, rel = O.check_close(_np(y), ref)
    assert ok, (err, bound, rel)


def test_fused_repeatable_full_size(monkeypatch):
    # the fused kernels exchange decoded weights between CTAs: repeated runs must agree bit for bit
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(4096, 2048, generator=g, device="cuda").to(torch.bfloat16)
    w = torch.randint(0, 256, (5120, 1024), generator=g, device="cuda", dtype=torch.uint8)
    s = torch.randint(118, 131, (5120, 64), generator=g, device="cuda", dtype=torch.uint8)
    first = _run(monkeypatch, "fused", x, w, s)
    for _ in range(3):
        assert torch.equal(_run(monkeypatch, "fused", x, w, s).view(torch.int16), first.view(torch.int16))
    assert soft.device_status() == 0


def test_fused_many_row_blocks_strided_weights(monkeypatch):
    # >= 4 row blocks with a weight view that is not contiguous: the fused mode
    # cannot use its decode-once copy and decodes inside the GEMM instead
    x, w, s = _inputs(1600, 384, 512, seed=33)
    wide = torch.cat([w, w], dim=1)
    y = _run(monkeypatch, "fused", x.cuda(), wide[:, :256].cuda(), s.cuda())
    ref = O.linear(_np(x), "bf16", w.numpy(), s.numpy())
    ok, err, bound, rel = O.check_close(_np(y), ref)
    assert ok, (err, bound, rel)
