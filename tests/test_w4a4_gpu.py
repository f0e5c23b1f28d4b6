"""W4A4 path: the OCP quantizer kernel (bit-exact vs the oracle) and the
block-scaled tcgen05 GEMM vs the reference semantics (dequant both operands,
one matmul; soft:468-475) within the north-star tolerance."""

import numpy as np
import pytest
import torch

import _gpu_ref as gref
from _paths import oracle, soft_module

pytestmark = pytest.mark.gpu
soft = soft_module()
O = oracle()


def _np(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_quantizer_bit_exact_vs_oracle(dtype):
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(64, 512, generator=g) * torch.logspace(-6, 6, 64).reshape(64, 1)).to(dtype)
    x[0, :32] = 0.0
    x[1, :32] = -0.0
    x[2, 5] = 1e-38
    x[3, :8] = torch.tensor([6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])  # ties to even at scale 127
    p, s = soft.quantize_mxfp4(x.cuda())
    rp, rs = O.quant_ocp_rne(x.float().numpy())
    np.testing.assert_array_equal(s.cpu().numpy(), rs)
    np.testing.assert_array_equal(p.cpu().numpy(), rp)


def _operands(m, n, k, seed, scale_mode="random"):
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(0, 256, (m, k // 2), generator=g, dtype=torch.uint8)
    b = torch.randint(0, 256, (n, k // 2), generator=g, dtype=torch.uint8)
    if scale_mode == "uniform":
        sa = torch.full((m, k // 32), 127, dtype=torch.uint8)
        sb = torch.full((n, k // 32), 127, dtype=torch.uint8)
    elif scale_mode == "rows":
        sa = (120 + torch.arange(m) % 13).to(torch.uint8)[:, None].repeat(1, k // 32)
        sb = (121 + torch.arange(n) % 11).to(torch.uint8)[:, None].repeat(1, k // 32)
    elif scale_mode == "kblocks":
        sa = (120 + torch.arange(k // 32) % 9).to(torch.uint8)[None, :].repeat(m, 1)
        sb = (124 + torch.arange(k // 32) % 7).to(torch.uint8)[None, :].repeat(n, 1)
    else:
        sa = torch.randint(118, 131, (m, k // 32), generator=g, dtype=torch.uint8)
        sb = torch.randint(118, 131, (n, k // 32), generator=g, dtype=torch.uint8)
    return a, sa, b, sb


@pytest.mark.parametrize("scale_mode", ["uniform", "rows", "kblocks", "random"])
@pytest.mark.parametrize("m,n,k", [(128, 256, 256), (200, 300, 384), (256, 512, 1024)])
def test_w4a4_matches_oracle(scale_mode, m, n, k):
    a, sa, b, sb = _operands(m, n, k, m + n + k, scale_mode)
    y = soft.gemm_mxfp4_w4a4(a.cuda(), sa.cuda(), b.cuda(), sb.cuda())
    ref = O.gemm_w4a4(a.numpy(), sa.numpy(), b.numpy(), sb.numpy(), "bf16")
    ok, err, bound, rel = O.check_close(_np(y), ref)
    assert ok, (scale_mode, err, bound, rel)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
def test_w4a4_output_dtypes(out_dtype):
    a, sa, b, sb = _operands(130, 264, 512, 3)
    y = soft.gemm_mxfp4_w4a4(a.cuda(), sa.cuda(), b.cuda(), sb.cuda(), out_dtype)
    assert y.dtype == out_dtype
    ref = O.gemm_w4a4(a.numpy(), sa.numpy(), b.numpy(), sb.numpy(), "fp32" if out_dtype == torch.float32 else "fp16")
    ok, err, bound, rel = O.check_close(_np(y), ref)
    assert ok, (err, bound, rel)


def test_w4a4_config3_full_size():
    # BF16 N(0,1) operands quantized with the OCP RNE quantizer
    g = torch.Generator(device="cuda").manual_seed(0)
    m, n, k = 8192, 4096, 4096
    xa = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    xb = torch.randn(n, k, generator=g, device="cuda").to(torch.bfloat16)
    a, sa = soft.quantize_mxfp4(xa)
    b, sb = soft.quantize_mxfp4(xb)
    y = soft.gemm_mxfp4_w4a4(a, sa, b, sb)
    # the reference path: dequant both to BF16, BF16 matmul
    ref = torch.matmul(gref.dequant(a, sa, torch.bfloat16), gref.dequant(b, sb, torch.bfloat16).t()).float()
    err = (y.float() - ref).abs()
    ulp = 2.0 ** (torch.floor(torch.log2(ref.abs().max())) - 7)
    assert err.max().item() <= 2 * ulp.item()
    assert (err.norm() / ref.norm()).item() <= 1e-3
    assert soft.device_status() == 0
