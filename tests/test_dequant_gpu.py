"""K0 dequant kernel vs the reference (golden fixtures) and the oracle: bit-exact."""

import numpy as np
import pytest
import torch

from _paths import bf16_to_f32, bits_to_f32, fp16_to_f32, golden, oracle, same_bits, soft_module

pytestmark = pytest.mark.gpu
soft = soft_module()
O = oracle()
DT = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}


def _np(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("name", ["fp32", "bf16", "fp16"])
def test_all_codes_all_scales_bit_exact_vs_reference(name):
    g = golden("dequant")
    out = soft.dequant_mxfp4(torch.from_numpy(g["packed"]).cuda(), torch.from_numpy(g["scales"]).cuda(), DT[name])
    exp = {"fp32": bits_to_f32, "bf16": bf16_to_f32, "fp16": fp16_to_f32}[name](g[f"out_{name}"])
    assert same_bits(_np(out), exp)


def test_known_answer_all_e2m1_codes():
    # test:81-92
    packed = torch.tensor([[c | ((c + 1) << 4) for c in range(0, 16, 2)] * 2], device="cuda", dtype=torch.uint8)
    scales = torch.full((1, 1), 127, device="cuda", dtype=torch.uint8)
    actual = soft.dequant_mxfp4(packed, scales)
    expected = torch.tensor([soft._MXFP4_E2M1_VALUES], device="cuda", dtype=torch.float32).repeat(1, 2)
    torch.testing.assert_close(actual, expected, rtol=0, atol=0)
    assert same_bits(_np(actual), np.tile(O.E2M1_VALUES, 2)[None])


@pytest.mark.parametrize("name", ["fp32", "bf16", "fp16"])
def test_random_tensor_bit_exact_vs_oracle(name):
    g = torch.Generator().manual_seed(3)
    packed = torch.randint(0, 256, (3, 257, 512), generator=g, dtype=torch.uint8)
    scales = torch.randint(0, 256, (3, 257, 32), generator=g, dtype=torch.uint8)
    out = soft.dequant_mxfp4(packed.cuda(), scales.cuda(), DT[name])
    assert tuple(out.shape) == (3, 257, 1024) and out.dtype == DT[name]
    assert same_bits(_np(out), O.dequant(packed.numpy(), scales.numpy(), name))


def test_empty_and_unaligned_views():
    empty = soft.dequant_mxfp4(torch.zeros(0, 16, dtype=torch.uint8, device="cuda"),
                               torch.zeros(0, 1, dtype=torch.uint8, device="cuda"))
    assert tuple(empty.shape) == (0, 32)
    base = torch.randint(0, 256, (4, 33), dtype=torch.uint8)
    packed = base[:, 1:]  # storage offset 1: not 16-byte aligned
    scales = torch.randint(110, 140, (4, 2), dtype=torch.uint8)
    out = soft.dequant_mxfp4(packed.cuda(), scales.cuda(), torch.bfloat16)
    assert same_bits(_np(out), O.dequant(packed.numpy(), scales.numpy(), "bf16"))
