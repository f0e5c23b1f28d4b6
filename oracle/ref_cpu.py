"""PyTorch-CPU port of the reference's safe path -- TEST/BENCH INFRASTRUCTURE.

Used only as the timed CPU baseline of ``bench.py`` (its ``cpu_baseline`` key
and the ``--impl reference`` arm) on the GPU box's host cores, where the
reference checkout itself is not available.  It performs the same torch
operations, in the same order, as the reference's ``safe`` backend:

* ``dequant``: soft:295-307 (nibble split, FP32 table lookup,
  ``exp2(code-127)`` with code 255 -> NaN, FP32 product, cast);
* ``linear``: soft:371-376 (dequant to x's dtype, ``torch.matmul(x, W^T)``,
  bias added after);
* ``moe_op``: soft:468-494 (per-expert ``nonzero``, gather, dequant,
  matmul, scale chain, route weight, scatter);
* ``moe_layer``: vllm:233-265 (gate_up op, SiLU*up, down op with route
  weights, top-k sum).

tests/test_oracle_golden.py checks it against the reference-generated fixtures.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

E2M1 = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0)


def dequant(packed: torch.Tensor, block_scales: torch.Tensor, dtype=torch.float32) -> torch.Tensor:
    codes = torch.stack((packed & 0x0F, packed >> 4), dim=-1).flatten(-2)
    table = torch.tensor(E2M1, device=packed.device, dtype=torch.float32)
    values = table[codes.long()]
    scale_codes = block_scales.repeat_interleave(32, dim=-1)
    scales = torch.exp2((scale_codes.to(torch.int16) - 127).to(torch.float32))
    scales = torch.where(scale_codes == 255, torch.full_like(scales, float("nan")), scales)
    return (values * scales).to(dtype)


def linear(x: torch.Tensor, packed: torch.Tensor, block_scales: torch.Tensor, bias=None) -> torch.Tensor:
    k = packed.shape[1] * 2
    x_2d = x.reshape(-1, k).contiguous()
    out = torch.matmul(x_2d, dequant(packed, block_scales, x.dtype).transpose(0, 1))
    if bias is not None:
        out = out + bias
    return out.reshape(*x.shape[:-1], packed.shape[0])


def moe_op(A, B, C, A_scale, B_scale, A_mx_scale, B_mx_scale, topk_weights, topk_ids, mul_routed_weight):
    dt = C.dtype
    acts = dequant(A, A_mx_scale, dt) if A.dtype == torch.uint8 else A.to(dt)
    C.zero_()
    g = A_scale.reshape(-1)[0].to(torch.float32)
    for e in range(B.shape[0]):
        pos = torch.nonzero(topk_ids == e, as_tuple=False)
        if pos.numel() == 0:
            continue
        t, j = pos[:, 0], pos[:, 1]
        out = torch.matmul(acts[t], dequant(B[e], B_mx_scale[e], dt).transpose(0, 1))
        out = out * g * B_scale[e].to(torch.float32)
        if mul_routed_weight:
            out = out * topk_weights[t, j, None]
        C[t, j] = out.to(dt)


def moe_layer(x, w13, s13, w2, s2, topk_weights, topk_ids):
    t, k = topk_ids.shape
    one = torch.ones(1)
    gate_up = torch.empty(t, k, w13.shape[1], dtype=x.dtype)
    moe_op(x, w13, gate_up, one, torch.ones(w13.shape[0]), None, s13, topk_weights, topk_ids, False)
    inter = gate_up.shape[-1] // 2
    routed = (F.silu(gate_up[..., :inter]) * gate_up[..., inter:]).reshape(t * k, inter)
    down = torch.empty(t * k, 1, w2.shape[1], dtype=x.dtype)
    moe_op(routed, w2, down, one, torch.ones(w2.shape[0]), None, s2, topk_weights.reshape(-1, 1),
           topk_ids.reshape(-1, 1), True)
    return down[:, 0].reshape(t, k, -1).sum(dim=1)
