"""Full-size GPU reference for parity properties (test infrastructure only).

A PyTorch restatement of the reference's safe path that runs on CUDA for the
BASELINE-sized checks the numpy oracle is too slow for: dequant with torch
elementwise ops (soft:295-307), ``torch.matmul`` in the compute dtype
(soft:371-373) and the per-expert safe MoE loop (soft:476-494) composed as the
vLLM layer (vllm:233-265).  The numpy oracle pins it on small shapes
(test_linear_gpu / test_moe_gpu compare both).
"""

import torch
import torch.nn.functional as F

E2M1 = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0)


def dequant(packed, scales, dtype):
    codes = torch.stack((packed & 0x0F, packed >> 4), dim=-1).flatten(-2)
    table = torch.tensor(E2M1, device=packed.device, dtype=torch.float32)
    values = table[codes.long()]
    sc = scales.repeat_interleave(32, dim=-1)
    mult = torch.exp2((sc.to(torch.int16) - 127).to(torch.float32))
    mult = torch.where(sc == 255, torch.full_like(mult, float("nan")), mult)
    return (values * mult).to(dtype)


def linear(x, packed, scales):
    return torch.matmul(x, dequant(packed, scales, x.dtype).t())


def moe_op(acts, packed, scales, topk_w, topk_ids, mul_routed_weight, out_dtype=torch.bfloat16):
    m, k = topk_ids.shape
    out = torch.zeros(m, k, packed.shape[1], dtype=out_dtype, device=acts.device)
    for e in range(packed.shape[0]):
        pos = torch.nonzero(topk_ids == e, as_tuple=False)
        if pos.numel() == 0:
            continue
        t, j = pos[:, 0], pos[:, 1]
        w = dequant(packed[e], scales[e], out_dtype)
        o = torch.matmul(acts[t].to(out_dtype), w.t())
        if mul_routed_weight:
            o = o * topk_w[t, j, None]
        out[t, j] = o.to(out_dtype)
    return out


def moe_layer(x, w13, s13, w2, s2, topk_w, topk_ids):
    gate_up = moe_op(x, w13, s13, topk_w, topk_ids, False)
    inter = gate_up.shape[-1] // 2
    routed = (F.silu(gate_up[..., :inter]) * gate_up[..., inter:]).reshape(-1, inter)
    down = moe_op(routed, w2, s2, topk_w.reshape(-1, 1), topk_ids.reshape(-1, 1), True)
    return down[:, 0].reshape(topk_ids.shape[0], topk_ids.shape[1], -1).sum(dim=1)
