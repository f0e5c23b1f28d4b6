"""K4 routing (bit-exact), K3 routed op and the K3+K5 MoE layer vs the
reference (golden), the oracle and the full-size PyTorch restatement."""

import numpy as np
import pytest
import torch

import _gpu_ref as gref
from _paths import bf16_to_f32, golden, oracle, soft_module

pytestmark = pytest.mark.gpu
soft = soft_module()
O = oracle()


def _np(t):
    return t.float().cpu().numpy()


def _bf16(bits):
    return torch.from_numpy(np.asarray(bits).view(np.int16)).view(torch.bfloat16)


# --------------------------------------------------------------------------- routing
@pytest.mark.parametrize("case", range(5))
@pytest.mark.parametrize("ids_dtype", [torch.int32, torch.int64])
def test_routing_matches_reference_make_routing(case, ids_dtype):
    g = golden("routing")
    pre = f"r{case}_"
    ids = torch.from_numpy(g[pre + "ids"]).to(ids_dtype).cuda()
    bm, e = int(g[pre + "block_m"]), int(g[pre + "num_experts"])
    sid, eid, post = soft.moe_route(ids, e, bm)
    n = int(post.item())
    assert n == int(g[pre + "post"][0])
    np.testing.assert_array_equal(sid[:n].cpu().numpy(), g[pre + "sorted"])
    np.testing.assert_array_equal(eid[: n // bm].cpu().numpy(), g[pre + "experts"])
    assert (eid[n // bm:] == -1).all()


@pytest.mark.parametrize("t,k,e,bm,offset", [(1, 1, 4, 128, 0), (4096, 8, 128, 128, 0), (3000, 8, 16, 128, 32),
                                             (777, 4, 64, 64, 0), (5, 2, 1024, 16, 0)])
def test_routing_local_experts_and_out_of_range(t, k, e, bm, offset):
    g = torch.Generator().manual_seed(t + e)
    ids = torch.randint(-3, offset + e + 40, (t, k), generator=g, dtype=torch.int64)
    sid, eid, post = soft.moe_route(ids.cuda(), e, bm, offset)
    rs, re_, rp = O.route_blocks(ids.numpy(), e, bm, offset)
    n = int(post.item())
    assert n == int(rp[0])
    np.testing.assert_array_equal(sid[:n].cpu().numpy(), rs)
    np.testing.assert_array_equal(eid[: n // bm].cpu().numpy(), re_)


# --------------------------------------------------------------------------- routed op
def _keys():
    return [(m, q, w) for m in (1, 2, 4, 8, 64) for q in (0, 1) for w in (0, 1)]


@pytest.mark.parametrize("m,qa,mrw", _keys())
def test_moe_op_matches_reference_golden(m, qa, mrw):
    # the reference's 20-case operator matrix (test:216-285), same tolerance gate
    g = golden("moe_op")
    pre = f"m{m}_q{qa}_w{mrw}_"
    if qa:
        a = torch.from_numpy(g[pre + "a"]).cuda()
        amx = torch.from_numpy(g[pre + "a_mx"]).cuda()
    else:
        a, amx = _bf16(g[pre + "a"]).cuda(), None
    b = torch.from_numpy(g[pre + "b"]).cuda()
    e = b.shape[0]
    c = torch.full((m, 2, b.shape[1]), float("nan"), dtype=torch.bfloat16, device="cuda")
    empty = torch.empty(0, device="cuda")
    soft.fused_moe_mxfp4_soft(a, b, c, torch.tensor([0.75], device="cuda"), torch.linspace(0.5, 1.25, e, device="cuda"),
                              amx, torch.from_numpy(g[pre + "b_mx"]).cuda(), torch.from_numpy(g[pre + "tw"]).cuda(),
                              torch.from_numpy(g[pre + "tid"]).cuda(), empty, empty, empty, bool(mrw), 2, False, False)
    ok, err, bound, rel = O.check_close(_np(c), bf16_to_f32(g[pre + "c"]))
    assert ok, (err, bound, rel)
    # reference test tolerance as well (test:285)
    torch.testing.assert_close(c.float().cpu(), torch.from_numpy(bf16_to_f32(g[pre + "c"])), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("c_dtype,a_dtype", [(torch.bfloat16, torch.bfloat16), (torch.float16, torch.float16),
                                             (torch.float32, torch.bfloat16), (torch.bfloat16, torch.float32),
                                             (torch.float16, torch.bfloat16)])
@pytest.mark.parametrize("m,n,k,e,top_k", [(37, 320, 256, 6, 3), (300, 256, 512, 16, 4)])
def test_moe_op_dtypes_and_dropped_routes(c_dtype, a_dtype, m, n, k, e, top_k):
    g = torch.Generator().manual_seed(m + n)
    a = torch.randn(m, k, generator=g).to(a_dtype)
    b = torch.randint(0, 256, (e, n, k // 2), generator=g, dtype=torch.uint8)
    bmx = torch.randint(116, 130, (e, n, k // 32), generator=g, dtype=torch.uint8)
    ids = torch.randint(0, e + 2, (m, top_k), generator=g, dtype=torch.int32)  # ids >= e are dropped
    tw = torch.rand(m, top_k, generator=g)
    a_scale = torch.tensor([0.75])
    b_scale = torch.linspace(0.5, 1.25, e)
    c = torch.full((m, top_k, n), 7.0, dtype=c_dtype, device="cuda")
    soft.fused_moe_mxfp4_soft(a.cuda(), b.cuda(), c, a_scale.cuda(), b_scale.cuda(), None, bmx.cuda(), tw.cuda(),
                              ids.cuda(), torch.empty(0), torch.empty(0), torch.empty(0), True, top_k, False, False)
    cname = {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}[c_dtype]
    ref = O.moe_op(_np(a), "fp32", None, b.numpy(), bmx.numpy(), a_scale.numpy(), b_scale.numpy(), tw.numpy(),
                   ids.numpy(), True, cname)
    got = _np(c)
    assert (got[ids.numpy() >= e] == 0).all()
    ok, err, bound, rel = O.check_close(got, ref)
    assert ok, (err, bound, rel)


@pytest.mark.parametrize("a_dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("lo,hi", [(118, 131), (140, 151), (100, 112)])
def test_moe_op_fp32_output_at_fp32_precision(a_dtype, lo, hi):
    # C = F32 makes the matmul FP32 (soft:405, 466-494): F16 weights would
    # overflow from scale code 143 on and flush small scales, BF16-rounded F32
    # activations would lose 16 bits; the split-activation path keeps both exact
    m, n, k, e, top_k = 45, 192, 384, 5, 2
    g = torch.Generator().manual_seed(lo + m)
    a = (torch.randn(m, k, generator=g) * 3).to(a_dtype)
    b = torch.randint(0, 256, (e, n, k // 2), generator=g, dtype=torch.uint8)
    bmx = torch.randint(lo, hi, (e, n, k // 32), generator=g, dtype=torch.uint8)
    ids = torch.randint(0, e, (m, top_k), generator=g, dtype=torch.int64)
    tw = torch.rand(m, top_k, generator=g)
    a_scale, b_scale = torch.tensor([0.75]), torch.linspace(0.5, 1.25, e)
    c = torch.full((m, top_k, n), 7.0, dtype=torch.float32, device="cuda")
    soft.fused_moe_mxfp4_soft(a.cuda(), b.cuda(), c, a_scale.cuda(), b_scale.cuda(), None, bmx.cuda(), tw.cuda(),
                              ids.cuda(), torch.empty(0), torch.empty(0), torch.empty(0), True, top_k, False, False)
    ref = O.moe_op(_np(a), "fp32", None, b.numpy(), bmx.numpy(), a_scale.numpy(), b_scale.numpy(), tw.numpy(),
                   ids.numpy(), True, "fp32")
    got = _np(c)
    assert np.isfinite(got).all() and np.isfinite(ref).all()
    ok, err, bound, rel = O.check_close(got, ref)
    assert ok, (err, bound, rel)
    # FP32 products and FP32 sums: far inside the BF16-scale gate
    assert rel < 1e-5, rel


# --------------------------------------------------------------------------- MoE layer
def test_moe_layer_matches_reference_golden():
    g = golden("moe_layer")
    y = soft.moe_layer_mxfp4(_bf16(g["x"]).cuda(), *(torch.from_numpy(g[k]).cuda() for k in ("w13", "s13", "w2", "s2")),
                             torch.from_numpy(g["tw"]).cuda(), torch.from_numpy(g["tid"]).cuda())
    ok, err, bound, rel = O.check_close(_np(y), bf16_to_f32(g["y"]))
    assert ok, (err, bound, rel)


# 16 and 100 routes per expert: the block-scaled routed GEMM with 32- and
# 128-route tiles
@pytest.mark.parametrize("m,top_k,e", [(64, 4, 16), (200, 4, 8)])
def test_moe_op_block_scaled_wide_range_activations(m, top_k, e):
    # BF16 activations whose 32-value blocks sit anywhere from 2^-30 to 2^30 and
    # span up to 2^24 inside a block, with all-zero blocks, signed zeros and
    # all-zero tokens: the block-scaled GEMM writes every activation as two E4M3
    # parts under per-block scales, which must stay within the tolerance of the
    # oracle's exact products on every route's row, not just overall
    n, k = 256, 512
    g = torch.Generator().manual_seed(91)
    mant = torch.randn(m, k, generator=g)
    block_exp = torch.randint(-30, 31, (m, k // 32, 1), generator=g).float().expand(m, k // 32, 32).reshape(m, k)
    spread = torch.randint(-24, 1, (m, k), generator=g).float()
    a = (mant * torch.exp2(block_exp + spread)).to(torch.bfloat16)
    a[::5, :32] = 0.0
    a[1::7, 32:64] = -0.0
    a[3] = 0.0
    b = torch.randint(0, 256, (e, n, k // 2), generator=g, dtype=torch.uint8)
    bmx = torch.randint(116, 130, (e, n, k // 32), generator=g, dtype=torch.uint8)
    ids = torch.stack([torch.randperm(e, generator=g)[:top_k] for _ in range(m)]).to(torch.int32)
    tw = torch.rand(m, top_k, generator=g)
    a_scale = torch.tensor([1.0])
    b_scale = torch.ones(e)
    c = torch.empty((m, top_k, n), dtype=torch.bfloat16, device="cuda")
    soft.fused_moe_mxfp4_soft(a.cuda(), b.cuda(), c, a_scale.cuda(), b_scale.cuda(), None, bmx.cuda(), tw.cuda(),
                              ids.cuda(), torch.empty(0), torch.empty(0), torch.empty(0), True, top_k, False, False)
    ref = O.moe_op(_np(a), "fp32", None, b.numpy(), bmx.numpy(), a_scale.numpy(), b_scale.numpy(), tw.numpy(),
                   ids.numpy(), True, "bf16")
    got = _np(c)
    assert np.isfinite(got).all()
    assert (got[3] == 0).all()
    for t in range(m):
        for j in range(top_k):
            ok, err, bound, rel = O.check_close(got[t, j], ref[t, j])
            assert ok, (t, j, err, bound, rel)


# routes per call: 2 (routed GEMV), 800 and 4104 (routed tensor-memory GEMM), 4096 over 16 experts (256 per
# expert: the CTA-pair GEMM)
@pytest.mark.parametrize("t,h,e,k,inter", [(1, 256, 8, 2, 128), (200, 512, 16, 4, 256), (513, 256, 64, 8, 384),
                                           (1024, 256, 16, 4, 128)])
def test_moe_layer_matches_oracle(t, h, e, k, inter):
    g = torch.Generator().manual_seed(t * 3 + e)
    x = torch.randn(t, h, generator=g).to(torch.bfloat16)
    w13 = torch.randint(0, 256, (e, 2 * inter, h // 2), generator=g, dtype=torch.uint8)
    s13 = torch.randint(118, 131, (e, 2 * inter, h // 32), generator=g, dtype=torch.uint8)
    w2 = torch.randint(0, 256, (e, h, inter // 2), generator=g, dtype=torch.uint8)
    s2 = torch.randint(114, 127, (e, h, inter // 32), generator=g, dtype=torch.uint8)
    tw, tid = torch.topk(torch.softmax(torch.randn(t, e, generator=g), -1), k, dim=-1)
    tw = tw / tw.sum(-1, keepdim=True)
    y = soft.moe_layer_mxfp4(x.cuda(), w13.cuda(), s13.cuda(), w2.cuda(), s2.cuda(), tw.cuda(), tid.cuda())
    ref = O.moe_layer(_np(x), w13.numpy(), s13.numpy(), w2.numpy(), s2.numpy(), tw.numpy(), tid.numpy())
    ok, err, bound, rel = O.check_close(_np(y), ref)
    assert ok, (err, bound, rel)
    # the layer equals the two-op composition of the vLLM adapter (vllm:240-265)
    gate_up = torch.empty(t, k, 2 * inter, dtype=torch.bfloat16, device="cuda")
    one = torch.ones(1, device="cuda")
    ones = torch.ones(e, device="cuda")
    empty = torch.empty(0, device="cuda")
    soft.fused_moe_mxfp4_soft(x.cuda(), w13.cuda(), gate_up, one, ones, None, s13.cuda(), tw.cuda(), tid.cuda(),
                              empty, empty, empty, False, k, False, False)
    routed = (torch.nn.functional.silu(gate_up[..., :inter]) * gate_up[..., inter:]).reshape(t * k, inter)
    down = torch.empty(t * k, 1, h, dtype=torch.bfloat16, device="cuda")
    soft.fused_moe_mxfp4_soft(routed, w2.cuda(), down, one, ones, None, s2.cuda(), tw.reshape(-1, 1).cuda(),
                              tid.reshape(-1, 1).cuda(), empty, empty, empty, True, 1, False, False)
    two_op = down[:, 0].reshape(t, k, h).sum(dim=1)
    assert torch.equal(two_op.view(torch.int16), y.view(torch.int16))


def test_moe_layer_out_of_range_ids_contribute_zero():
    t, h, e, k, inter = 70, 256, 6, 3, 128
    g = torch.Generator().manual_seed(77)
    x = torch.randn(t, h, generator=g).to(torch.bfloat16)
    w13 = torch.randint(0, 256, (e, 2 * inter, h // 2), generator=g, dtype=torch.uint8)
    s13 = torch.randint(118, 131, (e, 2 * inter, h // 32), generator=g, dtype=torch.uint8)
    w2 = torch.randint(0, 256, (e, h, inter // 2), generator=g, dtype=torch.uint8)
    s2 = torch.randint(114, 127, (e, h, inter // 32), generator=g, dtype=torch.uint8)
    tw = torch.rand(t, k, generator=g)
    tid = torch.randint(0, e, (t, k), generator=g)
    tid[::3, 1] = e          # past the last expert: dropped
    tid[5, :] = e + 7        # a token with every route dropped
    y = soft.moe_layer_mxfp4(x.cuda(), w13.cuda(), s13.cuda(), w2.cuda(), s2.cuda(), tw.cuda(), tid.cuda())
    ref = O.moe_layer(_np(x), w13.numpy(), s13.numpy(), w2.numpy(), s2.numpy(), tw.numpy(), tid.numpy())
    ok, err, bound, rel = O.check_close(_np(y), ref)
    assert ok, (err, bound, rel)
    assert torch.count_nonzero(y[5]).item() == 0


def test_moe_layer_config2_full_size():
    # BASELINE config 2 (Qwen3-30B-A3B layer): T=4096, H=2048, E=128, k=8, I=768
    t, h, e, k, inter = 4096, 2048, 128, 8, 768
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(t, h, generator=g, device="cuda").to(torch.bfloat16)
    w13 = torch.randint(0, 256, (e, 2 * inter, h // 2), generator=g, device="cuda", dtype=torch.uint8)
    s13 = torch.randint(118, 131, (e, 2 * inter, h // 32), generator=g, device="cuda", dtype=torch.uint8)
    w2 = torch.randint(0, 256, (e, h, inter // 2), generator=g, device="cuda", dtype=torch.uint8)
    s2 = torch.randint(118, 131, (e, h, inter // 32), generator=g, device="cuda", dtype=torch.uint8)
    logits = torch.randn(t, e, generator=g, device="cuda")
    tw, tid = torch.topk(torch.softmax(logits, -1), k, dim=-1)
    tw = tw / tw.sum(-1, keepdim=True)
    y = soft.moe_layer_mxfp4(x, w13, s13, w2, s2, tw, tid)
    ref = gref.moe_layer(x, w13, s13, w2, s2, tw, tid)
    err = (y.float() - ref.float()).abs()
    ulp = 2.0 ** (torch.floor(torch.log2(ref.float().abs().max())) - 7)
    assert err.max().item() <= 2 * ulp.item()
    assert (err.norm() / ref.float().norm()).item() <= 1e-3
    assert soft.device_status() == 0
