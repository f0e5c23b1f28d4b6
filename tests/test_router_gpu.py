"""Device router (softmax -> top-k -> renormalise, the routing vLLM hands the
adapter's _moe_apply at vllm:233) against torch's softmax + topk on the same
logits: ids identical, weights within 2e-6 relative (the FP32 softmax sums run
in a different order), and the routing feeds the MoE layer unchanged."""

import pytest
import torch

from _paths import soft_module

pytestmark = pytest.mark.gpu
soft = soft_module()


def _torch_route(logits, k, renorm):
    # torch's FP32 softmax, then the k largest with equal probabilities in
    # expert order (a stable sort; BF16/FP16 logits tie often)
    p = torch.softmax(logits.float(), dim=-1)
    ids = torch.argsort(-p, dim=-1, stable=True)[:, :k]
    w = torch.gather(p, 1, ids)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    return w, ids


@pytest.mark.parametrize("t,e,k", [(4096, 128, 8), (333, 64, 4), (7, 256, 32), (1, 1, 1), (100, 40, 6)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("renorm", [True, False])
def test_router_matches_torch(t, e, k, dtype, renorm):
    g = torch.Generator(device="cuda").manual_seed(t * 31 + e)
    logits = torch.randn(t, e, generator=g, device="cuda").to(dtype)
    w, ids = soft.moe_router(logits, k, renormalize=renorm)
    rw, rids = _torch_route(logits, k, renorm)
    assert w.dtype == torch.float32 and ids.dtype == torch.int32 and tuple(ids.shape) == (t, k)
    assert torch.equal(ids.long(), rids)
    torch.testing.assert_close(w, rw, rtol=2e-6, atol=1e-9)


def test_router_empty_and_errors():
    w, ids = soft.moe_router(torch.empty(0, 16, device="cuda"), 2)
    assert w.shape == (0, 2) and ids.shape == (0, 2)
    with pytest.raises(ValueError):
        soft.moe_router(torch.randn(4, 300, device="cuda"), 2)
    with pytest.raises(ValueError):
        soft.moe_router(torch.randn(4, 8, device="cuda"), 9)
    with pytest.raises(TypeError):
        soft.moe_router(torch.randn(4, 8, device="cuda").double(), 2)


def test_router_feeds_moe_layer():
    # config-2 shaped layer at reduced T: the device routing and torch's routing
    # give the same ids, so the layer's outputs agree to the weights' rounding
    t, h, e, k, inter = 256, 512, 32, 4, 128
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(t, h, generator=g, device="cuda").to(torch.bfloat16)
    w13 = torch.randint(0, 256, (e, 2 * inter, h // 2), generator=g, device="cuda", dtype=torch.uint8)
    s13 = torch.randint(118, 131, (e, 2 * inter, h // 32), generator=g, device="cuda", dtype=torch.uint8)
    w2 = torch.randint(0, 256, (e, h, inter // 2), generator=g, device="cuda", dtype=torch.uint8)
    s2 = torch.randint(118, 131, (e, h, inter // 32), generator=g, device="cuda", dtype=torch.uint8)
    logits = torch.randn(t, e, generator=g, device="cuda")
    tw, tid = soft.moe_router(logits, k)
    rw, rid = _torch_route(logits, k, True)
    y = soft.moe_layer_mxfp4(x, w13, s13, w2, s2, tw, tid)
    yr = soft.moe_layer_mxfp4(x, w13, s13, w2, s2, rw, rid)
    torch.testing.assert_close(y.float(), yr.float(), rtol=2e-2, atol=2e-2)
