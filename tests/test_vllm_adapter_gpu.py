"""The vLLM boundary on the GPU: adapter methods with the real operator module.

A compressed-tensors MXFP4 checkpoint written by compressed-tensors itself is
loaded with ``ct_checkpoint`` onto the GPU; the adapter's
``process_weights_after_loading`` / ``apply_weights`` / ``apply``
(vllm:68-70, 105-116, 215-265, restated in ``vllm_adapter``) run on
``SimpleNamespace`` layers exactly as vLLM calls them, with ``soft`` the
B200 operator module.  Results are checked against the oracle on the same
tensors and against the golden output of the reference adapter's own
``_moe_apply`` (``tests/golden/moe_layer.npz``); the two MoE forms must agree
bit for bit.
"""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from _paths import PKG, bf16_to_f32, golden, load_by_path, oracle, vllm_adapter

pytestmark = pytest.mark.gpu

va = vllm_adapter()
ct = load_by_path("mxfp4_ct_checkpoint", PKG / "ct_checkpoint.py")
O = oracle()
LAYER = "model.layers.0"


def _np(t):
    return t.float().cpu().numpy()


@pytest.fixture(scope="module")
def ckpt(ct_checkpoint_dir):
    return ct.MxFp4Checkpoint(ct_checkpoint_dir, device="cuda")


@pytest.mark.parametrize("backend", ["safe", "triton"])
def test_dense_layer_from_checkpoint(ckpt, monkeypatch, backend):
    monkeypatch.setenv("MXFP4_GFX936_BACKEND", backend)
    layer = ckpt.dense_layer(f"{LAYER}.self_attn.q_proj")
    va.dense_process_weights_after_loading(None, layer)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(3, 7, 256, generator=g).to(torch.bfloat16)
    bias = torch.randn(384, generator=g).to(torch.bfloat16)
    y = va.dense_apply_weights(None, layer, x.cuda(), bias.cuda())
    assert y.shape == (3, 7, 384) and y.dtype == torch.bfloat16
    w = layer.weight_packed.cpu().numpy()
    s = layer.weight_scale.cpu().numpy()
    ref = O.linear(_np(x).reshape(-1, 256), "bf16", w, s, _np(bias))
    ok, err, bound, rel = O.check_close(_np(y).reshape(-1, 384), ref)
    assert ok, (err, bound, rel)


def test_moe_layer_from_checkpoint_both_forms(ckpt, monkeypatch):
    layer = ckpt.moe_layer(f"{LAYER}.mlp.experts", 4)
    va.moe_process_weights_after_loading(None, layer)
    g = torch.Generator().manual_seed(5)
    t = 33
    x = torch.randn(t, 256, generator=g).to(torch.bfloat16)
    tw, tid = torch.topk(torch.softmax(torch.randn(t, 4, generator=g), -1), 2, dim=-1)
    tw = (tw / tw.sum(-1, keepdim=True)).float()
    tid = tid.to(torch.int32)
    monkeypatch.setattr(va, "MOE_FORM", "layer")
    y_layer = va.moe_apply(None, layer, x.cuda(), tw.cuda(), tid.cuda())
    monkeypatch.setattr(va, "MOE_FORM", "composition")
    y_comp = va.moe_apply(None, layer, x.cuda(), tw.cuda(), tid.cuda())
    assert torch.equal(y_layer.view(torch.int16), y_comp.view(torch.int16))
    ref = O.moe_layer(_np(x), *(getattr(layer, k).cpu().numpy() for k in
                                ("w13_weight", "w13_weight_scale", "w2_weight", "w2_weight_scale")),
                      tw.numpy(), tid.numpy())
    ok, err, bound, rel = O.check_close(_np(y_layer), ref)
    assert ok, (err, bound, rel)


@pytest.mark.parametrize("form", ["layer", "composition"])
def test_moe_apply_matches_reference_adapter_golden(monkeypatch, form):
    g = golden("moe_layer")
    layer = SimpleNamespace(activation="silu", w13_weight_packed=torch.from_numpy(g["w13"]).cuda(),
                            w13_weight_scale=torch.from_numpy(g["s13"]).cuda(),
                            w2_weight_packed=torch.from_numpy(g["w2"]).cuda(),
                            w2_weight_scale=torch.from_numpy(g["s2"]).cuda())
    va.moe_process_weights_after_loading(None, layer)
    monkeypatch.setattr(va, "MOE_FORM", form)
    x = torch.from_numpy(bf16_to_f32(g["x"])).to(torch.bfloat16).cuda()
    y = va.moe_apply(None, layer, x, torch.from_numpy(g["tw"]).cuda(), torch.from_numpy(g["tid"]).cuda())
    ok, err, bound, rel = O.check_close(_np(y), bf16_to_f32(g["y"]))
    assert ok, (err, bound, rel)
    assert np.isfinite(_np(y)).all()
