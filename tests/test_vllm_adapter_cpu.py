"""The vLLM compressed-tensors boundary, checked against the reference adapter on CPU.

The reference adapter (integration/vllm/vllm_mxfp4_gfx936.py) needs vLLM
0.15 to import, so its method bodies are compiled from the source with
``ast`` (as ``tests/golden/make_golden.py`` does) and run here on a
``SimpleNamespace`` layer next to this package's ``vllm_adapter``.  Both get
the same recording operator module (CPU restatement of the safe path from
``_gpu_ref``) as ``soft``: the calls each side makes into the operator module
(arguments and routing metadata) and the results must be identical.  The
reference source is only read when the reference checkout is present
(``MXFP4_REFERENCE_ROOT``); the GPU test runs the adapter with the real
operator module.
"""

import ast
import os
import subprocess
import sys
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch
import torch.nn.functional as F
from torch.nn.parameter import Parameter

import _gpu_ref as gref
from _paths import PKG, ROOT, load_by_path, vllm_adapter

REF = Path(os.getenv("MXFP4_REFERENCE_ROOT", "/root/reference"))
ADAPTER = REF / "integration" / "vllm" / "vllm_mxfp4_gfx936.py"
needs_ref = pytest.mark.skipif(not ADAPTER.is_file(), reason="reference checkout not present")

va = vllm_adapter()


class RecordingSoft:
    """Operator module stand-in: records every call, computes on CPU."""

    def __init__(self, make_routing=None):
        self.calls = []
        self._make_routing = make_routing

    def linear_mxfp4_soft(self, x, packed, scales, bias=None):
        self.calls.append(("linear", x.clone(), packed, scales, bias))
        y = gref.linear(x.reshape(-1, x.shape[-1]), packed, scales)
        if bias is not None:
            y = y + bias
        return y.reshape(*x.shape[:-1], packed.shape[0])

    def fused_moe_mxfp4_soft(self, A, B, C, A_scale, B_scale, A_mx_scale, B_mx_scale, topk_weights, topk_ids,
                             sorted_token_ids, expert_ids, num_tokens_post_padded, mul_routed_weight, top_k,
                             compute_type_a, compute_type_b):
        post = int(num_tokens_post_padded[0])
        block_m = sorted_token_ids.numel() // expert_ids.numel()
        self.calls.append(("moe_op", A.clone(), B, tuple(C.shape), C.dtype, A_scale.clone(), B_scale.clone(),
                           A_mx_scale, B_mx_scale, topk_weights.clone(), topk_ids.clone(),
                           sorted_token_ids[:post].clone(), expert_ids[:post // block_m].clone(), post,
                           mul_routed_weight, top_k, compute_type_a, compute_type_b))
        C.copy_(gref.moe_op(A, B, B_mx_scale, topk_weights, topk_ids, mul_routed_weight, out_dtype=C.dtype))

    def moe_route(self, topk_ids, num_experts, block_m=128, expert_offset=0):
        assert expert_offset == 0 and num_experts > int(topk_ids.max())
        # the device routing's metadata prefix is the reference's _make_routing
        return self._make_routing(topk_ids, block_m=block_m)

    def moe_layer_mxfp4(self, x, w13, w13_scale, w2, w2_scale, topk_weights, topk_ids):
        self.calls.append(("moe_layer", x.clone(), w13, w13_scale, w2, w2_scale, topk_weights, topk_ids))
        return gref.moe_layer(x, w13, w13_scale, w2, w2_scale, topk_weights, topk_ids)


def _compile_reference(soft, implementation="safe"):
    from compressed_tensors.compressors.nvfp4.helpers import unpack_fp4_from_uint8

    tree = ast.parse(ADAPTER.read_text())
    wanted = {"_dense_process_weights_after_loading", "_dense_apply_weights", "_moe_process_weights_after_loading",
              "_moe_apply", "_moe_gemm", "_make_routing", "_bf16_linear", "_bf16_moe_gemm", "_reference_dequant"}
    body = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in wanted]
    assert {n.name for n in body} == wanted
    ns = {"torch": torch, "F": F, "Parameter": Parameter, "soft": soft, "_IMPLEMENTATION": implementation,
          "_official_unpack_fp4": unpack_fp4_from_uint8}
    exec(compile(ast.Module(body=body, type_ignores=[]), str(ADAPTER), "exec"), ns)
    return SimpleNamespace(**{k: ns[k] for k in wanted})


def _same(a, b):
    if isinstance(a, torch.Tensor):
        return isinstance(b, torch.Tensor) and a.dtype == b.dtype and a.shape == b.shape and torch.equal(a, b)
    if isinstance(a, (tuple, list)):
        return len(a) == len(b) and all(_same(x, y) for x, y in zip(a, b))
    return a == b


def _weights(e, h, inter, seed):
    g = torch.Generator().manual_seed(seed)
    return SimpleNamespace(
        activation="silu",
        w13_weight_packed=torch.randint(0, 256, (e, 2 * inter, h // 2), generator=g, dtype=torch.uint8),
        w13_weight_scale=torch.randint(118, 131, (e, 2 * inter, h // 32), generator=g, dtype=torch.uint8),
        w2_weight_packed=torch.randint(0, 256, (e, h, inter // 2), generator=g, dtype=torch.uint8),
        w2_weight_scale=torch.randint(114, 127, (e, h, inter // 32), generator=g, dtype=torch.uint8))


def _routes(t, e, k, seed):
    g = torch.Generator().manual_seed(seed)
    tw, tid = torch.topk(torch.softmax(torch.randn(t, e, generator=g), -1), k, dim=-1)
    return (tw / tw.sum(-1, keepdim=True)).float(), tid.to(torch.int32)


@pytest.fixture
def sides(monkeypatch):
    ref_soft = RecordingSoft()
    ref = _compile_reference(ref_soft)
    ref_soft._make_routing = ref._make_routing
    own_soft = RecordingSoft(make_routing=ref._make_routing)
    monkeypatch.setattr(va, "soft", own_soft)
    return ref, ref_soft, own_soft


@needs_ref
@pytest.mark.parametrize("bias", [False, True])
def test_dense_apply_weights_matches_reference(sides, bias):
    ref, ref_soft, own_soft = sides
    g = torch.Generator().manual_seed(7)
    layer = SimpleNamespace(weight_packed=torch.randint(0, 256, (96, 128), generator=g, dtype=torch.uint8),
                            weight_scale=torch.randint(118, 131, (96, 8), generator=g, dtype=torch.uint8))
    x = torch.randn(2, 5, 256, generator=g).to(torch.bfloat16)
    b = torch.randn(96, generator=g).to(torch.bfloat16) if bias else None
    ref_layer, own_layer = SimpleNamespace(**vars(layer)), SimpleNamespace(**vars(layer))
    ref._dense_process_weights_after_loading(None, ref_layer)
    va.dense_process_weights_after_loading(None, own_layer)
    for name in ("weight_packed", "weight_scale"):
        r, o = getattr(ref_layer, name), getattr(own_layer, name)
        assert isinstance(o, Parameter) and not o.requires_grad and torch.equal(r, o)
    y_ref = ref._dense_apply_weights(None, ref_layer, x, b)
    y_own = va.dense_apply_weights(None, own_layer, x, b)
    assert _same(y_ref, y_own) and y_own.shape == (2, 5, 96)
    assert _same(ref_soft.calls, own_soft.calls) and len(own_soft.calls) == 1


@needs_ref
def test_moe_process_weights_matches_reference(sides):
    ref, _, _ = sides
    w = _weights(4, 256, 128, 3)
    ref_layer, own_layer = SimpleNamespace(**vars(w)), SimpleNamespace(**vars(w))
    ref._moe_process_weights_after_loading(None, ref_layer)
    va.moe_process_weights_after_loading(None, own_layer)
    assert sorted(vars(ref_layer)) == sorted(vars(own_layer))
    assert not hasattr(own_layer, "w13_weight_packed") and not hasattr(own_layer, "w2_weight_packed")
    for name in ("w13_weight", "w13_weight_scale", "w2_weight", "w2_weight_scale"):
        assert isinstance(getattr(own_layer, name), Parameter)
        assert torch.equal(getattr(ref_layer, name), getattr(own_layer, name))


@needs_ref
@pytest.mark.parametrize("form", ["composition", "layer"])
@pytest.mark.parametrize("t,e,k", [(1, 4, 2), (37, 8, 2), (130, 8, 4)])
def test_moe_apply_matches_reference(sides, monkeypatch, form, t, e, k):
    ref, ref_soft, own_soft = sides
    monkeypatch.setattr(va, "MOE_FORM", form)
    h, inter = 256, 128
    w = _weights(e, h, inter, t + e)
    layer = SimpleNamespace(**vars(w))
    va.moe_process_weights_after_loading(None, layer)
    x = torch.randn(t, h, generator=torch.Generator().manual_seed(t)).to(torch.bfloat16)
    tw, tid = _routes(t, e, k, t * 5 + e)
    y_ref = ref._moe_apply(None, layer, x, tw, tid)
    y_own = va.moe_apply(None, layer, x, tw, tid)
    assert _same(y_ref, y_own)
    if form == "composition":
        # same two operator calls with the same routing metadata and arguments
        assert len(own_soft.calls) == 2 and _same(ref_soft.calls, own_soft.calls)
    else:
        assert [c[0] for c in own_soft.calls] == ["moe_layer"]


@needs_ref
def test_moe_apply_rejects_what_reference_rejects(sides):
    ref, _, _ = sides
    w = _weights(4, 256, 128, 1)
    layer = SimpleNamespace(**vars(w))
    va.moe_process_weights_after_loading(None, layer)
    layer.activation = "gelu"
    x = torch.zeros(2, 256, dtype=torch.bfloat16)
    tw, tid = _routes(2, 4, 2, 0)
    with pytest.raises(NotImplementedError, match="silu"):
        ref._moe_apply(None, layer, x, tw, tid)
    with pytest.raises(NotImplementedError, match="silu"):
        va.moe_apply(None, layer, x, tw, tid)
    layer.activation = "silu"
    with pytest.raises(NotImplementedError, match="shared"):
        va.moe_apply(None, layer, x, tw, tid, shared_experts=object())
    layer.expert_map = torch.arange(4)
    with pytest.raises(NotImplementedError, match="expert_map"):
        va.moe_apply(None, layer, x, tw, tid)


@pytest.mark.parametrize("value,backend", [("safe", "safe"), ("triton", "triton"), ("reference", "safe"),
                                           ("bf16", "safe")])
def test_implementation_env_sets_backend(monkeypatch, value, backend):
    monkeypatch.setenv("MXFP4_IMPLEMENTATION", value)
    monkeypatch.setenv("MXFP4_GFX936_BACKEND", "unset")
    mod = load_by_path(f"mxfp4_vllm_adapter_{value}", PKG / "vllm_adapter.py")
    assert os.environ["MXFP4_GFX936_BACKEND"] == backend
    assert mod._IMPLEMENTATION == ("reference" if value == "bf16" else value)


def test_unknown_implementation_rejected(monkeypatch):
    monkeypatch.setenv("MXFP4_IMPLEMENTATION", "fast")
    monkeypatch.setenv("MXFP4_GFX936_BACKEND", "unset")
    with pytest.raises(ValueError, match="unknown MXFP4 implementation"):
        load_by_path("mxfp4_vllm_adapter_bad", PKG / "vllm_adapter.py")
    sys.modules.pop("mxfp4_vllm_adapter_bad", None)


_INSTALL_SCRIPT = r"""
import sys
from types import SimpleNamespace
import torch
sys.path.insert(0, sys.argv[1])
from _paths import vllm_adapter
va = vllm_adapter()
dense_cls, moe_cls = va.install()
assert dense_cls.__name__ == "CompressedTensorsW4A4Mxfp4", dense_cls
assert moe_cls.__name__ == "CompressedTensorsW4A4Mxfp4MoEMethod", moe_cls
assert dense_cls.apply_weights is va.dense_apply_weights
assert dense_cls.process_weights_after_loading is va.dense_process_weights_after_loading
assert moe_cls.apply is va.moe_apply
assert moe_cls.process_weights_after_loading is va.moe_process_weights_after_loading
# the patched methods run as vLLM 0.22 calls them (self is the scheme object)
layer = SimpleNamespace(weight_packed=torch.zeros(8, 64, dtype=torch.uint8),
                        weight_scale=torch.zeros(8, 4, dtype=torch.uint8))
dense_cls.process_weights_after_loading(object.__new__(dense_cls), layer)
assert isinstance(layer.weight_packed, torch.nn.Parameter)
m = SimpleNamespace(activation="silu", w13_weight_packed=torch.zeros(2, 4, 8, dtype=torch.uint8),
                    w13_weight_scale=torch.zeros(2, 4, 1, dtype=torch.uint8),
                    w2_weight_packed=torch.zeros(2, 16, 1, dtype=torch.uint8),
                    w2_weight_scale=torch.zeros(2, 16, 1, dtype=torch.uint8))
moe_cls.process_weights_after_loading(object.__new__(moe_cls), m)
assert hasattr(m, "w13_weight") and not hasattr(m, "w13_weight_packed")
try:
    moe_cls.apply(object.__new__(moe_cls), m, torch.zeros(1, 16, dtype=torch.bfloat16), torch.ones(1, 1),
                  torch.zeros(1, 1, dtype=torch.int32), object(), None)
except NotImplementedError as e:
    assert "shared" in str(e)
else:
    raise AssertionError("shared experts accepted")
print("INSTALL_OK")
"""


def test_install_patches_vllm_022_classes():
    pytest.importorskip("vllm")
    r = subprocess.run([sys.executable, "-c", _INSTALL_SCRIPT, str(ROOT / "tests")], capture_output=True,
                       text=True, timeout=600)
    assert "INSTALL_OK" in r.stdout, (r.stdout[-2000:], r.stderr[-4000:])
