"""vLLM compressed-tensors boundary of the B200 MXFP4 backend.

The reference's vLLM adapter (integration/vllm/vllm_mxfp4_gfx936.py) swaps
four methods of vLLM's compressed-tensors MXFP4 classes for calls into its
operator module.  This module restates those methods on this backend's
operator module (``moe_op_mxfp4_soft`` of this package, loaded by file path as
the adapter loads its own, vllm:38-51) and installs them into the vLLM that is
importable:

* ``dense_process_weights_after_loading`` (vllm:68-70): keep
  ``weight_packed`` ``[N, K/2]`` and ``weight_scale`` ``[N, K/32]`` (uint8)
  as frozen parameters.
* ``dense_apply_weights`` (vllm:105-116): ``linear_mxfp4_soft(x,
  layer.weight_packed, layer.weight_scale, bias)``.
* ``moe_process_weights_after_loading`` (vllm:215-230): rename
  ``w13_weight_packed`` / ``w2_weight_packed`` to ``w13_weight`` /
  ``w2_weight`` and freeze the four expert tensors.
* ``moe_apply`` (vllm:233-265): gate_up GEMM, SiLU(gate) * up, down GEMM with
  the route weights, top-k sum.  Two forms with the same bits:
  ``"layer"`` (default) is one ``moe_layer_mxfp4`` call (GLU and the route
  weight fused into the GEMM epilogues); ``"composition"`` is the adapter's
  own sequence of two ``fused_moe_mxfp4_soft`` calls (``moe_gemm``,
  vllm:149-185) with the routing metadata built on the device by
  ``moe_route`` instead of the adapter's host loop (``_make_routing``,
  vllm:119-146, same metadata).

``MXFP4_IMPLEMENTATION`` is read as the adapter reads it (vllm:29-36):
``safe`` (default), ``triton`` or ``reference`` (alias ``bf16``), and sets
``MXFP4_GFX936_BACKEND`` for the operator module.  ``triton`` selects this
backend's fused kernels.  ``reference`` selects the dequantize-then-BF16-matmul
products of the adapter's ``_bf16_linear`` / ``_bf16_moe_gemm``
(vllm:94-103, 188-212), which are the products of the safe backend
(soft:372-375, soft:478-494), so it runs the safe backend.

``install()`` patches vLLM 0.22's ``CompressedTensorsW4A4Mxfp4`` (dense) and
``CompressedTensorsW4A4Mxfp4MoEMethod``, or vLLM 0.15's
``CompressedTensorsW4A16Mxfp4`` where that class exists (the classes the
reference patches, vllm:268-275).  vLLM 0.22's MoE ``apply`` also passes
shared experts; this adapter covers the checkpoints the reference validates
(no shared experts, no vLLM expert map, route weights applied after the
experts) and raises ``NotImplementedError`` for the rest.
"""

from __future__ import annotations

import importlib
import importlib.util
import os
import sys
from pathlib import Path

import torch
import torch.nn.functional as F
from torch.nn.parameter import Parameter

_HERE = Path(__file__).resolve().parent

_IMPLEMENTATION = os.getenv("MXFP4_IMPLEMENTATION", "safe")
if _IMPLEMENTATION == "bf16":
    _IMPLEMENTATION = "reference"
if _IMPLEMENTATION not in ("reference", "safe", "triton"):
    raise ValueError(f"unknown MXFP4 implementation: {_IMPLEMENTATION}")
os.environ["MXFP4_GFX936_BACKEND"] = "triton" if _IMPLEMENTATION == "triton" else "safe"

ROUTING_BLOCK = 64  # the adapter's routing block (``_make_routing(topk_ids, block_m=64)``, vllm:119)
_MOE_FORMS = ("layer", "composition")
MOE_FORM = os.getenv("MXFP4_MOE_FORM", "layer")
if MOE_FORM not in _MOE_FORMS:
    raise ValueError(f"unknown MXFP4 MoE form: {MOE_FORM} (expected one of {_MOE_FORMS})")


def _load_soft_module():
    """The operator module, by file path (``MXFP4_SOFT_MODULE`` overrides)."""
    path = Path(os.getenv("MXFP4_SOFT_MODULE", _HERE / "moe_op_mxfp4_soft.py"))
    if not path.is_file():
        raise FileNotFoundError(f"MXFP4 soft module not found: {path}")
    if "moe_op_mxfp4_soft" in sys.modules:
        return sys.modules["moe_op_mxfp4_soft"]
    spec = importlib.util.spec_from_file_location("moe_op_mxfp4_soft", path)
    if spec is None or spec.loader is None:
        raise ImportError(f"cannot load MXFP4 soft module: {path}")
    module = importlib.util.module_from_spec(spec)
    sys.modules["moe_op_mxfp4_soft"] = module
    spec.loader.exec_module(module)
    return module


soft = _load_soft_module()


# ---------------------------------------------------------------------------
# dense W4A16 linear (vllm:68-70, 105-116)
# ---------------------------------------------------------------------------

def dense_process_weights_after_loading(self, layer):
    layer.weight_packed = Parameter(layer.weight_packed.data, requires_grad=False)
    layer.weight_scale = Parameter(layer.weight_scale.data, requires_grad=False)


def dense_apply_weights(self, layer, x, bias=None, input_quant_args=None, silu_quant_args=None):
    return soft.linear_mxfp4_soft(x, layer.weight_packed, layer.weight_scale, bias)


# ---------------------------------------------------------------------------
# routed MoE layer (vllm:149-185, 215-265)
# ---------------------------------------------------------------------------

def moe_gemm(activations, packed, scales, topk_ids, topk_weights, multiply_route_weights):
    """One routed GEMM of the composition: ``C[t, j] = A[t] · deq(B[ids[t, j]])ᵀ``
    (· ``topk_weights[t, j]`` with ``multiply_route_weights``) in
    ``activations``' dtype, unit tensor scales (vllm:149-185)."""
    sorted_ids, expert_ids, post_padded = soft.moe_route(topk_ids, packed.shape[0], block_m=ROUTING_BLOCK)
    output = torch.empty((topk_ids.shape[0], topk_ids.shape[1], packed.shape[1]),
                         dtype=activations.dtype, device=activations.device)
    a_scale = torch.ones(1, dtype=torch.float32, device=activations.device)
    b_scale = torch.ones(packed.shape[0], dtype=torch.float32, device=activations.device)
    soft.fused_moe_mxfp4_soft(activations, packed, output, a_scale, b_scale, None, scales, topk_weights,
                              topk_ids, sorted_ids, expert_ids, post_padded, multiply_route_weights,
                              topk_ids.shape[1], False, False)
    return output


def moe_process_weights_after_loading(self, layer):
    layer.w13_weight = Parameter(layer.w13_weight_packed.data, requires_grad=False)
    layer.w13_weight_scale = Parameter(layer.w13_weight_scale.data, requires_grad=False)
    layer.w2_weight = Parameter(layer.w2_weight_packed.data, requires_grad=False)
    layer.w2_weight_scale = Parameter(layer.w2_weight_scale.data, requires_grad=False)
    delattr(layer, "w13_weight_packed")
    delattr(layer, "w2_weight_packed")


def _check_moe_layer(layer, shared_experts):
    if layer.activation != "silu":
        raise NotImplementedError(f"the B200 MXFP4 adapter supports silu, got {layer.activation}")
    if shared_experts is not None:
        raise NotImplementedError("the B200 MXFP4 adapter has no shared-expert path")
    if getattr(layer, "expert_map", None) is not None:
        raise NotImplementedError("the B200 MXFP4 adapter expects all experts on this rank (no expert_map)")
    if getattr(layer, "apply_router_weight_on_input", False):
        raise NotImplementedError("the B200 MXFP4 adapter applies route weights after the experts")


def moe_apply(self, layer, x, topk_weights, topk_ids, shared_experts=None, shared_experts_input=None,
              use_nn_moe=False):
    _check_moe_layer(layer, shared_experts)
    if MOE_FORM == "layer" and x.dtype == torch.bfloat16:
        return soft.moe_layer_mxfp4(x, layer.w13_weight, layer.w13_weight_scale, layer.w2_weight,
                                    layer.w2_weight_scale, topk_weights, topk_ids)
    return moe_apply_composition(layer, x, topk_weights, topk_ids)


def moe_apply_composition(layer, x, topk_weights, topk_ids):
    """The adapter's own two-GEMM sequence (vllm:240-265)."""
    gate_up = moe_gemm(x, layer.w13_weight, layer.w13_weight_scale, topk_ids, topk_weights, False)
    intermediate_size = gate_up.shape[-1] // 2
    routed = (F.silu(gate_up[..., :intermediate_size]) * gate_up[..., intermediate_size:]).reshape(
        topk_ids.numel(), intermediate_size)
    down = moe_gemm(routed, layer.w2_weight, layer.w2_weight_scale, topk_ids.reshape(topk_ids.numel(), 1),
                    topk_weights.reshape(topk_ids.numel(), 1), True)
    return down[:, 0].reshape(topk_ids.shape[0], topk_ids.shape[1], x.shape[-1]).sum(dim=1)


# ---------------------------------------------------------------------------
# installation into vLLM (vllm:268-275)
# ---------------------------------------------------------------------------

_CT = "vllm.model_executor.layers.quantization.compressed_tensors"
_DENSE_CLASSES = (
    (f"{_CT}.schemes.compressed_tensors_w4a4_mxfp4", "CompressedTensorsW4A4Mxfp4"),  # vLLM 0.22
    (f"{_CT}.schemes.compressed_tensors_w4a16_mxfp4", "CompressedTensorsW4A16Mxfp4"),  # vLLM 0.15
)
_MOE_CLASSES = (
    (f"{_CT}.compressed_tensors_moe.compressed_tensors_moe_w4a4_mxfp4", "CompressedTensorsW4A4Mxfp4MoEMethod"),
    (f"{_CT}.compressed_tensors_moe", "CompressedTensorsW4A4Mxfp4MoEMethod"),
)


def _first_class(candidates):
    for module_name, class_name in candidates:
        try:
            module = importlib.import_module(module_name)
        except ImportError:
            continue
        cls = getattr(module, class_name, None)
        if cls is not None:
            return cls
    return None


def install():
    """Patch vLLM's compressed-tensors MXFP4 dense scheme and MoE method.

    Returns ``(dense_class, moe_class)``; raises ``ImportError`` when vLLM
    has neither class."""
    dense_cls = _first_class(_DENSE_CLASSES)
    moe_cls = _first_class(_MOE_CLASSES)
    if dense_cls is None or moe_cls is None:
        raise ImportError("vLLM's compressed-tensors MXFP4 classes were not found")
    dense_cls.process_weights_after_loading = dense_process_weights_after_loading
    dense_cls.apply_weights = dense_apply_weights
    moe_cls.process_weights_after_loading = moe_process_weights_after_loading
    moe_cls.apply = moe_apply
    return dense_cls, moe_cls
