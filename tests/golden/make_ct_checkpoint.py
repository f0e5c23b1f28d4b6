"""Write a small compressed-tensors MXFP4 checkpoint with compressed-tensors itself.

Test infrastructure: ``tests/test_ct_checkpoint_cpu.py`` and
``tests/test_vllm_adapter_gpu.py`` run this script (in a subprocess, with
``TORCHDYNAMO_DISABLE=1`` because compressed-tensors 0.15 compiles its FP4
rounding with ``torch.compile``) to get a checkpoint whose packing and scale
encoding come from the third-party writer, not from this repository::

    TORCHDYNAMO_DISABLE=1 python tests/golden/make_ct_checkpoint.py OUT_DIR

Contents (one Qwen3-MoE-shaped layer, hidden 256, intermediate 128, 4 experts):

* ``model.layers.0.self_attn.q_proj`` (384 x 256) and
  ``model.layers.0.mlp.experts.<e>.{gate,up,down}_proj``, compressed by
  ``MXFP4PackedCompressor.compress`` under the ``MXFP4A16`` preset scheme;
* ``model.layers.0.mlp.gate.weight`` (the router, left in bf16, listed under
  ``ignore``);
* two shards and ``model.safetensors.index.json``;
* ``expected.safetensors``: compressed-tensors' ``fake_quantize`` of every
  quantized weight (float32), i.e. the values the packed tensors stand for.

Scales are the power of two at or above ``amax / 6`` of each 32-value group.
"""

import json
import sys
from pathlib import Path

import torch
from compressed_tensors.compressors.mxfp4.base import MXFP4PackedCompressor
from compressed_tensors.quantization import preset_name_to_scheme
from compressed_tensors.quantization.lifecycle.forward import fake_quantize
from safetensors.torch import save_file

HIDDEN, INTER, EXPERTS, QROWS = 256, 128, 4, 384


def main(out):
    out = Path(out)
    out.mkdir(parents=True, exist_ok=True)
    scheme = preset_name_to_scheme("MXFP4A16", ["Linear"])
    g = torch.Generator().manual_seed(20261202)
    shards = [{}, {}]
    expected = {}

    def add(prefix, rows, cols, shard):
        w = torch.randn(rows, cols, generator=g) * torch.exp2(torch.randint(-3, 4, (rows, 1), generator=g).float())
        amax = w.reshape(rows, cols // 32, 32).abs().amax(-1).clamp_min(1e-30)
        scale = torch.exp2(torch.ceil(torch.log2(amax / 6.0)))
        state = MXFP4PackedCompressor.compress({"weight": w, "weight_scale": scale}, scheme)
        shards[shard][f"{prefix}.weight_packed"] = state["weight_packed"].contiguous()
        shards[shard][f"{prefix}.weight_scale"] = state["weight_scale"].contiguous()
        expected[prefix] = fake_quantize(w, scale, None, scheme.weights).float().contiguous()

    add("model.layers.0.self_attn.q_proj", QROWS, HIDDEN, 0)
    for e in range(EXPERTS):
        shard = 0 if e < EXPERTS // 2 else 1
        add(f"model.layers.0.mlp.experts.{e}.gate_proj", INTER, HIDDEN, shard)
        add(f"model.layers.0.mlp.experts.{e}.up_proj", INTER, HIDDEN, shard)
        add(f"model.layers.0.mlp.experts.{e}.down_proj", HIDDEN, INTER, shard)
    shards[1]["model.layers.0.mlp.gate.weight"] = torch.randn(EXPERTS, HIDDEN, generator=g).to(torch.bfloat16)

    weight_map = {}
    for i, tensors in enumerate(shards):
        name = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(tensors, str(out / name))
        weight_map.update({k: name for k in tensors})
    (out / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))
    save_file(expected, str(out / "expected.safetensors"))
    weights = scheme.weights.model_dump(mode="json")
    weights = {k: v for k, v in weights.items() if k in ("num_bits", "type", "symmetric", "group_size", "strategy",
                                                         "dynamic")}
    (out / "config.json").write_text(json.dumps({
        "architectures": ["Qwen3MoeForCausalLM"],
        "hidden_size": HIDDEN, "moe_intermediate_size": INTER, "num_experts": EXPERTS, "num_experts_per_tok": 2,
        "quantization_config": {
            "quant_method": "compressed-tensors",
            "format": "mxfp4-pack-quantized",
            "config_groups": {"group_0": {"targets": ["Linear"], "weights": weights,
                                          "format": "mxfp4-pack-quantized"}},
            "ignore": ["lm_head", "re:.*mlp.gate$"],
        },
    }, indent=1))


if __name__ == "__main__":
    main(sys.argv[1])
