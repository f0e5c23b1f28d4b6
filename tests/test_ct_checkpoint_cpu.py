"""Compressed-tensors MXFP4 checkpoint loader, checked on CPU.

The checkpoint comes from compressed-tensors' own MXFP4 compressor
(``tests/golden/make_ct_checkpoint.py``); the values each packed tensor stands
for are compressed-tensors' ``fake_quantize`` of the original weight.  The
loader's tensors, dequantized by the oracle, must equal those values exactly:
that pins the nibble order and the E8M0 scale encoding to the third-party
writer.  Stacking of the experts (gate rows then up rows, vllm:215-230),
row and expert shards, the index file and the format checks are covered too.
"""

import json
import shutil

import numpy as np
import pytest
import torch
from safetensors.torch import load_file

from _paths import PKG, load_by_path, oracle

ct = load_by_path("mxfp4_ct_checkpoint", PKG / "ct_checkpoint.py")
O = oracle()
LAYER = "model.layers.0"
EXPERTS = 4


def _deq(packed, scale):
    return O.dequant(packed.numpy(), scale.numpy(), "fp32")


@pytest.fixture(scope="module")
def expected(ct_checkpoint_dir):
    return load_file(str(ct_checkpoint_dir / "expected.safetensors"))


def test_dense_values_match_compressed_tensors(ct_checkpoint_dir, expected):
    ck = ct.MxFp4Checkpoint(ct_checkpoint_dir)
    packed, scale = ck.load_linear(f"{LAYER}.self_attn.q_proj")
    assert packed.dtype == torch.uint8 and tuple(packed.shape) == (384, 128)
    assert scale.dtype == torch.uint8 and tuple(scale.shape) == (384, 8)
    want = expected[f"{LAYER}.self_attn.q_proj"].numpy()
    assert np.array_equal(_deq(packed, scale), want)
    layer = ck.dense_layer(f"{LAYER}.self_attn.q_proj")
    assert torch.equal(layer.weight_packed, packed) and torch.equal(layer.weight_scale, scale)


def test_row_shard(ct_checkpoint_dir):
    ck = ct.MxFp4Checkpoint(ct_checkpoint_dir)
    full_p, full_s = ck.load_linear(f"{LAYER}.self_attn.q_proj")
    p, s = ck.load_linear(f"{LAYER}.self_attn.q_proj", rows=(96, 192))
    assert torch.equal(p, full_p[96:192]) and torch.equal(s, full_s[96:192])


def test_experts_stacked_gate_then_up(ct_checkpoint_dir, expected):
    ck = ct.MxFp4Checkpoint(ct_checkpoint_dir)
    w = ck.load_experts(f"{LAYER}.mlp.experts", EXPERTS)
    assert tuple(w["w13_weight_packed"].shape) == (EXPERTS, 256, 128)
    assert tuple(w["w13_weight_scale"].shape) == (EXPERTS, 256, 8)
    assert tuple(w["w2_weight_packed"].shape) == (EXPERTS, 256, 64)
    assert tuple(w["w2_weight_scale"].shape) == (EXPERTS, 256, 4)
    for e in range(EXPERTS):
        pre = f"{LAYER}.mlp.experts.{e}"
        w13 = _deq(w["w13_weight_packed"][e], w["w13_weight_scale"][e])
        want13 = np.concatenate((expected[f"{pre}.gate_proj"].numpy(), expected[f"{pre}.up_proj"].numpy()))
        assert np.array_equal(w13, want13)
        assert np.array_equal(_deq(w["w2_weight_packed"][e], w["w2_weight_scale"][e]),
                              expected[f"{pre}.down_proj"].numpy())


def test_expert_shard_and_moe_layer_object(ct_checkpoint_dir):
    ck = ct.MxFp4Checkpoint(ct_checkpoint_dir)
    full = ck.load_experts(f"{LAYER}.mlp.experts", EXPERTS)
    layer = ck.moe_layer(f"{LAYER}.mlp.experts", EXPERTS, experts=(1, 3))
    assert layer.activation == "silu"
    for k, v in full.items():
        assert torch.equal(getattr(layer, k), v[1:3])
    with pytest.raises(ValueError):
        ck.load_experts(f"{LAYER}.mlp.experts", EXPERTS, experts=(3, 5))


def test_single_file_without_index(ct_checkpoint_dir, tmp_path):
    # one shard only, found by scanning the directory
    shutil.copy(ct_checkpoint_dir / "model-00002-of-00002.safetensors", tmp_path / "model.safetensors")
    ck = ct.MxFp4Checkpoint(tmp_path)
    assert f"{LAYER}.mlp.gate.weight" in ck.names()
    p, s = ck.load_linear(f"{LAYER}.mlp.experts.3.down_proj")
    assert tuple(p.shape) == (256, 64) and tuple(s.shape) == (256, 4)
    with pytest.raises(KeyError):
        ck.load_linear(f"{LAYER}.self_attn.q_proj")


def test_format_checks(ct_checkpoint_dir, tmp_path):
    cfg = json.loads((ct_checkpoint_dir / "config.json").read_text())
    for f in ct_checkpoint_dir.glob("*.safetensors"):
        shutil.copy(f, tmp_path / f.name)
    shutil.copy(ct_checkpoint_dir / "model.safetensors.index.json", tmp_path / "model.safetensors.index.json")

    def write(c):
        (tmp_path / "config.json").write_text(json.dumps(c))

    bad = json.loads(json.dumps(cfg))
    bad["quantization_config"]["format"] = "nvfp4-pack-quantized"
    bad["quantization_config"]["config_groups"]["group_0"]["format"] = "nvfp4-pack-quantized"
    write(bad)
    with pytest.raises(ValueError, match="mxfp4-pack-quantized"):
        ct.MxFp4Checkpoint(tmp_path)
    bad = json.loads(json.dumps(cfg))
    bad["quantization_config"]["config_groups"]["group_0"]["weights"]["group_size"] = 16
    write(bad)
    with pytest.raises(ValueError, match="groups of 32"):
        ct.MxFp4Checkpoint(tmp_path)
    bad = json.loads(json.dumps(cfg))
    bad["quantization_config"]["quant_method"] = "fp8"
    write(bad)
    with pytest.raises(ValueError, match="compressed-tensors"):
        ct.MxFp4Checkpoint(tmp_path)
    write(cfg)
    ck = ct.MxFp4Checkpoint(tmp_path)
    # the unquantized router is not an MXFP4 linear
    with pytest.raises(KeyError):
        ck.load_linear(f"{LAYER}.mlp.gate")
