"""Compressed-tensors MXFP4 checkpoint loader (safetensors).

A checkpoint written in compressed-tensors' ``mxfp4-pack-quantized`` format
(compressed-tensors 0.15, ``MXFP4PackedCompressor``) stores, for every
quantized linear ``<prefix>``:

* ``<prefix>.weight_packed``: uint8 ``[N, K/2]``, E2M1 codes two per byte,
  column ``2i`` in the low nibble and ``2i+1`` in the high nibble
  (``pack_fp4_to_uint8``);
* ``<prefix>.weight_scale``: uint8 ``[N, K/32]``, one E8M0 exponent (bias
  127) per 32 consecutive columns (``compress_mx_scale``).

These are the tensors vLLM registers for the dense MXFP4 scheme and the
reference adapter's dense path keeps (vllm:68-70).  The experts of a
Qwen3-MoE checkpoint are per-expert linears
``<layer>.mlp.experts.<e>.{gate,up,down}_proj``; ``load_experts`` stacks them
the way vLLM's fused-MoE weight loader does for the adapter's MoE method
(vllm:215-230): ``w13_weight_packed`` ``[E, 2I, H/2]`` holds each expert's
gate rows then its up rows, ``w2_weight_packed`` ``[E, H, I/2]`` the down
projection, with the matching ``*_weight_scale``.

Tensors are read with ``safetensors.safe_open`` straight onto the target
device; a checkpoint split over several files is followed through its
``model.safetensors.index.json``.  Row ranges (column-parallel shards) and
expert ranges (expert-parallel shards) are cut before the copy.
"""

from __future__ import annotations

import json
from pathlib import Path
from types import SimpleNamespace

import torch
from safetensors import safe_open

FORMAT = "mxfp4-pack-quantized"
GROUP = 32


def _is_mxfp4_weights(args: dict) -> bool:
    return (args.get("num_bits") == 4 and args.get("type") == "float"
            and args.get("group_size") == GROUP)


class MxFp4Checkpoint:
    """One compressed-tensors MXFP4 checkpoint directory."""

    def __init__(self, path, device="cpu"):
        self.path = Path(path)
        self.device = torch.device(device)
        self.config = {}
        cfg = self.path / "config.json"
        if cfg.is_file():
            self.config = json.loads(cfg.read_text())
        self.quantization_config = self.config.get("quantization_config", {})
        self._check_format()
        self._files = self._index()

    # -- format --------------------------------------------------------------------------------
    def _check_format(self):
        q = self.quantization_config
        if not q:
            return  # bare safetensors: shapes and dtypes are still checked per tensor
        if q.get("quant_method") != "compressed-tensors":
            raise ValueError(f"not a compressed-tensors checkpoint: quant_method={q.get('quant_method')!r}")
        groups = q.get("config_groups", {})
        formats = {q.get("format")} | {g.get("format") for g in groups.values()}
        formats.discard(None)
        if FORMAT not in formats:
            raise ValueError(f"checkpoint format {sorted(formats)} is not {FORMAT!r}")
        weights = [g.get("weights") for g in groups.values() if g.get("weights")]
        if not weights or not all(_is_mxfp4_weights(w) for w in weights):
            raise ValueError("every config group must quantize weights as 4-bit float in groups of 32")

    # -- file index -----------------------------------------------------------------------------
    def _index(self):
        index = self.path / "model.safetensors.index.json"
        if index.is_file():
            weight_map = json.loads(index.read_text())["weight_map"]
            return {name: self.path / file for name, file in weight_map.items()}
        files = {}
        for file in sorted(self.path.glob("*.safetensors")):
            with safe_open(str(file), framework="pt") as f:
                for name in f.keys():
                    files[name] = file
        if not files:
            raise FileNotFoundError(f"no safetensors files under {self.path}")
        return files

    def names(self):
        return sorted(self._files)

    def tensor(self, name, rows=None):
        """One tensor, optionally rows ``rows = (start, stop)`` of dim 0, on the device."""
        file = self._files.get(name)
        if file is None:
            raise KeyError(f"tensor {name!r} is not in the checkpoint")
        with safe_open(str(file), framework="pt", device="cpu") as f:
            if rows is None:
                t = f.get_tensor(name)
            else:
                t = f.get_slice(name)[rows[0]:rows[1]]
        return t.to(self.device)

    # -- quantized linears ----------------------------------------------------------------------
    def load_linear(self, prefix, rows=None):
        """``(weight_packed [N, K/2], weight_scale [N, K/32])`` of ``prefix``."""
        packed = self.tensor(f"{prefix}.weight_packed", rows)
        scale = self.tensor(f"{prefix}.weight_scale", rows)
        if packed.dtype != torch.uint8 or scale.dtype != torch.uint8:
            raise TypeError(f"{prefix}: packed weights and E8M0 scales must be uint8, "
                            f"got {packed.dtype} and {scale.dtype}")
        if packed.ndim != 2 or scale.shape != (packed.shape[0], packed.shape[1] * 2 // GROUP):
            raise ValueError(f"{prefix}: weight_scale {tuple(scale.shape)} does not match "
                             f"weight_packed {tuple(packed.shape)} (one scale per {GROUP} values)")
        return packed, scale

    def dense_layer(self, prefix, rows=None):
        """A layer object carrying the dense scheme's attributes (vllm:68-70)."""
        packed, scale = self.load_linear(prefix, rows)
        return SimpleNamespace(weight_packed=packed, weight_scale=scale)

    def load_experts(self, prefix, num_experts, experts=None):
        """Stacked expert tensors under ``<prefix>.<e>.{gate,up,down}_proj``.

        ``experts = (first, stop)`` loads that range only (an expert-parallel
        shard).  Returns the four tensors of the MoE method before
        ``process_weights_after_loading`` (vllm:215-230)."""
        first, stop = experts if experts is not None else (0, num_experts)
        if not 0 <= first < stop <= num_experts:
            raise ValueError(f"expert range {first}:{stop} is outside 0:{num_experts}")
        w13, s13, w2, s2 = [], [], [], []
        for e in range(first, stop):
            gp, gs = self.load_linear(f"{prefix}.{e}.gate_proj")
            up, us = self.load_linear(f"{prefix}.{e}.up_proj")
            dp, ds = self.load_linear(f"{prefix}.{e}.down_proj")
            # gate/up [I, H/2], down [H, I/2]
            if gp.shape != up.shape or dp.shape[0] != gp.shape[1] * 2 or dp.shape[1] * 2 != gp.shape[0]:
                raise ValueError(f"{prefix}.{e}: gate/up/down shapes {tuple(gp.shape)} {tuple(up.shape)} "
                                 f"{tuple(dp.shape)} do not form one expert")
            w13.append(torch.cat((gp, up)))
            s13.append(torch.cat((gs, us)))
            w2.append(dp)
            s2.append(ds)
        return {
            "w13_weight_packed": torch.stack(w13),
            "w13_weight_scale": torch.stack(s13),
            "w2_weight_packed": torch.stack(w2),
            "w2_weight_scale": torch.stack(s2),
        }

    def moe_layer(self, prefix, num_experts, experts=None, activation="silu"):
        """A layer object carrying the MoE method's attributes before
        ``process_weights_after_loading`` (vllm:215-230)."""
        return SimpleNamespace(activation=activation, **self.load_experts(prefix, num_experts, experts))
