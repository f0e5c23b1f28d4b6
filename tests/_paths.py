"""Locations and loaders shared by the tests (test infrastructure only)."""

import importlib.util
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "mxfp4-gfx936_b200"
GOLDEN = ROOT / "tests" / "golden"


def load_by_path(name, path):
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    sys.modules[name] = module
    spec.loader.exec_module(module)
    return module


def oracle():
    return load_by_path("mxfp4_oracle", ROOT / "oracle" / "mxfp4_oracle.py")


def soft_module():
    """The drop-in operator module, loaded by file path as the reference test
    and the vLLM adapter load theirs (``MXFP4_SOFT_MODULE`` overrides)."""
    path = Path(os.getenv("MXFP4_SOFT_MODULE", PKG / "moe_op_mxfp4_soft.py"))
    return load_by_path("moe_op_mxfp4_soft", path)


def golden(name):
    return np.load(GOLDEN / f"{name}.npz")


def bits_to_f32(bits):
    bits = np.asarray(bits)
    if bits.dtype == np.uint16:
        raise TypeError("16-bit bits need a dtype; use bf16_to_f32 / fp16_to_f32")
    return bits.astype(np.uint32).view(np.float32)


def bf16_to_f32(bits):
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def fp16_to_f32(bits):
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def same_bits(a, b):
    """Bit-exact float comparison where any NaN equals any NaN."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    nan = np.isnan(a) & np.isnan(b)
    return bool(np.all((a.view(np.uint32) == b.view(np.uint32)) | nan))


def vllm_adapter(name="mxfp4_vllm_adapter"):
    """The package's vLLM adapter module.  Importing it sets
    ``MXFP4_GFX936_BACKEND`` from ``MXFP4_IMPLEMENTATION`` (as the reference
    adapter does); the variable is put back so other tests see their own."""
    saved = os.environ.get("MXFP4_GFX936_BACKEND")
    try:
        return load_by_path(name, PKG / "vllm_adapter.py")
    finally:
        if saved is None:
            os.environ.pop("MXFP4_GFX936_BACKEND", None)
        else:
            os.environ["MXFP4_GFX936_BACKEND"] = saved
