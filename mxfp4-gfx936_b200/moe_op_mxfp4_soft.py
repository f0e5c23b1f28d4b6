# SPDX-License-Identifier: MIT
"""B200 (sm_100a) drop-in for the ``moe_op_mxfp4_soft`` operator module.

This file replaces ``src/aiter/ops/triton/moe_op_mxfp4_soft.py`` of
lutianshu824/mxfp4-gfx936 ("soft" below) behind the same surface: the same
function names, argument order, dtypes, exception types and messages.  It is
self-contained so that it can be loaded by file path, the way the AITER entry,
the vLLM adapter and the reference test load the original
(``importlib.util.spec_from_file_location``; ``MXFP4_SOFT_MODULE``).

Every operator runs on the GPU through the C ABI of ``libmxfp4_b200.so``
(declared in ``include/mxfp4_b200.h``), found next to this file or at
``MXFP4_B200_LIBRARY``.  There is no CPU fallback and no Triton: a missing
library, a CPU tensor or a non-sm_100 device raises ``RuntimeError``.

Backend selection is explicit, as in soft:45-49.  ``MXFP4_GFX936_BACKEND``
(read on every call) selects how the dense linear runs:

* ``safe`` (default): explicit dequantisation of the weight into a workspace
  (the ``dequant_mxfp4`` kernel), then the tcgen05 GEMM on that BF16/FP16
  weight -- the structure of soft:371-373;
* ``triton`` (the reference's name, also what the vLLM adapter writes,
  vllm:34-36) and ``fused`` (the same mode under its B200 name): the weight is
  decoded inside the GEMM producer, the B200 counterpart of soft:176-274.
  There is no shape guard: both modes feed the same MMA sequence, so their
  results are identical bit for bit.

The routed-MoE op has one native path (device routing + grouped GEMM) for
every value.  With ``triton`` it also keeps the reference Triton path's input
contract (soft:409-430: unpacked activations and valid padded routing
metadata, else ``RuntimeError``); ``fused`` accepts packed activations and
empty metadata as well.  Any other value raises ``ValueError``.

The reference module's helpers keep their names and contracts (soft:34-62):
``_has_compatible_triton_compiler`` answers whether the prebuilt sm_100a
library loads on an sm_100 device (this backend's counterpart of the gfx936
compiler probe), ``_require_triton_compiler`` raises ``RuntimeError`` when it
does not, and ``_is_validated_triton_linear_shape`` keeps the reference's
M >= 370 and N >= 2048 rule.  The B200 fused path covers every shape, so the
operator does not consult that rule.
"""

from __future__ import annotations

import ctypes
import functools
import os
from pathlib import Path

import torch

_MXFP4_E2M1_VALUES = (
    0.0,
    0.5,
    1.0,
    1.5,
    2.0,
    3.0,
    4.0,
    6.0,
    -0.0,
    -0.5,
    -1.0,
    -1.5,
    -2.0,
    -3.0,
    -4.0,
    -6.0,
)

_BACKENDS = ("safe", "triton", "fused")
_FUSED_BACKENDS = ("triton", "fused")

# C ABI constants (include/mxfp4_b200.h)
_OK = 0
_ERR_INVALID_ARGUMENT = 1
_ERR_UNSUPPORTED_DEVICE = 2
_ERR_UNSUPPORTED = 6
_LINEAR_FUSED = 0
_LINEAR_SAFE = 1
_DTYPE_CODES = {
    torch.float32: 0,
    torch.bfloat16: 1,
    torch.float16: 2,
    torch.uint8: 3,
    torch.int32: 4,
    torch.int64: 5,
}
_BLOCK_M = 128  # rows per routed block of the grouped GEMM


def _library_path() -> Path:
    explicit = os.getenv("MXFP4_B200_LIBRARY")
    if explicit:
        return Path(explicit)
    return Path(__file__).resolve().parent / "libmxfp4_b200.so"


_VP = ctypes.c_void_p
_I64 = ctypes.c_int64
_INT = ctypes.c_int
_SZ = ctypes.c_size_t

_SIGNATURES = {
    "mxfp4_abi_version": (_INT, []),
    "mxfp4_last_error": (ctypes.c_char_p, []),
    "mxfp4_device_supported": (_INT, [_INT]),
    "mxfp4_device_status": (_INT, [_INT, _INT]),
    "mxfp4_dequant": (_INT, [_VP, _VP, _VP, _INT, _I64, _I64, _VP]),
    "mxfp4_linear_workspace_size": (_SZ, [_I64, _I64, _I64, _INT, _INT]),
    "mxfp4_linear_w4a16": (
        _INT,
        [_VP, _INT, _I64, _VP, _I64, _VP, _I64, _VP, _VP, _I64, _I64, _I64, _I64, _INT, _VP, _SZ, _VP],
    ),
    "mxfp4_linear_dequantized": (_INT, [_VP, _INT, _I64, _VP, _I64, _VP, _VP, _I64, _I64, _I64, _I64, _VP]),
    "mxfp4_quantize": (_INT, [_VP, _INT, _I64, _I64, _I64, _VP, _VP, _VP]),
    "mxfp4_moe_router": (_INT, [_VP, _INT, _I64, _INT, _INT, _INT, _VP, _VP, _VP]),
    "mxfp4_gemm_w4a4_workspace_size": (_SZ, [_I64, _I64, _I64]),
    "mxfp4_gemm_w4a4": (_INT, [_VP, _VP, _VP, _VP, _VP, _INT, _I64, _I64, _I64, _VP, _SZ, _VP]),
    "mxfp4_moe_route_capacity": (_I64, [_I64, _INT, _INT]),
    "mxfp4_moe_route_workspace_size": (_SZ, [_I64, _INT]),
    "mxfp4_moe_route": (_INT, [_VP, _INT, _I64, _INT, _INT, _INT, _INT, _VP, _VP, _VP, _I64, _VP, _SZ, _VP]),
    "mxfp4_fused_moe_workspace_size": (_SZ, [_I64, _INT, _INT, _I64, _I64, _INT, _INT]),
    "mxfp4_fused_moe": (
        _INT,
        [_VP, _INT, _VP, _VP, _VP, _VP, _VP, _VP, _INT, _VP, _INT, _VP, _INT, _I64, _INT, _INT, _I64, _I64,
         _INT, _VP, _SZ, _VP],
    ),
    "mxfp4_fused_moe_noalloc": (
        _INT,
        [_VP, _INT, _VP, _VP, _VP, _VP, _VP, _VP, _INT, _VP, _INT, _VP, _INT, _I64, _INT, _INT, _I64, _I64,
         _INT, _VP],
    ),
    "mxfp4_linear_w4a16_allgather": (
        _INT,
        [_VP, _INT, _I64, _VP, _I64, _VP, _I64, _VP, _VP, ctypes.POINTER(ctypes.c_void_p), _INT, _I64, _I64,
         _I64, _I64, _INT, _VP, _SZ, _VP],
    ),
    "mxfp4_linear_w4a16_allgather_mc": (
        _INT,
        [_VP, _INT, _I64, _VP, _I64, _VP, _I64, _VP, _VP, ctypes.POINTER(ctypes.c_void_p), _INT, _VP, _I64, _I64,
         _I64, _I64, _INT, _VP, _SZ, _VP],
    ),
    "mxfp4_peer_barrier": (_INT, [ctypes.POINTER(ctypes.c_void_p), _INT, _INT, _VP, _VP]),
    "mxfp4_peer_barrier_timed": (_INT, [ctypes.POINTER(ctypes.c_void_p), _INT, _INT, _VP, _I64, _VP]),
    "mxfp4_peer_barrier_reset": (_INT, [_VP, _INT, _VP, _VP]),
    "mxfp4_ipc_alloc": (_INT, [_SZ, ctypes.POINTER(ctypes.c_void_p), _VP]),
    "mxfp4_ipc_open": (_INT, [_VP, ctypes.POINTER(ctypes.c_void_p)]),
    "mxfp4_ipc_close": (_INT, [_VP]),
    "mxfp4_ipc_free": (_INT, [_VP]),
    "mxfp4_ep_moe_recv_capacity": (_I64, [_I64, _INT, _INT, _INT]),
    "mxfp4_ep_moe_workspace_size": (_SZ, [_I64, _INT, _INT, _I64, _I64]),
    "mxfp4_ep_moe_layer": (
        _INT,
        [_VP, _VP, _VP, _VP, _VP, _VP, _INT, _VP, _INT, _VP, _I64, _INT, _INT, _I64, _I64, _INT, _INT,
         ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
         ctypes.POINTER(ctypes.c_void_p), _I64, ctypes.POINTER(ctypes.c_void_p), _VP, _VP, _SZ, _VP],
    ),
    "mxfp4_moe_layer_workspace_size": (_SZ, [_I64, _INT, _INT, _I64, _I64]),
    "mxfp4_moe_layer": (
        _INT,
        [_VP, _VP, _VP, _VP, _VP, _VP, _INT, _VP, _INT, _VP, _I64, _INT, _INT, _I64, _I64, _VP, _SZ, _VP],
    ),
}


@functools.lru_cache(maxsize=1)
def _load_library():
    path = _library_path()
    if not path.is_file():
        raise RuntimeError(
            f"MXFP4 B200 backend library not found at {path}; build it with "
            "`python __graft_entry__.py` or set MXFP4_B200_LIBRARY"
        )
    try:
        lib = ctypes.CDLL(str(path))
    except OSError as exc:
        raise RuntimeError(f"cannot load MXFP4 B200 backend library {path}: {exc}") from exc
    for name, (restype, argtypes) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


@functools.lru_cache(maxsize=1)
def _has_compatible_native_library() -> bool:
    """True when the library loads and the current CUDA device is sm_100."""
    try:
        lib = _load_library()
    except RuntimeError:
        return False
    if not torch.cuda.is_available():
        return False
    return bool(lib.mxfp4_device_supported(torch.cuda.current_device()))


@functools.lru_cache(maxsize=1)
def _has_compatible_triton_compiler() -> bool:
    """soft:34-43 under the same name.  The fused backend's kernels come
    prebuilt for sm_100a, so its "compiler" is libmxfp4_b200.so itself: true
    when that library loads and the current CUDA device is sm_100."""
    return _has_compatible_native_library()


def _backend() -> str:
    """soft:45-49: ``MXFP4_GFX936_BACKEND`` read on every call, ``safe`` by
    default; ``triton`` and ``fused`` both select the fused-decode GEMM."""
    backend = os.getenv("MXFP4_GFX936_BACKEND", "safe")
    if backend not in _BACKENDS:
        raise ValueError(f"unknown gfx936 MXFP4 backend: {backend} (B200 backend: safe, triton or fused)")
    return backend


def _require_triton_compiler() -> None:
    """soft:52-57: the fused backend fails loud when its kernels cannot run."""
    if not _has_compatible_triton_compiler():
        raise RuntimeError(
            "MXFP4_GFX936_BACKEND=triton requires a compatible compiler; on B200 that is the prebuilt "
            "sm_100a library libmxfp4_b200.so on an sm_100 device (set MXFP4_B200_LIBRARY explicitly; "
            "TRITON_HIP_CLANG_PATH is not used by this backend)"
        )


def _is_validated_triton_linear_shape(m: int, n: int) -> bool:
    """soft:60-62: the shape range the reference validated its Triton linear
    on (M >= 370 and N >= 2048).  Kept for callers and tests that read it; the
    B200 fused linear covers every shape with the same bits as ``safe``."""
    return m >= 370 and n >= 2048


def _require_native_library() -> None:
    if not _has_compatible_native_library():
        raise RuntimeError(
            "the B200 MXFP4 backend requires libmxfp4_b200.so and an sm_100 CUDA device; "
            "set MXFP4_B200_LIBRARY explicitly"
        )


def _require_cuda(*tensors) -> torch.device:
    device = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "the B200 MXFP4 backend has no CPU path; all tensors must be on an sm_100 CUDA device"
            )
        if device is None:
            device = t.device
        elif t.device != device:
            raise RuntimeError("all tensors must be on the same CUDA device")
    _require_native_library()
    return device


def _check(rc: int) -> None:
    if rc == _OK:
        return
    msg = _load_library().mxfp4_last_error().decode(errors="replace")
    if rc == _ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    if rc == _ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(f"libmxfp4_b200 error {rc}: {msg}")


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _dense(t: torch.Tensor) -> torch.Tensor:
    """Contiguous and 16-byte aligned (TMA and vector loads need both)."""
    if not t.is_contiguous() or t.data_ptr() % 16 != 0:
        t = t.contiguous() if t.data_ptr() % 16 == 0 else t.clone(memory_format=torch.contiguous_format)
        if t.data_ptr() % 16 != 0:
            out = torch.empty(t.numel() + 16, dtype=t.dtype, device=t.device)
            t = out[: t.numel()].view(t.shape).copy_(t)
    return t


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


# ---------------------------------------------------------------------------
# dequant_mxfp4 (soft:277-307)
# ---------------------------------------------------------------------------

def dequant_mxfp4(
    packed: torch.Tensor,
    block_scales: torch.Tensor,
    dtype: torch.dtype = torch.float32,
) -> torch.Tensor:
    """Dequantize packed OCP MXFP4 E2M1 values with E8M0 block scales."""
    if packed.dtype != torch.uint8:
        raise TypeError(f"packed must be uint8, got {packed.dtype}")
    if block_scales.dtype != torch.uint8:
        raise TypeError(f"block_scales must be uint8, got {block_scales.dtype}")

    logical_k = packed.shape[-1] * 2
    if logical_k % 32 != 0:
        raise ValueError(f"logical K must be divisible by 32, got {logical_k}")
    if block_scales.shape[:-1] != packed.shape[:-1]:
        raise ValueError("packed and block_scales leading dimensions must match")
    if block_scales.shape[-1] * 32 != logical_k:
        raise ValueError("one E8M0 scale is required for every 32 MXFP4 values")
    device = _require_cuda(packed, block_scales)
    out_dtype = dtype if dtype in (torch.float32, torch.bfloat16, torch.float16) else torch.float32
    rows = packed.numel() // max(packed.shape[-1], 1) if packed.shape[-1] else 0
    out = torch.empty((*packed.shape[:-1], logical_k), dtype=out_dtype, device=device)
    if out.numel():
        p = _dense(packed)
        s = _dense(block_scales)
        with torch.cuda.device(device):
            _check(_load_library().mxfp4_dequant(
                _ptr(p), _ptr(s), _ptr(out), _DTYPE_CODES[out_dtype], rows, logical_k, _stream(device)))
    return out if out_dtype == dtype else out.to(dtype)


# ---------------------------------------------------------------------------
# linear_mxfp4_soft (soft:310-376)
# ---------------------------------------------------------------------------

def linear_mxfp4_soft(
    x: torch.Tensor,
    packed: torch.Tensor,
    block_scales: torch.Tensor,
    bias: torch.Tensor | None = None,
) -> torch.Tensor:
    """Weight-only OCP MXFP4 linear with an explicit backend."""
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError(f"x must be fp16 or bf16, got {x.dtype}")
    if packed.dtype != torch.uint8 or block_scales.dtype != torch.uint8:
        raise TypeError("packed weights and E8M0 scales must be uint8")
    if packed.ndim != 2 or block_scales.ndim != 2:
        raise ValueError("linear weights and scales must be 2D")
    logical_k = packed.shape[1] * 2
    if x.shape[-1] != logical_k:
        raise ValueError(f"input K {x.shape[-1]} does not match weight K {logical_k}")
    if logical_k % 128 != 0:
        raise ValueError(f"logical K must be divisible by 128, got {logical_k}")
    if block_scales.shape != (packed.shape[0], logical_k // 32):
        raise ValueError("one E8M0 scale is required for every 32 MXFP4 values")

    backend = _backend()
    if backend in _FUSED_BACKENDS:
        _require_triton_compiler()
    device = _require_cuda(x, packed, block_scales, bias)
    input_shape = x.shape
    n = packed.shape[0]
    x_2d = _dense(x.reshape(-1, logical_k))
    m = x_2d.shape[0]
    output = torch.empty((m, n), dtype=x.dtype, device=device)
    fused_bias = bias is not None and bias.dtype == x.dtype and tuple(bias.shape) == (n,)
    b = _dense(bias) if fused_bias else None
    w = _dense(packed)
    s = _dense(block_scales)
    mode = _LINEAR_FUSED if backend in _FUSED_BACKENDS else _LINEAR_SAFE
    lib = _load_library()
    if m:
        code = _DTYPE_CODES[x.dtype]
        ws_bytes = lib.mxfp4_linear_workspace_size(m, n, logical_k, code, mode)
        ws = _workspace(ws_bytes, device) if ws_bytes else None
        with torch.cuda.device(device):
            _check(lib.mxfp4_linear_w4a16(
                _ptr(x_2d), code, logical_k, _ptr(w), logical_k // 2, _ptr(s), logical_k // 32,
                _ptr(b), _ptr(output), n, m, n, logical_k, mode, _ptr(ws), ws_bytes, _stream(device)))
    if bias is not None and not fused_bias:
        output = output + bias
    return output.reshape(*input_shape[:-1], n)


def linear_dequantized(x: torch.Tensor, w_deq: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ w_deq.T`` (+ ``bias``) for weights already decoded by
    ``dequant_mxfp4`` into x's dtype: the matmul half of the safe path
    (soft:372-375) on the same kernels as ``linear_mxfp4_soft``, so
    ``linear_dequantized(x, dequant_mxfp4(W, S, x.dtype))`` has the bits of
    ``linear_mxfp4_soft(x, W, S)``.  K must be a multiple of 128."""
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError(f"x must be fp16 or bf16, got {x.dtype}")
    if w_deq.dtype != x.dtype or w_deq.ndim != 2:
        raise TypeError("w_deq must be a 2-D tensor of x's dtype")
    k = w_deq.shape[1]
    if x.shape[-1] != k or k % 128:
        raise ValueError(f"input K {x.shape[-1]} must match weight K {k}, a multiple of 128")
    device = _require_cuda(x, w_deq, bias)
    n = w_deq.shape[0]
    x_2d = _dense(x.reshape(-1, k))
    m = x_2d.shape[0]
    out = torch.empty((m, n), dtype=x.dtype, device=device)
    fused_bias = bias is not None and bias.dtype == x.dtype and tuple(bias.shape) == (n,)
    b = _dense(bias) if fused_bias else None
    w = _dense(w_deq)
    if m:
        with torch.cuda.device(device):
            _check(_load_library().mxfp4_linear_dequantized(
                _ptr(x_2d), _DTYPE_CODES[x.dtype], k, _ptr(w), k, _ptr(b), _ptr(out), n, m, n, k, _stream(device)))
    if bias is not None and not fused_bias:
        out = out + bias
    return out.reshape(*x.shape[:-1], n)


# ---------------------------------------------------------------------------
# fused_moe_mxfp4_soft (soft:379-494)
# ---------------------------------------------------------------------------

def fused_moe_mxfp4_soft(
    A: torch.Tensor,
    B: torch.Tensor,
    C: torch.Tensor,
    A_scale: torch.Tensor,
    B_scale: torch.Tensor,
    A_mx_scale: torch.Tensor | None,
    B_mx_scale: torch.Tensor,
    topk_weights: torch.Tensor,
    topk_ids: torch.Tensor,
    sorted_token_ids: torch.Tensor,
    expert_ids: torch.Tensor,
    num_tokens_post_padded: torch.Tensor,
    mul_routed_weight: bool,
    top_k: int,
    swizzle_mx_a: bool,
    swizzle_mx_b: bool,
) -> None:
    """Routed MXFP4 MoE GEMM on B200; writes the caller-owned ``C``.

    ``C[t, j, :] = A[t] . deq(B[e])^T * A_scale * B_scale[e]`` (times the
    route weight when ``mul_routed_weight``), with C's dtype as the compute
    dtype and the rounding points of soft:487-494, for e = topk_ids[t, j].
    With an FP32 ``C`` the products and sums are those of an FP32 matmul
    (soft:405, 466-494): activations are split exactly into BF16 parts and
    every part meets the exactly decoded BF16 weights with FP32 accumulation.
    Routes whose expert id lies outside ``[0, B.shape[0])`` leave zeros.  The
    padded routing metadata of the Triton path is validated like the
    reference's (backend ``triton``) and then ignored: the kernel derives its
    own route blocks from ``topk_ids`` on the device.
    """
    if swizzle_mx_a or swizzle_mx_b:
        raise NotImplementedError(
            "the gfx936 software fallback does not support swizzled scales; the B200 backend keeps that contract")
    if topk_ids.shape != topk_weights.shape or topk_ids.shape[1] != top_k:
        raise ValueError("top-k ids and weights must have matching (M, top_k) shapes")
    if B.dtype != torch.uint8 or B_mx_scale is None:
        raise TypeError("the gfx936 software fallback requires packed MXFP4 weights (B200 backend)")

    matmul_dtype = C.dtype
    if matmul_dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError(f"unsupported software fallback compute dtype: {matmul_dtype}")
    backend = _backend()
    if backend == "triton":
        # the reference Triton path's input contract (soft:409-430)
        _require_triton_compiler()
        routing_ready = (
            A.dtype != torch.uint8
            and sorted_token_ids.numel() > 0
            and expert_ids.numel() > 0
            and num_tokens_post_padded.numel() == 1
            and B.shape[-1] * 2 % 128 == 0
            and sorted_token_ids.numel() % expert_ids.numel() == 0
        )
        if not routing_ready:
            raise RuntimeError(
                "the experimental Triton MoE backend requires unpacked "
                "activations and valid padded routing metadata"
            )
        block_m = sorted_token_ids.numel() // expert_ids.numel()
        if block_m not in (16, 32, 64, 128):
            raise RuntimeError(f"unsupported Triton routing block size: {block_m}")
    del sorted_token_ids, expert_ids, num_tokens_post_padded

    if A.dtype == torch.uint8:
        if A_mx_scale is None:
            raise ValueError("packed MXFP4 activations require A_mx_scale")
        logical_k = A.shape[-1] * 2
    else:
        if A_mx_scale is not None:
            raise ValueError("unpacked activations must not provide A_mx_scale")
        if A.dtype not in (torch.float16, torch.bfloat16, torch.float32):
            raise TypeError(f"unsupported activation dtype: {A.dtype}")
        logical_k = A.shape[-1]
    num_experts, n = B.shape[0], B.shape[1]
    m = topk_ids.shape[0]
    if B.shape[2] * 2 != logical_k:
        raise ValueError(f"activation K {logical_k} does not match weight K {B.shape[2] * 2}")
    if logical_k % 128 != 0:
        raise ValueError(f"logical K must be divisible by 128, got {logical_k}")
    if tuple(B_mx_scale.shape) != (num_experts, n, logical_k // 32):
        raise ValueError("one E8M0 scale is required for every 32 MXFP4 values")
    if A.shape[0] != m:
        raise ValueError("A must have one row per token of topk_ids")
    if tuple(C.shape) != (m, top_k, n):
        raise ValueError(f"C must have shape {(m, top_k, n)}, got {tuple(C.shape)}")
    if topk_ids.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"topk_ids must be int32 or int64, got {topk_ids.dtype}")
    if topk_weights.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        raise TypeError(f"topk_weights must be a float tensor, got {topk_weights.dtype}")

    device = _require_cuda(A, B, C, A_scale, B_scale, A_mx_scale, B_mx_scale, topk_weights, topk_ids)
    a = _dense(A)
    amx = _dense(A_mx_scale) if A_mx_scale is not None else None
    b = _dense(B)
    bmx = _dense(B_mx_scale)
    a_scale = _dense(A_scale.reshape(-1)[:1].to(torch.float32))
    b_scale = _dense(B_scale.reshape(-1).to(torch.float32))
    if b_scale.numel() < num_experts:
        raise ValueError("B_scale needs one value per expert")
    tw = _dense(topk_weights)
    tid = _dense(topk_ids)
    c = C if (C.is_contiguous() and C.data_ptr() % 16 == 0) else torch.empty(
        (m, top_k, n), dtype=C.dtype, device=device)
    lib = _load_library()
    a_code, c_code = _DTYPE_CODES[a.dtype], _DTYPE_CODES[C.dtype]
    ws_bytes = lib.mxfp4_fused_moe_workspace_size(m, top_k, num_experts, n, logical_k, a_code, c_code)
    ws = _workspace(ws_bytes, device)
    with torch.cuda.device(device):
        _check(lib.mxfp4_fused_moe(
            _ptr(a), a_code, _ptr(amx), _ptr(b), _ptr(bmx), _ptr(a_scale), _ptr(b_scale),
            _ptr(tw), _DTYPE_CODES[tw.dtype], _ptr(tid), _DTYPE_CODES[tid.dtype], _ptr(c), c_code,
            m, top_k, num_experts, n, logical_k, 1 if mul_routed_weight else 0,
            _ptr(ws), ws_bytes, _stream(device)))
    if c is not C:
        C.copy_(c)


# ---------------------------------------------------------------------------
# B200 additions: device routing and the whole MoE layer
# ---------------------------------------------------------------------------

def moe_route(topk_ids: torch.Tensor, num_experts: int, block_m: int = _BLOCK_M,
              expert_offset: int = 0):
    """Device-side ``_make_routing`` (vllm:119-146) for local experts.

    Returns ``(sorted_token_ids, expert_ids, num_tokens_post_padded)`` with
    capacity-sized buffers: ``sorted_token_ids[:num_tokens_post_padded]`` and
    the first ``num_tokens_post_padded // block_m`` entries of ``expert_ids``
    are the metadata ``_make_routing(topk_ids - expert_offset, block_m)``
    produces when every id is local; trailing blocks have expert -1.
    """
    if topk_ids.dtype not in (torch.int32, torch.int64) or topk_ids.ndim != 2:
        raise TypeError("topk_ids must be a 2-D int32 or int64 tensor")
    device = _require_cuda(topk_ids)
    lib = _load_library()
    t, k = topk_ids.shape
    routes = t * k
    cap = int(lib.mxfp4_moe_route_capacity(routes, num_experts, block_m))
    sorted_ids = torch.empty(max(cap, 1), dtype=torch.int32, device=device)
    expert_ids = torch.empty(max(cap // block_m, 1), dtype=torch.int32, device=device)
    post = torch.empty(1, dtype=torch.int32, device=device)
    ws_bytes = lib.mxfp4_moe_route_workspace_size(routes, num_experts)
    ws = _workspace(ws_bytes, device)
    tid = _dense(topk_ids)
    with torch.cuda.device(device):
        _check(lib.mxfp4_moe_route(
            _ptr(tid), _DTYPE_CODES[tid.dtype], t, k, num_experts, expert_offset, block_m,
            _ptr(sorted_ids), _ptr(expert_ids), _ptr(post), cap, _ptr(ws), ws_bytes, _stream(device)))
    return sorted_ids[:cap], expert_ids[: cap // block_m], post


def moe_router(router_logits: torch.Tensor, top_k: int, renormalize: bool = True):
    """Softmax top-k routing on the device: the ``topk_weights`` (float32) and
    ``topk_ids`` (int32), both ``[M, top_k]``, that vLLM hands the adapter's
    ``_moe_apply`` (vllm:233).  Probabilities are an FP32 softmax over the
    experts; the top ``top_k`` come in descending order (equal values: the
    lower expert first) and, with ``renormalize``, are rescaled to sum to one.
    At most 256 experts and ``top_k <= min(32, experts)``."""
    if router_logits.ndim != 2:
        raise ValueError("router_logits must be 2-D [tokens, experts]")
    if router_logits.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        raise TypeError(f"router_logits must be float32, bfloat16 or float16, got {router_logits.dtype}")
    t, e = router_logits.shape
    if not 1 <= top_k <= min(32, e) or e > 256:
        raise ValueError(f"need 1 <= top_k <= min(32, experts) and experts <= 256, got top_k={top_k}, experts={e}")
    device = _require_cuda(router_logits)
    weights = torch.empty((t, top_k), dtype=torch.float32, device=device)
    ids = torch.empty((t, top_k), dtype=torch.int32, device=device)
    logits = _dense(router_logits)
    with torch.cuda.device(device):
        _check(_load_library().mxfp4_moe_router(_ptr(logits), _DTYPE_CODES[logits.dtype], t, e, top_k,
                                                int(bool(renormalize)), _ptr(weights), _ptr(ids), _stream(device)))
    return weights, ids


def moe_layer_mxfp4(x: torch.Tensor, w13: torch.Tensor, w13_scale: torch.Tensor, w2: torch.Tensor,
                    w2_scale: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
    """The routed-MoE layer of the vLLM adapter (``_moe_apply``, vllm:233-265).

    gate_up GEMM (gate = first ``inter`` rows of ``w13``) with SiLU(gate)*up
    fused in its epilogue, down GEMM with the route weight and the
    unpermute-scatter fused in its epilogue, then the top-k sum -- with the
    BF16 rounding points of the reference composition.
    """
    if x.dtype != torch.bfloat16:
        raise TypeError(f"x must be bf16, got {x.dtype}")
    for name, t in (("w13", w13), ("w13_scale", w13_scale), ("w2", w2), ("w2_scale", w2_scale)):
        if t.dtype != torch.uint8:
            raise TypeError(f"{name} must be uint8, got {t.dtype}")
    if topk_ids.shape != topk_weights.shape or topk_ids.ndim != 2:
        raise ValueError("top-k ids and weights must have matching (M, top_k) shapes")
    t, hidden = x.shape
    num_experts, two_inter = w13.shape[0], w13.shape[1]
    inter = two_inter // 2
    if w13.shape[2] * 2 != hidden or tuple(w2.shape) != (num_experts, hidden, inter // 2):
        raise ValueError("w13 must be [E, 2I, H/2] and w2 [E, H, I/2]")
    if tuple(w13_scale.shape) != (num_experts, two_inter, hidden // 32) or tuple(w2_scale.shape) != (
            num_experts, hidden, inter // 32):
        raise ValueError("one E8M0 scale is required for every 32 MXFP4 values")
    if topk_ids.shape[0] != t:
        raise ValueError("topk_ids must have one row per token")
    device = _require_cuda(x, w13, w13_scale, w2, w2_scale, topk_weights, topk_ids)
    lib = _load_library()
    top_k = topk_ids.shape[1]
    out = torch.empty((t, hidden), dtype=torch.bfloat16, device=device)
    ws_bytes = lib.mxfp4_moe_layer_workspace_size(t, top_k, num_experts, hidden, inter)
    ws = _workspace(ws_bytes, device)
    xs, tw, tid = _dense(x), _dense(topk_weights), _dense(topk_ids)
    with torch.cuda.device(device):
        _check(lib.mxfp4_moe_layer(
            _ptr(xs), _ptr(_dense(w13)), _ptr(_dense(w13_scale)), _ptr(_dense(w2)), _ptr(_dense(w2_scale)),
            _ptr(tw), _DTYPE_CODES[tw.dtype], _ptr(tid), _DTYPE_CODES[tid.dtype], _ptr(out),
            t, top_k, num_experts, hidden, inter, _ptr(ws), ws_bytes, _stream(device)))
    return out


def quantize_mxfp4(x: torch.Tensor):
    """BF16/FP32 -> (packed uint8 [..., K/2], E8M0 scales uint8 [..., K/32]).

    OCP MXFP4 with the W4A4 configuration's rounding: scale code
    floor(log2(fl32(max|x|/6))) + 127 per 32 values, elements rounded to
    nearest-even on the E2M1 grid and saturated at 6.
    """
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"x must be bf16 or fp32, got {x.dtype}")
    k = x.shape[-1]
    if k % 32:
        raise ValueError(f"K must be divisible by 32, got {k}")
    device = _require_cuda(x)
    x2 = _dense(x.reshape(-1, k))
    rows = x2.shape[0]
    packed = torch.empty((*x.shape[:-1], k // 2), dtype=torch.uint8, device=device)
    scales = torch.empty((*x.shape[:-1], k // 32), dtype=torch.uint8, device=device)
    if rows:
        with torch.cuda.device(device):
            _check(_load_library().mxfp4_quantize(_ptr(x2), _DTYPE_CODES[x.dtype], k, rows, k, _ptr(packed),
                                                  _ptr(scales), _stream(device)))
    return packed, scales


def gemm_mxfp4_w4a4(a_packed: torch.Tensor, a_scales: torch.Tensor, b_packed: torch.Tensor,
                    b_scales: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """W4A4: ``dequant(A) @ dequant(B)^T`` on the block-scaled tensor cores.

    The reference's packed-activation semantics (soft:468-475: both operands
    dequantised, one matmul with FP32 accumulation), computed natively with
    tcgen05 ``kind::mxf4`` and one E8M0 scale per 32 values on each side.
    """
    for name, t in (("a_packed", a_packed), ("a_scales", a_scales), ("b_packed", b_packed), ("b_scales", b_scales)):
        if t.dtype != torch.uint8:
            raise TypeError(f"{name} must be uint8, got {t.dtype}")
    if a_packed.ndim != 2 or b_packed.ndim != 2:
        raise ValueError("W4A4 operands must be 2D")
    if out_dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise TypeError(f"unsupported output dtype {out_dtype}")
    m, k = a_packed.shape[0], a_packed.shape[1] * 2
    n = b_packed.shape[0]
    if b_packed.shape[1] * 2 != k:
        raise ValueError("A and B must have the same K")
    if k % 128:
        raise ValueError(f"logical K must be divisible by 128, got {k}")
    if tuple(a_scales.shape) != (m, k // 32) or tuple(b_scales.shape) != (n, k // 32):
        raise ValueError("one E8M0 scale is required for every 32 MXFP4 values")
    device = _require_cuda(a_packed, a_scales, b_packed, b_scales)
    lib = _load_library()
    out = torch.empty((m, n), dtype=out_dtype, device=device)
    ws_bytes = lib.mxfp4_gemm_w4a4_workspace_size(m, n, k)
    ws = _workspace(ws_bytes, device)
    a, sa, b, sb = _dense(a_packed), _dense(a_scales), _dense(b_packed), _dense(b_scales)
    with torch.cuda.device(device):
        _check(lib.mxfp4_gemm_w4a4(_ptr(a), _ptr(sa), _ptr(b), _ptr(sb), _ptr(out), _DTYPE_CODES[out_dtype],
                                   m, n, k, _ptr(ws), ws_bytes, _stream(device)))
    return out


def device_status(device=None, clear: bool = True) -> int:
    """Device status word of the library (0 = ok; 4 = a bounded wait expired)."""
    dev = torch.cuda.current_device() if device is None else torch.device(device).index or 0
    return int(_load_library().mxfp4_device_status(dev, 1 if clear else 0))
