"""CPU oracle for the MXFP4 hot path -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module, and only as the checker (or as the timed
CPU baseline).  The CUDA library never calls into it and the operator module
never falls back to it.

It restates, in numpy, the algorithm of lutianshu824/mxfp4-gfx936 for the
path that the B200 library accelerates.  Every function cites the reference
lines it follows (paths relative to the reference project root):

* ``src/aiter/ops/triton/moe_op_mxfp4_soft.py`` ("soft") -- E2M1 table
  (soft:12-29), ``dequant_mxfp4`` (soft:277-307), the safe linear
  (soft:371-376) and the safe routed-MoE op (soft:466-494).
* ``integration/vllm/vllm_mxfp4_gfx936.py`` ("vllm") -- ``_make_routing``
  (vllm:119-146) and the MoE layer composition ``_moe_apply`` (vllm:233-265).
* ``tests/test_moe_mxfp4_soft.py`` ("test") -- the reference test quantizer
  ``torch_dynamic_mxfp4_quant`` (test:28-60).

Pinning: ``tests/golden/make_golden.py`` runs the reference's own code on CPU
(imported from the reference checkout) and stores its outputs under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks this module against
those fixtures (bit-exact for dequant, routing and quantizers; within the
stated tolerance for the GEMM-shaped functions, whose reduction order the
reference leaves to the BLAS library).

Dtype convention: tensors of a 16-bit float dtype are carried as float32
arrays whose values are already rounded to that dtype (every bf16 / fp16 value
is exact in float32).  ``dtype`` arguments are the strings ``"fp32"``,
``"bf16"`` and ``"fp16"``.
"""

from __future__ import annotations

import numpy as np

# soft:12-29 -- E2M1 code -> value; bit 3 is the sign, so code 8 is -0.0.
E2M1_VALUES = np.array(
    [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
     -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
    dtype=np.float32,
)

DTYPES = ("fp32", "bf16", "fp16")


# ---------------------------------------------------------------------------
# rounding helpers
# ---------------------------------------------------------------------------

def f32_to_bf16_bits(x) -> np.ndarray:
    """Round float32 -> bfloat16 (round to nearest even) and return the bits.

    NaN becomes the canonical 0x7FC0, as c10::BFloat16 does.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r = np.where(np.isnan(x), np.uint16(0x7FC0), r)
    return r


def bf16_bits_to_f32(bits) -> np.ndarray:
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def round_to(x, dtype: str) -> np.ndarray:
    """Round to ``dtype`` and return the result as float32 values."""
    x = np.asarray(x)
    if dtype == "fp32":
        return x.astype(np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(x.astype(np.float32)))
    if dtype == "fp16":
        with np.errstate(over="ignore", invalid="ignore"):
            return x.astype(np.float16).astype(np.float32)
    raise ValueError(f"unknown dtype {dtype!r}")


def _round_f64(x64, dtype: str) -> np.ndarray:
    # float64 -> float32 -> dtype.  The double rounding can move a result by
    # one unit of the target format in rare ties; parity tolerances cover it.
    return round_to(np.asarray(x64, dtype=np.float64).astype(np.float32), dtype)


# ---------------------------------------------------------------------------
# C1/C2: dequantisation (soft:277-307)
# ---------------------------------------------------------------------------

def unpack_codes(packed) -> np.ndarray:
    """uint8 [..., K/2] -> E2M1 codes uint8 [..., K]; low nibble = even K (soft:295)."""
    packed = np.asarray(packed, dtype=np.uint8)
    codes = np.stack((packed & 0x0F, packed >> 4), axis=-1)
    return codes.reshape(*packed.shape[:-1], packed.shape[-1] * 2)


def scale_multipliers(block_scales) -> np.ndarray:
    """E8M0 codes -> float32 2**(code-127); code 255 -> NaN (soft:299-306)."""
    s = np.asarray(block_scales, dtype=np.uint8)
    with np.errstate(over="ignore"):
        m = np.ldexp(np.ones(s.shape, dtype=np.float32), s.astype(np.int32) - 127)
    m = m.astype(np.float32)
    return np.where(s == 255, np.float32(np.nan), m).astype(np.float32)


def dequant(packed, block_scales, dtype: str = "fp32") -> np.ndarray:
    """``dequant_mxfp4`` (soft:277-307): FP32 value * FP32 scale, then cast."""
    packed = np.asarray(packed, dtype=np.uint8)
    block_scales = np.asarray(block_scales, dtype=np.uint8)
    k = packed.shape[-1] * 2
    if k % 32 != 0:
        raise ValueError(f"logical K must be divisible by 32, got {k}")
    if block_scales.shape[:-1] != packed.shape[:-1] or block_scales.shape[-1] * 32 != k:
        raise ValueError("one E8M0 scale is required for every 32 MXFP4 values")
    values = E2M1_VALUES[unpack_codes(packed)]
    scales = np.repeat(scale_multipliers(block_scales), 32, axis=-1)
    with np.errstate(over="ignore", invalid="ignore"):
        return round_to(values * scales, dtype)


# ---------------------------------------------------------------------------
# C3: dense W4A16 linear, safe path (soft:371-376)
# ---------------------------------------------------------------------------

def linear(x, x_dtype: str, packed, block_scales, bias=None) -> np.ndarray:
    """y = x . dequant(W)^T rounded to x's dtype, then ``+ bias`` (soft:371-375).

    The product is accumulated in float64 (an exact-as-possible stand-in for
    the BLAS FP32 accumulation) and rounded once.  ``bias`` (same dtype as x)
    is added afterwards with a second rounding, as ``output + bias`` does.
    """
    x = np.asarray(x, dtype=np.float32)
    k = x.shape[-1]
    w = dequant(packed, block_scales, x_dtype)
    y = _round_f64(x.reshape(-1, k).astype(np.float64) @ w.astype(np.float64).T, x_dtype)
    if bias is not None:
        y = round_to(y + np.asarray(bias, dtype=np.float32), x_dtype)
    return y.reshape(*x.shape[:-1], w.shape[0])


def gemm_w4a4(a_packed, a_scales, b_packed, b_scales, out_dtype: str = "bf16") -> np.ndarray:
    """Dense W4A4: dequant both operands to BF16, then one BF16 matmul.

    The reference's W4A4 semantics (soft:468-475 dequantises packed
    activations to the compute dtype before the same matmul as the weights).
    """
    a = dequant(a_packed, a_scales, "bf16").astype(np.float64)
    b = dequant(b_packed, b_scales, "bf16").astype(np.float64)
    return _round_f64(a @ b.T, out_dtype)


# ---------------------------------------------------------------------------
# C4: routed MoE op, safe path (soft:466-494)
# ---------------------------------------------------------------------------

def moe_op(A, a_dtype: str, A_mx_scale, B, B_mx_scale, a_scale, b_scale,
           topk_weights, topk_ids, mul_routed_weight: bool, c_dtype: str) -> np.ndarray:
    """Safe ``fused_moe_mxfp4_soft``; returns C [M, top_k, N] as float32 values.

    ``A`` is either a float array of ``a_dtype`` values or (``a_dtype ==
    "u8"``) packed MXFP4 with ``A_mx_scale``.  Rounding points follow
    soft:471-494 with C's dtype as the matmul dtype: the matmul output is
    rounded, multiplied by the FP32 ``A_scale`` and rounded, multiplied by
    ``B_scale[e]`` and rounded, then (optionally) multiplied by the FP32
    route weight and rounded a last time.  Experts outside ``[0, E)`` leave
    their rows zero (the loop at soft:478 never visits them).
    """
    B = np.asarray(B, dtype=np.uint8)
    B_mx_scale = np.asarray(B_mx_scale, dtype=np.uint8)
    topk_ids = np.asarray(topk_ids).astype(np.int64)
    topk_weights = np.asarray(topk_weights, dtype=np.float32)
    if a_dtype == "u8":
        acts = dequant(A, A_mx_scale, c_dtype)
    else:
        acts = round_to(np.asarray(A, dtype=np.float32), c_dtype)
    m, top_k = topk_ids.shape
    n = B.shape[1]
    C = np.zeros((m, top_k, n), dtype=np.float32)
    g = np.float32(np.asarray(a_scale, dtype=np.float32).reshape(-1)[0])
    bs = np.asarray(b_scale, dtype=np.float32).reshape(-1)
    for e in range(B.shape[0]):
        tok, slot = np.nonzero(topk_ids == e)
        if tok.size == 0:
            continue
        w = dequant(B[e], B_mx_scale[e], c_dtype).astype(np.float64)
        out = _round_f64(acts[tok].astype(np.float64) @ w.T, c_dtype)
        out = round_to(out * g, c_dtype)
        out = round_to(out * np.float32(bs[e]), c_dtype)
        if mul_routed_weight:
            out = round_to(out * topk_weights[tok, slot][:, None], c_dtype)
        C[tok, slot] = out
    return C


# ---------------------------------------------------------------------------
# a9: routing metadata (vllm:119-146)
# ---------------------------------------------------------------------------

def make_routing(topk_ids, block_m: int = 64):
    """``_make_routing``: per-expert blocks of ``block_m`` route ids.

    Route id r = t*top_k + j (flat index into topk_ids).  Experts are visited
    in ascending order (``torch.unique(sorted=True)``), route ids inside an
    expert ascend (``torch.nonzero``), each expert's list is cut into
    ``block_m`` chunks padded with ``T*top_k``.  Returns (sorted_ids int32,
    expert_ids int32, num_tokens_post_padded int32[1]).
    """
    flat = np.asarray(topk_ids).astype(np.int64).reshape(-1)
    pad = flat.size
    sorted_blocks, experts = [], []
    for e in np.unique(flat):
        routes = np.nonzero(flat == e)[0].astype(np.int32)
        for start in range(0, routes.size, block_m):
            chunk = routes[start:start + block_m]
            block = np.full(block_m, pad, dtype=np.int32)
            block[:chunk.size] = chunk
            sorted_blocks.append(block)
            experts.append(int(e))
    if not sorted_blocks:
        raise ValueError("topk_ids must contain at least one routed token")
    sorted_ids = np.concatenate(sorted_blocks)
    return (sorted_ids, np.asarray(experts, dtype=np.int32),
            np.asarray([sorted_ids.size], dtype=np.int32))


def route_blocks(topk_ids, num_experts: int, block_m: int, expert_offset: int = 0):
    """Routing restricted to local experts ``[expert_offset, expert_offset+E)``.

    For ids that are all local this equals ``make_routing`` with expert ids
    shifted by ``-expert_offset``; routes to other experts are dropped, which
    is what the safe op does with ids outside its weight tensor (soft:478).
    """
    flat = np.asarray(topk_ids).astype(np.int64).reshape(-1)
    pad = flat.size
    sorted_blocks, experts = [], []
    for e in range(num_experts):
        routes = np.nonzero(flat == e + expert_offset)[0].astype(np.int32)
        for start in range(0, routes.size, block_m):
            chunk = routes[start:start + block_m]
            block = np.full(block_m, pad, dtype=np.int32)
            block[:chunk.size] = chunk
            sorted_blocks.append(block)
            experts.append(e)
    if sorted_blocks:
        sorted_ids = np.concatenate(sorted_blocks)
    else:
        sorted_ids = np.zeros(0, dtype=np.int32)
    return (sorted_ids, np.asarray(experts, dtype=np.int32),
            np.asarray([sorted_ids.size], dtype=np.int32))


# ---------------------------------------------------------------------------
# a10: MoE layer composition (vllm:233-265)
# ---------------------------------------------------------------------------

def silu_bf16(g) -> np.ndarray:
    """``F.silu`` on a BF16 tensor: x / (1 + exp(-x)) in high precision, rounded."""
    g64 = np.asarray(g, dtype=np.float64)
    with np.errstate(over="ignore"):
        s = g64 / (1.0 + np.exp(-g64))
    return _round_f64(s, "bf16")


def moe_layer(x, w13, s13, w2, s2, topk_weights, topk_ids) -> np.ndarray:
    """``_moe_apply`` with the safe op, BF16 activations.

    gate_up = op(x, W13) without route weights (vllm:240-247); routed =
    bf16(silu(gate)) * up rounded (vllm:248-252); down = op(routed, W2) with
    the route weight, one route per row (vllm:253-262); the result is the
    FP32-accumulated sum over the top-k rows, rounded to BF16 (vllm:263-265).
    """
    topk_ids = np.asarray(topk_ids).astype(np.int64)
    topk_weights = np.asarray(topk_weights, dtype=np.float32)
    t, k = topk_ids.shape
    one = np.ones(1, dtype=np.float32)
    gate_up = moe_op(x, "bf16", None, w13, s13, one, np.ones(w13.shape[0], np.float32),
                     topk_weights, topk_ids, False, "bf16")
    inter = gate_up.shape[-1] // 2
    routed = round_to(silu_bf16(gate_up[..., :inter]) * gate_up[..., inter:], "bf16")
    routed = routed.reshape(t * k, inter)
    down = moe_op(routed, "bf16", None, w2, s2, one, np.ones(w2.shape[0], np.float32),
                  topk_weights.reshape(t * k, 1), topk_ids.reshape(t * k, 1), True, "bf16")
    summed = down[:, 0].reshape(t, k, -1).astype(np.float32).sum(axis=1, dtype=np.float32)
    return round_to(summed, "bf16")


def combine_topk(rows, top_k: int) -> np.ndarray:
    """Sum of ``top_k`` consecutive BF16 rows in FP32, rounded once (vllm:263-265)."""
    rows = np.asarray(rows, dtype=np.float32)
    t = rows.shape[0] // top_k
    return round_to(rows.reshape(t, top_k, -1).sum(axis=1, dtype=np.float32), "bf16")


# ---------------------------------------------------------------------------
# quantizers
# ---------------------------------------------------------------------------

def quant_reference_test(x):
    """The reference's test quantizer ``torch_dynamic_mxfp4_quant`` (test:28-60).

    amax is rounded up to a power of two by integer arithmetic on its bits,
    scale exponent = floor(log2(amax)) - 2 clamped to [-127, 127], elements are
    rounded half-up on the E2M1 grid by the ``(+1) >> 1`` trick and saturated
    at code 7.  Returns (packed uint8 [..., K/2], scales uint8 [..., K/32]).
    """
    x = np.asarray(x, dtype=np.float32)
    k = x.shape[-1]
    if k % 32:
        raise ValueError("test quantizer requires K divisible by 32")
    blocks = x.reshape(-1, k // 32, 32)
    amax = np.max(np.abs(blocks), axis=-1).astype(np.float32)
    ai = amax.view(np.int32).astype(np.int64)
    ai = ((ai + 0x200000) & 0xFF800000) & 0xFFFFFFFF
    amax_r = ai.astype(np.uint32).view(np.float32)
    with np.errstate(divide="ignore"):
        se = np.floor(np.log2(amax_r.astype(np.float32))) - 2
    se = np.clip(se, -127, 127).astype(np.float32)
    q = (blocks * np.exp2(-se).astype(np.float32)[..., None]).astype(np.float32)
    qi = q.view(np.int32).astype(np.int64)
    sign = (qi >> 31) & 1
    exponents = (qi >> 23) & 0xFF
    mant = qi & 0x7FFFFF
    adjusted = 127 - exponents - 1
    sub = (0x400000 | (mant >> 1))
    sub = np.where(adjusted >= 63, 0, sub >> np.clip(adjusted, 0, 62))
    mant = np.where(exponents < 127, sub, mant)
    exponents = np.where(exponents > 126, exponents, 126) - 126
    combined = (((exponents << 2) | (mant >> 21)) + 1) >> 1
    mag = np.where(combined < 7, combined, 7)
    codes = ((sign << 3) | mag).astype(np.uint8).reshape(*x.shape[:-1], k)
    packed = (codes[..., 0::2] | (codes[..., 1::2] << 4)).astype(np.uint8)
    scales = (se.astype(np.int64) + 127).astype(np.uint8).reshape(*x.shape[:-1], k // 32)
    return packed, scales


_E2M1_MAGS = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float64)


def quant_ocp_rne(x):
    """OCP MXFP4 quantizer of the W4A4 configuration.

    Per 32-element block: q = fl32(max|x| / 6) (IEEE FP32 division),
    e = floor(log2(q)) read from q's exponent, scale code = e + 127 clamped
    to [0, 254] (a zero block gets code 0 and all-zero elements); each element
    x / 2**(code-127) is rounded to the nearest E2M1 value with ties to the
    even code and saturated to +-6.  Returns (packed, scales) as uint8.
    """
    x = np.asarray(x, dtype=np.float32)
    k = x.shape[-1]
    if k % 32:
        raise ValueError("quantizer requires K divisible by 32")
    blocks = x.reshape(-1, k // 32, 32)
    bmax = np.max(np.abs(blocks), axis=-1).astype(np.float32)
    q = (bmax / np.float32(6.0)).astype(np.float32)
    _, ex = np.frexp(q.astype(np.float64))       # q = f * 2**ex, f in [0.5, 1)
    e = ex.astype(np.int64) - 1
    code = np.clip(e + 127, 0, 254)
    code = np.where(bmax == 0, 0, code).astype(np.int64)
    inv = np.ldexp(1.0, 127 - code).astype(np.float64)
    v = blocks.astype(np.float64) * inv[..., None]
    a = np.minimum(np.abs(v), 6.0)
    # nearest grid point, ties to the even code
    d = np.abs(a[..., None] - _E2M1_MAGS)
    best = np.argmin(d, axis=-1)
    dmin = np.take_along_axis(d, best[..., None], axis=-1)[..., 0]
    nxt = np.minimum(best + 1, 7)
    tie = (np.abs(a - _E2M1_MAGS[nxt]) == dmin) & (nxt != best)
    mag = np.where(tie & (best % 2 == 1), nxt, best)
    sign = (np.signbit(v) & (mag > 0)).astype(np.int64)
    codes = ((sign << 3) | mag).astype(np.uint8).reshape(*x.shape[:-1], k)
    packed = (codes[..., 0::2] | (codes[..., 1::2] << 4)).astype(np.uint8)
    scales = code.astype(np.uint8).reshape(*x.shape[:-1], k // 32)
    return packed, scales


# ---------------------------------------------------------------------------
# comparison helper used by the parity tests
# ---------------------------------------------------------------------------

def ulp_bf16(mag: float) -> float:
    """Spacing of BF16 values at magnitude ``mag`` (8 significant bits)."""
    mag = float(abs(mag))
    if mag == 0.0 or not np.isfinite(mag):
        return 2.0 ** -133
    return 2.0 ** (np.floor(np.log2(mag)) - 7)


def check_close(actual, expected, ulps: float = 2.0, rel_fro: float = 1e-3):
    """The north-star gate: max|err| <= ulps * ulp_bf16(max|ref|) and
    ||err||_F / ||ref||_F <= rel_fro.  Returns (ok, max_abs_err, bound, rel)."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    if a.shape != e.shape:
        return False, np.inf, 0.0, np.inf
    fin = np.isfinite(e)
    if not np.array_equal(np.isfinite(a), fin):
        return False, np.inf, 0.0, np.inf
    err = np.abs(a[fin] - e[fin])
    ref_max = float(np.max(np.abs(e[fin]))) if err.size else 0.0
    bound = ulps * ulp_bf16(ref_max)
    max_err = float(err.max()) if err.size else 0.0
    den = float(np.linalg.norm(e[fin]))
    rel = float(np.linalg.norm(err)) / den if den > 0 else (0.0 if max_err == 0 else np.inf)
    return (max_err <= bound and rel <= rel_fro), max_err, bound, rel
