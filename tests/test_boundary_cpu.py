"""Drop-in boundary checks that need no GPU.

Mirrors the reference's backend/fail-loud tests (test:63-78) for the B200
backend, checks that libmxfp4_b200.so exports every entry point that
include/mxfp4_b200.h declares, and that every validation error is raised with
the reference's exception type before any device work.
"""

import ctypes
import re

import numpy as np
import pytest
import torch

from _paths import PKG, ROOT, soft_module

soft = soft_module()


def _declared_symbols():
    text = (ROOT / "include" / "mxfp4_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|size_t|const char\*)\s+(mxfp4_\w+)\s*\(", text, re.M)))


def test_header_declares_the_abi():
    names = _declared_symbols()
    for required in ("mxfp4_dequant", "mxfp4_linear_w4a16", "mxfp4_fused_moe", "mxfp4_moe_route",
                     "mxfp4_moe_layer", "mxfp4_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(PKG / "libmxfp4_b200.so"))
    missing = [n for n in _declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing
    lib.mxfp4_abi_version.restype = ctypes.c_int
    assert lib.mxfp4_abi_version() == 1


def test_operator_module_binds_every_declared_symbol():
    assert set(_declared_symbols()) <= set(soft._SIGNATURES)
    soft._load_library()


def test_e2m1_table_matches_reference_constants():
    assert soft._MXFP4_E2M1_VALUES == (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                                       -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0)


def test_safe_backend_is_default(monkeypatch):
    monkeypatch.delenv("MXFP4_GFX936_BACKEND", raising=False)
    assert soft._backend() == "safe"


@pytest.mark.parametrize("value,expected", [("safe", "safe"), ("fused", "fused"), ("triton", "triton")])
def test_explicit_backend_values(monkeypatch, value, expected):
    monkeypatch.setenv("MXFP4_GFX936_BACKEND", value)
    assert soft._backend() == expected


def test_unknown_backend_fails_loud(monkeypatch):
    monkeypatch.setenv("MXFP4_GFX936_BACKEND", "unknown")
    with pytest.raises(ValueError, match="unknown gfx936 MXFP4 backend"):
        soft._backend()


def test_native_library_required(monkeypatch):
    monkeypatch.setattr(soft, "_has_compatible_native_library", lambda: False)
    with pytest.raises(RuntimeError, match="MXFP4_B200_LIBRARY"):
        soft._require_native_library()


def test_no_cpu_fallback():
    x = torch.randn(2, 128, dtype=torch.bfloat16)
    w = torch.zeros(64, 64, dtype=torch.uint8)
    s = torch.full((64, 4), 127, dtype=torch.uint8)
    with pytest.raises(RuntimeError, match="no CPU path|sm_100"):
        soft.linear_mxfp4_soft(x, w, s)
    with pytest.raises(RuntimeError, match="no CPU path|sm_100"):
        soft.dequant_mxfp4(w, s)


def test_dequant_validation_matches_reference():
    u8 = torch.uint8
    with pytest.raises(TypeError, match="packed must be uint8"):
        soft.dequant_mxfp4(torch.zeros(1, 16, dtype=torch.int32), torch.zeros(1, 1, dtype=u8))
    with pytest.raises(TypeError, match="block_scales must be uint8"):
        soft.dequant_mxfp4(torch.zeros(1, 16, dtype=u8), torch.zeros(1, 1))
    with pytest.raises(ValueError, match="divisible by 32"):
        soft.dequant_mxfp4(torch.zeros(1, 8, dtype=u8), torch.zeros(1, 1, dtype=u8))
    with pytest.raises(ValueError, match="leading dimensions"):
        soft.dequant_mxfp4(torch.zeros(2, 16, dtype=u8), torch.zeros(3, 1, dtype=u8))
    with pytest.raises(ValueError, match="every 32"):
        soft.dequant_mxfp4(torch.zeros(1, 16, dtype=u8), torch.zeros(1, 2, dtype=u8))


def test_linear_validation_matches_reference():
    u8 = torch.uint8
    w = torch.zeros(64, 64, dtype=u8)
    s = torch.zeros(64, 4, dtype=u8)
    with pytest.raises(TypeError, match="fp16 or bf16"):
        soft.linear_mxfp4_soft(torch.zeros(2, 128), w, s)
    with pytest.raises(TypeError, match="must be uint8"):
        soft.linear_mxfp4_soft(torch.zeros(2, 128, dtype=torch.bfloat16), w.int(), s)
    with pytest.raises(ValueError, match="2D"):
        soft.linear_mxfp4_soft(torch.zeros(2, 128, dtype=torch.bfloat16), w[None], s)
    with pytest.raises(ValueError, match="does not match weight K"):
        soft.linear_mxfp4_soft(torch.zeros(2, 256, dtype=torch.bfloat16), w, s)
    with pytest.raises(ValueError, match="divisible by 128"):
        soft.linear_mxfp4_soft(torch.zeros(2, 64, dtype=torch.bfloat16), w[:, :32], s[:, :2])
    with pytest.raises(ValueError, match="every 32"):
        soft.linear_mxfp4_soft(torch.zeros(2, 128, dtype=torch.bfloat16), w, s[:, :3])


def _moe_args(**over):
    m, k, n, e, top_k = 4, 128, 64, 4, 2
    args = dict(
        A=torch.zeros(m, k, dtype=torch.bfloat16), B=torch.zeros(e, n, k // 2, dtype=torch.uint8),
        C=torch.zeros(m, top_k, n, dtype=torch.bfloat16), A_scale=torch.ones(1), B_scale=torch.ones(e),
        A_mx_scale=None, B_mx_scale=torch.zeros(e, n, k // 32, dtype=torch.uint8),
        topk_weights=torch.ones(m, top_k), topk_ids=torch.zeros(m, top_k, dtype=torch.int64),
        sorted_token_ids=torch.empty(0), expert_ids=torch.empty(0), num_tokens_post_padded=torch.empty(0),
        mul_routed_weight=False, top_k=top_k, swizzle_mx_a=False, swizzle_mx_b=False)
    args.update(over)
    return args


def test_swizzled_scales_fail_loud():
    with pytest.raises(NotImplementedError, match="swizzled scales"):
        soft.fused_moe_mxfp4_soft(**_moe_args(swizzle_mx_a=True))
    with pytest.raises(NotImplementedError, match="swizzled scales"):
        soft.fused_moe_mxfp4_soft(**_moe_args(swizzle_mx_b=True))


def test_moe_validation_matches_reference():
    with pytest.raises(ValueError, match="matching"):
        soft.fused_moe_mxfp4_soft(**_moe_args(topk_weights=torch.ones(4, 3)))
    with pytest.raises(TypeError, match="packed MXFP4 weights"):
        soft.fused_moe_mxfp4_soft(**_moe_args(B=torch.zeros(4, 64, 64)))
    with pytest.raises(TypeError, match="compute dtype"):
        soft.fused_moe_mxfp4_soft(**_moe_args(C=torch.zeros(4, 2, 64, dtype=torch.int32)))
    with pytest.raises(ValueError, match="require A_mx_scale"):
        soft.fused_moe_mxfp4_soft(**_moe_args(A=torch.zeros(4, 64, dtype=torch.uint8)))
    with pytest.raises(ValueError, match="must not provide A_mx_scale"):
        soft.fused_moe_mxfp4_soft(**_moe_args(A_mx_scale=torch.zeros(4, 4, dtype=torch.uint8)))
    with pytest.raises(RuntimeError, match="no CPU path|sm_100"):
        soft.fused_moe_mxfp4_soft(**_moe_args())


def test_unknown_backend_rejected_by_ops(monkeypatch):
    monkeypatch.setenv("MXFP4_GFX936_BACKEND", "bogus")
    with pytest.raises(ValueError, match="unknown gfx936 MXFP4 backend"):
        soft.linear_mxfp4_soft(torch.zeros(2, 128, dtype=torch.bfloat16),
                               torch.zeros(64, 64, dtype=torch.uint8), torch.zeros(64, 4, dtype=torch.uint8))


def test_router_argument_checks_on_cpu():
    # the router rejects bad shapes, dtypes and sizes before it needs a GPU
    soft = soft_module()
    with pytest.raises(ValueError):
        soft.moe_router(torch.randn(8), 2)
    with pytest.raises(TypeError):
        soft.moe_router(torch.randn(4, 8, dtype=torch.float64), 2)
    with pytest.raises(ValueError):
        soft.moe_router(torch.randn(4, 300), 2)
    with pytest.raises(ValueError):
        soft.moe_router(torch.randn(4, 8), 9)
    with pytest.raises(ValueError):
        soft.moe_router(torch.randn(4, 64), 33)
    with pytest.raises(RuntimeError, match="no CPU path|sm_100"):
        soft.moe_router(torch.randn(4, 8), 2)  # valid arguments, but no CPU path


def _padded_rows(counts, block):
    return int(sum(-(-int(c) // block) * block for c in counts))


def test_routing_and_ep_capacities_hold_every_layout():
    # the capacities size device buffers before the routes are known: they must
    # hold the padded layout of any distribution of the routes over the experts
    lib = soft._load_library()
    rng = np.random.default_rng(0)
    for routes, experts, block in [(32768, 128, 128), (4096, 64, 256), (7, 3, 128), (0, 8, 64), (100, 1, 256)]:
        cap = lib.mxfp4_moe_route_capacity(routes, experts, block)
        assert cap % block == 0
        for dist_ in (rng.multinomial(routes, np.ones(experts) / experts), np.eye(experts, dtype=int)[0] * routes):
            assert _padded_rows(dist_, block) <= cap
    for t, k, e, world in [(512, 8, 128, 8), (2048, 8, 128, 2), (1, 1, 4, 4), (300, 4, 32, 1), (8, 8, 128, 8)]:
        cap = lib.mxfp4_ep_moe_recv_capacity(t, k, e, world)
        el = e // world
        # the owner pads every local expert to 256 rows (CTA-pair GEMM) when the
        # ranks' routes average 128 or more per local expert, else to 32 rows;
        # the layer reads the block back from the capacity (>= 383 rows per
        # local expert <=> 256-row blocks)
        block = 256 if world * t * k >= 128 * el else 32
        assert cap % block == 0
        assert (cap >= 383 * el) == (block == 256)
        # worst case for one owner: every route of every rank lands on its experts
        for dist_ in (rng.multinomial(world * t * k, np.ones(el) / el), np.eye(el, dtype=int)[0] * world * t * k):
            assert _padded_rows(dist_, block) <= cap
    assert lib.mxfp4_ep_moe_recv_capacity(10, 2, 10, 4) == 0  # experts must divide over the ranks
    assert lib.mxfp4_ep_moe_recv_capacity(-1, 2, 8, 4) == 0


def test_noalloc_checks_arguments_before_sizing_its_scratch():
    # a bad K or dtype is an invalid argument, not a scratch overflow; both
    # answers come from host validation before any device call
    lib = soft._load_library()
    null = ctypes.c_void_p(0)
    BF16, F32, I64 = 1, 0, 5

    def call(t, k, a_dtype=BF16, c_dtype=BF16, n=256):
        return lib.mxfp4_fused_moe_noalloc(null, a_dtype, null, null, null, null, null, null, F32, null, I64, null,
                                           c_dtype, t, 2, 8, n, k, 0, null)

    assert call(8, -128) == 1
    assert call(8, 100) == 1
    assert call(8, 128, a_dtype=7) == 1
    assert call(8, 128, c_dtype=3) == 1
    assert call(8, 128, n=0) == 1
    assert call(1 << 20, 128) == 5  # a valid request whose scratch exceeds the static array


def test_probe_library_exports_its_header():
    # the benchmark's tensor-core rate probe is a separate library with its own header
    text = (ROOT / "include" / "mxfp4_b200_probe.h").read_text()
    names = re.findall(r"^\s*int\s+(mxfp4_\w+)\s*\(", text, re.M)
    assert names == ["mxfp4_probe_mma_rate"]
    lib = ctypes.CDLL(str(PKG / "libmxfp4_b200_probe.so"))
    assert all(hasattr(lib, n) for n in names)
    # argument checks answer before any device call
    fn = lib.mxfp4_probe_mma_rate
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    assert fn(7, 10, None, None, None) == 1


def test_noalloc_limits_stated_in_the_header_hold():
    # include/mxfp4_b200.h states what the 8 MiB static scratch of
    # mxfp4_fused_moe_noalloc admits with BF16 A and C, 128 experts and top-8:
    # up to 7 tokens at K = 2048 and 112 at K = 768; the entry point compares
    # the workspace size of the call with the array's size
    lib = ctypes.CDLL(str(PKG / "libmxfp4_b200.so"))
    size = lib.mxfp4_fused_moe_workspace_size
    size.restype = ctypes.c_size_t
    size.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                     ctypes.c_int]
    BF16, limit = 1, 8 << 20
    for k, n, most in [(2048, 1536, 7), (768, 2048, 112)]:
        assert all(size(t, 8, 128, n, k, BF16, BF16) <= limit for t in range(1, most + 1))
        assert size(most + 1, 8, 128, n, k, BF16, BF16) > limit
    text = (ROOT / "include" / "mxfp4_b200.h").read_text()
    assert "up to 7 tokens at K = 2048 and 112" in text
