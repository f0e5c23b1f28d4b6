"""The allocation-free routed-MoE entry point, called through the C ABI.

``mxfp4_fused_moe_noalloc`` serves callers that cannot allocate device memory
when they call in (a plugin host or graph executor that owns all buffers, or a
fixed memory plan replayed under stream capture): it takes its routing scratch
from a static 8 MiB device array instead of a caller workspace.  Each call must
give the same output as ``mxfp4_fused_moe`` with a caller workspace; two calls
in a row with different routings check that nothing stale carries over from the
shared scratch.  This file is collected last so that a failure here does not
stop a ``-x`` run before the other tests ran; it also passes on its own in a
fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

from _paths import PKG, oracle

pytestmark = pytest.mark.gpu

F32, BF16, U8, I32, I64 = 0, 1, 3, 4, 5
ERR_WORKSPACE = 5


def _lib():
    lib = ctypes.CDLL(str(PKG / "libmxfp4_b200.so"))
    vp, i, i64, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
    lib.mxfp4_fused_moe.restype = i
    lib.mxfp4_fused_moe.argtypes = [vp, i, vp, vp, vp, vp, vp, vp, i, vp, i, vp, i, i64, i, i, i64, i64, i, vp, sz, vp]
    lib.mxfp4_fused_moe_noalloc.restype = i
    lib.mxfp4_fused_moe_noalloc.argtypes = [vp, i, vp, vp, vp, vp, vp, vp, i, vp, i, vp, i, i64, i, i, i64, i64, i, vp]
    lib.mxfp4_fused_moe_workspace_size.restype = sz
    lib.mxfp4_fused_moe_workspace_size.argtypes = [i64, i, i, i64, i64, i, i]
    lib.mxfp4_last_error.restype = ctypes.c_char_p
    return lib


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _case(seed, m, n, k, e, top_k):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(torch.bfloat16)
    b = torch.randint(0, 256, (e, n, k // 2), generator=g, dtype=torch.uint8)
    bmx = torch.randint(116, 130, (e, n, k // 32), generator=g, dtype=torch.uint8)
    ids = torch.randint(0, e + 1, (m, top_k), generator=g, dtype=torch.int64)  # id e is dropped
    tw = torch.rand(m, top_k, generator=g)
    a_scale = torch.tensor([0.75])
    b_scale = torch.linspace(0.5, 1.25, e)
    return [t.cuda() for t in (a, b, bmx, ids, tw, a_scale, b_scale)]


def _call(lib, case, workspace):
    a, b, bmx, ids, tw, a_scale, b_scale = case
    m, k = a.shape
    e, n = b.shape[0], b.shape[1]
    top_k = ids.shape[1]
    c = torch.full((m, top_k, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    common = (_p(a), BF16, None, _p(b), _p(bmx), _p(a_scale), _p(b_scale), _p(tw), F32, _p(ids), I64, _p(c), BF16,
              m, top_k, e, n, k, 1)
    if workspace is None:
        rc = lib.mxfp4_fused_moe_noalloc(*common, stream)
    else:
        ws = torch.empty(lib.mxfp4_fused_moe_workspace_size(m, top_k, e, n, k, BF16, BF16), dtype=torch.uint8,
                         device="cuda")
        rc = lib.mxfp4_fused_moe(*common, _p(ws), ws.numel(), stream)
    assert rc == 0, lib.mxfp4_last_error()
    torch.cuda.synchronize()
    return c


def test_noalloc_matches_workspace_entry_on_two_calls_in_a_row():
    lib = _lib()
    O = oracle()
    cases = [_case(1, 300, 320, 512, 16, 4), _case(2, 77, 256, 256, 8, 2)]
    for case in cases:
        got = _call(lib, case, None)
        want = _call(lib, case, "workspace")
        # same kernels, same order: identical bits
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
        a, b, bmx, ids, tw, a_scale, b_scale = (t.cpu() for t in case)
        ref = O.moe_op(a.float().numpy(), "bf16", None, b.numpy(), bmx.numpy(), a_scale.numpy(), b_scale.numpy(),
                       tw.numpy(), ids.numpy(), True, "bf16")
        ok, err, bound, rel = O.check_close(got.float().cpu().numpy(), ref)
        assert ok, (err, bound, rel)
        assert np.all(got.float().cpu().numpy()[ids.numpy() == b.shape[0]] == 0)


def test_noalloc_rejects_requests_beyond_its_static_scratch():
    lib = _lib()
    a = torch.zeros(8, 128, dtype=torch.bfloat16, device="cuda")
    # 2M routes need ~16 MB of routing scratch, above the 8 MiB static array
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.mxfp4_fused_moe_noalloc(_p(a), BF16, None, _p(a), _p(a), _p(a), _p(a), _p(a), F32, _p(a), I64, _p(a),
                                     BF16, 1 << 20, 2, 128, 256, 128, 0, stream)
    assert rc == ERR_WORKSPACE
    assert b"static" in lib.mxfp4_last_error()
