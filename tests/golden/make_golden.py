"""Generate the golden fixtures under tests/golden/ from the reference's own code.

Run in a container that has the reference checkout, with
``MXFP4_REFERENCE_ROOT`` set to its root directory::

    MXFP4_REFERENCE_ROOT=/path/to/reference python tests/golden/make_golden.py

The GPU box never runs this script; it only reads the ``.npz`` files it
writes.  What comes from where (paths relative to the reference root):

* the operator module ``src/aiter/ops/triton/moe_op_mxfp4_soft.py`` is loaded
  by file path exactly as the reference test does (test:10-19) and its
  ``safe`` backend runs on CPU tensors;
* the test quantizer ``torch_dynamic_mxfp4_quant`` is taken from the reference
  test module ``tests/test_moe_mxfp4_soft.py`` (test:28-60);
* ``_make_routing`` (vllm:119-146), ``_moe_apply`` (vllm:233-265),
  ``_moe_gemm`` (vllm:149-185) and ``_reference_dequant`` (vllm:73-91) are
  compiled from ``integration/vllm/vllm_mxfp4_gfx936.py`` by extracting those
  function definitions with ``ast`` (the module itself needs vLLM 0.15 and
  cannot be imported here); ``unpack_fp4_from_uint8`` comes from the installed
  compressed-tensors (0.15.0.1, ``compressors/nvfp4/helpers.py``).

Seeds: torch.manual_seed(20260810 + M) for the MoE op cases, 20260811 + M for
the linear cases, 20260812 for the 2048-K cases, as in the reference tests
(test:98, :115, :145, :220) but drawn on the CPU generator.
"""

from __future__ import annotations

import ast
import importlib.util
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REF = Path(os.getenv("MXFP4_REFERENCE_ROOT", ""))


def _load_by_path(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def load_reference():
    soft = _load_by_path("ref_moe_op_mxfp4_soft", REF / "src/aiter/ops/triton/moe_op_mxfp4_soft.py")
    os.environ["MXFP4_SOFT_MODULE"] = str(REF / "src/aiter/ops/triton/moe_op_mxfp4_soft.py")
    ref_test = _load_by_path("ref_test_moe_mxfp4_soft", REF / "tests/test_moe_mxfp4_soft.py")
    from compressed_tensors.compressors.nvfp4.helpers import unpack_fp4_from_uint8

    src_path = REF / "integration/vllm/vllm_mxfp4_gfx936.py"
    tree = ast.parse(src_path.read_text())
    wanted = {"_make_routing", "_moe_gemm", "_moe_apply", "_reference_dequant", "_bf16_moe_gemm"}
    body = [node for node in tree.body if isinstance(node, ast.FunctionDef) and node.name in wanted]
    module = ast.Module(body=body, type_ignores=[])
    ns = {"torch": torch, "F": F, "soft": soft, "_official_unpack_fp4": unpack_fp4_from_uint8,
          "_IMPLEMENTATION": "safe"}
    exec(compile(module, str(src_path), "exec"), ns)
    vllm_fns = types.SimpleNamespace(**{k: ns[k] for k in wanted})
    return soft, ref_test, vllm_fns


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def as_bits(t: torch.Tensor) -> np.ndarray:
    """Store any float tensor as its raw bits (uint16 / uint32)."""
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.float32:
        return t.contiguous().view(torch.int32).numpy().view(np.uint32).copy()
    raise TypeError(t.dtype)


def main() -> None:
    if not os.getenv("MXFP4_REFERENCE_ROOT"):
        raise SystemExit("set MXFP4_REFERENCE_ROOT to the reference checkout's root directory")
    soft, ref_test, vf = load_reference()
    os.environ["MXFP4_GFX936_BACKEND"] = "safe"
    quant = ref_test.torch_dynamic_mxfp4_quant
    out = {}

    # 1. dequant: all 16 codes in both nibble positions x all 256 scale codes
    row = torch.tensor([i | ((15 - i) << 4) for i in range(16)], dtype=torch.uint8)
    packed = row.repeat(256, 1)
    scales = torch.arange(256, dtype=torch.int32).to(torch.uint8).reshape(256, 1)
    dq = {"packed": packed.numpy(), "scales": scales.numpy()}
    for name, dt in (("fp32", torch.float32), ("bf16", torch.bfloat16), ("fp16", torch.float16)):
        dq[f"out_{name}"] = as_bits(soft.dequant_mxfp4(packed, scales, dt))
    # the reference's own known-answer vector (test:81-92)
    kat = torch.tensor([[c | ((c + 1) << 4) for c in range(0, 16, 2)] * 2], dtype=torch.uint8)
    dq["kat_packed"] = kat.numpy()
    dq["kat_out"] = as_bits(soft.dequant_mxfp4(kat, torch.full((1, 1), 127, dtype=torch.uint8)))
    dq["e2m1_values"] = np.asarray(soft._MXFP4_E2M1_VALUES, dtype=np.float32)
    np.savez_compressed(HERE / "dequant.npz", **dq)

    # 2. reference test quantizer on seeded inputs
    torch.manual_seed(1234)
    xq = torch.randn(16, 256) * torch.logspace(-3, 3, 16).reshape(16, 1)
    xq[3, :32] = 0.0                         # an all-zero block
    xq[5, 40] = 1e-30                        # a tiny value
    p, s = quant(xq)
    np.savez_compressed(HERE / "quant_test.npz", x=xq.numpy(), packed=p.numpy(), scales=s.numpy())

    # 3. safe linear (soft:310-376), BF16 and FP16, with and without bias
    cases = {}
    for idx, (m, n, k, seed, dt, with_bias) in enumerate([
        (1, 64, 128, 20260812, torch.bfloat16, False),
        (8, 64, 128, 20260819, torch.bfloat16, False),
        (16, 256, 2048, 20260811, torch.bfloat16, False),
        (5, 96, 256, 7, torch.bfloat16, True),
        (8, 64, 128, 11, torch.float16, False),
        (3, 64, 256, 13, torch.float16, True),
    ]):
        torch.manual_seed(seed)
        x = torch.randn(m, k, dtype=dt)
        w = torch.randn(n, k, dtype=dt)
        wp, ws = quant(w)
        bias = torch.randn(n, dtype=dt) if with_bias else None
        y = soft.linear_mxfp4_soft(x, wp, ws, bias)
        pre = f"c{idx}_"
        cases[pre + "x"] = as_bits(x)
        cases[pre + "w"] = wp.numpy()
        cases[pre + "s"] = ws.numpy()
        cases[pre + "y"] = as_bits(y)
        cases[pre + "dtype"] = np.array("bf16" if dt == torch.bfloat16 else "fp16")
        if bias is not None:
            cases[pre + "bias"] = as_bits(bias)
    np.savez_compressed(HERE / "linear.npz", **cases)

    # 4. safe MoE op: the reference's 20-case matrix (test:216-285) on CPU
    moe = {}
    for m in (1, 2, 4, 8, 64):
        for qa in (False, True):
            for mrw in (False, True):
                torch.manual_seed(20260810 + m)
                n, k, e, top_k = 64, 128, 4, 2
                a = torch.randn(m, k, dtype=torch.bfloat16)
                wts = torch.randn(e, n, k, dtype=torch.bfloat16)
                bp, bs = quant(wts)
                if qa:
                    ka, kas = quant(a)
                else:
                    ka, kas = a, None
                logits = torch.randn(m, e, dtype=torch.float32)
                tw, tid = torch.topk(torch.softmax(logits, dim=-1), k=top_k, dim=-1)
                c = torch.empty(m, top_k, n, dtype=torch.bfloat16)
                sa = torch.tensor([0.75], dtype=torch.float32)
                sb = torch.linspace(0.5, 1.25, e)
                empty = torch.empty(0)
                soft.fused_moe_mxfp4_soft(ka, bp, c, sa, sb, kas, bs, tw, tid,
                                          empty, empty, empty, mrw, top_k, False, False)
                pre = f"m{m}_q{int(qa)}_w{int(mrw)}_"
                moe[pre + "a"] = as_bits(a) if not qa else ka.numpy()
                if qa:
                    moe[pre + "a_mx"] = kas.numpy()
                moe[pre + "b"] = bp.numpy()
                moe[pre + "b_mx"] = bs.numpy()
                moe[pre + "tw"] = tw.numpy()
                moe[pre + "tid"] = tid.numpy()
                moe[pre + "c"] = as_bits(c)
    np.savez_compressed(HERE / "moe_op.npz", **moe)

    # 5. routing metadata (vllm:119-146)
    rt = {}
    g = torch.Generator().manual_seed(99)
    for idx, (t, top_k, e, bm) in enumerate([(16, 2, 4, 64), (333, 8, 32, 64), (1000, 8, 128, 128),
                                              (7, 4, 16, 16), (64, 1, 8, 32)]):
        logits = torch.randn(t, e, generator=g)
        ids = torch.topk(logits, k=top_k, dim=-1).indices.to(torch.int32)
        sid, eid, npp = vf._make_routing(ids, block_m=bm)
        pre = f"r{idx}_"
        rt[pre + "ids"] = ids.numpy()
        rt[pre + "block_m"] = np.array(bm)
        rt[pre + "num_experts"] = np.array(e)
        rt[pre + "sorted"] = sid.numpy()
        rt[pre + "experts"] = eid.numpy()
        rt[pre + "post"] = npp.numpy()
    np.savez_compressed(HERE / "routing.npz", **rt)

    # 6. MoE layer composition (vllm:233-265) with the safe op
    torch.manual_seed(20260901)
    t, h, e, top_k, inter = 24, 256, 8, 2, 128
    x = torch.randn(t, h, dtype=torch.bfloat16)
    w13 = torch.randn(e, 2 * inter, h, dtype=torch.bfloat16)
    w2 = torch.randn(e, h, inter, dtype=torch.bfloat16) * 0.1
    p13, s13 = quant(w13)
    p2, s2 = quant(w2)
    logits = torch.randn(t, e)
    tw, tid = torch.topk(torch.softmax(logits, dim=-1), k=top_k, dim=-1)
    tw = tw / tw.sum(dim=-1, keepdim=True)
    layer = types.SimpleNamespace(activation="silu", w13_weight=p13, w13_weight_scale=s13,
                                  w2_weight=p2, w2_weight_scale=s2)
    y = vf._moe_apply(None, layer, x, tw, tid)
    np.savez_compressed(HERE / "moe_layer.npz", x=as_bits(x), w13=p13.numpy(), s13=s13.numpy(),
                        w2=p2.numpy(), s2=s2.numpy(), tw=tw.numpy(), tid=tid.numpy(), y=as_bits(y))

    # 7. compressed-tensors independent dequant (vllm:73-91) on a small weight
    torch.manual_seed(5)
    wq = torch.randn(32, 128)
    pq, sq = quant(wq)
    sq[0, 0] = 255
    sq[1, 1] = 0
    sq[2, 2] = 254
    ref_dq = vf._reference_dequant(pq, sq, torch.float32)
    np.savez_compressed(HERE / "ct_dequant.npz", packed=pq.numpy(), scales=sq.numpy(), out=as_bits(ref_dq))

    for f in sorted(HERE.glob("*.npz")):
        print(f"{f.name}: {f.stat().st_size} bytes")


if __name__ == "__main__":
    sys.exit(main())
