"""Pin the CPU oracle against the reference's own outputs (CPU only).

The fixtures in tests/golden/ were produced by running the reference's code
(tests/golden/make_golden.py).  Integer/byte work and dequantisation must match
bit for bit; the GEMM-shaped results differ from the reference's CPU BLAS only
by reduction order and are held to the north-star tolerance
(max|err| <= 2 BF16 ulp of max|ref|, relative Frobenius <= 1e-3).
"""

import numpy as np
import pytest

from _paths import bf16_to_f32, bits_to_f32, fp16_to_f32, golden, oracle, same_bits

O = oracle()


def _unbits(bits, dtype):
    return {"bf16": bf16_to_f32, "fp16": fp16_to_f32}.get(dtype, bits_to_f32)(bits)


def test_e2m1_table_matches_reference():
    g = golden("dequant")
    assert same_bits(O.E2M1_VALUES, g["e2m1_values"])


def test_known_answer_all_codes_scale_127():
    # test:81-92: the E2M1 table itself at scale 127, bit-exact
    g = golden("dequant")
    out = O.dequant(g["kat_packed"], np.full((1, 1), 127, np.uint8), "fp32")
    assert same_bits(out, bits_to_f32(g["kat_out"]))
    assert same_bits(out[0, :16], O.E2M1_VALUES)


@pytest.mark.parametrize("dtype", ["fp32", "bf16", "fp16"])
def test_dequant_all_codes_all_scales_bit_exact(dtype):
    g = golden("dequant")
    out = O.dequant(g["packed"], g["scales"], dtype)
    assert same_bits(out, _unbits(g[f"out_{dtype}"], dtype))


def test_dequant_matches_compressed_tensors_reference():
    # vllm:73-91, the adapter's independent dequant (unpack + ldexp)
    g = golden("ct_dequant")
    assert same_bits(O.dequant(g["packed"], g["scales"], "fp32"), bits_to_f32(g["out"]))


def test_reference_test_quantizer_bit_exact():
    g = golden("quant_test")
    p, s = O.quant_reference_test(g["x"])
    np.testing.assert_array_equal(p, g["packed"])
    np.testing.assert_array_equal(s, g["scales"])


@pytest.mark.parametrize("case", range(6))
def test_linear_within_tolerance(case):
    g = golden("linear")
    pre = f"c{case}_"
    dt = str(g[pre + "dtype"])
    x = _unbits(g[pre + "x"], dt)
    bias = _unbits(g[pre + "bias"], dt) if pre + "bias" in g.files else None
    y = O.linear(x, dt, g[pre + "w"], g[pre + "s"], bias)
    ok, err, bound, rel = O.check_close(y, _unbits(g[pre + "y"], dt))
    assert ok, (err, bound, rel)


def _moe_keys():
    return [(m, q, w) for m in (1, 2, 4, 8, 64) for q in (0, 1) for w in (0, 1)]


@pytest.mark.parametrize("m,qa,mrw", _moe_keys())
def test_moe_op_within_tolerance(m, qa, mrw):
    g = golden("moe_op")
    pre = f"m{m}_q{qa}_w{mrw}_"
    if qa:
        a, adt, amx = g[pre + "a"], "u8", g[pre + "a_mx"]
    else:
        a, adt, amx = bf16_to_f32(g[pre + "a"]), "bf16", None
    e = g[pre + "b"].shape[0]
    c = O.moe_op(a, adt, amx, g[pre + "b"], g[pre + "b_mx"], np.array([0.75], np.float32),
                 np.linspace(0.5, 1.25, e).astype(np.float32), g[pre + "tw"], g[pre + "tid"],
                 bool(mrw), "bf16")
    ok, err, bound, rel = O.check_close(c, bf16_to_f32(g[pre + "c"]))
    assert ok, (err, bound, rel)


@pytest.mark.parametrize("case", range(5))
def test_make_routing_bit_exact(case):
    g = golden("routing")
    pre = f"r{case}_"
    sid, eid, post = O.make_routing(g[pre + "ids"], int(g[pre + "block_m"]))
    np.testing.assert_array_equal(sid, g[pre + "sorted"])
    np.testing.assert_array_equal(eid, g[pre + "experts"])
    np.testing.assert_array_equal(post, g[pre + "post"])
    # the local-expert restatement agrees when every id is local
    sid2, eid2, post2 = O.route_blocks(g[pre + "ids"], int(g[pre + "num_experts"]),
                                       int(g[pre + "block_m"]))
    present = np.unique(g[pre + "ids"])
    np.testing.assert_array_equal(sid2, sid)
    np.testing.assert_array_equal(eid2, eid)
    assert set(eid2.tolist()) == set(present.tolist())


def test_moe_layer_within_tolerance():
    g = golden("moe_layer")
    y = O.moe_layer(bf16_to_f32(g["x"]), g["w13"], g["s13"], g["w2"], g["s2"], g["tw"], g["tid"])
    ok, err, bound, rel = O.check_close(y, bf16_to_f32(g["y"]))
    assert ok, (err, bound, rel)


def test_ocp_quantizer_round_trip_properties():
    # BASELINE config-3 quantizer: every element lands on the nearest grid
    # point of its block scale (ties to even), saturating at 6.
    rng = np.random.default_rng(0)
    x = rng.standard_normal((8, 256)).astype(np.float32)
    x[0, :32] = 0.0
    p, s = O.quant_ocp_rne(x)
    assert s[0, 0] == 0 and not p[0, :16].any()
    deq = O.dequant(p, s, "fp32")
    blocks = x.reshape(8, 8, 32)
    bmax = np.abs(blocks).max(-1)
    scale = np.repeat(O.scale_multipliers(s), 32, -1).reshape(8, 8, 32)
    err = np.abs(deq.reshape(8, 8, 32) - np.clip(blocks, -6 * scale, 6 * scale))
    # half the widest grid step (2) at the block scale
    assert np.all(err <= scale + 1e-30)
    nz = bmax > 0
    e = np.floor(np.log2((bmax[nz] / np.float32(6)).astype(np.float32)))
    np.testing.assert_array_equal(s[nz].astype(int), (e + 127).astype(int))
    # exact ties go to the even code
    t = np.zeros((1, 32), np.float32)
    t[0, 0] = 6.0                     # block max 6 -> scale code 127
    t[0, 1:9] = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0]
    p, s = O.quant_ocp_rne(t)
    assert s[0, 0] == 127
    got = O.dequant(p, s, "fp32")[0, 1:9]
    np.testing.assert_array_equal(got, [0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 6.0])


# --------------------------------------------------------------------------
# the PyTorch-CPU port used as bench.py's CPU baseline (oracle/ref_cpu.py)
# --------------------------------------------------------------------------
import torch  # noqa: E402

from _paths import ROOT, load_by_path  # noqa: E402

R = load_by_path("mxfp4_ref_cpu", ROOT / "oracle" / "ref_cpu.py")


@pytest.mark.parametrize("dtype", ["fp32", "bf16", "fp16"])
def test_cpu_port_dequant_bit_exact(dtype):
    g = golden("dequant")
    tdt = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}[dtype]
    out = R.dequant(torch.from_numpy(g["packed"]), torch.from_numpy(g["scales"]), tdt)
    assert same_bits(out.float().numpy(), _unbits(g[f"out_{dtype}"], dtype))


@pytest.mark.parametrize("case", range(6))
def test_cpu_port_linear(case):
    g = golden("linear")
    pre = f"c{case}_"
    dt = str(g[pre + "dtype"])
    tdt = torch.bfloat16 if dt == "bf16" else torch.float16
    x = torch.from_numpy(g[pre + "x"].view(np.int16)).view(tdt)
    bias = torch.from_numpy(g[pre + "bias"].view(np.int16)).view(tdt) if pre + "bias" in g.files else None
    y = R.linear(x, torch.from_numpy(g[pre + "w"]), torch.from_numpy(g[pre + "s"]), bias)
    ok, err, bound, rel = O.check_close(y.float().numpy(), _unbits(g[pre + "y"], dt))
    assert ok, (err, bound, rel)


def test_cpu_port_moe_layer():
    g = golden("moe_layer")
    x = torch.from_numpy(g["x"].view(np.int16)).view(torch.bfloat16)
    y = R.moe_layer(x, *(torch.from_numpy(g[k]) for k in ("w13", "s13", "w2", "s2")),
                    torch.from_numpy(g["tw"]), torch.from_numpy(g["tid"]))
    ok, err, bound, rel = O.check_close(y.float().numpy(), bf16_to_f32(g["y"]))
    assert ok, (err, bound, rel)
