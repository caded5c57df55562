"""Pins the C oracle against the reference's own known answers and properties.

No GPU: these checks decide whether the oracle can be trusted as the parity
reference for the CUDA kernels.
"""

import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as orc
from tests import conformance as cf

GOLDEN = json.loads((Path(__file__).parent / "golden" / "golden.json").read_text())["cases"]


def _vals(spec):
    return np.array([float(x) for x in spec["values"]], np.float32).reshape(spec["dims"])


@pytest.mark.parametrize("case", [c for c in GOLDEN if c["op"] == "conv"], ids=lambda c: c["id"])
def test_conv_known_answers(case):
    o = case["options"]
    out = orc.conv(_vals(case["input"]), _vals(case["weight"]), o["strides"], o["dilations"], o["padding_before"],
                   o["padding_after"], o["groups"])
    assert list(out.shape) == case["out_dims"]
    assert out.reshape(-1).tolist() == [float(x) for x in case["expected"]]
    seq = orc.conv_f32_seq(_vals(case["input"]), _vals(case["weight"]), o["strides"], o["dilations"],
                           o["padding_before"], o["padding_after"], o["groups"])
    assert seq.reshape(-1).tolist() == [float(x) for x in case["expected"]]


@pytest.mark.parametrize("case", [c for c in GOLDEN if c["op"] == "conv_plan"], ids=lambda c: c["id"])
def test_conv_geometry_known_answers(case):
    o = case["options"]
    assert orc.conv_dims(case["input_dims"], case["weight_dims"], o["strides"], o["dilations"], o["padding_before"],
                         o["padding_after"]) == case["out_dims"]


@pytest.mark.parametrize("case", [c for c in GOLDEN if c["op"] == "attention"], ids=lambda c: c["id"])
def test_attention_known_answers(case):
    mask = None
    if case["mask"]:
        mask = np.array([float(x) for x in case["mask"]["values"]], np.float64).reshape(case["mask"]["dims"])
    out = orc.attention(_vals(case["q"]), _vals(case["k"]), _vals(case["v"]), mask, case["scale"], case["causal"])
    assert list(out.shape) == case["out_dims"]
    flat = out.reshape(-1)
    if "expected" in case:
        assert flat.tolist() == [float(x) for x in case["expected"]]
    else:
        exp = case["expected_prefix"]
        assert np.allclose(flat[: len(exp)], exp, rtol=0, atol=1e-5)


def test_reduction_known_answers():
    for case in (c for c in GOLDEN if c["op"] == "reduce_f32"):
        got = orc.reduce_f32(_vals(case["input"]), case["axes"], case["reduce"])
        assert got.reshape(-1).tolist() == np.array(case["expected"], np.float32).tolist(), case["id"]
    case = next(c for c in GOLDEN if c["op"] == "reduce_prime_tail")
    n = case["n"]
    values = np.ones(n, np.float32)
    values[17] = -1.0
    values[n - 1] = 2.0
    exp = case["expected"]
    for op, key in enumerate(("sum", "product", "min", "max")):
        assert orc.reduce_f32(values, [0], op).reshape(-1).tolist() == [np.float32(exp[key])]
    mean = np.float32(orc.reduce_f32(values, [0], 0).reshape(-1)[0]) / np.float32(n)
    assert mean == np.float32(exp["mean"])
    case = next(c for c in GOLDEN if c["op"] == "reduce_broadcast")
    scalar = np.broadcast_to(np.float32(1.25), (3, 2, 5))
    s = orc.reduce_f32(scalar, [0, 2], 0) / np.float32(15)
    assert s.tolist() == case["expected"]["mean_02_keep"]
    assert orc.reduce_f32(scalar, [1], 1).reshape(-1).tolist() == case["expected"]["product_1"]
    u = np.full((2, 3), 0xFFFFFFFF, np.uint32)
    assert orc.reduce_u32(u, [1], 0).tolist() == case["expected"]["u32_sum"]


def test_statistics_and_argmax_known_answers():
    case = next(c for c in GOLDEN if c["op"] == "softmax")
    st = orc.stats(_vals(case["input"]), case["axes"], 1e-5)
    assert np.allclose(st["softmax"][1], case["expected_row1"], atol=1e-6)
    assert abs(st["softmax"][0].sum() - 1.0) < 1e-6
    assert np.allclose(np.log(st["softmax"]), st["log_softmax"], atol=1e-5)
    case = next(c for c in GOLDEN if c["op"] == "layer_norm")
    st = orc.stats(_vals(case["input"]), case["axes"], case["eps"])
    assert np.allclose(st["norm"][1], case["expected_row1"], atol=1e-6)
    row0 = st["norm"][0].astype(np.float64)
    assert abs(row0.mean()) < 1e-6 and abs((row0 * row0).mean() - 1.0) < 1e-4
    case = next(c for c in GOLDEN if c["op"] == "argmax")
    assert orc.argmax_rows(_vals(case["input"])).tolist() == case["expected"]


def test_argmax_total_order_and_ties():
    x = np.array([[0.0, -0.0, 0.0], [-0.0, 0.0, -1.0], [3.0, 3.0, 3.0], [-np.inf, -5.0, -5.0]], np.float32)
    assert orc.argmax_rows(x).tolist() == [0, 1, 0, 1]


def test_low_rounding_witness():
    case = next(c for c in GOLDEN if c["op"] == "conv_low")
    x = _vals(case["input"])
    w = _vals(case["weight"])
    bits = orc.round_bits(x, "bf16")
    xd = orc.decode_bits(bits, "bf16")
    wd = orc.decode_bits(orc.round_bits(w, "bf16"), "bf16")
    out = orc.conv_f32_seq(xd, wd, [1], [1], [0], [0])
    assert out.reshape(-1).tolist() == [np.float32(v) for v in case["expected_f32"]]
    # The witness exposes premature low rounding (low.rs:89-93).
    once = orc.decode_bits(orc.round_bits(out, "bf16"), "bf16")
    assert float(once.reshape(-1)[0]) != case["expected_f32"][0]


def test_low_codec_matches_nearest_even():
    import torch

    rng = np.random.default_rng(7)
    x = np.concatenate([rng.standard_normal(4000).astype(np.float32) * 10,
                        np.array([0.0, -0.0, 1e-40, -1e-40, 3e38, -3e38, 65504.0, 65520.0, 1e-8], np.float32)])
    for name, dt in (("bf16", torch.bfloat16), ("f16", torch.float16)):
        want = torch.from_numpy(x).to(dt).view(torch.int16).numpy().view(np.uint16)
        assert (orc.round_bits(x, name) == want).all(), name
        finite = [b for b in range(0, 0x7C00 if name == "f16" else 0x7F80, 97)]
        dec = orc.decode_bits(np.array(finite, np.uint16), name)
        ref = torch.from_numpy(np.array(finite, np.uint16).view(np.int16)).view(dt).float().numpy()
        assert (dec == ref).all(), name


def test_conv_conformance_cases_are_exact_in_f32():
    """Dyadic fixtures: every partial sum is exact, so the f32 sequential
    oracle must equal the f64 oracle (the premise of conformance/
    convolution.rs:243-258)."""
    for case in cf.conv_cases():
        x, w = case.input.logical(), case.weight.logical()
        f64 = orc.conv(x, w, case.strides, case.dilations, case.padding_before, case.padding_after, case.groups)
        f32 = orc.conv_f32_seq(x, w, case.strides, case.dilations, case.padding_before, case.padding_after,
                               case.groups)
        assert f64.shape == f32.shape
        assert (f64 == f32.astype(np.float64)).all()


def test_conv_inexact_case_within_reference_bound():
    """The 65-tap inexact case (conformance/convolution.rs:259-280)."""
    x = np.array([(i - 30.0) / 37.0 for i in range(65)], np.float32)
    w = np.array([((i * 17) % 31) / 23.0 - 0.7 for i in range(65)], np.float32)
    exp = 0.0
    absolute = 0.0
    for a, b in zip(x.tolist(), w.tolist()):  # sequential f64 sum, as .sum::<f64>()
        exp += a * b
        absolute += abs(a * b)
    got = orc.conv_f32_seq(x.reshape(1, 1, 65), w.reshape(1, 1, 65), [1], [1], [0], [0]).reshape(-1)[0]
    assert abs(float(got) - exp) <= 2e-5 * absolute
    assert orc.conv(x.reshape(1, 1, 65), w.reshape(1, 1, 65), [1], [1], [0], [0]).reshape(-1)[0] == exp


def test_attention_oracle_threads_agree():
    case = cf.attention_cases()[4]
    a = orc.attention(case.q.logical(), case.k.logical(), case.v.logical(), nthreads=1)
    b = orc.attention(case.q.logical(), case.k.logical(), case.v.logical(), nthreads=4)
    assert (a == b).all()


def test_statistics_oracle_huge_offsets_finite():
    for row in cf.huge_offset_rows():
        st = orc.stats(row, [0], 1e-5)
        # Layer norm stays usable even when the reported variance overflows
        # (conformance/statistics.rs:412-430); log-probabilities may overflow.
        assert np.isfinite(st["norm"]).all() and np.isfinite(st["mean"]).all()


def test_reference_kernel_metadata_matches_the_references_own_unit_tests():
    """The second oracle's restated descriptors against the values the
    reference's own unit tests assert (compute-cuda/src/convolution.rs:171-189,
    reduction/dispatch.rs:195-199), and the attention descriptor's bounds."""
    from oracle import ref_kernels as ref

    meta, out_sp = ref.conv_metadata([2, 4, 5, 7], [140, 35, 7, 1], 11, [6, 2, 2, 3], [12, 6, 3, 1], 3,
                                     [2, 1], [1, 2], [1, 2], [0, 1], groups=2)
    assert out_sp == [3, 6]
    assert meta[:11] == [2, 2, 3, 6, 11, 3, 140, 35, 12, 6, 6]
    assert meta[11:] == [5, 7, 3, 6, 2, 3, 7, 1, 3, 1, 2, 1, 1, 2, 1, 2]
    assert ref.reduce_metadata([3, 5, 2], [1, 0, 3], [2, 0]) == [5, 0, 2, 3, 3, 1]
    # attention: every Q/K/V address the kernel forms stays inside the views
    q_shape, q_str, k_str, v_str = [2, 4, 70, 48], [13440, 3360, 48, 1], [8640, 4320, 48, 1], [5940, 2970, 33, 1]
    m = ref.attention_metadata(q_shape, q_str, 0, k_str, 0, v_str, 0, 2)
    rank, tail = 3, m[15:]
    dims = m[:3]

    def base(row, strides, offset, group):
        for d in (2, 1, 0):
            c = row % dims[d]
            row //= dims[d]
            if d == rank - 2:
                c //= group
            offset += c * strides[d]
        return offset

    rows = 2 * 4 * 70
    assert max(base(r, m[3:6], tail[0], 1) for r in range(rows)) + 47 * tail[4] < 2 * 4 * 70 * 48
    assert max(base(r, m[6:9], tail[1], tail[10]) for r in range(rows)) + 89 * tail[5] + 47 * tail[6] < 2 * 2 * 90 * 48
    assert max(base(r, m[9:12], tail[2], tail[10]) for r in range(rows)) + 89 * tail[7] + 32 * tail[8] < 2 * 2 * 90 * 33
