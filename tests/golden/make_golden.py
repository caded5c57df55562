"""Writes tests/golden/golden.json: the reference's own known-answer vectors.

The reference is Rust and cannot be built in this image, so its known
answers are transcribed here, each with the file and line of the test that
states it.  Before writing, this script re-reads every cited reference file
and asserts that the literal it transcribes is present at the cited lines, so
a transcription error fails loudly.  Run it where the reference tree is
mounted (it is not needed to run the tests):

    python tests/golden/make_golden.py /path/to/reference
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
F32_MAX = 3.4028234663852886e38

CASES = [
    # --- convolution oracle known answers
    {
        "id": "conv_cross_correlation_default",
        "op": "conv",
        "source": "crates/tensor-core/src/conformance/convolution.rs:323-330",
        "witness": ["(&[1, 1, 4], &[1., 2., 3., 4.])", "(&[1, 1, 2], &[2., -1.])", "assert_eq!(v, [0., 1., 2.]);"],
        "input": {"dims": [1, 1, 4], "values": [1, 2, 3, 4]},
        "weight": {"dims": [1, 1, 2], "values": [2, -1]},
        "options": {"strides": [1], "dilations": [1], "padding_before": [0], "padding_after": [0], "groups": 1},
        "out_dims": [1, 1, 3],
        "expected": [0, 1, 2],
    },
    {
        "id": "conv_strided_dilated_padded",
        "op": "conv",
        "source": "crates/tensor-core/src/conformance/convolution.rs:331-346",
        "witness": ["strides: vec![2],", "dilations: vec![2],", "padding_after: vec![2],", "[-2., 0., 8.]"],
        "input": {"dims": [1, 1, 4], "values": [1, 2, 3, 4]},
        "weight": {"dims": [1, 1, 2], "values": [2, -1]},
        "options": {"strides": [2], "dilations": [2], "padding_before": [1], "padding_after": [2], "groups": 1},
        "out_dims": [1, 1, 3],
        "expected": [-2, 0, 8],
    },
    {
        "id": "conv_grouped",
        "op": "conv",
        "source": "crates/tensor-core/src/conformance/convolution.rs:347-357",
        "witness": ["o.groups = 2;", "(&[1, 2, 2], &[1., 2., 10., 20.])", "(&[2, 1, 1], &[2., 3.])", "[2., 4., 30., 60.]"],
        "input": {"dims": [1, 2, 2], "values": [1, 2, 10, 20]},
        "weight": {"dims": [2, 1, 1], "values": [2, 3]},
        "options": {"strides": [1], "dilations": [1], "padding_before": [0], "padding_after": [0], "groups": 2},
        "out_dims": [1, 2, 2],
        "expected": [2, 4, 30, 60],
    },
    {
        "id": "host_conv1d_padded",
        "op": "conv",
        "source": "crates/tensor-core/src/host_tensor/tests.rs:96-101",
        "note": "host conv1d with bias 0.5; the bias composes separately, so the conv alone is the answer minus 0.5",
        "witness": ["vec![1.0, 2.0, 3.0, 4.0, 5.0]", "x.conv1d(&w, Some(&[0.5]), 1, 1)", "&[3.5, 6.5, 9.5, 12.5, 9.5]"],
        "input": {"dims": [1, 1, 5], "values": [1, 2, 3, 4, 5]},
        "weight": {"dims": [1, 1, 3], "values": [1, 1, 1]},
        "options": {"strides": [1], "dilations": [1], "padding_before": [1], "padding_after": [1], "groups": 1},
        "out_dims": [1, 1, 5],
        "expected": [3.0, 6.0, 9.0, 12.0, 9.0],
    },
    {
        "id": "conv_plan_grouped_asymmetric",
        "op": "conv_plan",
        "source": "crates/tensor-core/src/convolution.rs:141-171",
        "witness": ["strides: vec![2, 1],", "dilations: vec![1, 2],", "padding_before: vec![1, 2],",
                    "padding_after: vec![0, 1],", "groups: 4,", "assert_eq!(plan.output.dims(), [2, 8, 2, 8]);"],
        "input_dims": [2, 4, 5, 7],
        "weight_dims": [8, 1, 3, 2],
        "options": {"strides": [2, 1], "dilations": [1, 2], "padding_before": [1, 2], "padding_after": [0, 1], "groups": 4},
        "out_dims": [2, 8, 2, 8],
    },
    {
        "id": "conv_plan_3d",
        "op": "conv_plan",
        "source": "crates/tensor-core/src/convolution.rs:161-171",
        "witness": ["&s(&[1, 2, 5, 6, 7]),", "&s(&[4, 2, 2, 3, 4]),", "[1, 4, 4, 4, 4]"],
        "input_dims": [1, 2, 5, 6, 7],
        "weight_dims": [4, 2, 2, 3, 4],
        "options": {"strides": [1, 1, 1], "dilations": [1, 1, 1], "padding_before": [0, 0, 0], "padding_after": [0, 0, 0], "groups": 1},
        "out_dims": [1, 4, 4, 4, 4],
    },
    {
        "id": "conv_plan_metadata_case",
        "op": "conv_plan",
        "source": "crates/compute-cuda/src/convolution.rs:176-195",
        "witness": ["shape(&[2, 4, 5, 7])", "shape(&[6, 2, 2, 3])", "assert_eq!(plan.output.dims(), [2, 6, 3, 6]);"],
        "input_dims": [2, 4, 5, 7],
        "weight_dims": [6, 2, 2, 3],
        "options": {"strides": [2, 1], "dilations": [1, 2], "padding_before": [1, 2], "padding_after": [0, 1], "groups": 2},
        "out_dims": [2, 6, 3, 6],
    },
    # --- attention oracle known answers
    {
        "id": "attention_uniform_grouped",
        "op": "attention",
        "source": "crates/tensor-core/src/conformance/attention.rs:479-496",
        "witness": ["let q = shape(&[4, 1, 1]);", "let k = shape(&[2, 2, 1]);", "(&q, &[1., 2., 3., 4.]),",
                    "(&k, &[3., 5., 7., 11.]),", "(&v, &[2., 4., 6., 10.]),", "scale: Some(0.0),",
                    "assert_eq!(values, [3.0, 3.0, 8.0, 8.0]);"],
        "q": {"dims": [4, 1, 1], "values": [1, 2, 3, 4]},
        "k": {"dims": [2, 2, 1], "values": [3, 5, 7, 11]},
        "v": {"dims": [2, 2, 1], "values": [2, 4, 6, 10]},
        "mask": None,
        "scale": 0.0,
        "causal": None,
        "out_dims": [4, 1, 1],
        "expected": [3, 3, 8, 8],
    },
    {
        "id": "attention_bias_exclusion_signed_causal",
        "op": "attention",
        "source": "crates/tensor-core/src/conformance/attention.rs:498-514",
        "witness": ["let q = shape(&[3, 1]);", "(&q, &[1., 1., 1.]),", "(&k, &[0., 0.]),", "(&k, &[5., 17.]),",
                    "Some((&mask, &[0., f32::NEG_INFINITY])),", "causal: Some(-1),", "assert_eq!(values, [0.0, 5.0, 5.0]);"],
        "q": {"dims": [3, 1], "values": [1, 1, 1]},
        "k": {"dims": [2, 1], "values": [0, 0]},
        "v": {"dims": [2, 1], "values": [5, 17]},
        "mask": {"dims": [2], "values": [0.0, "-inf"]},
        "scale": None,
        "causal": -1,
        "out_dims": [3, 1],
        "expected": [0, 5, 5],
    },
    {
        "id": "host_causal_first_row",
        "op": "attention",
        "source": "crates/tensor-core/src/host_tensor/tests.rs:81-94",
        "note": "causal row 0 sees only key 0, so it equals V row 0; row 1 is checked by the oracle only",
        "witness": ["let v = Tensor::new(vec![2, 2], vec![10.0, 20.0, 30.0, 40.0]).unwrap();",
                    "assert!((causal_attn.data()[0] - 10.0).abs() < 1e-5);"],
        "q": {"dims": [2, 2], "values": [1, 0, 0, 1]},
        "k": {"dims": [2, 2], "values": [1, 0, 0, 1]},
        "v": {"dims": [2, 2], "values": [10, 20, 30, 40]},
        "mask": None,
        "scale": None,
        "causal": 0,
        "out_dims": [2, 2],
        "expected_prefix": [10, 20],
    },
    # --- reductions
    {
        "id": "reduce_min_signed_extrema",
        "op": "reduce_f32",
        "source": "crates/tensor-core/src/conformance/reduction.rs:145-155",
        "witness": ["(ReduceOp::Min, [f32::MAX, f32::MAX / 2.], f32::MAX / 2.),"],
        "input": {"dims": [2], "values": [F32_MAX, F32_MAX / 2]},
        "axes": [0], "reduce": 2, "expected": [F32_MAX / 2],
    },
    {
        "id": "reduce_max_signed_extrema",
        "op": "reduce_f32",
        "source": "crates/tensor-core/src/conformance/reduction.rs:145-155",
        "witness": ["(ReduceOp::Max, [-f32::MAX, -f32::MAX / 2.], -f32::MAX / 2.),"],
        "input": {"dims": [2], "values": [-F32_MAX, -F32_MAX / 2]},
        "axes": [0], "reduce": 3, "expected": [-F32_MAX / 2],
    },
    {
        "id": "reduce_prime_tail_131077",
        "op": "reduce_prime_tail",
        "source": "crates/tensor-core/src/conformance/reduction.rs:218-241",
        "witness": ["let n = 131_077;", "values[17] = -1.;", "values[n - 1] = 2.;", "&[(n - 1) as f32 / n as f32],"],
        "n": 131077,
        "expected": {"sum": 131076.0, "product": -2.0, "min": -1.0, "max": 2.0, "mean": 131076.0 / 131077.0},
    },
    {
        "id": "reduce_broadcast_scalar",
        "op": "reduce_broadcast",
        "source": "crates/tensor-core/src/conformance/reduction.rs:203-216",
        "witness": ["&[1.25; 2],", "&[1.5625; 15],", "[u32::MAX - 2; 2]"],
        "expected": {"mean_02_keep": [1.25, 1.25], "product_1": [1.5625] * 15, "u32_sum": [4294967293, 4294967293]},
    },
    # --- statistics and argmax
    {
        "id": "softmax_equal_large_logits",
        "op": "softmax",
        "source": "crates/tensor-core/src/host_tensor/tests.rs:52-60",
        "witness": ["vec![1.0, 2.0, 3.0, 1000.0, 1000.0, 1000.0]", "assert!((p - 1.0 / 3.0).abs() < 1e-6);"],
        "input": {"dims": [2, 3], "values": [1, 2, 3, 1000, 1000, 1000]},
        "axes": [1],
        "expected_row1": [1 / 3, 1 / 3, 1 / 3],
    },
    {
        "id": "layer_norm_constant_row",
        "op": "layer_norm",
        "source": "crates/tensor-core/src/host_tensor/tests.rs:3-16",
        "witness": ["vec![1.0, 2.0, 3.0, 4.0, 10.0, 10.0, 10.0, 10.0]", "assert!(v.abs() < 1e-6);"],
        "input": {"dims": [2, 4], "values": [1, 2, 3, 4, 10, 10, 10, 10]},
        "axes": [1],
        "eps": 1e-5,
        "expected_row1": [0, 0, 0, 0],
    },
    {
        "id": "argmax_topk_order",
        "op": "argmax",
        "source": "crates/tensor-core/src/host_tensor/tests.rs:36-48",
        "note": "topk(2) of [[1,0,0],[1,2,2]] gives indices [0,1,1,2]: the first index of each row is the argmax, lowest index on ties",
        "witness": ["vec![1.0, 0.0, 0.0, 1.0, 2.0, 2.0]", "assert_eq!(top.indices, vec![0, 1, 1, 2]);"],
        "input": {"dims": [2, 3], "values": [1, 0, 0, 1, 2, 2]},
        "expected": [0, 1],
    },
    # --- low-storage final rounding witness
    {
        "id": "low_conv_single_final_rounding_bf16",
        "op": "conv_low",
        "source": "crates/tensor-core/src/conformance/convolution/low.rs:75-96",
        "witness": ["LowDtype::Bf16 => 2_f32.powi(-8),", "&[1., half, half, half]", "let expected = 1f64 + 3. * f64::from(half);"],
        "dtype": "bf16",
        "input": {"dims": [1, 4, 1], "values": [1.0, 2 ** -8, 2 ** -8, 2 ** -8]},
        "weight": {"dims": [1, 4, 1], "values": [1.0, 1.0, 1.0, 1.0]},
        "expected_f32": [1.0 + 3 * 2 ** -8],
    },
]


def verify(reference: Path) -> None:
    for case in CASES:
        path, lines = case["source"].split(":")
        lo, hi = (int(x) for x in lines.split("-")) if "-" in lines else (int(lines), int(lines))
        text = (reference / path).read_text().splitlines()
        window = "\n".join(text[max(lo - 1, 0) : hi])
        for w in case["witness"]:
            if w not in window:
                raise SystemExit(f"{case['id']}: {w!r} not found in {case['source']}")


def main(argv: list[str]) -> int:
    if len(argv) != 2:
        raise SystemExit(f"usage: {argv[0]} <path of the reference checkout>")
    reference = Path(argv[1])
    verify(reference)
    (HERE / "golden.json").write_text(json.dumps({"cases": CASES}, indent=1) + "\n")
    print(f"wrote {len(CASES)} cases to {HERE / 'golden.json'}")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
