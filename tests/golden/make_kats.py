"""Writes tests/golden/reference_kats.json: the known-answer tests of the reference's own test
suite for the quantized-matmul path, transcribed from its Rust sources.

Each entry records its source (file:line in the reference) and a `literal` that must appear on
that line.  Run it with the reference tree's path (first argument, or REFERENCE_ROOT) and it
verifies every citation against the source before writing; without one it refuses.  The GPU box never needs the reference: the JSON is the
committed fixture.
"""
from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "reference_kats.json")

KATS = [
    # ---- src/weights.rs ------------------------------------------------------------------------
    dict(name="quantize_int8_preserves_values_approximately", src="src/weights.rs:204",
         literal="let values = vec![1.0, 2.0, -3.0, 4.0];",
         op="quantize_int8", values=[1.0, 2.0, -3.0, 4.0], block_size=4,
         expect=dict(block_size=4, num_elements=4, n_scales=1, dequant_close=0.02)),
    dict(name="quantize_int8_handles_zeros", src="src/weights.rs:232",
         literal="Weights::quantize_int8(&[0.0, 0.0, 0.0, 0.0], 2)",
         op="quantize_int8", values=[0.0, 0.0, 0.0, 0.0], block_size=2,
         expect=dict(data=[0, 0, 0, 0], scales=[1.0, 1.0], block_size=2, num_elements=4)),
    dict(name="quantize_int8_scale_is_absmax_over_127", src="src/weights.rs:251",
         literal="Weights::quantize_int8(&[1.0, -2.0, 4.0, 0.0, -10.0, 5.0, 1.0, 2.0], 4)",
         op="quantize_int8", values=[1.0, -2.0, 4.0, 0.0, -10.0, 5.0, 1.0, 2.0], block_size=4,
         expect=dict(scales_close=[[4.0, 127.0], [10.0, 127.0]], eps="f32::EPSILON")),
    dict(name="quantize_int8_handles_partial_final_block", src="src/weights.rs:262",
         literal="Weights::quantize_int8(&[1.0, 2.0, 3.0], 2)",
         op="quantize_int8", values=[1.0, 2.0, 3.0], block_size=2,
         expect=dict(block_size=2, num_elements=3, n_scales=2, scales_close=[[2.0, 127.0], [3.0, 127.0]],
                     eps="f32::EPSILON")),
    dict(name="quantize_int4_preserves_values_approximately", src="src/weights.rs:282",
         literal="let values = vec![1.0, 2.0, -3.0, 4.0];",
         op="quantize_int4", values=[1.0, 2.0, -3.0, 4.0], block_size=32,
         expect=dict(block_size=32, num_elements=4, n_scales=1, dequant_close=0.5)),
    dict(name="quantize_int4_handles_zeros", src="src/weights.rs:320",
         literal="Weights::quantize_int4(&[0.0, 0.0, 0.0, 0.0], 32)",
         op="quantize_int4", values=[0.0, 0.0, 0.0, 0.0], block_size=32,
         expect=dict(data=[0x88, 0x88], scales=[1.0], block_size=32, num_elements=4)),
    dict(name="quantize_int4_packing", src="src/weights.rs:339",
         literal="Weights::quantize_int4(&[7.0, -7.0], 32)",
         op="quantize_int4", values=[7.0, -7.0], block_size=32,
         expect=dict(data=[0x1F], scales=[1.0])),
    dict(name="quantize_int4_block_size", src="src/weights.rs:350",
         literal="Weights::quantize_int4(&[1.0, 2.0, 3.0, 4.0, -5.0, 6.0, -7.0, 8.0], 4)",
         op="quantize_int4", values=[1.0, 2.0, 3.0, 4.0, -5.0, 6.0, -7.0, 8.0], block_size=4,
         expect=dict(block_size=4, num_elements=8, n_scales=2, scales_close=[[4.0, 7.0], [8.0, 7.0]],
                     eps="f32::EPSILON")),
    # ---- src/matmul.rs -------------------------------------------------------------------------
    dict(name="dot_product_int8_matches_f32", src="src/matmul.rs:419",
         literal="let input = vec![0.5, -2.0, 1.5, 4.0];",
         op="matmul_vs_f32", qtype="int8", input=[0.5, -2.0, 1.5, 4.0], weight=[1.0, -0.5, 2.0, -3.0],
         out_features=1, in_features=4, block_size=4, tol=0.05),
    dict(name="matmul_with_int8_weights", src="src/matmul.rs:459",
         literal="let weight_int8 = Weights::quantize_int8(&weight_f32, 3);",
         op="matmul_vs_f32", qtype="int8", input=[1.0, 2.0, -1.0], weight=[1.5, -0.5, 2.0, 0.25, 3.0, -1.0],
         out_features=2, in_features=3, block_size=3, tol=0.05),
    dict(name="matmul_with_int4_weights", src="src/matmul.rs:477",
         literal="let weight_int4 = Weights::quantize_int4(&weight_f32, 4);",
         op="matmul_vs_f32", qtype="int4", input=[1.0, 2.0, -1.0], weight=[1.5, -0.5, 2.0, 0.25, 3.0, -1.0],
         out_features=2, in_features=3, block_size=4, tol=0.5),
    dict(name="matmul_large_output", src="src/matmul.rs:358",
         literal="let weight = Weights::F32(vec![1.0; 1000 * 100]);",
         op="matmul_f32_ones", out_features=1000, in_features=100, expect_all=100.0),
    dict(name="matmul_identity_matrix", src="src/matmul.rs:338",
         literal="let weight = Weights::F32(vec![1.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0, 1.0]);",
         also=[["src/matmul.rs:337", "let input = vec![1.0, 2.0, 3.0];"]],
         op="matmul_f32", input=[1.0, 2.0, 3.0], weight=[1.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0, 1.0],
         out_features=3, in_features=3, expect=[1.0, 2.0, 3.0], tol=1e-5),
    dict(name="matmul_known_values", src="src/matmul.rs:348",
         literal="let weight = Weights::F32(vec![1.0, 0.0, 0.0, 0.0, 1.0, 0.0]);",
         also=[["src/matmul.rs:347", "let input = vec![1.0, 2.0, 3.0];"]],
         op="matmul_f32", input=[1.0, 2.0, 3.0], weight=[1.0, 0.0, 0.0, 0.0, 1.0, 0.0],
         out_features=2, in_features=3, expect=[1.0, 2.0], tol=1e-5),
    # dot_product (src/matmul.rs:127-147) is one output row of an F32 matmul
    dict(name="dot_product_matches_scalar", src="src/matmul.rs:369", literal="let weight = vec![2.0, 3.0, 4.0, 5.0, 6.0];",
         also=[["src/matmul.rs:368", "let input = vec![1.0, 2.0, 3.0, 4.0, 5.0];"]],
         op="matmul_f32", input=[1.0, 2.0, 3.0, 4.0, 5.0], weight=[2.0, 3.0, 4.0, 5.0, 6.0],
         out_features=1, in_features=5, expect=[70.0], tol=0.0),
    dict(name="dot_product_large_aligned", src="src/matmul.rs:378", literal="let input = vec![1.0; 1024];",
         op="matmul_f32", input=[1.0] * 1024, weight=[1.0] * 1024, out_features=1, in_features=1024,
         expect=[1024.0], tol=0.0),
    dict(name="dot_product_with_remainder", src="src/matmul.rs:389",
         literal="let weight = vec![7.0, 6.0, 5.0, 4.0, 3.0, 2.0, 1.0];",
         also=[["src/matmul.rs:388", "let input = vec![1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0];"]],
         op="matmul_f32", input=[1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0], weight=[7.0, 6.0, 5.0, 4.0, 3.0, 2.0, 1.0],
         out_features=1, in_features=7, expect=[84.0], tol=0.0),
    # bf16 rows are the top 16 bits of the f32 values (`value.to_bits() >> 16`)
    dict(name="dot_product_bf16_matches_f32", src="src/matmul.rs:399",
         literal="let weight = vec![1.5, -0.25, 2.0, 0.125, -1.0];",
         also=[["src/matmul.rs:398", "let input = vec![1.0, -2.0, 0.5, 4.0, 3.0];"]],
         op="bf16_vs_f32", input=[1.0, -2.0, 0.5, 4.0, 3.0], weight=[1.5, -0.25, 2.0, 0.125, -1.0],
         out_features=1, in_features=5, against="widened", tol=1e-5),
    dict(name="matmul_with_bf16_weights", src="src/matmul.rs:449",
         literal="let output = matmul(&input, &Weights::Bf16(weight_bf16), 2, 3);",
         also=[["src/matmul.rs:443", "let weight_f32 = vec![1.5, -0.5, 2.0, 0.25, 3.0, -1.0];"]],
         op="bf16_vs_f32", input=[1.0, 2.0, -1.0], weight=[1.5, -0.5, 2.0, 0.25, 3.0, -1.0],
         out_features=2, in_features=3, against="f32", tol=1e-5),
    # ---- src/weights.rs: Weights::len (:35-46) ---------------------------------------------------
    dict(name="weights_len_f32", src="src/weights.rs:166", literal="let weights = Weights::F32(vec![0.0; 10]);",
         op="weights_len", kind="f32", data_len=10, expect=10),
    dict(name="weights_len_bf16", src="src/weights.rs:173", literal="let weights = Weights::Bf16(vec![0; 10]);",
         op="weights_len", kind="bf16", data_len=10, expect=10),
    dict(name="weights_len_int8", src="src/weights.rs:183", literal="block_size: 5,",
         op="weights_len", kind="int8", data_len=10, n_scales=2, block_size=5, num_elements=10, expect=10),
    dict(name="weights_len_int4", src="src/weights.rs:193", literal="data: vec![0; 5],",
         op="weights_len", kind="int4", data_len=5, n_scales=1, block_size=32, num_elements=10, expect=10),
    # ---- src/model.rs (quantize_weights block policy) -----------------------------------------
    dict(name="quantize_weights_quantizes_f32_weights", src="src/model.rs:630",
         literal="Weights::F32(vec![1.0, -2.0, 0.0, 4.0]),",
         op="quantize_weights", qtype="int8", values=[1.0, -2.0, 0.0, 4.0], out_features=2, in_features=2,
         expect=dict(data_len=4, block_size=2, num_elements=4, scales_close=[[2.0, 127.0], [4.0, 127.0]],
                     eps="f32::EPSILON")),
    dict(name="quantize_weights_quantizes_bf16_weights", src="src/model.rs:656",
         literal="(1.5_f32.to_bits() >> 16) as u16,",
         op="quantize_weights", qtype="int8", bf16=[0x3FC0, 0xC000], out_features=1, in_features=2,
         expect=dict(data_len=2, block_size=2, num_elements=2, scales_exact=[[2.0, 127.0]])),
    dict(name="quantize_weights_quantizes_f32_weights_to_int4", src="src/model.rs:679",
         literal="Weights::F32(vec![7.0, -7.0, 0.0, 3.0]),",
         op="quantize_weights", qtype="int4", values=[7.0, -7.0, 0.0, 3.0], out_features=2, in_features=2,
         expect=dict(data_len=2, scales=[1.0], block_size=32, num_elements=4)),
    # ---- tests/gguf.rs (Q8_0 -> Weights::Int8 block 32) ----------------------------------------
    dict(name="q8_0_dequantize_known_values", src="tests/gguf.rs:60",
         literal="data.extend_from_slice(&half::f16::from_f32(0.5).to_le_bytes());",
         op="q8_0", blocks=[[0x3800, list(range(-16, 16))]], n=32,
         expect=dict(dequant=[v * 0.5 for v in range(-16, 16)])),
    dict(name="tensor_weights_q8_0_returns_int8", src="tests/gguf.rs:78",
         literal="data.extend_from_slice(&half::f16::from_f32(0.25).to_le_bytes());",
         op="q8_0", blocks=[[0x3400, list(range(0, 32))], [0x3800, list(range(-16, 16))]], n=40,
         expect=dict(data=list(range(0, 32)) + list(range(-16, -8)), scales=[0.25, 0.5], block_size=32,
                     num_elements=40)),
    # ---- src/output_head.rs --------------------------------------------------------------------
    dict(name="argmax_returns_index_of_largest", src="src/output_head.rs:83",
         literal="assert_eq!(argmax(&[1.0, 3.0, 2.0]), 1);", op="argmax", values=[1.0, 3.0, 2.0], expect=1),
    dict(name="argmax_handles_negative_values", src="src/output_head.rs:88",
         literal="assert_eq!(argmax(&[-3.0, -1.0, -2.0]), 1);", op="argmax", values=[-3.0, -1.0, -2.0],
         expect=1),
    dict(name="greedy_returns_argmax_of_logits", src="src/output_head.rs:74",
         literal="OutputHead::new(vec![1.0, 0.0, 3.0, 0.0, 2.0, 0.0].into(), 3, 2);",
         op="greedy_f32", weight=[1.0, 0.0, 3.0, 0.0, 2.0, 0.0], vocab=3, hidden=2, hidden_state=[1.0, 1.0],
         expect=1),
    dict(name="logits_with_identity_weight", src="src/output_head.rs:53",
         literal="vec![1.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0, 1.0].into(),",
         also=[["src/output_head.rs:58", "let logits = output_head.logits(&[1.0, 2.0, 3.0]);"]],
         op="matmul_f32", input=[1.0, 2.0, 3.0], weight=[1.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0, 1.0],
         out_features=3, in_features=3, expect=[1.0, 2.0, 3.0], tol=0.0),
    dict(name="logits_returns_correct_length", src="src/output_head.rs:65",
         literal="OutputHead::new(vec![0.0; 12].into(), 4, 3);",
         op="matmul_f32", input=[1.0, 2.0, 3.0], weight=[0.0] * 12, out_features=4, in_features=3,
         expect=[0.0] * 4, tol=0.0),
    # ---- tests/metal_matmul.rs: the GPU backend's own parity tests ------------------------------
    # Inputs are index formulas: x_i = f32(i) % xm / xd - xs and w_i = f32((i*wa + wb) % wm) / wd - ws,
    # every operation in f32.  "expect" is the reference's CPU matmul ("matmul") or the test's
    # sequential sum (cpu_matmul_f32, "sequential"), each within the test's tolerance.
    dict(name="metal_matmul_identity", src="tests/metal_matmul.rs:61",
         literal="let weight = vec![1.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0, 1.0];",
         op="matmul_f32", input=[1.0, 2.0, 3.0], weight=[1.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0, 1.0],
         out_features=3, in_features=3, expect=[1.0, 2.0, 3.0], tol=1e-4),
    dict(name="metal_matmul_known_values", src="tests/metal_matmul.rs:74",
         literal="let weight = vec![1.0, 0.0, 0.0, 0.0, 1.0, 0.0];",
         op="matmul_f32", input=[1.0, 2.0, 3.0], weight=[1.0, 0.0, 0.0, 0.0, 1.0, 0.0],
         out_features=2, in_features=3, expect=[1.0, 2.0], tol=1e-4),
    dict(name="metal_matmul_large", src="tests/metal_matmul.rs:87", literal="let weight = vec![1.0; 1000 * 100];",
         op="matmul_f32_ones", out_features=1000, in_features=100, expect_all=100.0),
    dict(name="metal_matmul_matches_cpu", src="tests/metal_matmul.rs:106",
         literal=".map(|index| ((index * 17 + 11) % 23) as f32 / 7.0 - 1.5)",
         also=[["tests/metal_matmul.rs:103", ".map(|index| (index as f32 % 7.0) - 3.0)"]],
         op="formula_matmul", dtype="f32", out_features=16, in_features=17, x=[7.0, 1.0, 3.0],
         w=[17, 11, 23, 7.0, 1.5], expect="matmul", tol=1e-4, via=["host"]),
    dict(name="metal_matmul_bf16_matches_cpu", src="tests/metal_matmul.rs:126",
         literal=".map(|index| ((index * 17 + 11) % 23) as f32 / 7.0 - 1.5)",
         also=[["tests/metal_matmul.rs:123", ".map(|index| (index as f32 % 7.0) - 3.0)"]],
         op="formula_matmul", dtype="bf16", out_features=16, in_features=17, x=[7.0, 1.0, 3.0],
         w=[17, 11, 23, 7.0, 1.5], expect="matmul", tol=1e-4, via=["host"]),
    dict(name="metal_matmul_matches_cpu_transformer_dimensions", src="tests/metal_matmul.rs:156",
         literal=".map(|index| ((index * 29 + 7) % 37) as f32 / 19.0 - 0.95)",
         also=[["tests/metal_matmul.rs:153", ".map(|index| (index as f32 % 31.0) / 17.0 - 0.9)"]],
         op="formula_matmul", dtype="f32", out_features=2048, in_features=2048, x=[31.0, 17.0, 0.9],
         w=[29, 7, 37, 19.0, 0.95], expect="sequential", tol=1e-2, via=["host"]),
    dict(name="metal_matmul_multi_tile", src="tests/metal_matmul.rs:176",
         literal=".map(|index| ((index * 31 + 13) % 47) as f32 / 29.0 - 0.8)",
         also=[["tests/metal_matmul.rs:173", ".map(|index| (index as f32 % 43.0) / 23.0 - 0.85)"]],
         op="formula_matmul", dtype="f32", out_features=64, in_features=5504, x=[43.0, 23.0, 0.85],
         w=[31, 13, 47, 29.0, 0.8], expect="sequential", tol=1e-2, via=["host"]),
    dict(name="metal_buffer_matmul_matches_cpu", src="tests/metal_matmul.rs:196",
         literal=".map(|index| ((index * 17 + 11) % 23) as f32 / 7.0 - 1.5)",
         also=[["tests/metal_matmul.rs:193", ".map(|index| (index as f32 % 7.0) - 3.0)"]],
         op="formula_matmul", dtype="f32", out_features=16, in_features=17, x=[7.0, 1.0, 3.0],
         w=[17, 11, 23, 7.0, 1.5], expect="matmul", tol=1e-4, via=["host", "device"]),
    dict(name="weights_to_metal_f32", src="tests/metal_matmul.rs:218",
         literal="let weights = Weights::F32(vec![1.0, 2.0, 3.0, 4.0]);",
         op="dense_upload", dtype="f32", values=[1.0, 2.0, 3.0, 4.0], expect_len=4, expect_bytes=16),
    dict(name="weights_to_metal_bf16", src="tests/metal_matmul.rs:234",
         literal="let weights = Weights::Bf16(vec![f32_to_bf16(1.5), f32_to_bf16(-2.0)]);",
         op="dense_upload", dtype="bf16", values=[1.5, -2.0], expect_len=2, expect_bytes=4),
    dict(name="weights_to_metal_bf16_creates_metal_bf16", src="tests/metal_matmul.rs:251",
         literal="let weights = Weights::Bf16(vec![f32_to_bf16(0.5), f32_to_bf16(4.0), f32_to_bf16(-8.0)]);",
         op="dense_upload", dtype="bf16", values=[0.5, 4.0, -8.0], expect_len=3, expect_bytes=6),
    # ---- src/rmsnorm.rs, src/attention.rs, src/ffn.rs (decode-loop support ops) ----------------
    dict(name="rmsnorm_forward_normalizes_with_weights", src="src/rmsnorm.rs:48",
         literal="let rmsnorm = RmsNorm::new(vec![0.5, 1.0], 1e-6);", op="rmsnorm", x=[2.0, 4.0],
         weight=[0.5, 1.0], eps=1e-6, expect_close=[2.0 / 10.0 ** 0.5 * 0.5, 4.0 / 10.0 ** 0.5], tol=1e-5),
    dict(name="rmsnorm_forward_handles_zero_input", src="src/rmsnorm.rs:59",
         literal="let rmsnorm = RmsNorm::new(vec![1.0, 1.0], 1e-6);", op="rmsnorm", x=[0.0, 0.0],
         weight=[1.0, 1.0], eps=1e-6, expect_close=[0.0, 0.0], tol=0.0),
    dict(name="apply_rope_rotates_at_nonzero_position", src="src/attention.rs:229",
         literal="let mut values = vec![1.0, 0.0, 0.0, 1.0];", op="rope", x=[1.0, 0.0, 0.0, 1.0], head_dim=4,
         pos=1, theta=10.0, expect="cos(1), -sin(1/sqrt(10)), sin(1), cos(1/sqrt(10))", tol=1e-5),
    dict(name="silu_at_positive_value", src="src/ffn.rs:82", literal="assert_close(silu(1.0), 0.7310586);",
         op="silu", x=1.0, expect=0.7310586, tol=1e-5),
    dict(name="silu_at_negative_value", src="src/ffn.rs:87", literal="assert_close(silu(-1.0), -0.26894143);",
         op="silu", x=-1.0, expect=-0.26894143, tol=1e-5),
]


def reference_root() -> str:
    """The reference source tree whose lines the citations are checked against: the first
    command-line argument, else the REFERENCE_ROOT environment variable."""
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REFERENCE_ROOT", "")
    if not root:
        raise SystemExit("usage: make_kats.py <reference source tree> (or set REFERENCE_ROOT)")
    return root


def verify(root: str) -> None:
    for k in KATS:
        for src, literal in [[k["src"], k["literal"]]] + k.get("also", []):
            path, line = src.rsplit(":", 1)
            with open(os.path.join(root, path)) as f:
                lines = f.read().splitlines()
            text = lines[int(line) - 1]
            if literal not in text:
                raise SystemExit(f"{k['name']}: {src} does not contain {literal!r}: {text!r}")


def main() -> None:
    root = reference_root()
    if not os.path.isdir(root):
        raise SystemExit(f"reference tree {root} not found; the committed JSON stays as it is")
    verify(root)
    with open(OUT, "w") as f:  # one test per line
        f.write('{"source": "mizzy/pyxis test suite (Rust); transcribed by tests/golden/make_kats.py",\n "kats": [\n')
        f.write(",\n".join("  " + json.dumps(k) for k in KATS))
        f.write("\n ]\n}\n")
    print(f"wrote {OUT}: {len(KATS)} known-answer tests, all citations verified", file=sys.stderr)


if __name__ == "__main__":
    main()
