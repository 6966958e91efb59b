"""Regenerate the golden fixtures in this folder (run in a container that has the
reference tree; the GPU box only reads the committed outputs).

  python tests/golden/make_golden.py --reference <reference checkout>

Outputs
  dequant_golden.npz   seeded random Q4_K / Q5_K / Q6_K blocks (raw bytes) and their
                       dequantized values computed by the reference's own gguf-py numpy
                       dequantizers (vendor/llama.cpp/gguf-py/gguf/quants.py:475-572),
                       which apply the same per-element formula as quants.rs:181-249.
  known_answers.json   the expected values of the reference's known-answer unit tests
                       (quants.rs:3709-3772, real_math.rs:2919-3191, 4334-4440), each
                       with the construction it describes.
"""
import argparse
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def random_blocks(rng, n, size, d_offsets):
    raw = rng.integers(0, 256, size=(n, size), dtype=np.uint8)
    # realistic fp16 scales plus edge cases (zero, subnormal, negative, large)
    d = np.abs(rng.normal(0, 0.02, size=(n, len(d_offsets)))).astype(np.float16)
    d[0, :] = 0.0
    d[1, :] = np.float16(3.0e-7)          # subnormal half
    d[2, :] = -np.abs(d[2, :])
    d[3, :] = np.float16(1.5)
    for j, off in enumerate(d_offsets):
        raw[:, off:off + 2] = d[:, j:j + 1].view(np.uint8).reshape(n, 2)
    raw[4] = 0                              # an all-zero block
    return raw


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "vendor/llama.cpp/gguf-py"))
    from gguf import quants as gq  # noqa: E402

    rng = np.random.default_rng(20261201)
    out = {}
    for name, cls, size, d_offsets in (("q4k", gq.Q4_K, 144, [0, 2]), ("q5k", gq.Q5_K, 176, [0, 2]),
                                       ("q6k", gq.Q6_K, 210, [208])):
        raw = random_blocks(rng, 48, size, d_offsets)
        deq = cls.dequantize_blocks(raw.copy()).astype(np.float32)
        out[f"{name}_raw"] = raw
        out[f"{name}_out"] = deq
    np.savez_compressed(HERE / "dequant_golden.npz", **out)

    known = {
        "source": "reference unit tests (expected values copied as numbers; constructions restated)",
        "q4k_constructed_row": {
            "cite": "quants.rs:3725-3754, real_math.rs:3130-3170",
            "construction": "one Q4_K block: d=fp16(1.0), dmin=0, scales[0..4]=1, others 0, all qs bytes 0x11",
            "inputs": [1.0, 0.5], "expected": [128.0, 64.0]},
        "q6k_constructed_row": {
            "cite": "quants.rs:3757-3772, real_math.rs:3172-3191",
            "construction": "one Q6_K block: d=fp16(1.0), 16 scales=1, ql=qh=0",
            "inputs": [1.0, 0.5], "expected": [-8192.0, -4096.0]},
        "zero_blocks": {"cite": "quants.rs:3709-3722", "expected": 0.0},
        "q4k_top_k_four_rows": {
            "cite": "real_math.rs:4363-4400",
            "construction": "four constructed Q4_K rows with d = 1,2,3,4; input ones; k=2; no softcap",
            "argmax": 3, "top": [[3, 512.0], [2, 384.0]]},
        "q6k_top_k_pair": {
            "cite": "real_math.rs:4402-4440",
            "construction": "two constructed Q6_K rows with d = 1,2; input ones; k=2",
            "argmax": 0, "top": [[0, -8192.0], [1, -16384.0]]},
        "f32_top_k": {
            "cite": "real_math.rs:4334-4348",
            "rows": [[1.0, 0.0], [0.0, 2.0], [3.0, 0.0]], "input": [1.0, 1.0], "k": 2,
            "argmax": 2, "argmax_score": 3.0, "top": [[2, 3.0], [1, 2.0]]},
        "rms_norm_identity": {
            "cite": "real_math.rs:2919-2927", "x": [3.0, 4.0], "w": [1.0, 1.0], "tol": 1e-5},
        "gqa_limit_causality": {
            "cite": "real_math.rs:3081-3095", "q": [1.0, 0.0], "k": [[1.0, 0.0], [0.0, 1.0]],
            "v": [[10.0, 1.0], [100.0, 2.0]], "limit1_expected": [10.0, 1.0]},
        "gqa_window": {
            "cite": "real_math.rs:3097-3110", "q": [1.0, 0.0], "k": [[1.0, 0.0], [1.0, 0.0]],
            "v": [[10.0, 1.0], [100.0, 2.0]], "window1_expected": [100.0, 2.0], "full_expected": [55.0, 1.5]},
        "proportional_rope": {
            "cite": "real_math.rs:3007-3036", "x": [1, 2, 3, 4, 5, 6, 7, 8], "position": 1, "theta": 10000.0,
            "rotary_dim": 4, "unchanged": {"2": 3.0, "3": 4.0, "6": 7.0, "7": 8.0}},
    }
    (HERE / "known_answers.json").write_text(json.dumps(known, indent=1))
    print("wrote", HERE / "dequant_golden.npz", HERE / "known_answers.json")


if __name__ == "__main__":
    main()
