"""Writes tests/golden/reference_kat.json: the reference's own known-answer tests
for the hot path, transcribed with the file:line each value comes from.

The reference is Rust and cannot be built in this image, so its golden values
are taken from its test sources as text.  When the environment variable
REFERENCE_ROOT names a checkout of the reference, this script also re-reads
every cited line and fails if the literal it quotes is not there, so the
fixture cannot drift from its source.

Usage: REFERENCE_ROOT=<reference checkout> python tests/golden/make_kat.py
"""
from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("REFERENCE_ROOT", "")
KERNELS = "crates/ferrite-strata-cpu/tests/kernels.rs"
E2E = "crates/ferrite-strata-runtime/tests/end_to_end.rs"

# (id, source, line, literal quoted on that line, case)
CASES = [
    ("add_doubles", KERNELS, 142, "[2.0, 4.0, 6.0, 8.0]",
     {"op": "add", "a": [[1, 2], [3, 4]], "b": [[1, 2], [3, 4]], "out_shape": [2, 2],
      "want": [2, 4, 6, 8], "tol": 0.0}),
    ("add_elementwise", KERNELS, 156, "[11.0, 22.0]",
     {"op": "add", "a": [1, 2], "b": [10, 20], "out_shape": [2], "want": [11, 22], "tol": 0.0}),
    ("matmul_naive", KERNELS, 173, "[19.0, 22.0, 43.0, 50.0]",
     {"op": "matmul", "a": [[1, 2], [3, 4]], "b": [[5, 6], [7, 8]], "want": [19, 22, 43, 50], "tol": 0.0}),
    ("matmul_k_order", KERNELS, 189, "[8.0]",
     {"op": "matmul", "a": [[1, 1, 1, 1]], "b": [[2], [2], [2], [2]], "want": [8], "tol": 0.0}),
    ("softmax_row", KERNELS, 215, "[0.090_030_6, 0.244_728_4, 0.665_240_9]",
     {"op": "softmax", "x": [[1, 2, 3]], "want": [0.0900306, 0.2447284, 0.6652409], "tol": 1e-5}),
    ("softmax_uniform", KERNELS, 217, "[1.0 / 3.0; 3]",
     {"op": "softmax", "x": [[0, 0, 0]], "want": [1 / 3, 1 / 3, 1 / 3], "tol": 1e-6}),
    ("softmax_large_bias", KERNELS, 231, "[0.268_941_4, 0.731_058_6]",
     {"op": "softmax", "x": [[1000, 1001]], "want": [0.2689414, 0.7310586], "tol": 1e-5}),
    ("gelu_minus_one", KERNELS, 242, "[-0.158_655_2]",
     {"op": "gelu", "x": [-1.0], "want": [-0.1586552], "tol": 1e-5}),
    ("gelu_one", KERNELS, 244, "[0.841_344_8]",
     {"op": "gelu", "x": [1.0], "want": [0.8413448], "tol": 1e-5}),
    ("layer_norm_gamma_beta", KERNELS, 323, "[-1.0, 0.0]",
     {"op": "layer_norm", "x": [[1, 3]], "gamma": [2, 0], "beta": [1, 0], "eps": 1e-5,
      "want": [-1.0, 0.0], "tol": 1e-4}),
    ("linear_bias", KERNELS, 361, "[11.0, 22.0]",
     {"op": "linear", "x": [[1, 2]], "w": [[1, 0], [0, 1]], "bias": [10, 20], "want": [11, 22], "tol": 1e-6}),
    ("linear_no_bias", KERNELS, 390, "[7.0]",
     {"op": "linear", "x": [[3, 4]], "w": [[1, 1]], "bias": None, "want": [7], "tol": 1e-6}),
    ("transpose", KERNELS, 405, "[1.0, 4.0, 2.0, 5.0, 3.0, 6.0]",
     {"op": "transpose", "x": [[1, 2, 3], [4, 5, 6]], "want": [1, 4, 2, 5, 3, 6], "tol": 0.0}),
    ("expand_rows", KERNELS, 431, "[7.0, 8.0, 7.0, 8.0, 7.0, 8.0]",
     {"op": "expand", "x": [[7, 8]], "out_shape": [3, 2], "want": [7, 8, 7, 8, 7, 8], "tol": 0.0}),
    ("e2e_gelu_times_x", E2E, 144, "0.841_344_8",
     {"op": "gelu_mul", "x": [[1, 2, 3, 4], [5, 6, 7, 8]], "want_first": [0.8413448, 2 * 1.9544997],
      "tol": [1e-4, 1e-3]}),
]


def verify() -> None:
    if not REF or not os.path.isdir(REF):
        print("REFERENCE_ROOT not set to a reference checkout; transcription not re-checked", file=sys.stderr)
        return
    for cid, src, line, literal, _ in CASES:
        with open(os.path.join(REF, src)) as f:
            lines = f.read().splitlines()
        window = "\n".join(lines[line - 3:line + 2])
        if literal not in window:
            raise SystemExit(f"{cid}: `{literal}` not found near {src}:{line}")


def main() -> None:
    verify()
    out = [{"id": cid, "source": f"{src}:{line}", **case} for cid, src, line, _lit, case in CASES]
    with open(os.path.join(HERE, "reference_kat.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(f"wrote {len(out)} cases")


if __name__ == "__main__":
    main()
