"""Extract the reference's softmax known-answer vectors into softmax_golden.json.

The reference (sethigris/haelixe, Rust) pins its softmax kernel with the
"crucible" in haelixe-lab/src/main.rs and with finite-difference checks in
tests/tensor_tests.rs. It has no attention test. This script reads those two
files as text (the crate cannot be built here) and writes the inputs,
expected outputs and tolerances they contain, with their line numbers, so the
oracle can be checked against them without the reference present.

Usage: python tests/golden/make_golden.py [REFERENCE_ROOT]
"""
from __future__ import annotations

import json
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def _floats(s: str) -> list[float]:
    return [float(t.replace("f32", "").replace("_", "")) for t in re.findall(r"-?\d+\.\d+(?:e-?\d+)?(?:_?f32)?", s)]


def _find(lines, pattern, start=0):
    rx = re.compile(pattern)
    for i in range(start, len(lines)):
        if rx.search(lines[i]):
            return i
    raise SystemExit(f"pattern not found: {pattern}")


def main(ref_root: str) -> None:
    main_rs = os.path.join(ref_root, "haelixe-lab", "src", "main.rs")
    tests_rs = os.path.join(ref_root, "tests", "tensor_tests.rs")
    with open(main_rs) as f:
        L = f.read().split("\n")
    with open(tests_rs) as f:
        T = f.read().split("\n")

    cases = []
    # Stage 1: forward known values.
    i_in = _find(L, r"Shape::new\(\[1, 3\]\), &\[1\.0f32, 2\.0, 3\.0\]")
    i_ex = _find(L, r"let expected = \[", i_in)
    i_tol = _find(L, r"approx_eq\(y_data\[0\], expected\[0\], ([0-9.e-]+)\)", i_ex)
    cases.append({
        "name": "forward_known_values",
        "kind": "softmax_forward",
        "shape": [1, 3],
        "input": _floats(L[i_in].split("&[")[1]),
        "expected": _floats(L[i_ex]),
        "abs_tol": float(re.search(r"expected\[0\], ([0-9.e-]+)\)", L[i_tol]).group(1)),
        "source": f"haelixe-lab/src/main.rs:{i_in + 1}-{i_tol + 3}",
    })
    # Stage 2: numerical stability on extreme logits (finite output).
    i_in = _find(L, r"&\[1000\.0f32, 1001\.0, 1002\.0\]")
    cases.append({
        "name": "extreme_logits_finite",
        "kind": "softmax_finite",
        "shape": [1, 3],
        "input": _floats(L[i_in].split("&[")[1]),
        "source": f"haelixe-lab/src/main.rs:{i_in + 1}-{i_in + 8}",
    })
    # Stage 3: rows sum to one, values in [0, 1].
    i_sh = _find(L, r"Shape::new\(\[3, 4\]\)")
    i_vals = _find(L, r"-1\.0f32, 0\.0, 1\.0, 2\.0", i_sh)
    i_tol = _find(L, r"approx_eq\(sum, 1\.0, ([0-9.e-]+)\)", i_vals)
    cases.append({
        "name": "rows_sum_to_one",
        "kind": "softmax_simplex",
        "shape": [3, 4],
        "input": _floats(L[i_vals]),
        "abs_tol": float(re.search(r"approx_eq\(sum, 1\.0, ([0-9.e-]+)\)", L[i_tol]).group(1)),
        "source": f"haelixe-lab/src/main.rs:{i_sh + 1}-{i_tol + 1}",
    })
    # Stage 4: backward Jacobian with seed [1, 0, 0].
    i_in = _find(L, r"let mut x = Tensor::from_slice\(DType::F32, Shape::new\(\[1, 3\]\)")
    i_seed = _find(L, r"let grad_seed", i_in)
    i_ex = _find(L, r"let expected = \[", i_seed)
    i_tol = _find(L, r"approx_eq\(dx_data\[0\], expected\[0\], ([0-9.e-]+)\)", i_ex)
    cases.append({
        "name": "backward_jacobian_seed",
        "kind": "softmax_backward",
        "shape": [1, 3],
        "input": _floats(L[i_in].split("&[")[1]),
        "seed": _floats(L[i_seed].split("&[")[1]),
        "expected": _floats(L[i_ex]),
        "abs_tol": float(re.search(r"expected\[0\], ([0-9.e-]+)\)", L[i_tol]).group(1)),
        "source": f"haelixe-lab/src/main.rs:{i_in + 1}-{i_tol + 3}",
    })
    # Stage 5: d/dx sum(softmax(x)) == 0.
    i_in = _find(L, r"Shape::new\(\[1, 4\]\), &\[1\.0f32, 2\.0, 3\.0, 4\.0\]")
    i_tol = _find(L, r"v\.abs\(\) < ([0-9.e-]+)", i_in)
    cases.append({
        "name": "grad_of_sum_is_zero",
        "kind": "softmax_sum_grad",
        "shape": [1, 4],
        "input": _floats(L[i_in].split("&[")[1]),
        "abs_tol": float(re.search(r"v\.abs\(\) < ([0-9.e-]+)", L[i_tol]).group(1)),
        "source": f"haelixe-lab/src/main.rs:{i_in + 1}-{i_tol + 1}",
    })
    # tests/tensor_tests.rs: finite-difference constants and the softmax case.
    i_eps = _find(T, r"const EPS: f32 = ")
    i_tol = _find(T, r"const TOL: f32 = ")
    i_sm = _find(T, r"fn test_softmax_grad")
    i_data = _find(T, r"let data = vec!\[", i_sm)
    fd = {
        "eps": float(re.search(r"= ([0-9.e-]+);", T[i_eps]).group(1)),
        "tol": float(re.search(r"= ([0-9.e-]+);", T[i_tol]).group(1)),
        "softmax_input": _floats(T[i_data]),
        "source": f"tests/tensor_tests.rs:{i_eps + 1}-{i_tol + 1},{i_sm + 1}-{i_sm + 9}",
    }
    out = {"generated_by": "tests/golden/make_golden.py", "softmax_cases": cases, "finite_difference": fd}
    path = os.path.join(HERE, "softmax_golden.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")
    print(f"wrote {path}: {len(cases)} softmax cases")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
