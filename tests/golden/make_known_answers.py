"""Writes tests/golden/known_answers.json: the known-answer cases of the
reference's own runtime tests (JTPuffer/TempLit tests/test_metal_runtime.cpp
and the Metal-only block of tests/test_meta.cpp), restated as data.

Each case holds the op, its inputs, the expected output computed with the
same closed forms the reference test uses (in float32, as the C++ test
does), the tolerance the reference applies and the source line.  The
oracle (tests/test_oracle_golden.py) and the CUDA kernels
(tests/test_kernels_gpu.py) are both checked against this file.

Run:  python tests/golden/make_known_answers.py
"""
import json
import math
import os

import numpy as np

f32 = np.float32
SRC = "tests/test_metal_runtime.cpp"


def fl(x):
    return [float(f32(v)) for v in x]


def gelu(x):
    a = f32(0.7978845608)
    x = f32(x)
    return f32(0.5) * x * (f32(1) + np.tanh(a * (x + f32(0.044715) * x * x * x)))


def gelu_d(x):
    a, b = f32(0.7978845608), f32(0.044715)
    x = f32(x)
    x2 = x * x
    t = np.tanh(a * (x + b * x2 * x))
    return f32(0.5) * (f32(1) + t) + f32(0.5) * x * (f32(1) - t * t) * a * (f32(1) + f32(3) * b * x2)


def cases():
    c = []

    def add(name, op, inputs, expected, eps, line, **kw):
        d = {"name": name, "op": op, "inputs": inputs, "expected": expected, "eps": eps,
             "source": f"{SRC}:{line}"}
        d.update(kw)
        c.append(d)

    a, b = [1, 2, 3, 4], [5, 6, 7, 8]
    for op, exp in (("add", [6, 8, 10, 12]), ("sub", [-4] * 4), ("mul", [5, 12, 21, 32]),
                    ("div", fl([0.2, 1 / 3, 3 / 7, 0.5]))):
        add(f"binary_{op}", "binary", {"a": a, "a_shape": [2, 2], "b": b, "b_shape": [2, 2],
                                        "out_shape": [2, 2], "kind": op}, exp, 1e-5, "131-158")
    add("broadcast_row", "binary", {"a": [1, 2, 3, 4, 5, 6], "a_shape": [2, 3], "b": [10, 20, 30],
                                    "b_shape": [3], "out_shape": [2, 3], "kind": "add"},
        [11, 22, 33, 14, 25, 36], 1e-5, "160-174")
    for op, s, exp, eps in (("add", 3.0, [5, 7, 9, 11], 1e-5), ("div", 2.0, [1, 2, 3, 4], 1e-5),
                            ("pow", 3.0, [8, 64, 216, 512], 1e-3)):
        add(f"scalar_{op}", "scalar", {"x": [2, 4, 6, 8], "s": s, "kind": op}, exp, eps, "176-199")
    e1 = float(f32(1) / (f32(1) + np.exp(f32(-1))))
    e2 = float(f32(1) / (f32(1) + np.exp(f32(1))))
    e3 = float(f32(1) / (f32(1) + np.exp(f32(-2))))
    add("sigmoid", "unary", {"x": [0, 1, -1, 2], "kind": "sigmoid"}, [0.5, e1, e2, e3], 1e-5, "201-226")
    add("exp", "unary", {"x": [0, 1, -1, 2], "kind": "exp"},
        fl([1.0, math.exp(1), math.exp(-1), math.exp(2)]), 1e-5, "201-226")
    add("sqrt", "unary", {"x": [0, 1, 4, 9], "kind": "sqrt"}, [0, 1, 2, 3], 1e-5, "201-226")
    first = float(np.sqrt(f32(12.5) + f32(1e-6)))
    add("rms", "rms", {"x": [3, 4, 0, 0], "shape": [2, 2]}, [first, 1e-3], 1e-5, "228-244")
    add("rmsnorm", "rmsnorm", {"x": [3, 4, 0, 0], "shape": [2, 2]},
        fl([3 / first, 4 / first, 0, 0]), 1e-5, "228-244")
    xs = [-2, -1, 0, 1, 2]
    add("gelu", "unary", {"x": xs, "kind": "gelu"}, [float(gelu(x)) for x in xs], 1e-5, "246-279")
    add("gelu_derivative", "unary", {"x": xs, "kind": "gelu_derivative"},
        [float(gelu_d(x)) for x in xs], 1e-5, "246-279")
    add("matmul", "matmul", {"a": [1, 2, 3, 4, 5, 6], "a_shape": [2, 3], "b": [7, 8, 9, 10, 11, 12],
                             "b_shape": [3, 2]}, [58, 64, 139, 154], 1e-5, "281-305")
    add("matmul_batched", "matmul", {"a": [1, 2, 3, 4, 2, 0, 1, 2], "a_shape": [2, 2, 2],
                                     "b": [5, 6, 7, 8, 1, 3, 4, 2], "b_shape": [2, 2, 2]},
        [19, 22, 43, 50, 2, 6, 9, 7], 1e-5, "281-305")
    inp = [1, 2, 3, 4, 5, 6]
    add("sum_all", "sum_to_shape", {"x": inp, "shape": [2, 3], "out_shape": [1]}, [21], 1e-5, "344-374")
    add("sum_axis1", "sum_to_shape", {"x": inp, "shape": [2, 3], "out_shape": [2, 1]}, [6, 15], 1e-5, "344-374")
    add("sum_rows", "sum_to_shape", {"x": inp, "shape": [2, 3], "out_shape": [1, 3]}, [5, 7, 9], 1e-5, "344-374")
    add("max_rows", "max_to_shape", {"x": inp, "shape": [2, 3], "out_shape": [2, 1]}, [3, 6], 1e-5, "344-374")
    add("transpose", "transpose", {"x": inp, "shape": [2, 3], "dims": [-2, -1]}, [1, 4, 2, 5, 3, 6],
        1e-5, "344-374")
    x24 = list(range(1, 25))
    for name, shp, exp in (("non_adjacent", [1, 3, 1], [68, 100, 132]), ("adjacent", [2, 1, 1], [78, 222]),
                           ("all", [1, 1, 1], [300]), ("lower_rank", [4], [66, 72, 78, 84])):
        add(f"sum_to_shape_{name}", "sum_to_shape", {"x": x24, "shape": [2, 3, 4], "out_shape": shp},
            exp, 1e-5, "376-413")
    add("sum_to_shape_leading_singleton", "sum_to_shape",
        {"x": [1, 2, 3, 4], "shape": [1, 4], "out_shape": [4]}, [1, 2, 3, 4], 1e-5, "415-430")
    den = np.exp(f32(-2)) + np.exp(f32(-1)) + f32(1)
    lo, mid, hi = float(np.exp(f32(-2)) / den), float(np.exp(f32(-1)) / den), float(f32(1) / den)
    t = float(f32(1) / f32(3))
    add("softmax", "softmax", {"x": [1, 2, 3, 1, 1, 1], "shape": [2, 3]}, [lo, mid, hi, t, t, t], 1e-5, "432-472")
    add("softmax_rank4", "softmax", {"x": [1, 2, 3, 3, 2, 1, 1000, 1001, 1002, -1000, -1000, -1000],
                                     "shape": [2, 2, 1, 3]},
        [lo, mid, hi, hi, mid, lo, lo, mid, hi, t, t, t], 1e-5, "432-472")
    add("softmax_singleton", "softmax", {"x": [4, -7], "shape": [2, 1]}, [1, 1], 1e-5, "432-472")
    ld = float(np.log(den))
    logits = [1, 2, 3, 1, 1, 1, 1000, 1001, 1002, -1, -2, -3]
    add("cross_entropy", "cross_entropy", {"logits": logits, "shape": [2, 2, 3], "targets": [2, 0, 1, 2]},
        [ld, float(np.log(f32(3))), 1 + ld, 2 + ld], 1e-4, "474-507")
    add("cross_entropy_derivative", "cross_entropy_derivative",
        {"logits": logits, "shape": [2, 2, 3], "targets": [2, 0, 1, 2]},
        [lo, mid, hi - 1, -2 / 3, 1 / 3, 1 / 3, lo, mid - 1, hi, hi, mid, lo - 1], 1e-4, "474-507")
    large = [0.0] * 5000
    large[4097] = 100.0
    add("argmax_small", "argmax", {"x": [1, 4, 2, 9, 3, 5]}, [3], 0, "509-531")
    add("argmax_large", "argmax", {"x": large}, [4097], 0, "509-531")
    w = list(range(1, 13))
    add("embedding_lookup", "embedding_lookup", {"weights": w, "w_shape": [4, 3], "ids": [2, 0, 3, 1]},
        [7, 8, 9, 1, 2, 3, 10, 11, 12, 4, 5, 6], 1e-5, "533-549")
    vals = [1, 2, 3, 4, 5, 6, 10, 20, 30, 7, 8, 9]
    add("scatter_index", "scatter", {"values": vals, "ids": [2, 0, 2, 1], "n_rows": 4, "dim": 3, "base": None},
        [4, 5, 6, 7, 8, 9, 11, 22, 33, 0, 0, 0], 1e-5, "551-569")
    add("scatter_add_rows", "scatter", {"values": vals, "ids": [2, 0, 2, 1], "n_rows": 4, "dim": 3,
                                        "base": list(range(100, 112))},
        [104, 106, 108, 110, 112, 114, 117, 129, 141, 109, 110, 111], 1e-5, "571-593")
    add("gradient_clipping", "clip", {"grads": [[3, 4, 0], [12]], "max_norm": 1.0},
        {"sqnorm": 169.0, "clipped": [fl([3 / 13, 4 / 13, 0]), fl([12 / 13])]}, 1e-5, "595-615")
    # AdamW: two steps against the closed form, in float32 like the C++ test
    p = np.array([1, -2, 3, -4], dtype=f32)
    g = np.array([0.5, -0.25, 1.0, -0.75], dtype=f32)
    m1 = np.zeros(4, f32)
    m2 = np.zeros(4, f32)
    steps = []
    for step in (1, 2):
        c1 = f32(1) - f32(0.9) ** f32(step)
        c2 = f32(1) - f32(0.999) ** f32(step)
        m1 = f32(0.9) * m1 + f32(0.1) * g
        m2 = f32(0.999) * m2 + f32(0.001) * g * g
        p = p * f32(0.9999) - f32(0.01) * (m1 / c1) / (np.sqrt(m2 / c2) + f32(1e-8))
        steps.append(fl(p))
    add("adamw_two_steps", "adamw", {"param": [1, -2, 3, -4], "grad": [0.5, -0.25, 1.0, -0.75], "lr": 0.01,
                                     "beta1": 0.9, "beta2": 0.999, "eps": 1e-8, "weight_decay": 0.01},
        steps, 1e-5, "617-658")
    # Metal-only compiled-graph cases of tests/test_meta.cpp
    rmsv = float(np.sqrt(f32(12.5) + f32(1e-6)))
    c.append({"name": "compiled_rms_grad_sgd", "op": "rms_backward_sgd", "inputs": {"x": [3, 4], "lr": 1.0},
              "expected": fl([3 - 3 / (2 * rmsv), 4 - 4 / (2 * rmsv)]), "eps": 1e-5,
              "source": "tests/test_meta.cpp:230-247"})
    c.append({"name": "compiled_embedding_sgd", "op": "embedding_sgd",
              "inputs": {"weights": w, "w_shape": [4, 3], "ids": [2, 0, 2, 1], "lr": 0.5},
              "expected": [0.5, 1.5, 2.5, 3.5, 4.5, 5.5, 6.0, 7.0, 8.0, 10.0, 11.0, 12.0], "eps": 0,
              "source": "tests/test_meta.cpp:273-306"})
    c.append({"name": "compiled_cross_entropy_sgd", "op": "cross_entropy_sgd",
              "inputs": {"logits": [1, 2, 3, 1, 1, 1], "shape": [2, 3], "targets": [2, 0],
                         "root_grad": [2.0, 0.5], "lr": 1.0},
              "expected": fl([1 - 2 * lo, 2 - 2 * mid, 3 - 2 * (hi - 1), 1 + 1 / 3, 1 - 1 / 6, 1 - 1 / 6]),
              "eps": 1e-4, "source": "tests/test_meta.cpp:340-380"})
    return c


def main():
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "known_answers.json")
    with open(out, "w") as f:
        json.dump({"generator": "tests/golden/make_known_answers.py",
                   "reference": "JTPuffer/TempLit", "cases": cases()}, f, indent=1)
    print("wrote", out)


if __name__ == "__main__":
    main()
