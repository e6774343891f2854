"""Run one reference known-answer case on the GPU (C ABI) or on the oracle."""
from __future__ import annotations

import numpy as np

# ops of the reference whose C-ABI entry points exist in this build
GPU_OPS = {"matmul", "batch_matmul", "softmax", "add", "sub", "mul", "relu", "sigmoid", "swish",
           "tanh", "scale", "relu_backward", "sigmoid_backward", "swish_backward",
           "tanh_backward", "transpose", "group_norm", "conv2d", "conv_transpose2d",
           "conv2d_grad_bias", "sdpa", "concat", "upsample_nearest2d"}


def run_oracle(orc, case) -> np.ndarray:
    op, x, a = case["op"], case["inputs"], case["args"]
    if op == "matmul":
        return orc.matmul(x["a"], x["b"], a["m"], a["n"], a["k"])
    if op == "batch_matmul":
        return orc.batch_matmul(x["a"], x["b"], a["batch"], a["m"], a["n"], a["k"])
    if op == "softmax":
        return orc.softmax(x["x"], a["rows"], a["cols"])
    if op == "sdpa":
        return orc.attention(x["q"], x["k"], x["v"], a["bh"], a["seq"], a["dk"])
    if op == "conv2d":
        return orc.conv2d(x["input"], x["weight"], x["bias"], a["batch"], a["in_c"], a["in_h"],
                          a["in_w"], a["out_c"], a["kh"], a["kw"], tuple(a["stride"]),
                          tuple(a["padding"]), tuple(a["dilation"]), a["groups"])
    if op == "conv_transpose2d":
        return orc.conv_transpose2d(x["input"], x["weight"], x["bias"], a["batch"], a["in_c"],
                                    a["in_h"], a["in_w"], a["out_c"], a["kh"], a["kw"],
                                    tuple(a["stride"]), tuple(a["padding"]),
                                    tuple(a["output_padding"]), tuple(a["dilation"]), a["groups"])
    if op == "conv2d_grad_bias":
        return orc.conv2d_grad_bias(x["grad_out"], a["batch"], a["out_c"], a["out_h"], a["out_w"])
    if op == "group_norm":
        return orc.group_norm(x["x"], x["gamma"], x["beta"], a["batch"], a["channels"],
                              a["spatial"], a["groups"], a["eps"])
    if op == "transpose":
        return orc.transpose(x["a"], a["outer"], a["d0"], a["d1"], a["inner"])
    if op == "concat":
        return orc.concat(x["a"], x["b"], a["outer"], a["a_inner"], a["b_inner"])
    if op == "upsample_nearest2d":
        return orc.upsample_nearest2d(x["x"], a["batch"], a["channels"], a["in_h"], a["in_w"],
                                      a["scale_h"], a["scale_w"])
    if op == "scale":
        return orc.elementwise("scale", x["a"], None, a["s"])
    if op in ("add", "sub", "mul", "relu_backward", "sigmoid_backward", "swish_backward",
              "tanh_backward"):
        return orc.elementwise(op, x["a"], x["b"])
    if op in ("relu", "sigmoid", "swish", "tanh"):
        return orc.elementwise(op, x["a"])
    raise KeyError(op)


def run_gpu(dev, case) -> np.ndarray:
    op, x, a = case["op"], case["inputs"], case["args"]
    up = dev.upload
    if op == "matmul":
        return dev.read(dev.matmul(up(x["a"]), up(x["b"]), a["m"], a["n"], a["k"]))
    if op == "batch_matmul":
        return dev.read(dev.batch_matmul(up(x["a"]), up(x["b"]), a["batch"], a["m"], a["n"],
                                         a["k"]))
    if op == "softmax":
        return dev.read(dev.softmax(up(x["x"]), a["rows"], a["cols"]))
    if op == "sdpa":
        return dev.read(dev.scaled_dot_product_attention(up(x["q"]), up(x["k"]), up(x["v"]),
                                                         a["bh"], a["seq"], a["dk"]))
    if op == "conv2d":
        bias = up(x["bias"]) if x["bias"] is not None else None
        return dev.read(dev.conv2d(up(x["input"]), up(x["weight"]), bias, a["batch"], a["in_c"],
                                   a["in_h"], a["in_w"], a["out_c"], a["kh"], a["kw"],
                                   tuple(a["stride"]), tuple(a["padding"]), tuple(a["dilation"]),
                                   a["groups"]))
    if op == "conv_transpose2d":
        bias = up(x["bias"]) if x["bias"] is not None else None
        return dev.read(dev.conv_transpose2d(up(x["input"]), up(x["weight"]), bias, a["batch"],
                                             a["in_c"], a["in_h"], a["in_w"], a["out_c"],
                                             a["kh"], a["kw"], tuple(a["stride"]),
                                             tuple(a["padding"]), tuple(a["output_padding"]),
                                             tuple(a["dilation"]), a["groups"]))
    if op == "conv2d_grad_bias":
        return dev.read(dev.conv2d_grad_bias(up(x["grad_out"]), a["batch"], a["out_c"],
                                             a["out_h"], a["out_w"]))
    if op == "group_norm":
        return dev.read(dev.group_norm(up(x["x"]), up(x["gamma"]), up(x["beta"]), a["batch"],
                                       a["channels"], a["spatial"], a["groups"], a["eps"]))
    if op == "transpose":
        return dev.read(dev.transpose(up(x["a"]), a["outer"], a["d0"], a["d1"], a["inner"]))
    if op == "concat":
        return dev.read(dev.concat(up(x["a"]), up(x["b"]), a["outer"], a["a_inner"],
                                   a["b_inner"]))
    if op == "upsample_nearest2d":
        return dev.read(dev.upsample_nearest2d(up(x["x"]), a["batch"], a["channels"], a["in_h"],
                                               a["in_w"], a["scale_h"], a["scale_w"]))
    if op == "scale":
        return dev.read(dev.scale(up(x["a"]), a["s"]))
    if op in ("add", "sub", "mul", "relu_backward", "sigmoid_backward", "swish_backward",
              "tanh_backward"):
        return dev.read(getattr(dev, op)(up(x["a"]), up(x["b"])))
    if op in ("relu", "sigmoid", "swish"):
        return dev.read(getattr(dev, op)(up(x["a"])))
    if op == "tanh":
        return dev.read(dev.tanh_act(up(x["a"])))
    raise KeyError(op)


def check(case, got, want_oracle=None):
    """Compare `got` to the case's literal expectation (or the oracle)."""
    from conftest import assert_approx
    got = np.asarray(got, np.float32)
    if case.get("expect_slices"):
        for lo, hi, vals in case["expect_slices"]:
            assert_approx(got[lo:hi], vals, case["tol"])
        return
    if isinstance(case["expect"], list):
        want = np.asarray(case["expect"], np.float32)
        if case["exact"]:
            assert np.array_equal(got, want), f"{case['name']}: {got} != {want}"
        else:
            assert_approx(got, want, case["tol"])
    else:
        assert want_oracle is not None
        if case["exact"]:
            assert np.array_equal(got, np.asarray(want_oracle, np.float32)), case["name"]
        else:
            assert_approx(got, want_oracle, case["tol"])
    if case.get("row_sums"):
        cols = case["args"]["cols"]
        sums = got.reshape(-1, cols).astype(np.float64).sum(axis=1)
        assert np.all(np.abs(sums - 1.0) < case["row_sums"]), sums
