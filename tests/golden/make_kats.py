"""Generate tests/golden/reference_kats.json from the reference's unit tests.

Each case restates one `#[test]` of the any-gpu crate: the same inputs (the
Rust iterator expressions are rewritten as Python), the op call, and — where
the Rust test asserts literal values — those literal expected values.  Cases
whose Rust test compares against a CPU helper (`cpu_matmul`, `cpu_conv2d`,
`cpu_softmax`, `cpu_attention`, `cpu_group_norm`, `cpu_sigmoid`/`cpu_swish`)
carry `"expect": "oracle"`: the expected values come from the oracle, which is
itself pinned by the literal cases.  `"expect_err": true` marks the tests that
assert `is_err()`.

    python tests/golden/make_kats.py        # rewrites reference_kats.json
"""
from __future__ import annotations

import json
from pathlib import Path

OUT = Path(__file__).resolve().parent / "reference_kats.json"


def rng(lo, hi, f):
    return [float(f(i)) for i in range(lo, hi)]


def f32(x):
    import numpy as np
    return float(np.float32(x))


def cases():
    c = []

    def add(name, src, op, inputs, args, expect=None, tol=None, exact=False, expect_err=False,
            **extra):
        c.append(dict(name=name, source=src, op=op, inputs=inputs, args=args,
                      expect=expect if expect is not None else ("error" if expect_err else
                                                                "oracle"),
                      tol=tol, exact=exact, expect_err=expect_err, **extra))

    # ---------------------------------------------------- src/ops/conv.rs --
    add("matmul_2x2", "src/ops/conv.rs:633-638", "matmul",
        {"a": [1, 2, 3, 4], "b": [5, 6, 7, 8]}, {"m": 2, "n": 2, "k": 2},
        expect=[19, 22, 43, 50], exact=True)
    add("matmul_nonsquare_vs_cpu", "src/ops/conv.rs:641-648", "matmul",
        {"a": rng(1, 13, lambda x: x), "b": rng(1, 9, lambda x: f32(x) * f32(0.1))},
        {"m": 3, "n": 2, "k": 4}, tol=1e-4)
    add("matmul_1x1", "src/ops/conv.rs:651-654", "matmul", {"a": [3], "b": [7]},
        {"m": 1, "n": 1, "k": 1}, expect=[21], exact=True)
    add("matmul_17x13_vs_cpu", "src/ops/conv.rs:657-667", "matmul",
        {"a": rng(0, 17 * 11, lambda i: f32(f32(i) * f32(0.01)) - f32(0.5)),
         "b": rng(0, 11 * 13, lambda i: f32(f32(i) * f32(0.01)) - f32(0.3))},
        {"m": 17, "n": 13, "k": 11}, tol=1e-3)
    add("batch_matmul", "src/ops/conv.rs:672-677", "batch_matmul",
        {"a": [1, 2, 3, 4, 5, 6, 7, 8], "b": [1, 0, 0, 1, 2, 0, 0, 2]},
        {"batch": 2, "m": 2, "n": 2, "k": 2}, expect=[1, 2, 3, 4, 10, 12, 14, 16], exact=True)
    add("batch_matmul_nonsquare", "src/ops/conv.rs:680-686", "batch_matmul",
        {"a": [1, 2, 3, 4, 5, 6], "b": [1, 1, 1]}, {"batch": 1, "m": 2, "n": 1, "k": 3},
        expect=[6, 15], exact=True)
    conv = dict(stride=[1, 1], padding=[0, 0], dilation=[1, 1], groups=1)
    add("conv2d_3x3_vs_cpu", "src/ops/conv.rs:691-702", "conv2d",
        {"input": rng(1, 17, lambda x: x), "weight": [1, 0, -1, 1, 0, -1, 1, 0, -1],
         "bias": [0]},
        dict(batch=1, in_c=1, in_h=4, in_w=4, out_c=1, kh=3, kw=3, **conv), tol=1e-5)
    add("conv2d_1x1_kernel", "src/ops/conv.rs:705-718", "conv2d",
        {"input": [1, 2, 3, 4, 10, 20, 30, 40], "weight": [1.0, 0.5, 0.0, 1.0, -1.0, 2.0],
         "bias": [0, 0, 0]},
        dict(batch=1, in_c=2, in_h=2, in_w=2, out_c=3, kh=1, kw=1, **conv),
        expect_slices=[[0, 4, [6, 12, 18, 24]], [4, 8, [10, 20, 30, 40]]], tol=1e-5)
    add("conv2d_padding_vs_cpu", "src/ops/conv.rs:721-731", "conv2d",
        {"input": rng(1, 10, lambda x: x), "weight": [1.0] * 9, "bias": None},
        dict(batch=1, in_c=1, in_h=3, in_w=3, out_c=1, kh=3, kw=3, stride=[1, 1],
             padding=[1, 1], dilation=[1, 1], groups=1), tol=1e-5)
    add("conv2d_stride2", "src/ops/conv.rs:734-741", "conv2d",
        {"input": rng(1, 17, lambda x: x), "weight": [1.0], "bias": None},
        dict(batch=1, in_c=1, in_h=4, in_w=4, out_c=1, kh=1, kw=1, stride=[2, 2],
             padding=[0, 0], dilation=[1, 1], groups=1), expect=[1, 3, 9, 11], exact=True)
    add("conv2d_5x5_kernel_vs_cpu", "src/ops/conv.rs:744-755", "conv2d",
        {"input": rng(0, 64, lambda i: f32(i) * f32(0.1)),
         "weight": [1.0 if i == 12 else 0.0 for i in range(25)], "bias": None},
        dict(batch=1, in_c=1, in_h=8, in_w=8, out_c=1, kh=5, kw=5, stride=[1, 1],
             padding=[2, 2], dilation=[1, 1], groups=1), tol=1e-4)
    add("conv2d_multichannel_vs_cpu", "src/ops/conv.rs:758-770", "conv2d",
        {"input": rng(0, 2 * 3 * 16, lambda i: f32(f32(i) * f32(0.01)) - f32(0.5)),
         "weight": rng(0, 2 * 3 * 9, lambda i: f32(f32(i) * f32(0.02)) - f32(0.3)),
         "bias": [0.1, -0.2]},
        dict(batch=2, in_c=3, in_h=4, in_w=4, out_c=2, kh=3, kw=3, stride=[1, 1],
             padding=[1, 1], dilation=[1, 1], groups=1), tol=1e-3)
    add("conv2d_with_bias", "src/ops/conv.rs:773-781", "conv2d",
        {"input": [0.0] * 4, "weight": [0.0], "bias": [42.0]},
        dict(batch=1, in_c=1, in_h=2, in_w=2, out_c=1, kh=1, kw=1, **conv),
        expect=[42, 42, 42, 42], exact=True)
    add("conv_transpose2d_stride2", "src/ops/conv.rs:786-793", "conv_transpose2d",
        {"input": [1, 2, 3, 4], "weight": [1.0], "bias": None},
        dict(batch=1, in_c=1, in_h=2, in_w=2, out_c=1, kh=1, kw=1, stride=[2, 2],
             padding=[0, 0], output_padding=[0, 0], dilation=[1, 1], groups=1),
        expect=[1, 0, 2, 0, 0, 0, 3, 0, 4], tol=1e-5)
    add("conv_transpose2d_3x3_kernel", "src/ops/conv.rs:796-803", "conv_transpose2d",
        {"input": [5.0], "weight": [1.0] * 9, "bias": None},
        dict(batch=1, in_c=1, in_h=1, in_w=1, out_c=1, kh=3, kw=3, stride=[1, 1],
             padding=[0, 0], output_padding=[0, 0], dilation=[1, 1], groups=1),
        expect=[5.0] * 9, tol=1e-5)
    add("matmul_a_size_mismatch", "src/ops/conv.rs:808-812", "matmul",
        {"a": [1, 2, 3], "b": [1, 2, 3, 4]}, {"m": 2, "n": 2, "k": 2}, expect_err=True)
    add("matmul_b_size_mismatch", "src/ops/conv.rs:815-819", "matmul",
        {"a": [1, 2, 3, 4], "b": [1, 2, 3]}, {"m": 2, "n": 2, "k": 2}, expect_err=True)
    add("conv2d_input_size_mismatch", "src/ops/conv.rs:822-826", "conv2d",
        {"input": [1.0] * 10, "weight": [1.0] * 9, "bias": None},
        dict(batch=1, in_c=1, in_h=4, in_w=4, out_c=1, kh=3, kw=3, **conv), expect_err=True)
    add("conv2d_weight_size_mismatch", "src/ops/conv.rs:829-833", "conv2d",
        {"input": [1.0] * 16, "weight": [1.0] * 5, "bias": None},
        dict(batch=1, in_c=1, in_h=4, in_w=4, out_c=1, kh=3, kw=3, **conv), expect_err=True)
    add("conv2d_bias_size_mismatch", "src/ops/conv.rs:836-841", "conv2d",
        {"input": [1.0] * 16, "weight": [1.0] * 9, "bias": [1.0, 2.0]},
        dict(batch=1, in_c=1, in_h=4, in_w=4, out_c=1, kh=3, kw=3, **conv), expect_err=True)
    add("batch_matmul_vs_cpu", "src/ops/conv.rs:846-866", "batch_matmul",
        {"a": rng(0, 3 * 4 * 5, lambda i: f32(f32(i) * f32(0.01)) - f32(0.3)),
         "b": rng(0, 3 * 5 * 3, lambda i: f32(f32(i) * f32(0.02)) - f32(0.1))},
        {"batch": 3, "m": 4, "n": 3, "k": 5}, tol=1e-3)
    add("conv2d_grad_bias_basic", "src/ops/conv.rs:907-922", "conv2d_grad_bias",
        {"grad_out": [1, 2, 3, 4]}, dict(batch=1, out_c=1, out_h=2, out_w=2), expect=[10],
        tol=1e-5)
    add("conv2d_grad_bias_two_channels", "src/ops/conv.rs:907-922", "conv2d_grad_bias",
        {"grad_out": [1, 2, 3, 4, 5, 6, 7, 8]}, dict(batch=1, out_c=2, out_h=2, out_w=2),
        expect=[10, 26], tol=1e-5)

    # ----------------------------------------------- src/ops/attention.rs --
    add("softmax_vs_cpu", "src/ops/attention.rs:232-242", "softmax",
        {"x": [1, 2, 3, -1, 0, 1, 5, 5, 5]}, {"rows": 3, "cols": 3}, tol=1e-4, row_sums=1e-4)
    add("softmax_large_values", "src/ops/attention.rs:245-253", "softmax",
        {"x": [1000, 1001, 1002]}, {"rows": 1, "cols": 3}, tol=1e-4, row_sums=1e-4)
    add("softmax_single_element", "src/ops/attention.rs:256-259", "softmax", {"x": [42]},
        {"rows": 1, "cols": 1}, expect=[1.0], tol=1e-5)
    add("attention_vs_cpu", "src/ops/attention.rs:262-272", "sdpa",
        {"q": rng(0, 12, lambda i: f32(f32(i) * f32(0.1)) - f32(0.3)),
         "k": rng(0, 12, lambda i: f32(f32(i) * f32(0.05)) + f32(0.1)),
         "v": rng(0, 12, lambda i: f32(f32(i) * f32(0.2)) - f32(0.5))},
        {"bh": 1, "seq": 3, "dk": 4}, tol=1e-3)
    add("attention_uniform_qk", "src/ops/attention.rs:275-285", "sdpa",
        {"q": [1, 1, 1, 1], "k": [1, 1, 1, 1], "v": [0, 10, 20, 30]},
        {"bh": 1, "seq": 2, "dk": 2}, expect=[10, 20, 10, 20], tol=1e-3)
    add("softmax_size_mismatch", "src/ops/attention.rs:312-315", "softmax", {"x": [1, 2, 3]},
        {"rows": 2, "cols": 3}, expect_err=True)

    # ---------------------------------------------------- src/ops/norm.rs --
    add("group_norm_per_channel", "src/ops/norm.rs:483-490", "group_norm",
        {"x": [1, 3, 2, 4], "gamma": [1, 1], "beta": [0, 0]},
        dict(batch=1, channels=2, spatial=2, groups=2, eps=1e-5), expect=[-1, 1, -1, 1], tol=1e-3)
    add("group_norm_single_group", "src/ops/norm.rs:493-505", "group_norm",
        {"x": [1, 2, 3, 4], "gamma": [1.0] * 4, "beta": [0.0] * 4},
        dict(batch=1, channels=4, spatial=1, groups=1, eps=1e-5), tol=1e-3)
    add("group_norm_with_affine", "src/ops/norm.rs:508-514", "group_norm",
        {"x": [1, 3, 2, 4], "gamma": [2.0, 0.5], "beta": [1.0, -1.0]},
        dict(batch=1, channels=2, spatial=2, groups=2, eps=1e-5), expect=[-1, 3, -1.5, -0.5],
        tol=1e-3)
    add("group_norm_batched_vs_cpu", "src/ops/norm.rs:517-528", "group_norm",
        {"x": rng(0, 24, lambda i: f32(f32(i) * f32(0.1)) - f32(0.5)),
         "gamma": [1.0, 2.0, 0.5, 1.5], "beta": [0.0, 1.0, -1.0, 0.5]},
        dict(batch=2, channels=4, spatial=3, groups=2, eps=1e-5), tol=1e-3)
    add("group_norm_constant_input", "src/ops/norm.rs:531-541", "group_norm",
        {"x": [5.0] * 8, "gamma": [1.0, 1.0], "beta": [0.0, 0.0]},
        dict(batch=1, channels=2, spatial=4, groups=2, eps=1e-5), expect=[0.0] * 8, tol=1e-3)
    add("group_norm_channels_not_divisible", "src/ops/norm.rs:544-549", "group_norm",
        {"x": [1.0] * 5, "gamma": [1.0] * 5, "beta": [0.0] * 5},
        dict(batch=1, channels=5, spatial=1, groups=2, eps=1e-5), expect_err=True)
    add("group_norm_input_size_mismatch", "src/ops/norm.rs:552-557", "group_norm",
        {"x": [1.0] * 10, "gamma": [1.0] * 4, "beta": [0.0] * 4},
        dict(batch=1, channels=4, spatial=4, groups=2, eps=1e-5), expect_err=True)

    # --------------------------------------------- src/ops/elementwise.rs --
    add("add", "src/ops/elementwise.rs:264-269", "add",
        {"a": [1, 2, 3, 4], "b": [10, 20, 30, 40]}, {}, expect=[11, 22, 33, 44], exact=True)
    add("add_odd_size", "src/ops/elementwise.rs:272-279", "add",
        {"a": rng(0, 13, lambda i: i), "b": rng(0, 13, lambda i: i * 10.0)}, {},
        expect=[float(i + i * 10.0) for i in range(13)], exact=True)
    add("add_single_element", "src/ops/elementwise.rs:282-285", "add", {"a": [42], "b": [-42]},
        {}, expect=[0.0], exact=True)
    add("sub", "src/ops/elementwise.rs:288-293", "sub", {"a": [10, 20, 30], "b": [1, 2, 3]},
        {}, expect=[9, 18, 27], exact=True)
    add("mul", "src/ops/elementwise.rs:296-301", "mul",
        {"a": [1, 2, 3, 4], "b": [10, 20, 30, 40]}, {}, expect=[10, 40, 90, 160], exact=True)
    add("mul_zeros", "src/ops/elementwise.rs:304-309", "mul", {"a": [1, 2, 3], "b": [0, 0, 0]},
        {}, expect=[0, 0, 0], exact=True)
    add("relu", "src/ops/elementwise.rs:312-316", "relu", {"a": [-2, -1, 0, 1, 2]}, {},
        expect=[0, 0, 0, 1, 2], exact=True)
    add("relu_all_negative", "src/ops/elementwise.rs:319-322", "relu",
        {"a": [-100.0, -0.001, -1e-10]}, {}, expect=[0, 0, 0], exact=True)
    add("sigmoid_vs_cpu", "src/ops/elementwise.rs:325-330", "sigmoid",
        {"a": [-50.0, -10.0, -1.0, 0.0, 1.0, 10.0, 50.0]}, {}, tol=1e-4)
    add("swish_vs_cpu", "src/ops/elementwise.rs:333-338", "swish",
        {"a": [-5.0, -2.0, -1.0, 0.0, 1.0, 2.0, 5.0]}, {}, tol=1e-4)
    add("tanh_vs_cpu", "src/ops/elementwise.rs:341-346", "tanh",
        {"a": [-10.0, -1.0, 0.0, 1.0, 10.0]}, {}, tol=1e-4)
    add("scale", "src/ops/elementwise.rs:349-352", "scale", {"a": [1, 2, 3, 4]}, {"s": 0.5},
        expect=[0.5, 1.0, 1.5, 2.0], exact=True)
    add("scale_zero", "src/ops/elementwise.rs:355-358", "scale", {"a": [99.0, -99.0]},
        {"s": 0.0}, expect=[0.0, 0.0], exact=True)
    add("scale_negative", "src/ops/elementwise.rs:361-364", "scale", {"a": [1.0, -2.0, 3.0]},
        {"s": -2.0}, expect=[-2.0, 4.0, -6.0], exact=True)
    add("add_length_mismatch", "src/ops/elementwise.rs:369-373", "add",
        {"a": [1, 2], "b": [1, 2, 3]}, {}, expect_err=True)
    add("sub_length_mismatch", "src/ops/elementwise.rs:376-380", "sub", {"a": [1], "b": [1, 2]},
        {}, expect_err=True)
    add("mul_length_mismatch", "src/ops/elementwise.rs:383-387", "mul",
        {"a": [1, 2, 3], "b": [1]}, {}, expect_err=True)
    add("add_vs_cpu", "src/ops/elementwise.rs:392-398", "add",
        {"a": rng(0, 100, lambda i: f32(f32(i) * f32(0.3)) - f32(15.0)),
         "b": rng(0, 100, lambda i: f32(f32(i) * f32(-0.2)) + f32(10.0))}, {}, tol=1e-5)
    add("sub_vs_cpu", "src/ops/elementwise.rs:401-407", "sub",
        {"a": rng(0, 100, lambda i: f32(i) * f32(0.7)),
         "b": rng(0, 100, lambda i: f32(i) * f32(0.3))}, {}, tol=1e-5)
    add("mul_vs_cpu", "src/ops/elementwise.rs:410-416", "mul",
        {"a": rng(0, 100, lambda i: f32(f32(i) * f32(0.1)) - f32(5.0)),
         "b": rng(0, 100, lambda i: f32(f32(i) * f32(0.05)) + f32(0.5))}, {}, tol=1e-4)
    add("relu_backward_vs_cpu", "src/ops/elementwise.rs:421-427", "relu_backward",
        {"a": [1, 2, 3, 4, 5], "b": [-1.0, 0.5, 0.0, -0.1, 2.0]}, {},
        expect=[0.0, 2.0, 0.0, 0.0, 5.0], tol=1e-5)
    add("sigmoid_backward_vs_cpu", "src/ops/elementwise.rs:430-436", "sigmoid_backward",
        {"a": [1.0, 1.0, 1.0], "b": [0.5, 0.7311, 0.2689]}, {},
        expect=[f32(g * s * (1.0 - s)) for g, s in zip([1.0] * 3, [0.5, 0.7311, 0.2689])],
        tol=1e-3)
    add("swish_backward_vs_cpu", "src/ops/elementwise.rs:439-448", "swish_backward",
        {"a": [1.0] * 4, "b": [0.0, 1.0, -1.0, 2.0]}, {}, tol=1e-3)
    add("tanh_backward_vs_cpu", "src/ops/elementwise.rs:451-457", "tanh_backward",
        {"a": [1.0] * 4, "b": [0.0, 0.7616, -0.7616, 0.9951]}, {},
        expect=[1.0 - t * t for t in [0.0, 0.7616, -0.7616, 0.9951]], tol=1e-3)

    # ---------------------------------------------- src/ops/tensor_ops.rs --
    add("transpose_2d", "src/ops/tensor_ops.rs:407-411", "transpose",
        {"a": [1, 2, 3, 4, 5, 6]}, dict(outer=1, d0=2, d1=3, inner=1),
        expect=[1, 4, 2, 5, 3, 6], exact=True)
    add("transpose_square", "src/ops/tensor_ops.rs:414-419", "transpose",
        {"a": [1, 2, 3, 4, 5, 6, 7, 8, 9]}, dict(outer=1, d0=3, d1=3, inner=1),
        expect=[1, 4, 7, 2, 5, 8, 3, 6, 9], exact=True)
    add("transpose_batched", "src/ops/tensor_ops.rs:422-432", "transpose",
        {"a": list(range(1, 13))}, dict(outer=2, d0=2, d1=3, inner=1),
        expect=[1, 4, 2, 5, 3, 6, 7, 10, 8, 11, 9, 12], exact=True)
    add("transpose_1x_n", "src/ops/tensor_ops.rs:435-441", "transpose",
        {"a": [1, 2, 3, 4, 5]}, dict(outer=1, d0=1, d1=5, inner=1), expect=[1, 2, 3, 4, 5],
        exact=True)
    add("concat_flat", "src/ops/tensor_ops.rs:379-382", "concat",
        {"a": [1, 2, 3], "b": [4, 5, 6]}, dict(outer=1, a_inner=3, b_inner=3),
        expect=[1, 2, 3, 4, 5, 6], exact=True)
    add("concat_asymmetric", "src/ops/tensor_ops.rs:385-391", "concat",
        {"a": [1, 2], "b": [3, 4, 5]}, dict(outer=1, a_inner=2, b_inner=3),
        expect=[1, 2, 3, 4, 5], exact=True)
    add("concat_batched_channel_axis", "src/ops/tensor_ops.rs:394-404", "concat",
        {"a": [10, 20, 30, 40], "b": [1, 2, 3, 4, 5, 6, 7, 8]},
        dict(outer=2, a_inner=2, b_inner=4),
        expect=[10, 20, 1, 2, 3, 4, 30, 40, 5, 6, 7, 8], exact=True)

    # ------------------------------------------------ src/ops/upsample.rs --
    add("upsample_2x", "src/ops/upsample.rs:161-170", "upsample_nearest2d",
        {"x": [1, 2, 3, 4]}, dict(batch=1, channels=1, in_h=2, in_w=2, scale_h=2, scale_w=2),
        expect=[1, 1, 2, 2, 1, 1, 2, 2, 3, 3, 4, 4, 3, 3, 4, 4], exact=True)
    add("upsample_3x_vs_cpu", "src/ops/upsample.rs:173-179", "upsample_nearest2d",
        {"x": rng(1, 7, lambda x: x)},
        dict(batch=1, channels=1, in_h=2, in_w=3, scale_h=3, scale_w=3), exact=True)
    add("upsample_batched_multichannel_vs_cpu", "src/ops/upsample.rs:182-188",
        "upsample_nearest2d", {"x": rng(0, 24, lambda i: i)},
        dict(batch=2, channels=3, in_h=2, in_w=2, scale_h=2, scale_w=2), exact=True)
    add("upsample_1x1", "src/ops/upsample.rs:191-195", "upsample_nearest2d", {"x": [7]},
        dict(batch=1, channels=1, in_h=1, in_w=1, scale_h=3, scale_w=3), expect=[7] * 9,
        exact=True)
    return c


def main():
    data = {"generator": "tests/golden/make_kats.py",
            "reference": "cochranblock/any-gpu unit tests (file:line per case)",
            "cases": cases()}
    OUT.write_text(json.dumps(data, indent=1) + "\n")
    print(f"wrote {len(data['cases'])} cases to {OUT}")


if __name__ == "__main__":
    main()
