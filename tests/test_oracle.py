"""CPU tests: the oracle against the reference's own known answers (pinning
it), against float64 numpy on seeded inputs, and the reference's numeric
gradient check for conv2d_grad_weight (src/ops/conv.rs:871-904)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import KATS
from kat_runner import check, run_oracle

LITERAL = [c for c in KATS if isinstance(c["expect"], list) or c.get("expect_slices")]
VS_CPU = [c for c in KATS if c["expect"] == "oracle"]


@pytest.mark.parametrize("case", LITERAL, ids=[c["name"] for c in LITERAL])
def test_oracle_matches_reference_literal(orc, case):
    got = run_oracle(orc, case)
    check(case, got)


def _f64_reference(case):
    op, x, a = case["op"], case["inputs"], case["args"]
    f = lambda v: np.asarray(v, np.float64)
    if op == "matmul":
        return (f(x["a"]).reshape(a["m"], a["k"]) @ f(x["b"]).reshape(a["k"], a["n"])).ravel()
    if op == "batch_matmul":
        A = f(x["a"]).reshape(a["batch"], a["m"], a["k"])
        B = f(x["b"]).reshape(a["batch"], a["k"], a["n"])
        return (A @ B).ravel()
    if op == "softmax":
        X = f(x["x"]).reshape(a["rows"], a["cols"])
        E = np.exp(X - X.max(1, keepdims=True))
        return (E / E.sum(1, keepdims=True)).ravel()
    if op == "sdpa":
        s, d = a["seq"], a["dk"]
        Q, K, V = (f(x[n]).reshape(-1, s, d) for n in "qkv")
        S = Q @ K.transpose(0, 2, 1) / np.sqrt(d)
        P = np.exp(S - S.max(-1, keepdims=True))
        P /= P.sum(-1, keepdims=True)
        return (P @ V).ravel()
    return None


@pytest.mark.parametrize("case", VS_CPU, ids=[c["name"] for c in VS_CPU])
def test_oracle_vs_float64(orc, case):
    want = _f64_reference(case)
    if want is None:
        pytest.skip("no float64 restatement for this op")
    got = run_oracle(orc, case)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)


def test_oracle_conv_grad_weight_numeric(orc):
    # src/ops/conv.rs:871-904: loss = sum(conv2d(x, w)), eps 1e-3, tol 1e-2
    x = [v * 0.1 for v in range(1, 17)]
    w = np.array([0.5, -0.5, 0.3, -0.3], np.float32)
    gw = orc.conv2d_grad_weight(x, np.ones(9, np.float32), 1, 1, 4, 4, 1, 3, 3, 2, 2, 1, 1, 0, 0,
                                1, 1, 1)
    eps = np.float32(1e-3)
    for i in range(4):
        wp, wm = w.copy(), w.copy()
        wp[i] += eps
        wm[i] -= eps
        sp = orc.conv2d(x, wp, None, 1, 1, 4, 4, 1, 2, 2).sum(dtype=np.float32)
        sm = orc.conv2d(x, wm, None, 1, 1, 4, 4, 1, 2, 2).sum(dtype=np.float32)
        assert abs(gw[i] - (sp - sm) / (2 * eps)) < 1e-2


@pytest.mark.parametrize("m,n,k", [(64, 48, 96), (17, 13, 11), (128, 256, 64)])
def test_oracle_matmul_random(orc, m, n, k):
    r = np.random.default_rng(7)
    a = r.uniform(-1, 1, m * k).astype(np.float32)
    b = r.uniform(-1, 1, k * n).astype(np.float32)
    got = orc.matmul(a, b, m, n, k)
    want = a.astype(np.float64).reshape(m, k) @ b.astype(np.float64).reshape(k, n)
    assert orc.rel_fro(got, want) < 1e-6
    np.testing.assert_array_equal(got, orc.matmul(a, b, m, n, k, threads=True))


def test_oracle_conv2d_random(orc):
    r = np.random.default_rng(3)
    N, C, H, W, O = 2, 4, 9, 7, 6
    x = r.standard_normal(N * C * H * W).astype(np.float32)
    w = r.standard_normal(O * C * 9).astype(np.float32)
    bias = r.standard_normal(O).astype(np.float32)
    got = orc.conv2d(x, w, bias, N, C, H, W, O, 3, 3, (1, 1), (1, 1), (1, 1), 1)
    xp = np.pad(x.reshape(N, C, H, W).astype(np.float64), ((0, 0), (0, 0), (1, 1), (1, 1)))
    wf = w.reshape(O, C, 3, 3).astype(np.float64)
    want = np.zeros((N, O, H, W))
    for i in range(3):
        for j in range(3):
            want += np.einsum("nchw,oc->nohw", xp[:, :, i:i + H, j:j + W], wf[:, :, i, j])
    want += bias[None, :, None, None]
    assert orc.rel_fro(got, want) < 1e-6
    np.testing.assert_array_equal(got, orc.conv2d(x, w, bias, N, C, H, W, O, 3, 3, (1, 1),
                                                  (1, 1), (1, 1), 1, threads=True))


def test_oracle_group_norm_random(orc):
    r = np.random.default_rng(5)
    N, C, S, G = 3, 8, 50, 4
    x = r.standard_normal(N * C * S).astype(np.float32)
    g = r.standard_normal(C).astype(np.float32)
    b = r.standard_normal(C).astype(np.float32)
    got = orc.group_norm(x, g, b, N, C, S, G, 1e-5)
    X = x.reshape(N, G, -1).astype(np.float64)
    Y = (X - X.mean(-1, keepdims=True)) / np.sqrt(X.var(-1, keepdims=True) + 1e-5)
    want = Y.reshape(N, C, S) * g[None, :, None] + b[None, :, None]
    assert orc.rel_fro(got, want) < 1e-5


def test_oracle_attention_random(orc):
    r = np.random.default_rng(9)
    bh, s, d = 3, 33, 16
    q, k, v = (r.standard_normal(bh * s * d).astype(np.float32) for _ in range(3))
    got = orc.attention(q, k, v, bh, s, d)
    case = {"op": "sdpa", "inputs": {"q": q, "k": k, "v": v}, "args": {"seq": s, "dk": d}}
    assert orc.rel_fro(got, _f64_reference(case)) < 1e-5
    np.testing.assert_array_equal(got, orc.attention(q, k, v, bh, s, d, threads=True))


def test_oracle_causal_first_row_is_v0(orc):
    r = np.random.default_rng(1)
    q, k, v = (r.standard_normal(2 * 5 * 4).astype(np.float32) for _ in range(3))
    out = orc.attention(q, k, v, 2, 5, 4, causal=True).reshape(2, 5, 4)
    np.testing.assert_allclose(out[:, 0], v.reshape(2, 5, 4)[:, 0], rtol=1e-6)


def test_oracle_rmsnorm_rope(orc):
    r = np.random.default_rng(2)
    x = r.standard_normal(4 * 64).astype(np.float32)
    w = r.standard_normal(64).astype(np.float32)
    got = orc.rmsnorm(x, w, 4, 64, 1e-5)
    X = x.reshape(4, 64).astype(np.float64)
    want = X / np.sqrt((X * X).mean(1, keepdims=True) + 1e-5) * w
    assert orc.rel_fro(got, want) < 1e-6
    # RoPE at position 0 is the identity; rotation preserves pair norms
    xr = r.standard_normal(1 * 3 * 2 * 8).astype(np.float32)
    y = orc.rope(xr, 1, 3, 2, 8).reshape(3, 2, 8)
    np.testing.assert_allclose(y[0], xr.reshape(3, 2, 8)[0], rtol=1e-6)
    X = xr.reshape(3, 2, 8)
    np.testing.assert_allclose(y[..., :4] ** 2 + y[..., 4:] ** 2,
                               X[..., :4] ** 2 + X[..., 4:] ** 2, rtol=1e-5)


def gn_backward_f64(dy, x, gamma, n, c, s, g, eps):
    """Gradients of group_norm from torch autograd in float64: an implementation
    independent of the reference's shaders (which have no tests of their own)."""
    import torch
    X = torch.tensor(np.asarray(x, np.float64).reshape(n, c, s), requires_grad=True)
    G = torch.tensor(np.asarray(gamma, np.float64), requires_grad=True)
    B = torch.zeros(c, dtype=torch.float64, requires_grad=True)
    Y = torch.nn.functional.group_norm(X, g, G, B, eps)
    Y.backward(torch.tensor(np.asarray(dy, np.float64).reshape(n, c, s)))
    return X.grad.numpy().ravel(), G.grad.numpy(), B.grad.numpy()


@pytest.mark.parametrize("n,c,s,g", [(2, 4, 3, 2), (2, 6, 37, 3), (1, 8, 64, 1)])
def test_oracle_group_norm_backward_vs_autograd(orc, n, c, s, g):
    """The oracle's restatement of SHADER_GN_BACK_* (src/ops/norm.rs:97-205)
    against torch autograd in float64."""
    r = np.random.default_rng(n * 100 + s)
    x = r.standard_normal(n * c * s).astype(np.float32)
    dy = r.standard_normal(n * c * s).astype(np.float32)
    gamma = (1 + 0.2 * r.standard_normal(c)).astype(np.float32)
    got = orc.group_norm_backward(dy, x, gamma, n, c, s, g, 1e-5)
    want = gn_backward_f64(dy, x, gamma, n, c, s, g, 1e-5)
    for a, b in zip(got, want):
        assert orc.rel_fro(a, b) <= 1e-4


def test_oracle_adamw_vs_float64(orc):
    """The oracle's restatement of SHADER_ADAMW (src/optim.rs:22-51) against the
    same update in float64 (the reference has no test of its own for AdamW)."""
    r = np.random.default_rng(11)
    n = 1000
    p, g = r.standard_normal(n).astype(np.float32), r.standard_normal(n).astype(np.float32)
    m, v = np.zeros(n, np.float32), np.zeros(n, np.float32)
    P, M, V = p.astype(np.float64), np.zeros(n), np.zeros(n)
    lr, b1, b2, eps, wd = 1e-3, 0.9, 0.999, 1e-8, 0.01
    for t in (1, 2, 3):
        p, m, v = orc.adamw(p, g, m, v, lr, b1, b2, eps, wd, t)
        M = b1 * M + (1 - b1) * g
        V = b2 * V + (1 - b2) * g.astype(np.float64) ** 2
        P = P * (1 - lr * wd) - lr * (M / (1 - b1 ** t)) / (np.sqrt(V / (1 - b2 ** t)) + eps)
    # v differs by ~1e-5: the shader's 1 - beta2 is 0.0009999871 in f32
    assert orc.rel_fro(p, P) <= 1e-6 and orc.rel_fro(m, M) <= 1e-6 and orc.rel_fro(v, V) <= 1e-4


def test_oracle_adamw_reference_tests(orc):
    """The reference's own AdamW tests (src/optim.rs:149-240), on the oracle."""
    one = lambda *x: np.array(x, np.float32)
    z = lambda n: np.zeros(n, np.float32)
    p, _, _ = orc.adamw(one(1, 2, 3), one(0.1, 0.2, 0.3), z(3), z(3), 0.01, weight_decay=0.0)
    assert (p < one(1, 2, 3)).all()                                  # test_adamw_basic
    p, m, v = one(10), z(1), z(1)
    for t in range(1, 11):                                           # test_adamw_multiple_steps
        p, m, v = orc.adamw(p, one(1), m, v, 0.1, weight_decay=0.0, step=t)
    assert p[0] < 10.0
    p, _, _ = orc.adamw(one(10), one(0), z(1), z(1), 0.01, weight_decay=0.1)
    assert abs(p[0] - 9.99) <= 1e-3                                  # test_adamw_weight_decay
    p, _, _ = orc.adamw(one(5), one(-1), z(1), z(1), 0.01, weight_decay=0.0)
    assert p[0] > 5.0                                                # test_adamw_negative_gradient


def test_oracle_tape_ops_vs_numpy(orc):
    """The restated tape shaders (src/ops/tensor_ops.rs, upsample.rs,
    attention.rs:72-87) against numpy on random shapes."""
    r = np.random.default_rng(11)
    a = r.standard_normal((5, 7)).astype(np.float32)
    b = r.standard_normal((5, 3)).astype(np.float32)
    np.testing.assert_array_equal(orc.concat(a, b, 5, 7, 3), np.concatenate([a, b], 1).ravel())
    ab = np.concatenate([a, b], 1)
    np.testing.assert_array_equal(orc.slice_per_block(ab, 5, 3, 7, 10), b.ravel())
    v = r.standard_normal(5).astype(np.float32)
    np.testing.assert_array_equal(orc.add_broadcast(a, v, 5, 7), (a + v[:, None]).ravel())
    np.testing.assert_allclose(orc.sum_inner(a, 5, 7), a.astype(np.float64).sum(1), rtol=1e-5)
    np.testing.assert_allclose(orc.sum_rows(a, 5, 7), a.astype(np.float64).sum(0), rtol=1e-5,
                               atol=1e-6)
    x = r.standard_normal((2, 3, 4, 5)).astype(np.float32)
    up = x.repeat(2, axis=2).repeat(3, axis=3)
    np.testing.assert_array_equal(orc.upsample_nearest2d(x, 2, 3, 4, 5, 2, 3), up.ravel())
    go = r.standard_normal(up.shape).astype(np.float32)
    want = go.reshape(2, 3, 4, 2, 5, 3).astype(np.float64).sum((3, 5))
    np.testing.assert_allclose(orc.upsample_nearest2d_backward(go, 2, 3, 4, 5, 2, 3),
                               want.ravel(), rtol=1e-5, atol=1e-6)
    t = r.standard_normal(a.size).astype(np.float32)
    d = a.ravel().astype(np.float64) - t
    np.testing.assert_allclose(orc.mse_loss(a, t)[0], (d * d).mean(), rtol=1e-5)


@pytest.mark.parametrize("causal", [False, True])
def test_oracle_attention_backward_matches_float64(orc, causal):
    """The oracle's attention backward (the reference's SDPA composition
    differentiated with its own matmul / scale rules and the softmax Jacobian)
    against float64 autograd of the same function."""
    import torch
    bh, s, d = 3, 40, 16
    r = np.random.default_rng(8 + causal)
    q, k, v, do = (r.standard_normal(bh * s * d).astype(np.float32) for _ in range(4))
    got = orc.attention_backward(q, k, v, do, bh, s, d, causal=causal)
    Q, K, V = (torch.tensor(x.reshape(bh, s, d), dtype=torch.float64, requires_grad=True)
               for x in (q, k, v))
    sc = Q @ K.transpose(1, 2) / np.sqrt(d)
    if causal:
        sc = sc.masked_fill(torch.ones(s, s, dtype=torch.bool).triu(1), float("-inf"))
    (torch.softmax(sc, -1) @ V).backward(torch.tensor(do.reshape(bh, s, d), dtype=torch.float64))
    for g, w in zip(got, (Q.grad, K.grad, V.grad)):
        w = w.numpy().ravel()
        assert np.linalg.norm(g - w) / np.linalg.norm(w) < 1e-5
