"""Reverse-mode autograd tape over the C ABI (reference: `Tape`, src/autograd.rs:1-480).

Same surface as the reference: `leaf`, the recorded forward ops (`add`, `sub`,
`mul`, `scale`, `relu`, `sigmoid`, `swish`, `tanh_act`, `matmul`, `mse_loss`,
`conv2d`, `concat`, `group_norm`, `upsample_nearest2d`, `add_broadcast`,
`add_per_col`), `read`, `read_grad` and `backward(loss)`, with tensor ids
numbered in creation order.  Every forward and backward step is one call of
the library's kernels; the backward rules are the reference's
(src/autograd.rs:281-476):

* Matmul: dA = dC B^T and dB = A^T dC as single GEMMs with a transposed
  operand (the reference transposes A and B first, :357-366);
* Conv2d: dX = conv_transpose2d(dC, W) with the output padding that recovers
  the input size, dW = conv2d_grad_weight, db = conv2d_grad_bias (:376-427);
* GroupNorm: group_norm_backward (:439-449); Concat: slice_per_block
  (:429-437); UpsampleNearest2d: its backward (:451-456); AddBroadcast /
  AddPerCol: sum_inner / sum_rows for the bias (:458-474);
* MseLoss: 2 (pred - target) / n, the upstream gradient not applied, as in
  the reference (:368-374, the loss is the tape's last node).

Two ops have no reference counterpart.  `linear` records matmul + bias +
activation as a single op whose forward is one GEMM with the bias (and a
ReLU) in its epilogue, and whose backward is the activation's mask, the two
GEMMs and the bias's `sum_rows`.  `scaled_dot_product_attention` records the
fused attention forward as one op; its backward (`agpu_sdpa_backward`) is the
reference's SDPA composition (src/ops/attention.rs:149-169) differentiated
with its matmul and scale rules and the softmax Jacobian.

Gradients are accumulated with `add` into a fresh buffer (:267-279); the
pass-through gradients of Add, Sub and the broadcast adds share the upstream
buffer instead of copying it (buffers are never written after creation).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np

from . import AnyGpuError, GpuBuffer, GpuDevice

_SHAPE = 1  # AGPU_ERR_SHAPE


@dataclass(frozen=True)
class TensorId:
    """Index of a tensor on its tape (reference: `TensorId(u32)`)."""
    index: int


@dataclass
class _Entry:
    op: str
    output: TensorId
    args: Dict


class Tape:
    """Records forward ops on one device and runs their backward in reverse."""

    def __init__(self, dev: GpuDevice):
        self.dev = dev
        self._entries: List[_Entry] = []
        self._bufs: List[GpuBuffer] = []
        self._grads: List[Optional[GpuBuffer]] = []

    # ----------------------------------------------------------- plumbing --
    def _push(self, buf: GpuBuffer, op: str, **args) -> TensorId:
        tid = TensorId(len(self._bufs))
        self._bufs.append(buf)
        self._grads.append(None)
        self._entries.append(_Entry(op, tid, args))
        return tid

    def buf(self, t: TensorId) -> GpuBuffer:
        return self._bufs[t.index]

    def leaf(self, data) -> TensorId:
        """Register a parameter or input (reference :85-92)."""
        return self._push(self.dev.upload(data), "leaf")

    def read(self, t: TensorId) -> np.ndarray:
        return self.dev.read(self._bufs[t.index])

    def read_grad(self, t: TensorId) -> Optional[np.ndarray]:
        g = self._grads[t.index]
        return None if g is None else self.dev.read(g)

    def grad(self, t: TensorId) -> Optional[GpuBuffer]:
        """The gradient buffer itself (stays on the device)."""
        return self._grads[t.index]

    def _accum(self, t: TensorId, g: GpuBuffer) -> None:
        cur = self._grads[t.index]
        self._grads[t.index] = g if cur is None else self.dev.add(cur, g)

    # ------------------------------------------------------- forward ops --
    def add(self, a, b):
        return self._push(self.dev.add(self.buf(a), self.buf(b)), "add", a=a, b=b)

    def sub(self, a, b):
        return self._push(self.dev.sub(self.buf(a), self.buf(b)), "sub", a=a, b=b)

    def mul(self, a, b):
        return self._push(self.dev.mul(self.buf(a), self.buf(b)), "mul", a=a, b=b)

    def scale(self, a, s: float):
        return self._push(self.dev.scale(self.buf(a), s), "scale", a=a, s=s)

    def relu(self, a):
        return self._push(self.dev.relu(self.buf(a)), "relu", a=a)

    def sigmoid(self, a):
        return self._push(self.dev.sigmoid(self.buf(a)), "sigmoid", a=a)

    def swish(self, a):
        return self._push(self.dev.swish(self.buf(a)), "swish", a=a)

    def tanh_act(self, a):
        return self._push(self.dev.tanh_act(self.buf(a)), "tanh", a=a)

    def matmul(self, a, b, m: int, n: int, k: int):
        out = self.dev.matmul(self.buf(a), self.buf(b), m, n, k)
        return self._push(out, "matmul", a=a, b=b, m=m, n=n, k=k)

    def mse_loss(self, pred, target):
        out = self.dev.mse_loss(self.buf(pred), self.buf(target))
        return self._push(out, "mse", pred=pred, target=target)

    def conv2d(self, input, weight, bias, batch, in_c, in_h, in_w, out_c, kh, kw,
               stride=(1, 1), padding=(0, 0), dilation=(1, 1), groups=1):
        out_h = (in_h + 2 * padding[0] - dilation[0] * (kh - 1) - 1) // stride[0] + 1
        out_w = (in_w + 2 * padding[1] - dilation[1] * (kw - 1) - 1) // stride[1] + 1
        out = self.dev.conv2d(self.buf(input), self.buf(weight),
                              self.buf(bias) if bias is not None else None, batch, in_c, in_h,
                              in_w, out_c, kh, kw, tuple(stride), tuple(padding),
                              tuple(dilation), groups)
        return self._push(out, "conv2d", input=input, weight=weight, bias=bias, batch=batch,
                          in_c=in_c, in_h=in_h, in_w=in_w, out_c=out_c, out_h=out_h,
                          out_w=out_w, kh=kh, kw=kw, stride=tuple(stride),
                          padding=tuple(padding), dilation=tuple(dilation), groups=groups)

    def concat(self, a, b, outer: int, a_inner: int, b_inner: int):
        out = self.dev.concat(self.buf(a), self.buf(b), outer, a_inner, b_inner)
        return self._push(out, "concat", a=a, b=b, outer=outer, a_inner=a_inner,
                          b_inner=b_inner)

    def group_norm(self, input, gamma, beta, batch, channels, spatial, groups, eps):
        out = self.dev.group_norm(self.buf(input), self.buf(gamma), self.buf(beta), batch,
                                  channels, spatial, groups, eps)
        return self._push(out, "group_norm", input=input, gamma=gamma, beta=beta, batch=batch,
                          channels=channels, spatial=spatial, groups=groups, eps=eps)

    def upsample_nearest2d(self, input, batch, channels, in_h, in_w, scale_h, scale_w):
        out = self.dev.upsample_nearest2d(self.buf(input), batch, channels, in_h, in_w,
                                          scale_h, scale_w)
        return self._push(out, "upsample", input=input, batch=batch, channels=channels,
                          in_h=in_h, in_w=in_w, scale_h=scale_h, scale_w=scale_w)

    def add_broadcast(self, a, b, outer: int, inner: int):
        out = self.dev.add_broadcast(self.buf(a), self.buf(b), outer, inner)
        return self._push(out, "add_broadcast", a=a, b=b, outer=outer, inner=inner)

    def add_per_col(self, a, b, rows: int, cols: int):
        out = self.dev.add_per_col(self.buf(a), self.buf(b), rows, cols)
        return self._push(out, "add_per_col", a=a, b=b, rows=rows, cols=cols)

    def linear(self, x, w, bias, m: int, n: int, k: int, act: str = "none"):
        """act(x @ w + bias[col]) as ONE recorded op and one launch: the bias
        and the activation run in the GEMM's epilogue (`agpu_gemm_ex`).  No
        reference counterpart: it records what `matmul` -> `add_per_col` ->
        `relu` record as three ops (three launches, two [m, n] intermediates)
        and has the same gradients.  `bias` may be None; `act` is "none",
        "relu" (the ReLU mask is read from the output, so no pre-activation
        is kept) or "swish" (its backward needs the pre-activation, so the
        GEMM fuses only the bias and the swish is a second launch)."""
        codes = {"none": 0, "relu": 2, "swish": 0}
        if act not in codes:
            raise ValueError(f"linear: act must be one of {sorted(codes)}, got {act!r}")
        out = self.dev.gemm_ex(self.buf(x), self.buf(w), 1, m, n, k,
                               bias=None if bias is None else self.buf(bias), act=codes[act])
        pre = None
        if act == "swish":
            pre, out = out, self.dev.swish(out)
        return self._push(out, "linear", a=x, b=w, bias=bias, m=m, n=n, k=k, act=act, pre=pre)

    def scaled_dot_product_attention(self, q, k, v, batch_heads: int, seq_len: int, d_k: int,
                                     causal: bool = False):
        """softmax(Q K^T / sqrt(d_k)) V per head as one recorded op (the fused
        forward kernel); gradients for Q, K and V from agpu_sdpa_backward."""
        f = self.dev.sdpa_causal if causal else self.dev.scaled_dot_product_attention
        out = f(self.buf(q), self.buf(k), self.buf(v), batch_heads, seq_len, d_k)
        return self._push(out, "sdpa", q=q, k=k, v=v, bh=batch_heads, s=seq_len, d=d_k,
                          causal=causal)

    # ----------------------------------------------------------- backward --
    def backward(self, loss: TensorId) -> None:
        """Gradients of every recorded tensor w.r.t. the 1-element `loss`
        (reference :281-477); a loss of another size raises AnyGpuError
        (AGPU_ERR_SHAPE), as the reference's `ensure!` returns Err."""
        if self._bufs[loss.index].len != 1:
            raise AnyGpuError(_SHAPE, "backward: loss must be a scalar (1 element)")
        d = self.dev
        self._grads[loss.index] = d.upload(np.ones(1, np.float32))
        for e in reversed(self._entries):
            g = self._grads[e.output.index]
            if g is None or e.op == "leaf":
                continue
            a = e.args
            if e.op == "add":
                self._accum(a["a"], g)
                self._accum(a["b"], g)
            elif e.op == "sub":
                self._accum(a["a"], g)
                self._accum(a["b"], d.scale(g, -1.0))
            elif e.op == "mul":
                ga = d.mul(g, self.buf(a["b"]))
                gb = d.mul(g, self.buf(a["a"]))
                self._accum(a["a"], ga)
                self._accum(a["b"], gb)
            elif e.op == "scale":
                self._accum(a["a"], d.scale(g, a["s"]))
            elif e.op == "relu":
                self._accum(a["a"], d.relu_backward(g, self.buf(a["a"])))
            elif e.op == "sigmoid":
                self._accum(a["a"], d.sigmoid_backward(g, self.buf(e.output)))
            elif e.op == "swish":
                self._accum(a["a"], d.swish_backward(g, self.buf(a["a"])))
            elif e.op == "tanh":
                self._accum(a["a"], d.tanh_backward(g, self.buf(e.output)))
            elif e.op == "matmul":
                m, n, k = a["m"], a["n"], a["k"]
                ga = d.gemm(g, self.buf(a["b"]), 1, m, k, n, trans_b=True)   # dC B^T
                gb = d.gemm(self.buf(a["a"]), g, 1, k, n, m, trans_a=True)   # A^T dC
                self._accum(a["a"], ga)
                self._accum(a["b"], gb)
            elif e.op == "mse":
                pred, target = a["pred"], a["target"]
                n = self._bufs[pred.index].len
                diff = d.sub(self.buf(pred), self.buf(target))
                self._accum(pred, d.scale(diff, 2.0 / n))
            elif e.op == "conv2d":
                self._conv2d_backward(g, a)
            elif e.op == "concat":
                comb = a["a_inner"] + a["b_inner"]
                ga = d.slice_per_block(g, a["outer"], a["a_inner"], 0, comb)
                gb = d.slice_per_block(g, a["outer"], a["b_inner"], a["a_inner"], comb)
                self._accum(a["a"], ga)
                self._accum(a["b"], gb)
            elif e.op == "group_norm":
                di, dg, db = d.group_norm_backward(g, self.buf(a["input"]), self.buf(a["gamma"]),
                                                   a["batch"], a["channels"], a["spatial"],
                                                   a["groups"], a["eps"])
                self._accum(a["input"], di)
                self._accum(a["gamma"], dg)
                self._accum(a["beta"], db)
            elif e.op == "upsample":
                gi = d.upsample_nearest2d_backward(g, a["batch"], a["channels"], a["in_h"],
                                                   a["in_w"], a["scale_h"], a["scale_w"])
                self._accum(a["input"], gi)
            elif e.op == "add_broadcast":
                self._accum(a["a"], g)
                self._accum(a["b"], d.sum_inner(g, a["outer"], a["inner"]))
            elif e.op == "add_per_col":
                self._accum(a["a"], g)
                self._accum(a["b"], d.sum_rows(g, a["rows"], a["cols"]))
            elif e.op == "linear":
                m, n, k = a["m"], a["n"], a["k"]
                if a["act"] == "relu":  # out > 0 exactly where the pre-activation is
                    g = d.relu_backward(g, self.buf(e.output))
                elif a["act"] == "swish":
                    g = d.swish_backward(g, a["pre"])
                self._accum(a["a"], d.gemm(g, self.buf(a["b"]), 1, m, k, n, trans_b=True))
                self._accum(a["b"], d.gemm(self.buf(a["a"]), g, 1, k, n, m, trans_a=True))
                if a["bias"] is not None:
                    self._accum(a["bias"], d.sum_rows(g, m, n))
            elif e.op == "sdpa":
                dq, dk, dv = d.sdpa_backward(self.buf(a["q"]), self.buf(a["k"]), self.buf(a["v"]),
                                             g, a["bh"], a["s"], a["d"], a["causal"])
                self._accum(a["q"], dq)
                self._accum(a["k"], dk)
                self._accum(a["v"], dv)
            else:  # pragma: no cover - every recorded op is handled above
                raise KeyError(e.op)

    def _conv2d_backward(self, g: GpuBuffer, a: Dict) -> None:
        d = self.dev
        (sh, sw), (ph, pw), (dh, dw) = a["stride"], a["padding"], a["dilation"]
        # output padding that makes the transposed conv recover the input size
        oph = a["in_h"] - ((a["out_h"] - 1) * sh - 2 * ph + dh * (a["kh"] - 1) + 1)
        opw = a["in_w"] - ((a["out_w"] - 1) * sw - 2 * pw + dw * (a["kw"] - 1) + 1)
        if oph < 0 or opw < 0:
            raise AnyGpuError(_SHAPE, "negative output_pad in conv backward")
        gi = d.conv_transpose2d(g, self.buf(a["weight"]), None, a["batch"], a["out_c"],
                                a["out_h"], a["out_w"], a["in_c"], a["kh"], a["kw"], (sh, sw),
                                (ph, pw), (oph, opw), (dh, dw), a["groups"])
        gw = d.conv2d_grad_weight(self.buf(a["input"]), g, a["batch"], a["in_c"], a["in_h"],
                                  a["in_w"], a["out_c"], a["out_h"], a["out_w"], a["kh"],
                                  a["kw"], sh, sw, ph, pw, dh, dw, a["groups"])
        gb = (d.conv2d_grad_bias(g, a["batch"], a["out_c"], a["out_h"], a["out_w"])
              if a["bias"] is not None else None)
        self._accum(a["input"], gi)
        self._accum(a["weight"], gw)
        if gb is not None:
            self._accum(a["bias"], gb)


__all__ = ["Tape", "TensorId"]
