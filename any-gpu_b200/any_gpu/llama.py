"""LLaMA-style decoder layer forward composed from the library's ops.

Everything runs in libagpu kernels on caller-owned device memory (raw
pointers, one stream); this module only sequences the launches:

    h1  = rmsnorm(x, w_attn_norm)                       [T, d]      T = B*S
    qkv = h1 @ Wqkv                                     [T, 3d]     packed [B,S,3,H,Dh]
    q,k = rope(q), rope(k)       (in place, positions = sequence index)
    o   = sdpa(q, k, v)          (strided: read straight from qkv, written [B,S,H,Dh])
    x2  = x + o @ Wo             (residual fused in the GEMM epilogue)
    h2  = rmsnorm(x2, w_ffn_norm)
    a   = swish(h2 @ Wg) * (h2 @ Wu)                    [T, F]   (SwiGLU)
    y   = x2 + a @ Wd            (residual fused in the GEMM epilogue)

Weights are row-major [in, out] (x @ W).  Wgu [d, 2F] packs Wg and Wu: when
F % 32 == 0 in 32-column blocks (gate block j = columns [64j, 64j+32), up
block j = [64j+32, 64j+64)), so that the gate/up GEMM's epilogue writes
swish(gate) * up directly (gemm_ex act 3); otherwise as [Wg | Wu], with a
separate swish * up pass.  Attention is non-causal by default (the
reference's SDPA is non-causal); `causal=True` masks future keys.
"""
from __future__ import annotations

from dataclasses import dataclass

F32 = 4


@dataclass
class LlamaDims:
    batch: int
    seq: int
    d_model: int
    heads: int
    ffn: int
    eps: float = 1e-5
    rope_base: float = 10000.0
    causal: bool = False

    @property
    def tokens(self) -> int:
        return self.batch * self.seq

    @property
    def head_dim(self) -> int:
        return self.d_model // self.heads

    @property
    def fused_swiglu(self) -> bool:
        """Wgu in interleaved 32-column gate/up blocks, SwiGLU in the GEMM epilogue."""
        return self.ffn % 32 == 0

    def gemm_flops(self) -> float:
        t, d, f = self.tokens, self.d_model, self.ffn
        return 2.0 * t * (4 * d * d + 3 * d * f)

    def attention_flops(self) -> float:
        s = self.seq
        full = 4.0 * self.batch * self.heads * s * s * self.head_dim
        return full / 2 if self.causal else full

    def workspace_elems(self) -> dict:
        t, d, f = self.tokens, self.d_model, self.ffn
        return {"h": t * d, "qkv": t * 3 * d, "o": t * d, "x2": t * d,
                "gu": 1 if self.fused_swiglu else t * 2 * f, "a": t * f}


def layer_forward(dev, dims: LlamaDims, x, w, ws, y, stream: int = 0) -> None:
    """x, y: device pointers [T, d]; w: dict of weight pointers (attn_norm [d],
    wqkv [d,3d], wo [d,d], ffn_norm [d], wgu [d,2F], wd [F,d]); ws: dict of
    workspace pointers sized by dims.workspace_elems()."""
    B, S, d, H, Fd = dims.batch, dims.seq, dims.d_model, dims.heads, dims.ffn
    T, Dh = dims.tokens, dims.head_dim
    dev.launch_rmsnorm(x, w["attn_norm"], ws["h"], T, d, dims.eps, stream)
    dev.launch_gemm_ex(ws["h"], w["wqkv"], ws["qkv"], 1, T, 3 * d, d, stream=stream)
    q, k, v = ws["qkv"], ws["qkv"] + d * F32, ws["qkv"] + 2 * d * F32
    dev.launch_rope(q, q, B, S, H, Dh, 3 * d, dims.rope_base, stream)
    dev.launch_rope(k, k, B, S, H, Dh, 3 * d, dims.rope_base, stream)
    qkv_st = (3 * d, Dh, S * 3 * d)
    o_st = (d, Dh, S * d)
    dev.launch_sdpa_strided(q, k, v, ws["o"], B, H, S, Dh, qkv_st, qkv_st, qkv_st, o_st,
                            dims.causal, stream)
    dev.launch_gemm_ex(ws["o"], w["wo"], ws["x2"], 1, T, d, d, resid_ptr=x, stream=stream)
    dev.launch_rmsnorm(ws["x2"], w["ffn_norm"], ws["h"], T, d, dims.eps, stream)
    if dims.fused_swiglu:
        dev.launch_gemm_ex(ws["h"], w["wgu"], ws["a"], 1, T, 2 * Fd, d, act=3, stream=stream)
    else:
        dev.launch_gemm_ex(ws["h"], w["wgu"], ws["gu"], 1, T, 2 * Fd, d, stream=stream)
        dev.launch_swish_mul(ws["gu"], ws["gu"] + Fd * F32, ws["a"], T, Fd, 2 * Fd, 2 * Fd, Fd,
                             stream)
    dev.launch_gemm_ex(ws["a"], w["wd"], y, 1, T, d, Fd, resid_ptr=ws["x2"], stream=stream)
