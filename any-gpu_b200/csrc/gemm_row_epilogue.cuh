// Row-statistics epilogues of the GEMMs, applied once to a finished output
// element (row `row` of batch item `b`, column `col`): the two products of
// the attention backward that consume per-row vectors.
//
//   act 4 (probabilities): C = exp2(acc * scale - rowvec[b, row]), 0 where
//         `causal` and col > row -- softmax probabilities from scores and the
//         rows' saved base-2 log-sum-exp;
//   act 5 (softmax backward): C = aux[b, row, col] * (acc - rowvec[b, row])
//         * scale -- with aux = P and rowvec = D = rowsum(dO o O), the
//         softmax Jacobian-vector product of acc = dO V^T, scaled.
//
// Internal to the library (agpu_gemm_ex accepts act 0-3 only).
#pragma once

namespace agpu {

struct RowEpilogue {
  const float* rowvec = nullptr;  // [batch, M]
  const float* aux = nullptr;     // [batch, M, N] (act 5)
  float scale = 1.0f;
  int causal = 0;                 // act 4: zero above the diagonal
};

// Four consecutive columns col..col+3 of one row; `aux4` = aux at that
// element (act 5), `rv` = rowvec[b, row].
__device__ __forceinline__ float4 row_epilogue(float4 v, int act, const RowEpilogue& re,
                                               float rv, const float* aux4, int row, int col) {
  if (act == 4) {
    float4 o;
    o.x = (re.causal && col > row) ? 0.f : exp2f(v.x * re.scale - rv);
    o.y = (re.causal && col + 1 > row) ? 0.f : exp2f(v.y * re.scale - rv);
    o.z = (re.causal && col + 2 > row) ? 0.f : exp2f(v.z * re.scale - rv);
    o.w = (re.causal && col + 3 > row) ? 0.f : exp2f(v.w * re.scale - rv);
    return o;
  }
  const float4 p = __ldg(reinterpret_cast<const float4*>(aux4));
  return make_float4(p.x * (v.x - rv) * re.scale, p.y * (v.y - rv) * re.scale,
                     p.z * (v.z - rv) * re.scale, p.w * (v.w - rv) * re.scale);
}

__device__ __forceinline__ float row_epilogue1(float v, int act, const RowEpilogue& re, float rv,
                                               const float* aux1, int row, int col) {
  if (act == 4) return (re.causal && col > row) ? 0.f : exp2f(v * re.scale - rv);
  return __ldg(aux1) * (v - rv) * re.scale;
}

}  // namespace agpu
