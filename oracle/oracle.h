/* oracle.h -- TEST INFRASTRUCTURE ONLY: CPU restatement of the reference's
 * CPU implementations (see oracle.c).  Not linked into the product. */
#ifndef AGPU_ORACLE_H
#define AGPU_ORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif
int oracle_num_threads(void);
void oracle_matmul(const float* a, const float* b, float* out, int64_t m, int64_t n, int64_t k);
void oracle_matmul_mt(const float* a, const float* b, float* out, int64_t m, int64_t n, int64_t k);
void oracle_batch_matmul(const float* a, const float* b, float* out, int64_t batch, int64_t m,
                         int64_t n, int64_t k);
void oracle_batch_matmul_mt(const float* a, const float* b, float* out, int64_t batch, int64_t m,
                            int64_t n, int64_t k);
void oracle_softmax(const float* x, float* out, int64_t rows, int64_t cols);
void oracle_softmax_mt(const float* x, float* out, int64_t rows, int64_t cols);
void oracle_attention(const float* q, const float* k, const float* v, float* out, int64_t bh,
                      int64_t seq, int64_t dk);
void oracle_attention_mt(const float* q, const float* k, const float* v, float* out, int64_t bh,
                         int64_t seq, int64_t dk);
void oracle_attention_causal(const float* q, const float* k, const float* v, float* out,
                             int64_t bh, int64_t seq, int64_t dk);
int64_t oracle_conv_out(int64_t in, int64_t k, int64_t stride, int64_t pad, int64_t dil);
void oracle_conv2d(const float* input, const float* weight, const float* bias, float* out,
                   int64_t batch, int64_t in_c, int64_t in_h, int64_t in_w, int64_t out_c,
                   int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                   int64_t dh, int64_t dw, int64_t groups);
void oracle_conv2d_mt(const float* input, const float* weight, const float* bias, float* out,
                      int64_t batch, int64_t in_c, int64_t in_h, int64_t in_w, int64_t out_c,
                      int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                      int64_t dh, int64_t dw, int64_t groups);
void oracle_conv_transpose2d(const float* input, const float* weight, const float* bias,
                             float* out, int64_t batch, int64_t in_c, int64_t in_h, int64_t in_w,
                             int64_t out_c, int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                             int64_t ph, int64_t pw, int64_t oph, int64_t opw, int64_t dh,
                             int64_t dw, int64_t groups);
void oracle_conv2d_grad_weight(const float* input, const float* grad_out, float* grad_w,
                               int64_t batch, int64_t in_c, int64_t in_h, int64_t in_w,
                               int64_t out_c, int64_t out_h, int64_t out_w, int64_t kh,
                               int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                               int64_t dh, int64_t dw, int64_t groups);
void oracle_conv2d_grad_bias(const float* grad_out, float* grad_b, int64_t batch, int64_t out_c,
                             int64_t out_h, int64_t out_w);
void oracle_group_norm(const float* input, const float* gamma, const float* beta, float* out,
                       int64_t batch, int64_t channels, int64_t spatial, int64_t groups,
                       float eps);
void oracle_group_norm_mt(const float* input, const float* gamma, const float* beta, float* out,
                          int64_t batch, int64_t channels, int64_t spatial, int64_t groups,
                          float eps);
void oracle_group_norm_backward(const float* grad_out, const float* input, const float* gamma,
                                float* d_input, float* d_gamma, float* d_beta, int64_t batch,
                                int64_t channels, int64_t spatial, int64_t groups, float eps);
float oracle_sigmoid1(float x);
float oracle_swish1(float x);
void oracle_elementwise(int op, const float* a, const float* b, float s, float* out, int64_t n);
void oracle_transpose(const float* a, float* out, int64_t outer, int64_t d0, int64_t d1,
                      int64_t inner);
void oracle_add_per_col(const float* a, const float* b, float* out, int64_t rows, int64_t cols);
void oracle_rmsnorm(const float* x, const float* w, float* out, int64_t rows, int64_t cols,
                    float eps);
void oracle_rope(const float* x, float* out, int64_t batch, int64_t seq, int64_t heads,
                 int64_t dim, float base);
#ifdef __cplusplus
}
#endif
#endif
