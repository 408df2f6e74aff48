#ifndef QWANTO_ATTENTION_H
#define QWANTO_ATTENTION_H

/*
 * The reference's linear-attention API (c/qwanto_attention.h:11-69), served
 * by qwn_cuda.so with the same names, signatures and struct layout.  `state`
 * is CUDA managed memory [n_heads][head_dim][head_dim] fp32, readable on the
 * host like the reference's malloc'd state; decode and prefill run the GPU
 * kernels of qwn_linear_attention_* (bit-identical to the reference's AVX2 /
 * AVX-512 rounding order for head_dim % 8 == 0) and return after the outputs
 * are back in the caller's buffers.  head_dim 1..512.
 */

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef QWN_REF_API
#define QWN_REF_API __attribute__((visibility("default")))
#endif

/* c/qwanto_attention.h:11-15 */
typedef struct {
    int n_heads;
    int head_dim;
    float *state; /* managed: [n_heads][head_dim][head_dim] */
} QwantoLinearAttentionState;

/* <- c/qwanto_attention.c:11-19: 0, or -1 */
QWN_REF_API int qwanto_linear_attention_init(QwantoLinearAttentionState *state, int n_heads, int head_dim);
/* <- c/qwanto_attention.c:21-25 */
QWN_REF_API void qwanto_linear_attention_reset(QwantoLinearAttentionState *state);
/* <- c/qwanto_attention.c:27-32 */
QWN_REF_API void qwanto_linear_attention_destroy(QwantoLinearAttentionState *state);
/* <- c/qwanto_attention.c:34-142: Q/K/V/O [n_heads][head_dim] */
QWN_REF_API void qwanto_linear_attention_decode(QwantoLinearAttentionState *state,
                                                const float *Q, const float *K, const float *V,
                                                float decay, float *O);
/* <- c/qwanto_attention.c:144-156: Q/K/V/O [seq_len][n_heads][head_dim] */
QWN_REF_API void qwanto_linear_attention_prefill(QwantoLinearAttentionState *state,
                                                 const float *Q, const float *K, const float *V,
                                                 float decay, int seq_len, float *O);

#ifdef __cplusplus
}
#endif

#endif /* QWANTO_ATTENTION_H */
