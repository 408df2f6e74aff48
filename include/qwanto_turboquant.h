#ifndef QWANTO_TURBOQUANT_H
#define QWANTO_TURBOQUANT_H

/*
 * The reference's typed KV-cache API (c/qwanto_turboquant.h:11-156): cache
 * mode and ABI-v1 byte contract, the contiguous Q8 cache and the TurboQuant
 * 3.5-bit cache, served by qwn_cuda.so with the same names, signatures,
 * constants and struct layouts (TurboQuantBlock is the packed 32-byte block).
 *
 * Behind it: the caches' buffers (packed_k/v, scales_k/v) are CUDA managed
 * memory in the reference's own byte layout, so callers may index them on
 * the host or hand pointers into them to qwn_turboquant_quantize_token, as
 * the reference decoder does (c/qwanto_decode.c:1765-1766).  Quantization,
 * the per-token dot/accumulate helpers and the attention heads run as GPU
 * kernels: codes and scales bit-exact with the reference (IEEE division,
 * round-to-nearest-even / roundf, the truncating fp16 of the TurboQuant
 * parameters), attention within |d| <= 1e-4 + 1e-3 |ref|.  The _avx2, _vnni
 * and _avx512 names are kept for source compatibility and run the same GPU
 * kernels as the _scalar ones.  Pointers may be host, pinned, managed or
 * device memory.  Every call returns after its results are in place.
 */

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef QWN_REF_API
#define QWN_REF_API __attribute__((visibility("default")))
#endif

#define TURBOQUANT_GROUP_SIZE 64
#define TURBOQUANT_BLOCK_BYTES 32
#define TURBOQUANT_PAYLOAD_BYTES 28

#define QWN_KV_CACHE_ABI_VERSION 1u
#define QWN_KV_CACHE_PAGE_SIZE 16u

/* c/qwanto_turboquant.h:29-34 */
typedef enum {
    QWN_KV_CACHE_FP16 = 0,
    QWN_KV_CACHE_Q8 = 1,
    QWN_KV_CACHE_TURBOQUANT_Q4 = 2,
    QWN_KV_CACHE_AUTO = 3
} QwnKvCacheMode;

/* c/qwanto_turboquant.h:36-49 */
typedef struct {
    uint32_t struct_size;
    uint32_t abi_version;
    uint32_t cache_dtype;
    uint32_t block_size;
    uint32_t scale_bytes;
    uint32_t zero_point_bytes;
    uint32_t key_layout;
    uint32_t value_layout;
    uint32_t page_size;
    uint32_t alignment;
    uint32_t valid_token_count;
    uint32_t reserved[5];
} QwnKvCacheContract;

/* <- c/qwanto_turboquant.c:20-27 */
QWN_REF_API const char *qwn_kv_cache_mode_name(QwnKvCacheMode mode);
/* <- c/qwanto_turboquant.c:29-38: "fp16", "q8", "turboquant-q4" | "qwn-q4-kv", "auto" */
QWN_REF_API int qwn_kv_cache_mode_parse(const char *text, QwnKvCacheMode *mode);
/* <- c/qwanto_turboquant.c:40-59 */
QWN_REF_API void qwn_kv_cache_contract_init(QwnKvCacheContract *contract, QwnKvCacheMode mode,
                                            uint32_t valid_token_count);

/* c/qwanto_turboquant.h:57-63 */
#pragma pack(push, 1)
typedef struct {
    uint16_t scale_fp16;      /* range = max - min, truncated to fp16 */
    uint16_t zero_point_fp16; /* min, truncated to fp16 */
    uint8_t packed_data[TURBOQUANT_PAYLOAD_BYTES]; /* 4 x (8 pairs of 4+3 bits in 7 bytes) */
} TurboQuantBlock;
#pragma pack(pop)

/* c/qwanto_turboquant.h:65-76 */
typedef struct {
    uint8_t *packed_k;       /* managed: [max_tokens][token_stride_k] */
    uint8_t *packed_v;
    int n_channels;
    int n_tokens;
    int max_tokens;
    int n_heads;
    int head_dim;
    size_t token_stride_k;
    size_t token_stride_v;
    size_t total_bytes;
} TurboQuantCache;

/* c/qwanto_turboquant.h:80-94 */
typedef struct {
    int8_t *packed_k;        /* managed: [max_tokens][n_channels] */
    int8_t *packed_v;
    float *scales_k;         /* managed: [max_tokens][ceil(n_channels/64)] */
    float *scales_v;
    int n_channels;
    int n_tokens;
    int max_tokens;
    int n_heads;
    int head_dim;
    size_t token_stride;
    size_t scale_stride;
    size_t total_bytes;
    QwnKvCacheContract contract;
} QwnQ8Cache;

/* <- c/qwanto_turboquant.c:588-614 */
QWN_REF_API int qwn_q8_cache_init(QwnQ8Cache *cache, int max_tokens, int n_heads, int head_dim);
/* <- c/qwanto_turboquant.c:617-624 */
QWN_REF_API void qwn_q8_cache_free(QwnQ8Cache *cache);
/* <- c/qwanto_turboquant.c:626-630 */
QWN_REF_API void qwn_q8_cache_reset(QwnQ8Cache *cache);
/* <- c/qwanto_turboquant.c:632-646 (quantizer :555-586), on the GPU */
QWN_REF_API int qwn_q8_cache_append(QwnQ8Cache *cache, const float *key, const float *value, int n_channels);
/* <- c/qwanto_turboquant.c:648-662 */
QWN_REF_API float qwn_q8_cache_dot_key_scalar(const QwnQ8Cache *cache, int token, int channel_offset,
                                              const float *query, int dim);
/* <- c/qwanto_turboquant.c:664-676 */
QWN_REF_API void qwn_q8_cache_accum_value_scalar(const QwnQ8Cache *cache, int token, int channel_offset,
                                                 float score, float *ctx, int dim);
/* <- c/qwanto_turboquant.c:678-705: tokens [0, pos]; scores_scratch receives
 * exp(score - max) per token, as the reference leaves it */
QWN_REF_API void qwn_q8_cache_attention_head(const float *query, const QwnQ8Cache *cache, int kv_head_idx,
                                             int pos, float scale, float *scores_scratch, float *ctx_out);

/* <- c/qwanto_turboquant.c:515-541 */
QWN_REF_API int qwn_turboquant_init(TurboQuantCache *cache, int max_tokens, int n_heads, int head_dim);
/* <- c/qwanto_turboquant.c:545-550 */
QWN_REF_API void qwn_turboquant_free(TurboQuantCache *cache);
/* <- c/qwanto_turboquant.c:162-213 (with pack_16_values :125-140), on the GPU */
QWN_REF_API void qwn_turboquant_quantize_token(const float *src, uint8_t *dst_blocks, int n_channels);
/* <- c/qwanto_turboquant.c:218-252 */
QWN_REF_API float qwn_turboquant_dot_key_scalar(const float *query, const uint8_t *key_blocks, int dim);
/* <- c/qwanto_turboquant.c:254-284 */
QWN_REF_API void qwn_turboquant_accum_value_scalar(float score, const uint8_t *value_blocks, float *ctx, int dim);
/* <- c/qwanto_turboquant.c:289-502 (ISA variants; the same GPU kernels here) */
QWN_REF_API float qwn_turboquant_dot_key_avx2(const float *query, const uint8_t *key_blocks, int dim);
QWN_REF_API void qwn_turboquant_accum_value_avx2(float score, const uint8_t *value_blocks, float *ctx, int dim);
QWN_REF_API float qwn_turboquant_dot_key_vnni(const float *query, const uint8_t *key_blocks, int dim);
QWN_REF_API void qwn_turboquant_accum_value_vnni(float score, const uint8_t *value_blocks, float *ctx, int dim);
QWN_REF_API float qwn_turboquant_dot_key_avx512(const float *query, const uint8_t *key_blocks, int dim);
QWN_REF_API void qwn_turboquant_accum_value_avx512(float score, const uint8_t *value_blocks, float *ctx, int dim);
/* <- c/qwanto_turboquant.c:707-768: tokens [0, pos]; scores_scratch receives
 * the softmax probabilities */
QWN_REF_API void qwn_turboquant_attention_head(const float *query, const TurboQuantCache *cache, int layer,
                                               int head_idx, int kv_head_idx, int pos, float scale,
                                               float *scores_scratch, float *ctx_out);
/* <- c/qwanto_turboquant.c:773-792: output[h * head_dim] = dot of query head h
 * with token 0's key blocks of head h */
QWN_REF_API void qwn_turboquant_matmul_avx512(const TurboQuantCache *cache, const float *query, float *output,
                                              int n_heads, int head_dim);

#ifdef __cplusplus
}
#endif

#endif /* QWANTO_TURBOQUANT_H */
