#ifndef QWN_PAGED_KV_H
#define QWN_PAGED_KV_H

/*
 * The reference's paged fp16 KV-cache API (c/qwn_paged_kv.h:12-85), served
 * by qwn_cuda.so: same names, signatures, struct layouts and constants, so a
 * caller built against the reference header links against this library
 * instead of c/qwn_paged_kv.c.
 *
 * Behind it: key_data / val_data are CUDA managed memory (valid on the host
 * and on the device, laid out [block][layer][kv_head][16][head_dim] fp16 as
 * the reference documents them); qwn_paged_kv_write converts on the GPU and
 * both attention calls run one GPU kernel per call.  The free stack and the
 * block tables stay plain host integers, exactly as the reference exposes
 * them in these structs.  Every call is synchronous on return, like the
 * reference's; calls run on the calling thread's current CUDA device.
 */

#include <stdint.h>
#include <stddef.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef QWN_REF_API
#define QWN_REF_API __attribute__((visibility("default")))
#endif

#define QWN_PAGE_BLOCK_SIZE 16  /* tokens per physical block (c/qwn_paged_kv.h:12) */
#define QWN_KV_PAGE_BYTES 16384 /* allocation alignment (c/qwn_paged_kv.h:13) */

/* c/qwn_paged_kv.h:15-25 */
typedef struct {
    uint16_t *key_data;    /* managed: [total_blocks][layers][kv_heads][16][head_dim] fp16 */
    uint16_t *val_data;    /* managed: same layout */
    int *free_stack;       /* host: LIFO of free block ids, initially total-1-i */
    int free_top;
    int total_blocks;
    int layers;
    int kv_heads;
    int head_dim;
    size_t block_bytes;    /* bytes of one block across all layers (K or V) */
} QwnKVBlockPool;

/* c/qwn_paged_kv.h:27-36 */
typedef struct {
    int req_id;
    int num_tokens;
    int max_tokens;
    int *block_ids;        /* host: physical block of each logical block */
    int block_count;
    int block_capacity;
    int prefill_remaining; /* prompt tokens not yet prefilled */
    int prefill_offset;
} QwnBlockTable;

/* c/qwn_paged_kv.h:38-41 */
typedef struct {
    int max_chunk_tokens;
    int active_requests;
} QwnChunkedScheduler;

/* <- c/qwn_paged_kv.c:42-80: 0, or -1 (bad geometry, no CUDA device, no memory) */
QWN_REF_API int qwn_kv_pool_init(QwnKVBlockPool *pool, int total_blocks, int layers, int kv_heads, int head_dim);
/* <- c/qwn_paged_kv.c:82-93 */
QWN_REF_API void qwn_kv_pool_free(QwnKVBlockPool *pool);
/* <- c/qwn_paged_kv.c:95-98: pop the free stack, -1 when empty */
QWN_REF_API int qwn_kv_pool_alloc_block(QwnKVBlockPool *pool);
/* <- c/qwn_paged_kv.c:100-103 */
QWN_REF_API void qwn_kv_pool_free_block(QwnKVBlockPool *pool, int block_id);
/* <- c/qwn_paged_kv.c:105-113 */
QWN_REF_API int qwn_block_table_init(QwnBlockTable *bt, int req_id, int initial_capacity);
/* <- c/qwn_paged_kv.c:115-138 */
QWN_REF_API int qwn_block_table_append_token(QwnKVBlockPool *pool, QwnBlockTable *bt);
/* <- c/qwn_paged_kv.c:140-149 */
QWN_REF_API void qwn_block_table_free(QwnKVBlockPool *pool, QwnBlockTable *bt);
/* <- c/qwn_paged_kv.c:151-198: fp32 K/V rows [kv_heads][head_dim] -> fp16 on the GPU */
QWN_REF_API int qwn_paged_kv_write(QwnKVBlockPool *pool, const QwnBlockTable *bt, int layer,
                                   int token_pos, const float *k, const float *v);
/* <- c/qwn_paged_kv.c:225-297: one head over tokens [0, num_tokens); scores_scratch
 * receives the softmax probabilities */
QWN_REF_API void qwn_paged_attention_head(const QwnKVBlockPool *pool, const QwnBlockTable *bt,
                                          int layer, int head_idx, int kv_head_idx,
                                          const float *q_head, float *scores_scratch,
                                          float *out_ctx_head);
/* <- c/qwn_paged_kv.c:299-382: the same result; the gather scratch buffers are
 * accepted and left untouched (the GPU kernel reads the pages in place) */
QWN_REF_API void qwn_paged_attention_gather_head(const QwnKVBlockPool *pool, const QwnBlockTable *bt,
                                                 int layer, int head_idx, int kv_head_idx,
                                                 const float *q_head, uint16_t *k_gather_scratch,
                                                 uint16_t *v_gather_scratch, float *scores_scratch,
                                                 float *out_ctx_head);
/* <- c/qwn_paged_kv.c:384-388 */
QWN_REF_API void qwn_scheduler_init(QwnChunkedScheduler *sched, int max_chunk_tokens);
/* <- c/qwn_paged_kv.c:390-396: 1 for a decode step, else min(prefill_remaining, max_chunk_tokens) */
QWN_REF_API int qwn_scheduler_next_chunk(const QwnChunkedScheduler *sched, const QwnBlockTable *bt);

#ifdef __cplusplus
}
#endif

#endif /* QWN_PAGED_KV_H */
