#ifndef QWANTO_PAGEDEVICTION_H
#define QWANTO_PAGEDEVICTION_H

/*
 * The reference's token-level eviction API (c/qwanto_pagedeviction.h:16-70),
 * served by qwn_cuda.so with the same names, signatures, constants and the
 * same 16-byte QwnVToken / QwnPagedEvictionPool layouts.  This bookkeeping is
 * host code (O(active tokens) per call on a caller-owned struct), with the
 * reference's results bit for bit: insert at slot active_count, sinks for
 * token_id < 4, EMA 0.8*old + 0.2*new on non-sink slots (one fused multiply-
 * add, as the reference compiles), prune in index order from slot 4, auto-
 * prune to 90% of the physical pool.  The GPU's page-level eviction is
 * qwn_kv_evict (qwn_kv_b200.h).
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

#define QWN_VTOKEN_MAX_CAPACITY 32768
#define QWN_VTOKEN_SINK_TOKENS 4

/* c/qwanto_pagedeviction.h:19-25 */
typedef struct {
    uint32_t token_id;
    float importance_score;
    uint32_t physical_slot;
    bool is_sink;
    bool is_active;
} QwnVToken;

/* c/qwanto_pagedeviction.h:27-34 */
typedef struct {
    QwnVToken virtual_tokens[QWN_VTOKEN_MAX_CAPACITY];
    uint32_t active_count;
    uint32_t max_capacity;
    uint32_t physical_pool_size;
    float eviction_threshold;
    uint64_t total_evictions;
} QwnPagedEvictionPool;

/* <- c/qwanto_pagedeviction.c:7-22 */
QWN_REF_API int qwn_paged_eviction_init(QwnPagedEvictionPool *pool, uint32_t max_capacity,
                                        uint32_t physical_pool_size, float eviction_threshold);
/* <- c/qwanto_pagedeviction.c:24-52: 0, -1 (bad arguments) or -2 (capacity) */
QWN_REF_API int qwn_paged_eviction_insert(QwnPagedEvictionPool *pool, uint32_t token_id,
                                          float initial_importance, uint32_t *assigned_physical_slot);
/* <- c/qwanto_pagedeviction.c:54-70 */
QWN_REF_API void qwn_paged_eviction_update_scores(QwnPagedEvictionPool *pool, const float *attention_scores,
                                                  uint32_t sequence_length);
/* <- c/qwanto_pagedeviction.c:72-93: tokens evicted */
QWN_REF_API uint32_t qwn_paged_eviction_prune(QwnPagedEvictionPool *pool, uint32_t target_retained_tokens);
/* <- c/qwanto_pagedeviction.c:95-103 */
QWN_REF_API float qwn_paged_eviction_memory_waste_pct(const QwnPagedEvictionPool *pool);

#ifdef __cplusplus
}
#endif

#endif /* QWANTO_PAGEDEVICTION_H */
