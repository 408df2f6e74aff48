#ifndef QWN_KV_B200_H
#define QWN_KV_B200_H

/*
 * Paged, batched, device-resident quantized KV-cache entry points of
 * qwn_cuda.so (extension of ABI version 1).
 *
 * The reference keeps the quantized caches as contiguous per-layer arrays on
 * the host (c/qwanto_turboquant.c:515-543, :588-615) and pages only its fp16
 * cache (c/qwn_paged_kv.c:42-198); its GPU ABI moves host buffers on every
 * call (c/cuda/qwn_cuda_abi.h:130-149).  These entry points compose the
 * reference block table with the reference codecs on the GPU:
 *
 *   qwn_kv_pool_*      <- QwnKVBlockPool / qwn_kv_pool_init/free
 *                         (c/qwn_paged_kv.h:15-25, :44-53)
 *   qwn_kv_seq_append  <- qwn_block_table_append_token, once per sequence in
 *                         batch order (c/qwn_paged_kv.c:115-138)
 *   qwn_kv_decode      <- qwn_q8_cache_append + qwn_q8_cache_attention_head
 *                         (c/qwanto_turboquant.c:632-705) and the TurboQuant
 *                         pair qwn_turboquant_quantize_token +
 *                         qwn_turboquant_attention_head (:162-213, :707-768),
 *                         for every sequence and query head of one layer
 *   qwn_kv_evict       <- qwn_paged_eviction_update_scores/prune
 *                         (c/qwanto_pagedeviction.c:54-93), lifted to pages
 *
 * All pointers named *_dev are device pointers; host_* are host pointers.
 * Calls that take a stream enqueue work on it (NULL = the CUDA default
 * stream) and return without synchronising;
 * device-side failures (pool exhausted, bad page id, a wait that timed out)
 * are latched in a status word read by qwn_kv_pool_check().
 * Status codes are QwnCudaStatus (qwn_cuda_abi.h).
 */

#include "qwn_cuda_abi.h"

#ifdef __cplusplus
extern "C" {
#endif

#define QWN_KV_B200_VERSION 1u

/* capability bits reported by qwn_cuda_abi_query in addition to ABI v1's */
enum {
    QWN_CUDA_CAP_PAGED_KV = 1ull << 6,        /* qwn_kv_pool_* / qwn_kv_decode */
    QWN_CUDA_CAP_TQ_KV = 1ull << 7,           /* 4-bit and 3.5-bit codecs */
    QWN_CUDA_CAP_BATCHED_DEVICE = 1ull << 8,  /* device-pointer batched decode */
    QWN_CUDA_CAP_SPLIT_KV_MERGE = 1ull << 9,  /* partial (m,l,o) export + merge */
    QWN_CUDA_CAP_PAGE_EVICTION = 1ull << 10,  /* page scores, eviction, compaction */
    QWN_CUDA_CAP_LINEAR_ATTENTION = 1ull << 11 /* qwn_linear_attention_* */
};

typedef enum {
    QWN_KV_CODEC_Q8_B64_F32 = 1,  /* reference Q8: fp32 scale per 64 channels */
    QWN_KV_CODEC_Q8_HEAD_F16 = 2, /* int8 per token-head, fp16 absmax scale */
    QWN_KV_CODEC_TQ35_G64 = 3,    /* reference TurboQuant 4/3-bit, groups of 64 */
    QWN_KV_CODEC_Q4_G32 = 4,      /* 4-bit, groups of 32, fp16 range + fp16 min */
    QWN_KV_CODEC_F16 = 5          /* fp16 K and V, round to nearest even: the reference's paged
                                     pool (qwn_paged_kv_write, c/qwn_paged_kv.c:151-198) */
} QwnKvCodec;

/* device status bits latched by kernels */
enum {
    QWN_KV_STATUS_POOL_EXHAUSTED = 1u << 0,
    QWN_KV_STATUS_TABLE_OVERFLOW = 1u << 1,
    QWN_KV_STATUS_BAD_PAGE = 1u << 2,
    QWN_KV_STATUS_BAD_SEQUENCE = 1u << 3,
    QWN_KV_STATUS_WAIT_TIMEOUT = 1u << 4,
    QWN_KV_STATUS_BAD_LENGTH = 1u << 5,
    QWN_KV_STATUS_PEER_TIMEOUT = 1u << 6  /* a rank's partial did not arrive (qwn_kv_decode_split) */
};

typedef struct {
    QwnCudaAbiHeader header;
    int32_t device_id;
    uint32_t codec;             /* QwnKvCodec */
    uint32_t layers;
    uint32_t kv_heads;
    uint32_t head_dim;          /* must be 128 */
    uint32_t page_tokens;       /* multiple of 16 (16 = QWN_PAGE_BLOCK_SIZE) */
    uint32_t total_pages;       /* physical pages in the pool */
    uint32_t max_seqs;          /* sequence slots (block tables) */
    uint32_t max_pages_per_seq;
    uint32_t max_query_heads;   /* largest query_heads used with this pool */
    uint64_t permutation_seed;  /* 0: free stack total-1-i, as qwn_kv_pool_init;
                                   else a seeded Fisher-Yates permutation of it */
    uint64_t memory_budget_bytes; /* 0: no budget beyond the device's free memory */
} QwnKvPoolOptions;

typedef struct { QwnCudaAbiHeader header; void *opaque; } QwnKvPoolHandle;

typedef struct {
    QwnCudaAbiHeader header;
    void *pages_dev;            /* [total_pages][layers][kv_heads][page_tokens/16][tile_bytes] */
    int32_t *page_table_dev;    /* [max_seqs][max_pages_per_seq], -1 = none */
    int32_t *seq_lens_dev;      /* [max_seqs] tokens */
    int32_t *seq_pages_dev;     /* [max_seqs] pages held */
    int32_t *free_stack_dev;    /* [total_pages] */
    int32_t *free_top_dev;      /* [1] */
    float *page_scores_dev;     /* [max_seqs][max_pages_per_seq] eviction EMA */
    uint32_t *status_dev;       /* [1] QWN_KV_STATUS_* bits */
    uint64_t tile_bytes, page_bytes, pool_bytes, scratch_bytes;
    uint32_t attention_ctas, attention_warps; /* persistent grid of qwn_kv_decode */
    uint32_t reserved;
} QwnKvPoolInfo;

QWN_CUDA_ABI_API int qwn_kv_pool_create(const QwnKvPoolOptions *options, QwnKvPoolHandle *pool);
QWN_CUDA_ABI_API int qwn_kv_pool_destroy(QwnKvPoolHandle *pool);
QWN_CUDA_ABI_API int qwn_kv_pool_get_info(const QwnKvPoolHandle *pool, QwnKvPoolInfo *info);
/* empty every sequence and rebuild the free stack; synchronous */
QWN_CUDA_ABI_API int qwn_kv_pool_reset(QwnKvPoolHandle *pool);
/* return and clear the latched status bits (and, after a wait timeout, the
 * split-KV merge counters an abandoned merge left behind).  The pool's work
 * may run on any of the caller's streams, so this synchronises the device. */
QWN_CUDA_ABI_API int qwn_kv_pool_check(QwnKvPoolHandle *pool, uint32_t *status_bits);

/* Grow sequences: sequence seq_ids[i] gains counts[i] tokens (1 when
 * counts_dev is NULL; seq_ids_dev NULL means 0..num_seqs-1).  Pages are
 * popped from the LIFO free stack in batch order.  All-or-nothing: when the
 * pool cannot hold the request nothing changes and POOL_EXHAUSTED latches. */
QWN_CUDA_ABI_API int qwn_kv_seq_append(QwnKvPoolHandle *pool, uint32_t num_seqs,
                                       const int32_t *seq_ids_dev, const int32_t *counts_dev,
                                       void *stream);

typedef struct {
    QwnCudaAbiHeader header;
    uint32_t layer;
    uint32_t num_seqs;
    const int32_t *seq_ids_dev; /* [num_seqs] or NULL = 0..num_seqs-1 */
    uint32_t query_heads;       /* multiple of kv_heads, at most 8 per kv head */
    float scale;                /* softmax scale; 0 = 1/sqrt(128) */
    const float *query_dev;     /* [num_seqs][query_heads][128] fp32 */
    const float *key_dev;       /* [num_seqs][kv_heads][128] fp32 of the newest token, or NULL */
    const float *value_dev;     /* same shape as key_dev */
    float *output_dev;          /* [num_seqs][query_heads][128] fp32 */
    float *page_mass_dev;       /* optional [max_seqs][max_pages_per_seq]: per-page
                                   attention mass summed over query heads */
    uint32_t attend_limit;      /* attend tokens [0, min(len, attend_limit)); 0 = len */
    uint32_t reserved;
    void *stream;               /* cudaStream_t; NULL = the CUDA default stream */
} QwnKvDecodeRequest;

/* One layer of decode for a batch: when key_dev/value_dev are given, the
 * newest token of each sequence (position len-1, reserved by
 * qwn_kv_seq_append) is quantized into its page; then GQA attention over the
 * sequence's pages (query head h reads kv head h / (query_heads/kv_heads)). */
QWN_CUDA_ABI_API int qwn_kv_decode(QwnKvPoolHandle *pool, const QwnKvDecodeRequest *request);

/* Quantize-on-append only: the newest token (position len-1) of each
 * sequence of the batch, for one layer (qwn_q8_cache_append /
 * qwn_turboquant_quantize_token, c/qwanto_turboquant.c:632-646, :162-213).
 * key/value: [num_seqs][kv_heads][128] fp32 device arrays. */
QWN_CUDA_ABI_API int qwn_kv_append(QwnKvPoolHandle *pool, uint32_t layer, uint32_t num_seqs,
                                   const int32_t *seq_ids_dev, const float *key_dev,
                                   const float *value_dev, void *stream);

/* Partial attention for split-KV across devices: like qwn_kv_decode without
 * append over tokens [t_begin, t_end), writing the base-2 partial state
 * m[q_head], l[q_head], o[q_head][128] (o unnormalised) per sequence. */
typedef struct {
    QwnCudaAbiHeader header;
    uint32_t layer, num_seqs;
    const int32_t *seq_ids_dev;
    uint32_t query_heads;
    float scale;
    const float *query_dev;
    float *m_dev;               /* [num_seqs][query_heads] */
    float *l_dev;               /* [num_seqs][query_heads] */
    float *o_dev;               /* [num_seqs][query_heads][128] */
    uint32_t t_begin, t_end;    /* token range; t_end 0 = len */
    void *stream;
} QwnKvPartialRequest;
QWN_CUDA_ABI_API int qwn_kv_partial(QwnKvPoolHandle *pool, const QwnKvPartialRequest *request);

/* out[s][h][:] = merge over parts p of (m, l, o)[p][s][h] */
QWN_CUDA_ABI_API int qwn_kv_merge_partials(uint32_t parts, uint32_t rows, const float *m_dev,
                                           const float *l_dev, const float *o_dev,
                                           float *out_dev, void *stream);
/* The same merge with each part packed as one block of rows*130 floats:
 * o[rows][128], then m[rows], then l[rows] (the layout qwn_kv_partial writes
 * when its o/m/l pointers point into one block), so a single all-gather of
 * the blocks carries every part.  No counterpart in the reference (its
 * decoder has no split-KV path); the merge rule is qwn_kv_merge_partials'. */
QWN_CUDA_ABI_API int qwn_kv_merge_partials_packed(uint32_t parts, uint32_t rows, const float *packed_dev,
                                                  float *out_dev, void *stream);

/* ---- split-KV over the GPUs of one node, exchange fused into attention ----
 * Each rank attends its token range of one sequence.  The warp that completes
 * a (sequence, kv head) segment's partial state (m, l, o) stores it into every
 * rank's exchange buffer with plain peer stores over NVLink, raises that
 * segment's flag there, waits (bounded) for every rank's flag of the segment in
 * its own buffer and merges the ranks' partials in rank order: every rank ends
 * with the same output rows, and no collective or merge launch follows.  This
 * replaces qwn_kv_partial + an all-gather + qwn_kv_merge_partials_packed; the
 * reference's decoder has no split-KV path (its merge rule is the one of
 * qwn_kv_merge_partials).
 * Exchange buffer of a rank: flags [2 parities][QWN_KV_MAX_RANKS senders]
 * [QWN_KV_EXCHANGE_SEGMENTS] u32, then blocks [2][QWN_KV_MAX_RANKS] of
 * max_rows*130 floats (o[max_rows][128], m[max_rows], l[max_rows]).  Calls
 * alternate parities, so a rank one call ahead never overwrites a block that
 * a slower rank is still merging. */
#define QWN_KV_MAX_RANKS 8u
#define QWN_KV_EXCHANGE_SEGMENTS 64u

/* bytes of one rank's exchange buffer for rows of up to max_rows query heads */
QWN_CUDA_ABI_API int qwn_kv_exchange_bytes(uint32_t max_rows, uint64_t *bytes);
/* allocate and zero this rank's exchange buffer on device_id; ipc_handle
 * (64 bytes) receives the CUDA IPC handle the other ranks open */
QWN_CUDA_ABI_API int qwn_kv_exchange_alloc(int32_t device_id, uint64_t bytes, void **buffer_dev,
                                           void *ipc_handle);
QWN_CUDA_ABI_API int qwn_kv_exchange_free(int32_t device_id, void *buffer_dev);
/* map another rank's buffer (its 64-byte IPC handle) into this process on device_id */
QWN_CUDA_ABI_API int qwn_kv_exchange_open(int32_t device_id, const void *ipc_handle, void **buffer_dev);
QWN_CUDA_ABI_API int qwn_kv_exchange_close(int32_t device_id, void *buffer_dev);

typedef struct {
    QwnCudaAbiHeader header;
    uint32_t rank, world;                /* world <= QWN_KV_MAX_RANKS */
    uint32_t max_rows;                   /* row capacity the buffers were sized for */
    uint32_t reserved;
    void *buffers[QWN_KV_MAX_RANKS];     /* rank p's exchange buffer as mapped here; [rank] = own */
    uint64_t timeout_ns;                 /* bound on each wait for a rank's partial; 0 = 2 s */
} QwnKvPeerSet;

typedef struct {
    QwnCudaAbiHeader header;
    uint32_t layer;
    uint32_t query_heads;               /* multiple of kv_heads, at most 8 per kv head, <= max_rows */
    const int32_t *seq_ids_dev;         /* [1]: the sequence, or NULL = sequence 0 */
    float scale;                        /* softmax scale; 0 = 1/sqrt(128) */
    uint32_t epoch;                     /* 1, 2, 3, ...: one per call, the same on every rank */
    const float *query_dev;             /* [query_heads][128] */
    const float *key_dev;               /* newest token [kv_heads][128] on the rank whose range runs to the
                                           end of the sequence (t_end 0), stored before it is read; else NULL */
    const float *value_dev;
    float *output_dev;                  /* [query_heads][128]: the merged rows, the same on every rank */
    uint32_t t_begin, t_end;            /* this rank's token range, t_end 0 = to the end; must hold tokens */
    const QwnKvPeerSet *peers;
    void *stream;
} QwnKvSplitRequest;
QWN_CUDA_ABI_API int qwn_kv_decode_split(QwnKvPoolHandle *pool, const QwnKvSplitRequest *request);

/* Store tokens [first_pos, first_pos+n_tokens) of one sequence and layer
 * (already reserved with qwn_kv_seq_append): key/value [n_tokens][kv_heads][128]. */
QWN_CUDA_ABI_API int qwn_kv_store_tokens(QwnKvPoolHandle *pool, int32_t seq_id, uint32_t layer,
                                         uint32_t first_pos, uint32_t n_tokens,
                                         const float *key_dev, const float *value_dev,
                                         void *stream);

/* Synthetic inputs: x = Irwin-Hall(12) sample of the counter-based
 * generator (seed, kind, seq, layer, index); kind 1 = Q, 2 = K, 3 = V.
 * Row i of out_dev is position pos_dev[i] of sequence seq_ids_dev[i]:
 * out[i][c] = x(index = pos*width + c), times 8 where outlier_mask_dev[c]. */
QWN_CUDA_ABI_API int qwn_kv_generate_rows(float *out_dev, uint32_t rows, uint32_t width,
                                          uint32_t kind, uint64_t seed, uint32_t layer,
                                          const int32_t *seq_ids_dev, const int32_t *pos_dev,
                                          const uint8_t *outlier_mask_dev, void *stream);
/* Grow sequences to lens (pages in batch order, like qwn_kv_seq_append) and
 * fill every layer with quantized synthetic K/V of those positions.
 * outlier_mask_host: optional [layers][kv_heads*128] (1 = K channel x8). */
QWN_CUDA_ABI_API int qwn_kv_prefill_synthetic(QwnKvPoolHandle *pool, uint32_t num_seqs,
                                              const int32_t *host_seq_ids,
                                              const int32_t *host_lens, uint64_t seed,
                                              const uint8_t *outlier_mask_host, void *stream);

typedef struct {
    QwnCudaAbiHeader header;
    uint32_t num_seqs;
    const int32_t *seq_ids_dev;   /* or NULL = 0..num_seqs-1 */
    const float *page_mass_dev;   /* [max_seqs][max_pages_per_seq] from qwn_kv_decode */
    const uint8_t *flags_dev;     /* [num_seqs]: 1 = evict this sequence now */
    uint32_t token_budget;
    uint32_t reserved;
    void *stream;
} QwnKvEvictRequest;
/* score = 0.8*score + 0.2*mass on every page of the batch; then for each
 * flagged sequence longer than the budget, evict its lowest-score pages
 * (page 0 and the last page protected, ties to the lower index) until
 * len <= budget, compact the table and push the freed pages on the free
 * stack in ascending logical order, sequences in batch order. */
QWN_CUDA_ABI_API int qwn_kv_evict(QwnKvPoolHandle *pool, const QwnKvEvictRequest *request);

/* End-to-end decode step through host buffers (the plugin path with copies
 * inside): grows every sequence 0..num_seqs-1 by one token, copies the
 * layers' inputs host->device, runs qwn_kv_decode per layer and copies the
 * outputs back; returns after the last copy.  The layers move in up to seven
 * chunks (the first and the last layer alone): each chunk's layers launch
 * back to back while the next chunk's inputs and the previous chunk's
 * outputs are in flight on two copy streams.  Host arrays are
 * [layers][num_seqs][heads][128] fp32 (heads = query_heads for query/output,
 * kv_heads for key/value); pinned host memory gives overlapped copies. */
typedef struct {
    QwnCudaAbiHeader header;
    uint32_t num_layers, num_seqs, query_heads;
    float scale;
    const float *host_query;
    const float *host_key;
    const float *host_value;
    float *host_output;
} QwnKvHostStepRequest;
QWN_CUDA_ABI_API int qwn_kv_decode_step_host(QwnKvPoolHandle *pool,
                                             const QwnKvHostStepRequest *request,
                                             QwnCudaTelemetry *telemetry);

/* Decode attention that allocates nothing.  This entry point has no
 * counterpart in the reference; it exists for callers that cannot allocate
 * device memory at the moment they need attention: a server that gave all
 * free HBM to its own arena at start-up, a latency-critical loop that cannot
 * afford cudaMalloc/cudaFree synchronising the device, or an FFI caller that
 * holds only raw device pointers to a KV pool laid out as qwn_kv_pool_* lays
 * it out (QwnKvPoolInfo gives them) and no pool handle.
 * It runs the qwn_kv_decode attention (no append) with its scratch in a
 * fixed device array inside the library (about 4.3 MB per device, held until
 * the process exits).  Limits: num_seqs x kv_heads <= 256; query heads per kv
 * head <= 8; head_dim 128; every codec of QwnKvCodec (Q8_B64_F32, Q8_HEAD_F16,
 * TQ35_G64, Q4_G32, F16).  pages_dev, query_dev and output_dev must be
 * 16-byte aligned and the int32 arrays 4-byte aligned (INVALID_ARGUMENT
 * otherwise, before anything is launched).  All calls on a device share the
 * array: calls whose work may overlap on the GPU race and must be ordered by
 * the caller.  The first call on a device sets the array up (looks up its
 * address); make it before any stream capture. */
typedef struct {
    QwnCudaAbiHeader header;
    int32_t device_id;
    uint32_t codec;
    uint32_t layers, kv_heads, head_dim, page_tokens;  /* pool geometry */
    uint32_t total_pages, max_seqs, max_pages_per_seq;
    uint32_t layer, num_seqs, query_heads;
    float scale;                    /* 0 = 1/sqrt(128) */
    const void *pages_dev;
    const int32_t *page_table_dev;  /* [max_seqs][max_pages_per_seq] */
    const int32_t *seq_lens_dev;    /* [max_seqs] */
    const int32_t *seq_ids_dev;     /* [num_seqs] or NULL = 0..num_seqs-1 */
    const float *query_dev;         /* [num_seqs][query_heads][128] */
    float *output_dev;              /* [num_seqs][query_heads][128] */
    uint32_t *status_dev;           /* optional QWN_KV_STATUS_* bits */
    void *stream;                   /* NULL = the CUDA default stream */
} QwnKvStaticAttentionRequest;
QWN_CUDA_ABI_API int qwn_kv_attention_static(const QwnKvStaticAttentionRequest *request);

/* copy a device range to/from host (tests and tools without a CUDA runtime) */
QWN_CUDA_ABI_API int qwn_kv_memcpy_d2h(void *host, const void *dev, uint64_t bytes);
QWN_CUDA_ABI_API int qwn_kv_memcpy_h2d(void *dev, const void *host, uint64_t bytes);
/* kernel launches issued by this library since load (for evidence in runs) */
QWN_CUDA_ABI_API uint64_t qwn_kv_launch_count(void);

/* ---- linear attention on a device-resident state ------------------------
 * Mirrors QwantoLinearAttentionState and qwanto_linear_attention_init/reset/
 * destroy/decode/prefill (c/qwanto_attention.h:11-72, c/qwanto_attention.c:
 * 11-156); the first three fields keep the reference struct's order, with
 * `state` a DEVICE pointer to [n_heads][head_dim][head_dim] fp32 (row = key
 * dim, column = value dim).  Per token and head:
 *     S[i][j] = fma(decay, S[i][j], RN(k_i * v_j)),
 *     O[j]    = fma chain over i = 0..head_dim-1 of q_i * S[i][j] from 0,
 * the reference's AVX2/AVX-512 order and rounding, so states and outputs are
 * bit-identical to the reference built with -mavx2 -mfma for head_dim % 8 ==
 * 0 (its SIMD paths).  Batched sequences are more heads: n_heads = sequences
 * x heads with q/k/v/o laid out [seq_len][n_heads][head_dim].
 * head_dim 1..512.  The *_host call copies host buffers in and out and
 * synchronises, like the reference call it replaces; the others enqueue on
 * `stream` (NULL = default stream) and return. */
typedef struct {
    int32_t n_heads;
    int32_t head_dim;
    float *state;          /* device [n_heads][head_dim][head_dim] fp32 */
    int32_t device_id;
    uint32_t reserved;
    void *staging;         /* library-owned device scratch of the *_host call */
    uint64_t staging_bytes;
} QwnLinearAttentionState;

/* <- qwanto_linear_attention_init (c/qwanto_attention.c:11-19): allocates and zeroes */
QWN_CUDA_ABI_API int qwn_linear_attention_init(QwnLinearAttentionState *state, int32_t device_id,
                                               int32_t n_heads, int32_t head_dim);
/* <- qwanto_linear_attention_reset (c/qwanto_attention.c:21-25) */
QWN_CUDA_ABI_API int qwn_linear_attention_reset(QwnLinearAttentionState *state, void *stream);
/* <- qwanto_linear_attention_destroy (c/qwanto_attention.c:27-32) */
QWN_CUDA_ABI_API int qwn_linear_attention_destroy(QwnLinearAttentionState *state);
/* <- qwanto_linear_attention_decode (c/qwanto_attention.c:34-142); q/k/v/o [n_heads][head_dim] */
QWN_CUDA_ABI_API int qwn_linear_attention_decode(QwnLinearAttentionState *state, const float *q_dev,
                                                 const float *k_dev, const float *v_dev, float decay,
                                                 float *o_dev, void *stream);
/* <- qwanto_linear_attention_prefill (c/qwanto_attention.c:144-156); [seq_len][n_heads][head_dim] */
QWN_CUDA_ABI_API int qwn_linear_attention_prefill(QwnLinearAttentionState *state, const float *q_dev,
                                                  const float *k_dev, const float *v_dev, float decay,
                                                  int32_t seq_len, float *o_dev, void *stream);
/* the same prefill on HOST buffers (copies in, runs, copies out, synchronises) */
QWN_CUDA_ABI_API int qwn_linear_attention_prefill_host(QwnLinearAttentionState *state, const float *q,
                                                       const float *k, const float *v, float decay,
                                                       int32_t seq_len, float *o);

#ifdef __cplusplus
}
#endif

#endif /* QWN_KV_B200_H */
