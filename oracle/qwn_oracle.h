/*
 * qwn_oracle.h -- CPU restatement of Qwanto's quantized KV-cache path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the parity checker for the CUDA
 * implementation in qwanto_b200/csrc.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg may load it, and only to check results or
 * to time the CPU baseline.  The product library never links or calls it.
 *
 * Every function cites the reference routine it restates (paths relative to
 * the reference checkout, e.g. c/qwanto_turboquant.c:573).  Where the
 * reference has no implementation (the paged quantized layout, the per-head
 * fp16 Q8 codec, the 4-bit group-32 codec, page-level eviction) the function
 * is this project's own specification, stated in plain C so that the CUDA
 * kernels and this file can be compared bit for bit.
 *
 * Pinning: the reference-exact codecs (Q8 with fp32 scale per 64 channels,
 * TurboQuant 3.5-bit groups of 64), the block table and the token-level
 * eviction API are checked against the reference's own functions compiled
 * from its sources into oracle/_ref (see oracle/Makefile) and against the
 * reference tests' analytic inputs (c/tests/test_kv_cache.c:29-59).
 */
#ifndef QWN_ORACLE_H
#define QWN_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Codec identifiers; the same numbers are used by include/qwn_kv_b200.h. */
enum {
    QOR_CODEC_Q8_B64_F32 = 1,  /* reference Q8: int8, fp32 scale per 64 channels */
    QOR_CODEC_Q8_HEAD_F16 = 2, /* int8 per token-head, fp16 absmax scale */
    QOR_CODEC_TQ35_G64 = 3,    /* reference TurboQuant: 4/3-bit alternating, groups of 64 */
    QOR_CODEC_Q4_G32 = 4,      /* 4-bit, groups of 32, fp16 range + fp16 min */
    QOR_CODEC_F16 = 5          /* fp16 K and V, the reference's paged pool format */
};

#define QOR_HEAD_DIM 128   /* the paged layout is defined for head_dim 128 */
#define QOR_TILE_TOKENS 16 /* a page is page_tokens/16 contiguous tiles */

/* ---- deterministic synthetic inputs ------------------------------------ */
uint64_t qor_mix64(uint64_t x);
/* ~N(0,1) sample: Irwin-Hall sum of twelve 16-bit uniforms, exact in fp32. */
float qor_normal(uint64_t seed, uint64_t stream, uint64_t index);
void qor_fill_normal(uint64_t seed, uint64_t stream, uint64_t first_index,
                     float *out, size_t n);
/* stream id for tensor kind (1=Q, 2=K, 3=V), sequence and layer */
uint64_t qor_stream(uint32_t kind, uint32_t seq, uint32_t layer);
/* Fisher-Yates permutation of the initial LIFO free stack (total-1-i). */
void qor_permuted_free_stack(uint64_t seed, int total, int32_t *stack);
/* pick `count` outlier channels out of `channels` (partial Fisher-Yates) */
void qor_outlier_channels(uint64_t seed, uint32_t layer, int channels, int count,
                          uint8_t *mask);

/* ---- fp16 conversions ---------------------------------------------------- */
uint16_t qor_f32_to_f16_rne(float f);
float qor_f16_to_f32(uint16_t h);
/* the reference's truncating conversions, c/qwanto_turboquant.c:84-123 */
uint16_t qor_tq_f32_to_f16(float f);
float qor_tq_f16_to_f32(uint16_t h);

/* ---- codecs on logical rows -------------------------------------------- */
/* c/qwanto_turboquant.c:555-586 (qwn_q8_round, qwn_q8_scale_for,
 * qwn_q8_quantize_vector).  Writes exactly n codes and ceil(n/64) scales. */
void qor_q8_b64_quantize(const float *src, int n, int8_t *codes, float *scales);
/* per token-head: scale16 = RNE fp16(max|v|/127), q = rint(clamp(v/scale16)) */
void qor_q8_head_quantize(const float *src, int n, int8_t *codes, uint16_t *scale16);
/* c/qwanto_turboquant.c:162-213 incl. pack_16_values (:125-140).
 * Output: ceil(n/64) reference blocks of 32 bytes. */
void qor_tq35_quantize(const float *src, int n, uint8_t *blocks);
/* unpack one 32-byte reference block (c/qwanto_turboquant.c:142-157) */
void qor_tq35_unpack(const uint8_t *block, uint8_t codes[64], uint16_t *range16,
                     uint16_t *min16);
/* 4-bit groups of 32: the reference TurboQuant rules of
 * c/qwanto_turboquant.c:171-206 with group 32 and every code 4-bit. */
void qor_q4g32_quantize(const float *src, int n, uint8_t *codes,
                        uint16_t *range16, uint16_t *min16);

/* ---- paged layout (this project's format) ------------------------------ */
size_t qor_tile_bytes(int codec);
/* quantize K and V (head_dim 128 each) and store them at slot t of a tile */
void qor_tile_store(int codec, uint8_t *tile, int t, const float *k, const float *v);
/* read back logical codes/params of slot t. codes: int8 for Q8 codecs,
 * 0..15 for the 4-bit and 3.5-bit codecs.  params: Q8_B64 -> 2 floats,
 * Q8_HEAD -> 1 (scale), TQ35 -> 4 (range,min per group of 64),
 * Q4_G32 -> 8 (range,min per group of 32).  Params are returned as the
 * decoded fp32 values of the stored fields. */
void qor_tile_load(int codec, const uint8_t *tile, int t, int is_value,
                   int16_t codes[128], float *params);
/* dequantised value of element d of slot t (K if is_value == 0) */
float qor_tile_dequant(int codec, const uint8_t *tile, int t, int is_value, int d);

/* ---- page pool / block table (c/qwn_paged_kv.c:42-149) ------------------ */
typedef struct {
    int codec, layers, kv_heads, page_tokens;
    int total_pages, max_seqs, max_pages_per_seq;
    size_t tile_bytes, page_bytes;
    uint8_t *pages;           /* [total_pages][layers][kv_heads][tiles][tile] */
    int32_t *free_stack;
    int32_t free_top;
    int32_t *page_table;      /* [max_seqs][max_pages_per_seq] */
    int32_t *lens;            /* tokens per sequence */
    int32_t *npages;          /* pages per sequence */
    float *page_score;        /* [max_seqs][max_pages_per_seq] eviction EMA */
} QorPool;

int qor_pool_init(QorPool *p, int codec, int layers, int kv_heads, int page_tokens,
                  int total_pages, int max_seqs, int max_pages_per_seq,
                  uint64_t perm_seed);
/* with_pages 0: block tables, free stack and scores only (pages NULL), for
 * pools whose page bytes would not fit in host memory; writes and
 * attention are then unavailable */
int qor_pool_init_ex(QorPool *p, int codec, int layers, int kv_heads, int page_tokens,
                     int total_pages, int max_seqs, int max_pages_per_seq,
                     uint64_t perm_seed, int with_pages);
void qor_pool_free(QorPool *p);
/* add counts[i] tokens to sequence seq_ids[i], in array order, allocating
 * pages from the LIFO free stack like qwn_block_table_append_token
 * (c/qwn_paged_kv.c:115-138).  Returns 0, or -1 when the pool is exhausted
 * (no state is changed then). */
int qor_pool_append(QorPool *p, int n, const int32_t *seq_ids, const int32_t *counts);
/* store K,V ([kv_heads][128] each) of token `pos` of `seq` in `layer` */
int qor_pool_write_token(QorPool *p, int seq, int layer, int pos, const float *k,
                         const float *v);
uint8_t *qor_pool_tile(QorPool *p, int seq, int layer, int kv_head, int pos);
/* store the synthetic rows of generator layer gen_layer for positions
 * [first, last) of seq into `layer` (K x 8 where k_outlier_mask[c] != 0) */
int qor_pool_fill_synthetic(QorPool *p, int seq, int layer, int gen_layer, int first, int last,
                            uint64_t seed, const uint8_t *k_outlier_mask);
/* GQA decode attention over tokens [0,len) of one sequence and layer, in
 * the reference's arithmetic order (c/qwanto_turboquant.c:678-705 for Q8,
 * :707-768 with the scalar dot/accum of :218-284 for TurboQuant).  Query
 * head h reads kv head (h*kv_heads)/query_heads.  out: [query_heads][128]. */
void qor_pool_attention(const QorPool *p, int seq, int layer, int len,
                        const float *q, int query_heads, float scale, float *out,
                        float *token_probs /* optional [query_heads][len] */);

/* ---- split-KV (m, l, o) merge ------------------------------------------- */
/* partial over a token range in base-2 log domain: m = max(s*log2e),
 * l = sum 2^(s*log2e - m), o[d] = sum 2^(..) v[d] (unnormalised) */
void qor_partial_attention(const QorPool *p, int seq, int layer, int t0, int t1,
                           const float *q, int query_heads, float scale,
                           float *m, float *l, float *o);
void qor_merge_partials(int nparts, int query_heads, const float *m, const float *l,
                        const float *o, float *out);

/* ---- eviction ------------------------------------------------------------ */
/* token-level vToken pool, c/qwanto_pagedeviction.c:7-103 */
#define QOR_VTOKEN_MAX_CAPACITY 32768
#define QOR_VTOKEN_SINK_TOKENS 4
typedef struct {
    uint32_t token_id;
    float importance_score;
    uint32_t physical_slot;
    uint8_t is_sink;
    uint8_t is_active;
} QorVToken;
typedef struct {
    QorVToken tokens[QOR_VTOKEN_MAX_CAPACITY];
    uint32_t active_count, max_capacity, physical_pool_size;
    float eviction_threshold;
    uint64_t total_evictions;
} QorEvictionPool;
int qor_vtoken_init(QorEvictionPool *p, uint32_t max_capacity, uint32_t physical,
                    float threshold);
int qor_vtoken_insert(QorEvictionPool *p, uint32_t token_id, float importance,
                      uint32_t *slot);
void qor_vtoken_update_scores(QorEvictionPool *p, const float *scores, uint32_t n,
                              int fused);
uint32_t qor_vtoken_prune(QorEvictionPool *p, uint32_t target);
float qor_vtoken_waste_pct(const QorEvictionPool *p);

/* page-level eviction + compaction (this project's specification):
 * score = 0.8*score + 0.2*mass on every live page (fp32, no contraction);
 * for each flagged sequence (ascending index) with len > budget: page 0
 * and the last page are protected; evict the lowest-score pages (ties to
 * the lower logical index) until len <= budget, compact the survivors in
 * order, and push the freed physical pages on the free stack in ascending
 * logical order.  mass: [max_seqs][max_pages_per_seq].  Returns the number
 * of pages evicted. */
int qor_pool_evict(QorPool *p, int nseqs, const int32_t *seq_ids, const float *mass,
                   const uint8_t *flags, int token_budget);
/* seeded Bernoulli(prob) eviction trigger for (seed, step, seq) */
int qor_evict_trigger(uint64_t seed, uint32_t step, uint32_t seq, double prob);

/* ---- linear attention (c/qwanto_attention.c:34-156) -------------------- */
/* One decode step over n_heads states of head_dim x head_dim (row i = key
 * dim, column j = value dim): S[i][j] = fma(decay, S[i][j], RN(k_i * v_j)),
 * then O[j] = fma chain over i ascending of q_i * S[i][j] starting from 0 --
 * the order and roundings of the reference's AVX2/AVX-512 paths. */
void qor_linear_attention_decode(float *state, int n_heads, int head_dim, const float *q,
                                 const float *k, const float *v, float decay, float *o);

#ifdef __cplusplus
}
#endif
#endif
