/*
 * ref_shim.c -- drives the reference's own CPU KV-cache functions the way
 * its decoder does, for the CPU baseline and for pinning the oracle.
 *
 * TEST / BASELINE INFRASTRUCTURE ONLY.  Linked into oracle/_ref/libqwnref.so
 * together with the reference sources compiled in place (oracle/Makefile).
 *
 * The decode step mirrors c/qwanto_decode.c:1725-1799: per layer, append the
 * token's K/V (qwn_q8_cache_append / qwn_turboquant_quantize_token), then an
 * OpenMP loop over query heads calling qwn_q8_cache_attention_head or
 * qwn_turboquant_attention_head with kv head (int)(h / (H/HK)) and
 * scale 1/sqrtf(head_dim).  For a batch the OpenMP loop runs over
 * (sequence x query head), as the batched reference would.
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "qwanto_turboquant.h"
#include "qwn_oracle.h"
#include "qwn_paged_kv.h"

typedef struct {
    int codec; /* 1 = reference Q8, 3 = reference TurboQuant, 5 = reference fp16 paged pool */
    int nseq, layers, heads, kv_heads, head_dim;
    uint64_t seed;
    int32_t *lens;            /* current tokens per sequence */
    QwnQ8Cache *q8;           /* [nseq][layers] */
    TurboQuantCache *tq;      /* [nseq][layers] */
    float *q, *k, *v, *ctx;   /* per-sequence scratch rows */
    float *scores;            /* [nseq*heads][max_ctx] */
    int max_ctx;
    /* codec 5: the decoder's fp16 paged path (c/qwanto_decode.c:1600-1604,
     * :1807-1835): one block pool, a block table per sequence, per-thread
     * gather scratch */
    QwnKVBlockPool fpool;
    QwnBlockTable *bt;
    uint16_t *kg, *vg;
    int nthreads;
} QrefBatch;

void qref_batch_destroy(void *handle);

static void gen_row(uint64_t seed, uint32_t kind, int seq, int layer, int pos, int width,
                    float *out) {
    qor_fill_normal(seed, qor_stream(kind, (uint32_t)seq, (uint32_t)layer),
                    (uint64_t)pos * (uint64_t)width, out, (size_t)width);
}

static int append_token(QrefBatch *b, int s, int l, int pos, const float *k, const float *v) {
    int KV = b->kv_heads * b->head_dim;
    if (b->codec == 5) return qwn_paged_kv_write(&b->fpool, &b->bt[s], l, pos, k, v);
    if (b->codec == 1) return qwn_q8_cache_append(&b->q8[(size_t)s * b->layers + l], k, v, KV);
    TurboQuantCache *c = &b->tq[(size_t)s * b->layers + l];
    int bph = (b->head_dim + TURBOQUANT_GROUP_SIZE - 1) / TURBOQUANT_GROUP_SIZE;
    for (int h = 0; h < b->kv_heads; h++) {
        size_t ho = (size_t)h * bph * TURBOQUANT_BLOCK_BYTES;
        qwn_turboquant_quantize_token(k + (size_t)h * b->head_dim,
                                      c->packed_k + (size_t)pos * c->token_stride_k + ho, b->head_dim);
        qwn_turboquant_quantize_token(v + (size_t)h * b->head_dim,
                                      c->packed_v + (size_t)pos * c->token_stride_v + ho, b->head_dim);
    }
    c->n_tokens = pos + 1;
    return 0;
}

void *qref_batch_create(int codec, int nseq, const int32_t *lens, int layers, int heads,
                        int kv_heads, int head_dim, int max_new, uint64_t seed) {
    QrefBatch *b = (QrefBatch *)calloc(1, sizeof(QrefBatch));
    if (!b) return NULL;
    b->codec = codec; b->nseq = nseq; b->layers = layers; b->heads = heads;
    b->kv_heads = kv_heads; b->head_dim = head_dim; b->seed = seed;
    b->lens = (int32_t *)malloc(sizeof(int32_t) * (size_t)nseq);
    int maxlen = 0;
    for (int s = 0; s < nseq; s++) { b->lens[s] = lens[s]; if (lens[s] > maxlen) maxlen = lens[s]; }
    b->max_ctx = maxlen + max_new;
    size_t nc = (size_t)nseq * (size_t)layers;
    if (codec == 1) b->q8 = (QwnQ8Cache *)calloc(nc, sizeof(QwnQ8Cache));
    else if (codec == 3) b->tq = (TurboQuantCache *)calloc(nc, sizeof(TurboQuantCache));
    int KV = kv_heads * head_dim;
    b->q = (float *)malloc(sizeof(float) * (size_t)nseq * heads * head_dim);
    b->k = (float *)malloc(sizeof(float) * (size_t)nseq * KV);
    b->v = (float *)malloc(sizeof(float) * (size_t)nseq * KV);
    b->ctx = (float *)malloc(sizeof(float) * (size_t)nseq * heads * head_dim);
    b->scores = (float *)malloc(sizeof(float) * (size_t)nseq * heads * (size_t)b->max_ctx);
    int fail = 0;
    if (codec == 5) {
        int blocks = 0;
        for (int s = 0; s < nseq; s++) blocks += (lens[s] + max_new + QWN_PAGE_BLOCK_SIZE - 1) / QWN_PAGE_BLOCK_SIZE;
        b->bt = (QwnBlockTable *)calloc((size_t)nseq, sizeof(QwnBlockTable));
        fail = !b->bt || qwn_kv_pool_init(&b->fpool, blocks + nseq, layers, kv_heads, head_dim) != 0;
        /* the blocks of every prefill token, in sequence order (the pool's
         * LIFO free stack is not thread-safe) */
        for (int s = 0; s < nseq && !fail; s++) {
            fail = qwn_block_table_init(&b->bt[s], s, (b->lens[s] + max_new) / QWN_PAGE_BLOCK_SIZE + 1) != 0;
            for (int t = 0; t < lens[s] && !fail; t++) fail = qwn_block_table_append_token(&b->fpool, &b->bt[s]) != 0;
        }
        b->nthreads = omp_get_max_threads();
        b->kg = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)b->nthreads * b->max_ctx * head_dim);
        b->vg = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)b->nthreads * b->max_ctx * head_dim);
        fail = fail || !b->kg || !b->vg;
    }
    for (int s = 0; s < nseq && !fail && codec != 5; s++)
        for (int l = 0; l < layers && !fail; l++) {
            int cap = lens[s] + max_new;
            if (codec == 1) fail = qwn_q8_cache_init(&b->q8[(size_t)s * layers + l], cap, kv_heads, head_dim) != 0;
            else fail = qwn_turboquant_init(&b->tq[(size_t)s * layers + l], cap, kv_heads, head_dim) != 0;
        }
    if (fail) { qref_batch_destroy(b); return NULL; }
    /* prefill: tokens [0, len) of every (sequence, layer), parallel over caches */
    #pragma omp parallel
    {
        float *kr = (float *)malloc(sizeof(float) * (size_t)KV);
        float *vr = (float *)malloc(sizeof(float) * (size_t)KV);
        #pragma omp for schedule(dynamic, 1)
        for (long c = 0; c < (long)nc; c++) {
            int s = (int)(c / layers), l = (int)(c % layers);
            for (int t = 0; t < lens[s]; t++) {
                gen_row(seed, 2, s, l, t, KV, kr);
                gen_row(seed, 3, s, l, t, KV, vr);
                append_token(b, s, l, t, kr, vr);
            }
        }
        free(kr); free(vr);
    }
    return b;
}

/* one decode step of every sequence through `layers_run` layers (the first
 * layers of the model); returns the number of seq-steps done (nseq) */
int qref_batch_step(void *handle, int layers_run) {
    QrefBatch *b = (QrefBatch *)handle;
    int H = b->heads, HK = b->kv_heads, HD = b->head_dim, KV = HK * HD;
    float ratio = (float)H / (float)HK;
    float scale = 1.0f / sqrtf((float)HD);
    if (b->codec == 5) /* one block-table append per token, before the layers */
        for (int s = 0; s < b->nseq; s++)
            if (qwn_block_table_append_token(&b->fpool, &b->bt[s]) != 0) return -1;
    for (int l = 0; l < layers_run && l < b->layers; l++) {
        /* inputs of this step (position = current length) */
        #pragma omp parallel for schedule(static)
        for (int s = 0; s < b->nseq; s++) {
            int pos = b->lens[s];
            gen_row(b->seed, 1, s, l, pos, H * HD, b->q + (size_t)s * H * HD);
            gen_row(b->seed, 2, s, l, pos, KV, b->k + (size_t)s * KV);
            gen_row(b->seed, 3, s, l, pos, KV, b->v + (size_t)s * KV);
            append_token(b, s, l, pos, b->k + (size_t)s * KV, b->v + (size_t)s * KV);
        }
        #pragma omp parallel for schedule(dynamic, 1)
        for (long w = 0; w < (long)b->nseq * H; w++) {
            int s = (int)(w / H), h = (int)(w % H);
            int kh = (int)((float)h / ratio);
            int pos = b->lens[s];
            float *sc = b->scores + (size_t)w * b->max_ctx;
            const float *qh = b->q + ((size_t)s * H + h) * HD;
            float *out = b->ctx + ((size_t)s * H + h) * HD;
            if (b->codec == 5) {
                size_t g = (size_t)omp_get_thread_num() * b->max_ctx * HD;
                qwn_paged_attention_gather_head(&b->fpool, &b->bt[s], l, h, (h * HK) / H, qh, b->kg + g,
                                                b->vg + g, sc, out);
            } else if (b->codec == 1)
                qwn_q8_cache_attention_head(qh, &b->q8[(size_t)s * b->layers + l], kh, pos, scale, sc, out);
            else
                qwn_turboquant_attention_head(qh, &b->tq[(size_t)s * b->layers + l], l, h, kh, pos,
                                              scale, sc, out);
        }
    }
    for (int s = 0; s < b->nseq; s++) b->lens[s]++;
    return b->nseq;
}

const float *qref_batch_ctx(void *handle) { return ((QrefBatch *)handle)->ctx; }

void qref_batch_destroy(void *handle) {
    QrefBatch *b = (QrefBatch *)handle;
    if (!b) return;
    size_t nc = (size_t)b->nseq * (size_t)b->layers;
    for (size_t c = 0; c < nc; c++) {
        if (b->q8) qwn_q8_cache_free(&b->q8[c]);
        if (b->tq) qwn_turboquant_free(&b->tq[c]);
    }
    if (b->bt) {
        for (int s = 0; s < b->nseq; s++) qwn_block_table_free(&b->fpool, &b->bt[s]);
        free(b->bt);
    }
    if (b->codec == 5) qwn_kv_pool_free(&b->fpool);
    free(b->kg); free(b->vg);
    free(b->q8); free(b->tq); free(b->lens); free(b->q); free(b->k); free(b->v);
    free(b->ctx); free(b->scores); free(b);
}

/* The reference's fp16 pool write (c/qwn_paged_kv.c:151-198) of n token-head
 * rows of head_dim values: k/v [n][head_dim] fp32 -> k16/v16 [n][head_dim]
 * fp16 bits, read back from a one-block pool (n <= 16).  Pins the oracle's
 * fp32 -> fp16 rounding. */
int qref_f16_write(const float *k, const float *v, int n, int head_dim, uint16_t *k16, uint16_t *v16) {
    if (n <= 0 || n > QWN_PAGE_BLOCK_SIZE) return -1;
    QwnKVBlockPool pool;
    QwnBlockTable bt;
    if (qwn_kv_pool_init(&pool, 1, 1, 1, head_dim) != 0) return -1;
    int rc = qwn_block_table_init(&bt, 0, 1);
    for (int t = 0; t < n && rc == 0; t++) rc = qwn_block_table_append_token(&pool, &bt);
    for (int t = 0; t < n && rc == 0; t++)
        rc = qwn_paged_kv_write(&pool, &bt, 0, t, k + (size_t)t * head_dim, v + (size_t)t * head_dim);
    if (rc == 0) {
        int blk = bt.block_ids[0];
        size_t base = (size_t)blk * QWN_PAGE_BLOCK_SIZE * head_dim;
        memcpy(k16, pool.key_data + base, sizeof(uint16_t) * (size_t)n * head_dim);
        memcpy(v16, pool.val_data + base, sizeof(uint16_t) * (size_t)n * head_dim);
    }
    qwn_block_table_free(&pool, &bt);
    qwn_kv_pool_free(&pool);
    return rc;
}

int qref_max_threads(void) { return omp_get_max_threads(); }
void qref_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }
