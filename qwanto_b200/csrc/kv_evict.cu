// Page attention mass, score-based page eviction and compaction.
//
// The reference evicts at token level in a host-side vToken pool
// (c/qwanto_pagedeviction.c:24-93) and has no page-level policy.  Lifted to
// pages here:
//   mass(page)  = sum over query heads of the softmax probability of the
//                 page's tokens (exported by the attention kernel per tile
//                 as (sum_t 2^(s_t - m_tile), m_tile) and rescaled by the
//                 final (m, l) of the segment);
//   score(page) = 0.8*score + 0.2*mass, two IEEE roundings then an add
//                 (the EMA of c/qwanto_pagedeviction.c:64-68);
//   eviction    = for each flagged sequence (batch order) longer than the
//                 budget: protect page 0 (the attention-sink tokens 0-3,
//                 c/qwanto_pagedeviction.h:17) and the last page, drop the
//                 lowest scores (ties to the lower logical index) until
//                 len <= budget, compact, push the freed physical pages on the
//                 LIFO free stack in ascending logical order
//                 (qwn_kv_pool_free_block, c/qwn_paged_kv.c:100-103).
#include <cub/block/block_scan.cuh>

#include "kv_internal.cuh"

namespace qkv {
namespace {

__global__ void fill_f32_kernel(float *p, float v, size_t n) {
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x)
        p[e] = v;
}

__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// one CTA per batch entry
__global__ void page_mass_kernel(uint32_t n, const int32_t *seq_ids, const int32_t *lens, uint32_t kv_heads,
                                 uint32_t group, uint32_t tpp, uint32_t mp, const float2 *tile_mass,
                                 const float2 *seg_ml, float *page_mass) {
    const uint32_t i = blockIdx.x;
    if (i >= n) return;
    __shared__ unsigned long long s_prefix;
    if (threadIdx.x == 0) s_prefix = 0ull;
    __syncthreads();
    unsigned long long part = 0;
    for (uint32_t k = threadIdx.x; k < i; k += blockDim.x) {
        const int32_t sq = seq_ids ? seq_ids[k] : (int32_t)k;
        part += (unsigned long long)((lens[sq] + 15) / 16) * kv_heads;
    }
    atomicAdd(&s_prefix, part);
    __syncthreads();
    const uint64_t prefix = s_prefix;
    const int32_t seq = seq_ids ? seq_ids[i] : (int32_t)i;
    const uint32_t ntiles = (uint32_t)((lens[seq] + 15) / 16);
    const uint32_t npages = (ntiles + tpp - 1) / tpp;
    for (uint32_t lp = threadIdx.x; lp < npages; lp += blockDim.x) {
        float mass = 0.f;
        for (uint32_t h = 0; h < kv_heads; h++) {
            const uint32_t s_idx = i * kv_heads + h;
            for (uint32_t g = 0; g < group; g++) {
                const float2 ml = seg_ml[(size_t)s_idx * kMaxGroup + g];
                const float inv = ml.y > 0.f ? 1.0f / ml.y : 0.f;
                for (uint32_t tt = 0; tt < tpp; tt++) {
                    const uint32_t tile = lp * tpp + tt;
                    if (tile >= ntiles) break;
                    const float2 um = tile_mass[(prefix + (uint64_t)h * ntiles + tile) * kMaxGroup + g];
                    mass += um.x * ex2f(um.y - ml.x) * inv;
                }
            }
        }
        page_mass[(size_t)seq * mp + lp] = mass;
    }
}

// EMA on every page of the entry, then rank the candidates of a flagged entry
__global__ void evict_rank_kernel(uint32_t n, const int32_t *seq_ids, const float *mass, const uint8_t *flags,
                                  uint32_t budget, const int32_t *lens, const int32_t *npages, float *scores,
                                  uint8_t *dead, int32_t *count, uint32_t P, uint32_t mp) {
    const uint32_t i = blockIdx.x;
    if (i >= n) return;
    const int32_t seq = seq_ids ? seq_ids[i] : (int32_t)i;
    const int32_t np = npages[seq];
    float *sc = scores + (size_t)seq * mp;
    for (int32_t lp = threadIdx.x; lp < np; lp += blockDim.x)
        sc[lp] = __fadd_rn(__fmul_rn(0.8f, sc[lp]), __fmul_rn(0.2f, mass[(size_t)seq * mp + lp]));
    __syncthreads();
    int32_t ne = 0;
    const int32_t len = lens[seq];
    if (flags[i] && len > (int32_t)budget && np >= 3) {
        ne = (len - (int32_t)budget + (int32_t)P - 1) / (int32_t)P;
        if (ne > np - 2) ne = np - 2;
    }
    uint8_t *dd = dead + (size_t)i * mp;
    for (int32_t c = threadIdx.x; c < np; c += blockDim.x) {
        uint8_t d = 0;
        if (ne > 0 && c >= 1 && c <= np - 2) {
            const float s = sc[c];
            int32_t rank = 0;
            for (int32_t o = 1; o <= np - 2; o++) {
                const float so = sc[o];
                rank += (so < s || (so == s && o < c)) ? 1 : 0;
            }
            d = rank < ne ? 1 : 0;
        }
        dd[c] = d;
    }
    if (threadIdx.x == 0) count[i] = ne;
}

// free-stack pushes and table compaction, entries in batch order
__global__ void __launch_bounds__(1024) evict_compact_kernel(uint32_t n, const int32_t *seq_ids,
                                                             const uint8_t *dead, const int32_t *count,
                                                             int32_t *lens, int32_t *npages, int32_t *table,
                                                             float *scores, int32_t *free_stack,
                                                             int32_t *free_top, uint32_t P, uint32_t mp,
                                                             uint32_t total_pages, uint32_t *epoch) {
    using Scan = cub::BlockScan<int, 1024>;
    __shared__ typename Scan::TempStorage tmp;
    int32_t top = *free_top;
    for (uint32_t i = 0; i < n; i++) {
        const int32_t ne = count[i];
        if (ne <= 0) continue;
        const int32_t seq = seq_ids ? seq_ids[i] : (int32_t)i;
        const int32_t np = npages[seq];
        int32_t *tb = table + (size_t)seq * mp;
        float *sc = scores + (size_t)seq * mp;
        const uint8_t *dd = dead + (size_t)i * mp;
        int dead_before = 0;
        for (int32_t base = 0; base < np; base += 1024) {
            const int32_t lp = base + (int32_t)threadIdx.x;
            const int d = (lp < np) ? dd[lp] : 0;
            int32_t pg = 0;
            float s = 0.f;
            if (lp < np) { pg = tb[lp]; s = sc[lp]; }
            int off, agg;
            Scan(tmp).ExclusiveSum(d, off, agg);
            __syncthreads();
            if (lp < np) {
                if (d) {
                    if (top + dead_before + off < (int32_t)total_pages) free_stack[top + dead_before + off] = pg;
                } else {
                    const int32_t dst = lp - (dead_before + off);
                    tb[dst] = pg;
                    sc[dst] = s;
                }
            }
            dead_before += agg;
            __syncthreads();
        }
        for (int32_t lp = np - ne + (int32_t)threadIdx.x; lp < np; lp += 1024) {
            tb[lp] = -1;
            sc[lp] = 0.f;
        }
        top += dead_before;
        if (threadIdx.x == 0) {
            npages[seq] = np - dead_before;
            lens[seq] -= dead_before * (int32_t)P;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        *free_top = top;
        atomicAdd(epoch, 1u);  // lengths and tables changed: cached attention plans are stale
    }
}

}  // namespace

cudaError_t launch_fill_f32(float *p, float v, size_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    fill_f32_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, 1024), 256, 0, s>>>(p, v, n);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_page_mass(Pool *p, uint32_t n, const int32_t *seq_ids, uint32_t query_heads,
                             float *page_mass, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    page_mass_kernel<<<n, 128, 0, s>>>(n, seq_ids, p->seq_lens, p->kv_heads, query_heads / p->kv_heads,
                                       p->tiles_per_page, p->max_pages_per_seq, p->tile_mass, p->seg_ml,
                                       page_mass);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_evict(Pool *p, uint32_t n, const int32_t *seq_ids, const float *mass, const uint8_t *flags,
                         uint32_t budget, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    plans_invalidated(p);  // compaction moves the plans' epoch
    evict_rank_kernel<<<n, 256, 0, s>>>(n, seq_ids, mass, flags, budget, p->seq_lens, p->seq_pages,
                                        p->page_scores, p->evict_dead, p->evict_count, p->page_tokens,
                                        p->max_pages_per_seq);
    count_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    evict_compact_kernel<<<1, 1024, 0, s>>>(n, seq_ids, p->evict_dead, p->evict_count, p->seq_lens,
                                            p->seq_pages, p->page_table, p->page_scores, p->free_stack,
                                            p->free_top, p->page_tokens, p->max_pages_per_seq, p->total_pages,
                                            p->plans);
    count_launch();
    return cudaGetLastError();
}

}  // namespace qkv
