// Paged quantized KV pool: lifecycle, page allocation, quantize-on-append,
// synthetic prefill and the exported qwn_kv_* entry points.

#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "kv_internal.cuh"
#include "kv_store.cuh"

namespace qkv {

std::atomic<uint64_t> g_launches{0};
static std::mutex g_err_mu;
static std::string g_last_error;

void set_error(const char *msg) {
    std::lock_guard<std::mutex> lk(g_err_mu);
    g_last_error = msg ? msg : "qwn_cuda error";
}
void set_cuda_error(const char *what, cudaError_t e) {
    char buf[256];
    std::snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
    set_error(buf);
}
std::string last_error() {
    std::lock_guard<std::mutex> lk(g_err_mu);
    return g_last_error;
}

size_t attention_smem_bytes(uint32_t codec, int hg);
const void *attention_kernel_ptr(uint32_t codec, int hg);

namespace {

struct StoreGeo {
    uint8_t *pages;
    uint64_t page_bytes;
    uint32_t tile_bytes, tpp, page_tokens, kv_heads, mp, total_pages, max_seqs;
    const int32_t *page_table;
    const int32_t *seq_lens;
    uint32_t *status;
};

__device__ __forceinline__ uint8_t *tile_for(const StoreGeo &g, int32_t seq, uint32_t layer,
                                             uint32_t head, int32_t pos) {
    const uint32_t lp = (uint32_t)pos / g.page_tokens;
    if (lp >= g.mp) { latch(g.status, QWN_KV_STATUS_TABLE_OVERFLOW); return nullptr; }
    const int32_t pg = g.page_table[(size_t)seq * g.mp + lp];
    if (pg < 0 || (uint32_t)pg >= g.total_pages) { latch(g.status, QWN_KV_STATUS_BAD_PAGE); return nullptr; }
    const uint32_t tin = ((uint32_t)pos % g.page_tokens) / 16u;
    return g.pages + (size_t)pg * g.page_bytes +
           ((size_t)(layer * g.kv_heads + head) * g.tpp + tin) * g.tile_bytes;
}

// append the newest token (position len-1) of each sequence in the batch
template <int CODEC>
__global__ void append_kernel(StoreGeo g, uint32_t layer, uint32_t n, const int32_t *seq_ids,
                              const float *key, const float *value) {
    const uint32_t wg = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (wg >= n * g.kv_heads) return;
    const uint32_t i = wg / g.kv_heads, h = wg % g.kv_heads;
    const int32_t seq = seq_ids ? seq_ids[i] : (int32_t)i;
    if (seq < 0 || (uint32_t)seq >= g.max_seqs) { if (lane == 0) latch(g.status, QWN_KV_STATUS_BAD_SEQUENCE); return; }
    const int32_t pos = g.seq_lens[seq] - 1;
    if (pos < 0) { if (lane == 0) latch(g.status, QWN_KV_STATUS_BAD_LENGTH); return; }
    uint8_t *tile = tile_for(g, seq, layer, h, pos);
    if (!tile) return;
    const size_t row = ((size_t)i * g.kv_heads + h) * kHeadDim;
    const float4 k = reinterpret_cast<const float4 *>(key + row)[lane];
    const float4 v = reinterpret_cast<const float4 *>(value + row)[lane];
    store_token<CODEC>(tile, pos & 15, k, v, lane);
}

// store tokens [first, first+n) of one sequence (key/value [n][HK][128])
template <int CODEC>
__global__ void store_tokens_kernel(StoreGeo g, int32_t seq, uint32_t layer, uint32_t first,
                                    uint32_t n, const float *key, const float *value) {
    const uint32_t wg = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (wg >= n * g.kv_heads) return;
    const uint32_t tk = wg / g.kv_heads, h = wg % g.kv_heads;
    const int32_t pos = (int32_t)(first + tk);
    if (pos >= g.seq_lens[seq]) { if (lane == 0) latch(g.status, QWN_KV_STATUS_BAD_LENGTH); return; }
    uint8_t *tile = tile_for(g, seq, layer, h, pos);
    if (!tile) return;
    const size_t row = ((size_t)tk * g.kv_heads + h) * kHeadDim;
    const float4 k = reinterpret_cast<const float4 *>(key + row)[lane];
    const float4 v = reinterpret_cast<const float4 *>(value + row)[lane];
    store_token<CODEC>(tile, pos & 15, k, v, lane);
}

// synthetic prefill of one sequence: every (layer, position, head)
template <int CODEC>
__global__ void prefill_kernel(StoreGeo g, int32_t seq, uint32_t layers, uint32_t len, uint64_t seed,
                               const uint8_t *mask) {
    const int lane = threadIdx.x & 31;
    const uint64_t total = (uint64_t)layers * len * g.kv_heads;
    const uint64_t nw = (uint64_t)gridDim.x * (blockDim.x >> 5);
    const uint32_t width = g.kv_heads * kHeadDim;
    for (uint64_t wg = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); wg < total; wg += nw) {
        const uint32_t h = (uint32_t)(wg % g.kv_heads);
        const uint32_t pos = (uint32_t)((wg / g.kv_heads) % len);
        const uint32_t layer = (uint32_t)(wg / ((uint64_t)g.kv_heads * len));
        uint8_t *tile = tile_for(g, seq, layer, h, (int32_t)pos);
        if (!tile) continue;
        const uint64_t kk = gen_key(seed, 2, (uint32_t)seq, layer), kvv = gen_key(seed, 3, (uint32_t)seq, layer);
        const uint64_t base = (uint64_t)pos * width + h * kHeadDim + 4 * lane;
        float kx[4], vx[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            kx[i] = gen_normal(kk, base + i);
            vx[i] = gen_normal(kvv, base + i);
            if (mask && mask[(size_t)layer * width + h * kHeadDim + 4 * lane + i]) kx[i] *= 8.0f;
        }
        store_token<CODEC>(tile, (int)(pos & 15), make_float4(kx[0], kx[1], kx[2], kx[3]),
                           make_float4(vx[0], vx[1], vx[2], vx[3]), lane);
    }
}

__global__ void generate_kernel(float *out, uint32_t rows, uint32_t width, uint32_t kind, uint64_t seed,
                                uint32_t layer, const int32_t *seq_ids, const int32_t *pos,
                                const uint8_t *mask) {
    const uint64_t total = (uint64_t)rows * width;
    for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t r = (uint32_t)(e / width), c = (uint32_t)(e % width);
        const uint32_t seq = seq_ids ? (uint32_t)seq_ids[r] : r;
        const uint64_t key = gen_key(seed, kind, seq, layer);
        float x = gen_normal(key, (uint64_t)pos[r] * width + c);
        if (mask && mask[c]) x *= 8.0f;
        out[e] = x;
    }
}

// qwn_block_table_append_token for every sequence of the batch, in order:
// pages popped from the top of the LIFO free stack (c/qwn_paged_kv.c:95-138).
// One warp: a shuffle scan over chunks of 32 sequences gives each sequence
// its offset on the stack; the first pass only checks, so a request that does
// not fit changes nothing.
__device__ __forceinline__ int warp_excl_scan(int v, int &total) {
    const int lane = threadIdx.x & 31;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    total = __shfl_sync(0xffffffffu, x, 31);
    return x - v;
}

__global__ void __launch_bounds__(32) seq_append_kernel(uint32_t n, const int32_t *seq_ids, const int32_t *counts,
                                                        int32_t *lens, int32_t *npages, int32_t *table,
                                                        float *scores, const int32_t *free_stack,
                                                        int32_t *free_top, uint32_t P, uint32_t mp,
                                                        uint32_t max_seqs, uint32_t *status, uint32_t *epoch) {
    const int lane = threadIdx.x;
    // the attention launch that follows (a programmatic dependent) may bring
    // its CTAs up now; it waits for this kernel's completion before its first
    // global access (the host never lets it start early after this kernel)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    int total = 0;
    uint32_t bad = 0;
    for (uint32_t base = 0; base < n; base += 32) {
        const uint32_t i = base + lane;
        int need = 0;
        if (i < n) {
            const int32_t seq = seq_ids ? seq_ids[i] : (int32_t)i;
            if (seq < 0 || (uint32_t)seq >= max_seqs) {
                bad |= QWN_KV_STATUS_BAD_SEQUENCE;
            } else {
                const int32_t cnt = counts ? counts[i] : 1;
                const int32_t np_new = (lens[seq] + cnt + (int32_t)P - 1) / (int32_t)P;
                if (cnt < 0 || np_new > (int32_t)mp) bad |= QWN_KV_STATUS_TABLE_OVERFLOW;
                need = max(0, np_new - npages[seq]);
            }
        }
        int chunk;
        warp_excl_scan(need, chunk);
        total += chunk;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    const int32_t top = *free_top;
    if (bad || total > top) {
        if (lane == 0) latch(status, bad ? bad : QWN_KV_STATUS_POOL_EXHAUSTED);
        return;
    }
    int carry = 0;
    for (uint32_t base = 0; base < n; base += 32) {
        const uint32_t i = base + lane;
        int need = 0, seq = 0, cnt = 0, np = 0;
        if (i < n) {
            seq = seq_ids ? seq_ids[i] : (int32_t)i;
            cnt = counts ? counts[i] : 1;
            np = npages[seq];
            need = max(0, (lens[seq] + cnt + (int32_t)P - 1) / (int32_t)P - np);
        }
        int chunk;
        const int off = warp_excl_scan(need, chunk);
        if (i < n) {
            for (int k = 0; k < need; k++) {
                table[(size_t)seq * mp + np + k] = free_stack[top - 1 - (carry + off + k)];
                scores[(size_t)seq * mp + np + k] = 1.0f;
            }
            npages[seq] = np + need;
            lens[seq] += cnt;
        }
        carry += chunk;
    }
    if (lane == 0) {
        *free_top = top - carry;
        atomicAdd(epoch, 1u);  // lengths and tables changed: cached attention plans are stale
    }
}

__global__ void iota_i32(int32_t *p, size_t n) {
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x)
        p[e] = (int32_t)e;
}

StoreGeo store_geo(Pool *p) {
    StoreGeo g;
    g.pages = p->pages;
    g.page_bytes = p->page_bytes;
    g.tile_bytes = (uint32_t)p->tile_bytes;
    g.tpp = p->tiles_per_page;
    g.page_tokens = p->page_tokens;
    g.kv_heads = p->kv_heads;
    g.mp = p->max_pages_per_seq;
    g.total_pages = p->total_pages;
    g.max_seqs = p->max_seqs;
    g.page_table = p->page_table;
    g.seq_lens = p->seq_lens;
    g.status = p->status;
    return g;
}

template <template <int> class K, class... Args>
cudaError_t dispatch_store(uint32_t codec, dim3 grid, dim3 block, cudaStream_t s, Args... args) {
    switch (codec) {
        case QWN_KV_CODEC_Q8_HEAD_F16: K<QWN_KV_CODEC_Q8_HEAD_F16>::launch(grid, block, s, args...); break;
        case QWN_KV_CODEC_Q8_B64_F32: K<QWN_KV_CODEC_Q8_B64_F32>::launch(grid, block, s, args...); break;
        case QWN_KV_CODEC_TQ35_G64: K<QWN_KV_CODEC_TQ35_G64>::launch(grid, block, s, args...); break;
        case QWN_KV_CODEC_Q4_G32: K<QWN_KV_CODEC_Q4_G32>::launch(grid, block, s, args...); break;
        case QWN_KV_CODEC_F16: K<QWN_KV_CODEC_F16>::launch(grid, block, s, args...); break;
        default: return cudaErrorNotSupported;
    }
    count_launch();
    return cudaGetLastError();
}
template <int C> struct AppendL {
    template <class... A> static void launch(dim3 g, dim3 b, cudaStream_t s, A... a) {
        append_kernel<C><<<g, b, 0, s>>>(a...);
    }
};
template <int C> struct StoreL {
    template <class... A> static void launch(dim3 g, dim3 b, cudaStream_t s, A... a) {
        store_tokens_kernel<C><<<g, b, 0, s>>>(a...);
    }
};
template <int C> struct PrefillL {
    template <class... A> static void launch(dim3 g, dim3 b, cudaStream_t s, A... a) {
        prefill_kernel<C><<<g, b, 0, s>>>(a...);
    }
};

}  // namespace

cudaError_t launch_seq_append(Pool *p, uint32_t n, const int32_t *seq_ids, const int32_t *counts,
                              cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    plans_invalidated(p);
    {
        // this kernel lets the next launch start its CTAs early, so the next
        // attention launch must not read anything before its dependency wait
        std::lock_guard<std::mutex> lk(p->last_mu);
        p->last_attn.valid = false;
    }
    seq_append_kernel<<<1, 32, 0, s>>>(n, seq_ids, counts, p->seq_lens, p->seq_pages, p->page_table,
                                         p->page_scores, p->free_stack, p->free_top, p->page_tokens,
                                         p->max_pages_per_seq, p->max_seqs, p->status, p->plans);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_append(Pool *p, uint32_t layer, uint32_t n, const int32_t *seq_ids, const float *key,
                          const float *value, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const uint32_t warps = n * p->kv_heads;
    return dispatch_store<AppendL>(p->codec, dim3((warps + 3) / 4), dim3(128), s, store_geo(p), layer, n,
                                   seq_ids, key, value);
}

cudaError_t launch_store_tokens(Pool *p, int32_t seq, uint32_t layer, uint32_t first, uint32_t n,
                                const float *key, const float *value, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const uint32_t warps = n * p->kv_heads;
    return dispatch_store<StoreL>(p->codec, dim3((warps + 3) / 4), dim3(128), s, store_geo(p), seq, layer,
                                  first, n, key, value);
}

cudaError_t launch_generate(float *out, uint32_t rows, uint32_t width, uint32_t kind, uint64_t seed,
                            uint32_t layer, const int32_t *seq_ids, const int32_t *pos, const uint8_t *mask,
                            cudaStream_t s) {
    const uint64_t total = (uint64_t)rows * width;
    if (total == 0) return cudaSuccess;
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((total + 255) / 256, 148u * 16u);
    generate_kernel<<<blocks, 256, 0, s>>>(out, rows, width, kind, seed, layer, seq_ids, pos, mask);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_pool_init_state(Pool *p, cudaStream_t s) {
    cudaError_t e;
    if ((e = cudaMemsetAsync(p->page_table, 0xFF, sizeof(int32_t) * (size_t)p->max_seqs * p->max_pages_per_seq, s)))
        return e;
    if ((e = cudaMemsetAsync(p->seq_lens, 0, sizeof(int32_t) * p->max_seqs, s))) return e;
    if ((e = cudaMemsetAsync(p->seq_pages, 0, sizeof(int32_t) * p->max_seqs, s))) return e;
    if ((e = cudaMemsetAsync(p->page_scores, 0, sizeof(float) * (size_t)p->max_seqs * p->max_pages_per_seq, s)))
        return e;
    if ((e = cudaMemsetAsync(p->status, 0, sizeof(uint32_t), s))) return e;
    if ((e = cudaMemsetAsync(p->counters, 0, sizeof(uint32_t) * counter_count(p), s))) return e;
    // no cached attention plan survives (epoch 0, every record's key invalid)
    plans_invalidated(p);
    if ((e = cudaMemsetAsync(p->plans, 0xFF, sizeof(uint32_t) * plan_words(p), s))) return e;
    if ((e = cudaMemsetAsync(p->plans, 0, sizeof(uint32_t), s))) return e;
    // free stack: total-1-i, optionally permuted (Fisher-Yates on the host)
    std::vector<int32_t> stack(p->total_pages);
    for (uint32_t i = 0; i < p->total_pages; i++) stack[i] = (int32_t)(p->total_pages - 1 - i);
    if (p->perm_seed) {
        auto mix = [](uint64_t x) {
            uint64_t z = x + 0x9E3779B97F4A7C15ull;
            z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
            z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
            return z ^ (z >> 31);
        };
        const uint64_t key = mix(p->perm_seed ^ 0x5045524Dull);
        for (int64_t i = (int64_t)p->total_pages - 1; i > 0; i--) {
            const uint64_t j = mix(key + (uint64_t)i) % (uint64_t)(i + 1);
            std::swap(stack[(size_t)i], stack[(size_t)j]);
        }
    }
    if ((e = cudaMemcpyAsync(p->free_stack, stack.data(), sizeof(int32_t) * stack.size(),
                             cudaMemcpyHostToDevice, s)))
        return e;
    const int32_t top = (int32_t)p->total_pages;
    if ((e = cudaMemcpyAsync(p->free_top, &top, sizeof(int32_t), cudaMemcpyHostToDevice, s))) return e;
    return cudaStreamSynchronize(s);  // the host vectors above go out of scope
}

}  // namespace qkv

using namespace qkv;

// ===========================================================================
// exported entry points
// ===========================================================================
extern "C" {

QWN_CUDA_ABI_API uint64_t qwn_kv_launch_count(void) { return g_launches.load(); }

QWN_CUDA_ABI_API int qwn_kv_memcpy_d2h(void *host, const void *dev, uint64_t bytes) {
    cudaError_t e = cudaMemcpy(host, dev, bytes, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_memcpy_d2h", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}
QWN_CUDA_ABI_API int qwn_kv_memcpy_h2d(void *dev, const void *host, uint64_t bytes) {
    cudaError_t e = cudaMemcpy(dev, host, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_memcpy_h2d", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}

static void pool_release(Pool *p) {
    cudaSetDevice(p->device);
    cudaFree(p->pages); cudaFree(p->page_table); cudaFree(p->seq_lens); cudaFree(p->seq_pages);
    cudaFree(p->free_stack); cudaFree(p->free_top); cudaFree(p->page_scores); cudaFree(p->status);
    cudaFree(p->partials); cudaFree(p->counters); cudaFree(p->plans); cudaFree(p->tile_mass); cudaFree(p->seg_ml);
    cudaFree(p->evict_dead); cudaFree(p->evict_count); cudaFree(p->ident);
    cudaFree(p->stage_q); cudaFree(p->stage_k); cudaFree(p->stage_v); cudaFree(p->stage_o);
    if (p->status_host) cudaFreeHost(p->status_host);
    if (p->step_t0) cudaEventDestroy(p->step_t0);
    if (p->step_t1) cudaEventDestroy(p->step_t1);
    for (uint32_t i = 0; i < p->layer_events; i++) {
        cudaEventDestroy(p->layer_in_ev[i]);
        cudaEventDestroy(p->layer_out_ev[i]);
    }
    delete[] p->layer_in_ev;
    delete[] p->layer_out_ev;
    if (p->stream) cudaStreamDestroy(p->stream);
    if (p->copy_stream) cudaStreamDestroy(p->copy_stream);
    if (p->out_stream) cudaStreamDestroy(p->out_stream);
    delete p;
}

QWN_CUDA_ABI_API int qwn_kv_pool_create(const QwnKvPoolOptions *o, QwnKvPoolHandle *out) {
    if (!o || !out || !header_ok(o->header, sizeof(*o)) || !header_ok(out->header, sizeof(*out))) {
        set_error("qwn_kv_pool_create: bad header");
        return QWN_CUDA_STATUS_ABI_MISMATCH;
    }
    const size_t tb = tile_bytes_of(o->codec);
    if (!tb || o->head_dim != (uint32_t)kHeadDim || o->layers == 0 || o->kv_heads == 0 ||
        o->page_tokens == 0 || o->page_tokens % 16 || o->total_pages == 0 || o->max_seqs == 0 ||
        o->max_pages_per_seq == 0) {
        set_error("qwn_kv_pool_create: unsupported geometry (head_dim must be 128, page_tokens a multiple of 16)");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    const uint32_t mq = o->max_query_heads ? o->max_query_heads : o->kv_heads * kMaxGroup;
    if (mq % o->kv_heads || mq / o->kv_heads > (uint32_t)kMaxGroup) {
        set_error("qwn_kv_pool_create: query heads must be a multiple of kv_heads, at most 8 per kv head");
        return QWN_CUDA_STATUS_UNSUPPORTED;
    }
    if (cudaSetDevice(o->device_id) != cudaSuccess) {
        set_cuda_error("cudaSetDevice", cudaGetLastError());
        return QWN_CUDA_STATUS_UNAVAILABLE;
    }
    Pool *p = new (std::nothrow) Pool();
    if (!p) return QWN_CUDA_STATUS_OUT_OF_MEMORY;
    p->device = o->device_id;
    p->codec = o->codec;
    p->layers = o->layers;
    p->kv_heads = o->kv_heads;
    p->page_tokens = o->page_tokens;
    p->tiles_per_page = o->page_tokens / 16;
    p->total_pages = o->total_pages;
    p->max_seqs = o->max_seqs;
    p->max_pages_per_seq = o->max_pages_per_seq;
    p->max_query_heads = mq;
    p->perm_seed = o->permutation_seed;
    p->tile_bytes = tb;
    p->page_bytes = tb * p->tiles_per_page * (size_t)o->layers * o->kv_heads;
    p->pool_bytes = p->page_bytes * (size_t)o->total_pages;

    // persistent attention grids, resident CTAs x SMs, per kernel variant
    // (one or two head groups of four query heads)
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, p->device);
    uint32_t ctas[2] = {0, 0};
    for (int hg = 1; hg <= 2; hg++) {
        int per_sm = 0;
        const void *kern = attention_kernel_ptr(p->codec, hg);
        const size_t smem = attention_smem_bytes(p->codec, hg);
        if (kern) {
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kWarpsPerCta * 32, smem);
        }
        if (per_sm < 1) per_sm = 1;
        ctas[hg - 1] = (uint32_t)(sms > 0 ? sms : 148) * (uint32_t)per_sm;
    }
    p->attn_ctas = ctas[0];
    p->attn_ctas2 = ctas[1];
    p->attn_warps = (ctas[0] > ctas[1] ? ctas[0] : ctas[1]) * kWarpsPerCta;
    p->max_segments = (uint64_t)o->max_seqs * o->kv_heads;
    p->max_units = (uint64_t)o->max_seqs * o->max_pages_per_seq * p->tiles_per_page * o->kv_heads;
    const size_t part_bytes = ((size_t)p->attn_warps + p->max_segments) * kPartialFloats * sizeof(float);
    const size_t mass_bytes = (size_t)p->max_units * kMaxGroup * sizeof(float2);
    const size_t segml_bytes = (size_t)p->max_segments * kMaxGroup * sizeof(float2);
    const size_t table_elems = (size_t)o->max_seqs * o->max_pages_per_seq;
    p->scratch_bytes = part_bytes + mass_bytes + segml_bytes + counter_count(p) * sizeof(uint32_t) +
                       plan_words(p) * sizeof(uint32_t) + table_elems;

    size_t free_b = 0, total_b = 0;
    cudaMemGetInfo(&free_b, &total_b);
    const uint64_t need = p->pool_bytes + p->scratch_bytes + table_elems * 8 + (size_t)o->total_pages * 4;
    if ((o->memory_budget_bytes && need > o->memory_budget_bytes) || need > free_b) {
        delete p;
        set_error("qwn_kv_pool_create: pool does not fit the memory budget / free device memory");
        return QWN_CUDA_STATUS_OUT_OF_MEMORY;
    }
    bool ok = cudaStreamCreateWithFlags(&p->stream, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&p->copy_stream, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&p->out_stream, cudaStreamNonBlocking) == cudaSuccess &&
              cudaMalloc(&p->pages, p->pool_bytes) == cudaSuccess &&
              cudaMalloc(&p->page_table, sizeof(int32_t) * table_elems) == cudaSuccess &&
              cudaMalloc(&p->seq_lens, sizeof(int32_t) * o->max_seqs) == cudaSuccess &&
              cudaMalloc(&p->seq_pages, sizeof(int32_t) * o->max_seqs) == cudaSuccess &&
              cudaMalloc(&p->free_stack, sizeof(int32_t) * o->total_pages) == cudaSuccess &&
              cudaMalloc(&p->free_top, sizeof(int32_t)) == cudaSuccess &&
              cudaMalloc(&p->page_scores, sizeof(float) * table_elems) == cudaSuccess &&
              cudaMalloc(&p->status, sizeof(uint32_t)) == cudaSuccess &&
              cudaMalloc(&p->partials, part_bytes) == cudaSuccess &&
              cudaMalloc(&p->counters, sizeof(uint32_t) * counter_count(p)) == cudaSuccess &&
              cudaMalloc(&p->plans, sizeof(uint32_t) * plan_words(p)) == cudaSuccess &&
              cudaMalloc(&p->tile_mass, mass_bytes) == cudaSuccess &&
              cudaMalloc(&p->seg_ml, segml_bytes) == cudaSuccess &&
              cudaMalloc(&p->evict_dead, table_elems) == cudaSuccess &&
              cudaMalloc(&p->evict_count, sizeof(int32_t) * o->max_seqs) == cudaSuccess &&
              cudaMalloc(&p->ident, sizeof(int32_t) * o->max_seqs) == cudaSuccess;
    if (!ok) {
        set_cuda_error("qwn_kv_pool_create: allocation", cudaGetLastError());
        pool_release(p);
        return QWN_CUDA_STATUS_OUT_OF_MEMORY;
    }
    cudaMemsetAsync(p->pages, 0, p->pool_bytes, p->stream);
    iota_i32<<<(o->max_seqs + 255) / 256, 256, 0, p->stream>>>(p->ident, o->max_seqs);
    count_launch();
    cudaError_t e = launch_pool_init_state(p, p->stream);
    if (e != cudaSuccess) {
        set_cuda_error("qwn_kv_pool_create: init", e);
        pool_release(p);
        return QWN_CUDA_STATUS_RUNTIME_ERROR;
    }
    std::memset(out, 0, sizeof(*out));
    qwn_cuda_abi_header_init(&out->header, sizeof(*out));
    out->opaque = p;
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_pool_destroy(QwnKvPoolHandle *h) {
    Pool *p = pool_from(h);
    if (!p) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    cudaSetDevice(p->device);
    cudaDeviceSynchronize();
    pool_release(p);
    h->opaque = nullptr;
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_pool_get_info(const QwnKvPoolHandle *h, QwnKvPoolInfo *info) {
    Pool *p = pool_from(h);
    if (!p || !info || !header_ok(info->header, sizeof(*info))) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    std::memset(info, 0, sizeof(*info));
    qwn_cuda_abi_header_init(&info->header, sizeof(*info));
    info->pages_dev = p->pages;
    info->page_table_dev = p->page_table;
    info->seq_lens_dev = p->seq_lens;
    info->seq_pages_dev = p->seq_pages;
    info->free_stack_dev = p->free_stack;
    info->free_top_dev = p->free_top;
    info->page_scores_dev = p->page_scores;
    info->status_dev = p->status;
    info->tile_bytes = p->tile_bytes;
    info->page_bytes = p->page_bytes;
    info->pool_bytes = p->pool_bytes;
    info->scratch_bytes = p->scratch_bytes;
    info->attention_ctas = p->attn_ctas;
    info->attention_warps = p->attn_warps;
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_pool_reset(QwnKvPoolHandle *h) {
    Pool *p = pool_from(h);
    if (!p) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lk(p->mu);
    cudaSetDevice(p->device);
    cudaError_t e = launch_pool_init_state(p, p->stream);
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_pool_reset", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_pool_check(QwnKvPoolHandle *h, uint32_t *bits) {
    Pool *p = pool_from(h);
    if (!p || !bits) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    cudaSetDevice(p->device);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_pool_check", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    uint32_t st = 0;
    cudaMemcpy(&st, p->status, sizeof(st), cudaMemcpyDeviceToHost);
    cudaMemset(p->status, 0, sizeof(uint32_t));
    if (st & QWN_KV_STATUS_WAIT_TIMEOUT)  // an abandoned merge leaves counters behind
        cudaMemset(p->counters, 0, sizeof(uint32_t) * counter_count(p));
    *bits = st;
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_seq_append(QwnKvPoolHandle *h, uint32_t n, const int32_t *seq_ids,
                                       const int32_t *counts, void *stream) {
    Pool *p = pool_from(h);
    if (!p || n > p->max_seqs) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    cudaSetDevice(p->device);
    cudaError_t e = launch_seq_append(p, n, seq_ids, counts, stream_of(p, stream));
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_seq_append", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}

static int decode_impl(Pool *p, const QwnKvDecodeRequest *r, cudaStream_t s) {
    if (r->layer >= p->layers || r->num_seqs > p->max_seqs || !r->query_dev || !r->output_dev ||
        r->query_heads == 0 || r->query_heads % p->kv_heads || r->query_heads > p->max_query_heads ||
        ((r->key_dev == nullptr) != (r->value_dev == nullptr))) {
        set_error("qwn_kv_decode: invalid request");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    cudaError_t e = cudaSuccess;
    // attention over the whole sequence ends in the tile of the newest token:
    // the attention kernel quantizes and stores it before reading that tile
    const bool fuse = r->key_dev && r->attend_limit == 0;
    if (r->key_dev && !fuse)
        e = launch_append(p, r->layer, r->num_seqs, r->seq_ids_dev, r->key_dev, r->value_dev, s);
    if (e == cudaSuccess) {
        AttnLaunch a{};
        if (fuse) {
            a.new_k = r->key_dev;
            a.new_v = r->value_dev;
        }
        a.layer = r->layer;
        a.num_seqs = r->num_seqs;
        a.query_heads = r->query_heads;
        a.attend_limit = r->attend_limit;
        a.seq_ids = r->seq_ids_dev;
        a.query = r->query_dev;
        a.output = r->output_dev;
        a.scale = r->scale > 0.f ? r->scale : 1.0f / std::sqrt((float)kHeadDim);
        a.page_mass = r->page_mass_dev;
        e = launch_attention(p, a, s);
    }
    if (e == cudaSuccess && r->page_mass_dev) {
        e = launch_page_mass(p, r->num_seqs, r->seq_ids_dev, r->query_heads, r->page_mass_dev, s);
    }
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_decode", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_decode(QwnKvPoolHandle *h, const QwnKvDecodeRequest *r) {
    Pool *p = pool_from(h);
    if (!p || !r || !header_ok(r->header, sizeof(*r))) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    cudaSetDevice(p->device);
    return decode_impl(p, r, stream_of(p, r->stream));
}

QWN_CUDA_ABI_API int qwn_kv_append(QwnKvPoolHandle *h, uint32_t layer, uint32_t n, const int32_t *seq_ids,
                                   const float *key, const float *value, void *stream) {
    Pool *p = pool_from(h);
    if (!p || layer >= p->layers || n > p->max_seqs || !key || !value) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    cudaSetDevice(p->device);
    cudaError_t e = launch_append(p, layer, n, seq_ids, key, value, stream_of(p, stream));
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_append", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_partial(QwnKvPoolHandle *h, const QwnKvPartialRequest *r) {
    Pool *p = pool_from(h);
    if (!p || !r || !header_ok(r->header, sizeof(*r)) || r->layer >= p->layers || !r->query_dev ||
        !r->m_dev || !r->l_dev || !r->o_dev || r->query_heads % p->kv_heads ||
        r->query_heads > p->max_query_heads || r->num_seqs > p->max_seqs) {
        set_error("qwn_kv_partial: invalid request");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    cudaSetDevice(p->device);
    AttnLaunch a{};
    a.layer = r->layer;
    a.num_seqs = r->num_seqs;
    a.query_heads = r->query_heads;
    a.seq_ids = r->seq_ids_dev;
    a.query = r->query_dev;
    a.scale = r->scale > 0.f ? r->scale : 1.0f / std::sqrt((float)kHeadDim);
    a.part_m = r->m_dev;
    a.part_l = r->l_dev;
    a.part_o = r->o_dev;
    a.t_begin = r->t_begin;
    a.t_end = r->t_end;
    cudaStream_t s = stream_of(p, r->stream);
    // rows whose range is empty are never visited by a warp: mark them empty
    cudaError_t e = cudaMemsetAsync(r->l_dev, 0, sizeof(float) * r->num_seqs * r->query_heads, s);
    if (e == cudaSuccess) {
        e = launch_fill_f32(r->m_dev, -INFINITY, (size_t)r->num_seqs * r->query_heads, s);
    }
    if (e == cudaSuccess) e = launch_attention(p, a, s);
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_partial", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_merge_partials(uint32_t parts, uint32_t rows, const float *m, const float *l,
                                           const float *o, float *out, void *stream) {
    if (!m || !l || !o || !out || parts == 0) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    cudaError_t e = launch_merge(parts, rows, m, l, o, out, rows, (size_t)rows * kHeadDim,
                                 static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_merge_partials", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_merge_partials_packed(uint32_t parts, uint32_t rows, const float *packed, float *out,
                                                  void *stream) {
    if (!packed || !out || parts == 0) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    const size_t stride = (size_t)rows * (kHeadDim + 2);
    const float *o = packed, *m = packed + (size_t)rows * kHeadDim, *l = m + rows;
    cudaError_t e = launch_merge(parts, rows, m, l, o, out, stride, stride, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_merge_partials_packed", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}

// ---- split-KV exchange buffers (CUDA IPC over the node's NVLink fabric) ----
static size_t exchange_bytes(uint32_t max_rows) {
    return 2ull * QWN_KV_MAX_RANKS * QWN_KV_EXCHANGE_SEGMENTS * 4 +
           2ull * QWN_KV_MAX_RANKS * max_rows * (kHeadDim + 2) * sizeof(float);
}

QWN_CUDA_ABI_API int qwn_kv_exchange_bytes(uint32_t max_rows, uint64_t *bytes) {
    if (!bytes || max_rows == 0) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    *bytes = exchange_bytes(max_rows);
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_exchange_alloc(int32_t device, uint64_t bytes, void **buf, void *ipc_handle) {
    if (!buf || !ipc_handle || bytes == 0) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    *buf = nullptr;
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaMalloc(buf, bytes);
    if (e == cudaSuccess) e = cudaMemset(*buf, 0, bytes);
    cudaIpcMemHandle_t hd{};
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&hd, *buf);
    if (e != cudaSuccess) {
        if (*buf) cudaFree(*buf);
        *buf = nullptr;
        set_cuda_error("qwn_kv_exchange_alloc", e);
        return e == cudaErrorMemoryAllocation ? QWN_CUDA_STATUS_OUT_OF_MEMORY : QWN_CUDA_STATUS_RUNTIME_ERROR;
    }
    static_assert(sizeof(hd) == 64, "CUDA IPC handles are 64 bytes");
    std::memcpy(ipc_handle, &hd, sizeof(hd));
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_exchange_free(int32_t device, void *buf) {
    if (!buf) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    cudaSetDevice(device);
    cudaError_t e = cudaFree(buf);
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_exchange_free", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_exchange_open(int32_t device, const void *ipc_handle, void **buf) {
    if (!buf || !ipc_handle) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    cudaIpcMemHandle_t hd;
    std::memcpy(&hd, ipc_handle, sizeof(hd));
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaIpcOpenMemHandle(buf, hd, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_exchange_open", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_exchange_close(int32_t device, void *buf) {
    if (!buf) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    cudaSetDevice(device);
    cudaError_t e = cudaIpcCloseMemHandle(buf);
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_exchange_close", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_decode_split(QwnKvPoolHandle *h, const QwnKvSplitRequest *r) {
    Pool *p = pool_from(h);
    if (!p || !r || !header_ok(r->header, sizeof(*r))) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    const QwnKvPeerSet *ps = r->peers;
    bool ok = ps && header_ok(ps->header, sizeof(*ps)) && ps->world >= 1 && ps->world <= QWN_KV_MAX_RANKS &&
              ps->rank < ps->world && r->epoch != 0 && r->layer < p->layers && r->query_dev && r->output_dev &&
              r->query_heads && r->query_heads % p->kv_heads == 0 && r->query_heads <= p->max_query_heads &&
              r->query_heads <= ps->max_rows && p->kv_heads <= QWN_KV_EXCHANGE_SEGMENTS &&
              (r->t_end == 0 || r->t_end > r->t_begin) && ((r->key_dev == nullptr) == (r->value_dev == nullptr)) &&
              (r->key_dev == nullptr || r->t_end == 0);
    for (uint32_t k = 0; ok && k < ps->world; k++) ok = ps->buffers[k] != nullptr;
    if (!ok) {
        set_error("qwn_kv_decode_split: invalid request");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    cudaSetDevice(p->device);
    AttnLaunch a{};
    a.layer = r->layer;
    a.num_seqs = 1;
    a.query_heads = r->query_heads;
    a.seq_ids = r->seq_ids_dev;
    a.query = r->query_dev;
    a.output = r->output_dev;
    a.scale = r->scale > 0.f ? r->scale : 1.0f / std::sqrt((float)kHeadDim);
    a.t_begin = r->t_begin;
    a.t_end = r->t_end;
    a.new_k = r->key_dev;
    a.new_v = r->value_dev;
    a.peers = ps;
    a.epoch = r->epoch;
    cudaError_t e = launch_attention(p, a, stream_of(p, r->stream));
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_decode_split", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_store_tokens(QwnKvPoolHandle *h, int32_t seq, uint32_t layer, uint32_t first,
                                         uint32_t n, const float *key, const float *value, void *stream) {
    Pool *p = pool_from(h);
    if (!p || seq < 0 || (uint32_t)seq >= p->max_seqs || layer >= p->layers || !key || !value)
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    cudaSetDevice(p->device);
    cudaError_t e = launch_store_tokens(p, seq, layer, first, n, key, value, stream_of(p, stream));
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_store_tokens", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_generate_rows(float *out, uint32_t rows, uint32_t width, uint32_t kind,
                                          uint64_t seed, uint32_t layer, const int32_t *seq_ids,
                                          const int32_t *pos, const uint8_t *mask, void *stream) {
    if (!out || !pos) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    cudaError_t e = launch_generate(out, rows, width, kind, seed, layer, seq_ids, pos, mask,
                                    static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_generate_rows", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_prefill_synthetic(QwnKvPoolHandle *h, uint32_t n, const int32_t *host_seq_ids,
                                              const int32_t *host_lens, uint64_t seed,
                                              const uint8_t *mask_host, void *stream) {
    Pool *p = pool_from(h);
    if (!p || !host_seq_ids || !host_lens || n > p->max_seqs) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    cudaSetDevice(p->device);
    cudaStream_t s = stream_of(p, stream);
    int32_t *d_ids = nullptr, *d_cnt = nullptr;
    uint8_t *d_mask = nullptr;
    const size_t mask_bytes = (size_t)p->layers * p->kv_heads * kHeadDim;
    cudaError_t e = cudaMalloc(&d_ids, sizeof(int32_t) * n);
    if (e == cudaSuccess) e = cudaMalloc(&d_cnt, sizeof(int32_t) * n);
    if (e == cudaSuccess && mask_host) e = cudaMalloc(&d_mask, mask_bytes);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_ids, host_seq_ids, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_cnt, host_lens, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess && mask_host) e = cudaMemcpyAsync(d_mask, mask_host, mask_bytes, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = launch_seq_append(p, n, d_ids, d_cnt, s);
    for (uint32_t i = 0; e == cudaSuccess && i < n; i++) {
        if (host_lens[i] <= 0) continue;
        const uint64_t warps = (uint64_t)p->layers * (uint64_t)host_lens[i] * p->kv_heads;
        const uint32_t blocks = (uint32_t)std::min<uint64_t>((warps + 3) / 4, 148ull * 32ull);
        e = dispatch_store<PrefillL>(p->codec, dim3(blocks), dim3(128), s, store_geo(p), host_seq_ids[i],
                                     p->layers, (uint32_t)host_lens[i], seed, (const uint8_t *)d_mask);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaFree(d_ids);
    cudaFree(d_cnt);
    cudaFree(d_mask);
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_prefill_synthetic", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_evict(QwnKvPoolHandle *h, const QwnKvEvictRequest *r) {
    Pool *p = pool_from(h);
    if (!p || !r || !header_ok(r->header, sizeof(*r)) || !r->page_mass_dev || !r->flags_dev ||
        r->num_seqs > p->max_seqs)
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    cudaSetDevice(p->device);
    cudaError_t e = launch_evict(p, r->num_seqs, r->seq_ids_dev, r->page_mass_dev, r->flags_dev,
                                 r->token_budget, stream_of(p, r->stream));
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_evict", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_kv_decode_step_host(QwnKvPoolHandle *h, const QwnKvHostStepRequest *r,
                                             QwnCudaTelemetry *tel) {
    Pool *p = pool_from(h);
    if (!p || !r || !header_ok(r->header, sizeof(*r)) || !r->host_query || !r->host_key || !r->host_value ||
        !r->host_output || r->num_layers == 0 || r->num_layers > p->layers || r->num_seqs == 0 ||
        r->num_seqs > p->max_seqs || r->query_heads % p->kv_heads || r->query_heads > p->max_query_heads) {
        set_error("qwn_kv_decode_step_host: invalid request");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    std::lock_guard<std::mutex> lk(p->mu);
    cudaSetDevice(p->device);
    const size_t q_el = (size_t)r->num_seqs * r->query_heads * kHeadDim;
    const size_t kv_el = (size_t)r->num_seqs * p->kv_heads * kHeadDim;
    const size_t lq = q_el * r->num_layers, lkv = kv_el * r->num_layers;
    cudaError_t e = cudaSuccess;
    if (lq > p->stage_q_elems || lkv > p->stage_kv_elems) {
        cudaFree(p->stage_q); cudaFree(p->stage_k); cudaFree(p->stage_v); cudaFree(p->stage_o);
        p->stage_q = p->stage_k = p->stage_v = p->stage_o = nullptr;
        p->stage_q_elems = p->stage_kv_elems = 0;
        if ((e = cudaMalloc(&p->stage_q, lq * 4)) || (e = cudaMalloc(&p->stage_o, lq * 4)) ||
            (e = cudaMalloc(&p->stage_k, lkv * 4)) || (e = cudaMalloc(&p->stage_v, lkv * 4))) {
            set_cuda_error("qwn_kv_decode_step_host: staging", e);
            return QWN_CUDA_STATUS_OUT_OF_MEMORY;
        }
        p->stage_q_elems = lq;
        p->stage_kv_elems = lkv;
    }
    if (r->num_layers > p->layer_events) {
        for (uint32_t i = 0; i < p->layer_events; i++) {
            cudaEventDestroy(p->layer_in_ev[i]);
            cudaEventDestroy(p->layer_out_ev[i]);
        }
        delete[] p->layer_in_ev;
        delete[] p->layer_out_ev;
        p->layer_in_ev = new cudaEvent_t[r->num_layers];
        p->layer_out_ev = new cudaEvent_t[r->num_layers];
        for (uint32_t i = 0; i < r->num_layers; i++) {
            cudaEventCreateWithFlags(&p->layer_in_ev[i], cudaEventDisableTiming);
            cudaEventCreateWithFlags(&p->layer_out_ev[i], cudaEventDisableTiming);
        }
        p->layer_events = r->num_layers;
    }
    if (!p->step_t0) {
        if ((e = cudaEventCreate(&p->step_t0)) || (e = cudaEventCreate(&p->step_t1)) ||
            (e = cudaMallocHost(&p->status_host, sizeof(uint32_t)))) {
            set_cuda_error("qwn_kv_decode_step_host: set-up", e);
            return QWN_CUDA_STATUS_RUNTIME_ERROR;
        }
    }
    cudaEvent_t t0 = p->step_t0, t1 = p->step_t1;
    cudaEventRecord(t0, p->stream);
    // The layers go in chunks: the first and the last of one layer, the rest
    // in about five spans.  Each chunk's inputs arrive on the copy stream, the
    // compute stream waits for them once and then launches the chunk's layers
    // back to back -- with no stream operation between two attention
    // launches, so each may start early on the SMs the one before leaves --
    // and the chunk's outputs go back on the output stream as soon as its
    // last layer is done, while the next chunk computes.
    const uint32_t NL = r->num_layers;
    constexpr uint32_t kChunks = 7;  // at most: the first layer, five spans, the last layer
    uint32_t bounds[kChunks + 1];
    uint32_t nchunks = 0;
    bounds[0] = 0;
    {
        const uint32_t mid = NL > 2 ? NL - 2 : 0;  // layers between the first and the last
        const uint32_t span = mid ? (mid + kChunks - 3) / (kChunks - 2) : 1;
        uint32_t at = 1;
        bounds[++nchunks] = 1;  // the first layer alone: compute starts after one layer's copy
        while (NL > 1 && at < NL - 1) {
            at = at + span < NL - 1 ? at + span : NL - 1;
            bounds[++nchunks] = at;
        }
        if (NL > 1) bounds[++nchunks] = NL;  // the last layer alone: its copy out is the only tail
    }
    for (uint32_t c = 0; c < nchunks && e == cudaSuccess; c++) {
        const uint32_t a = bounds[c], n = bounds[c + 1] - a;
        e = cudaMemcpyAsync(p->stage_q + a * q_el, r->host_query + a * q_el, n * q_el * 4, cudaMemcpyHostToDevice,
                            p->copy_stream);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(p->stage_k + a * kv_el, r->host_key + a * kv_el, n * kv_el * 4,
                                cudaMemcpyHostToDevice, p->copy_stream);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(p->stage_v + a * kv_el, r->host_value + a * kv_el, n * kv_el * 4,
                                cudaMemcpyHostToDevice, p->copy_stream);
        if (e == cudaSuccess) e = cudaEventRecord(p->layer_in_ev[c], p->copy_stream);
    }
    if (e == cudaSuccess) e = launch_seq_append(p, r->num_seqs, nullptr, nullptr, p->stream);
    for (uint32_t c = 0; c < nchunks && e == cudaSuccess; c++) {
        e = cudaStreamWaitEvent(p->stream, p->layer_in_ev[c], 0);
        for (uint32_t L = bounds[c]; L < bounds[c + 1] && e == cudaSuccess; L++) {
            QwnKvDecodeRequest d{};
            qwn_cuda_abi_header_init(&d.header, sizeof(d));
            d.layer = L;
            d.num_seqs = r->num_seqs;
            d.query_heads = r->query_heads;
            d.scale = r->scale;
            d.query_dev = p->stage_q + L * q_el;
            d.key_dev = p->stage_k + L * kv_el;
            d.value_dev = p->stage_v + L * kv_el;
            d.output_dev = p->stage_o + L * q_el;
            if (decode_impl(p, &d, p->stream) != QWN_CUDA_STATUS_OK) e = cudaErrorLaunchFailure;
        }
        if (e == cudaSuccess) e = cudaEventRecord(p->layer_out_ev[c], p->stream);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(p->out_stream, p->layer_out_ev[c], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(r->host_output + bounds[c] * q_el, p->stage_o + bounds[c] * q_el,
                                (bounds[c + 1] - bounds[c]) * q_el * 4, cudaMemcpyDeviceToHost, p->out_stream);
    }
    // the status word comes back with the step (no separate synchronous read)
    if (e == cudaSuccess) e = cudaMemcpyAsync(p->status_host, p->status, sizeof(uint32_t), cudaMemcpyDeviceToHost,
                                              p->stream);
    if (e == cudaSuccess) e = cudaEventRecord(t1, p->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(p->copy_stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(p->out_stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(p->stream);
    float ms = 0.f;
    if (e == cudaSuccess) cudaEventElapsedTime(&ms, t0, t1);
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_decode_step_host", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    // clear a latched status word, as qwn_kv_pool_check does, so that one
    // error fails this step and not every later one; an abandoned split-KV
    // merge (wait timeout) also leaves counters that must restart at 0
    const uint32_t st = *p->status_host;
    if (st) e = cudaMemset(p->status, 0, sizeof(uint32_t));
    if (e == cudaSuccess && (st & QWN_KV_STATUS_WAIT_TIMEOUT))
        e = cudaMemset(p->counters, 0, sizeof(uint32_t) * counter_count(p));
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_decode_step_host: status", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    if (tel && header_ok(tel->header, sizeof(*tel))) {
        // one page-allocation launch, then one fused append + attention launch per layer
        tel->kv_cache_kernel_count += 1ull + r->num_layers;
        tel->kv_cache_upload_bytes += (uint64_t)(lq + 2 * lkv) * 4;
        tel->kv_cache_kernel_ms += ms;
        std::snprintf(tel->kv_cache_kernel_type, sizeof(tel->kv_cache_kernel_type), "paged-b200-split-kv");
    }
    if (st & QWN_KV_STATUS_POOL_EXHAUSTED) {
        set_error("paged KV pool exhausted");
        return QWN_CUDA_STATUS_OUT_OF_MEMORY;
    }
    if (st) {
        set_error("device status latched an error (see qwn_kv_pool_check)");
        return QWN_CUDA_STATUS_RUNTIME_ERROR;
    }
    return QWN_CUDA_STATUS_OK;
}

}  // extern "C"
