// The reference's own C APIs, served by qwn_cuda.so on the GPU:
//   qwn_paged_kv.h         (c/qwn_paged_kv.h:12-85)        fp16 block pool, block tables, paged attention
//   qwanto_turboquant.h    (c/qwanto_turboquant.h:11-156)  cache mode/contract, Q8 and TurboQuant caches
//   qwanto_attention.h     (c/qwanto_attention.h:11-69)    linear attention
//   qwanto_pagedeviction.h (c/qwanto_pagedeviction.h:16-70) token-level eviction bookkeeping
//
// A caller built against the reference headers links against this library
// instead of the reference's .c files.  The structs keep the reference
// layouts; their data buffers are CUDA managed memory (valid on the host and
// the device, in the reference's byte layout), their integer bookkeeping
// (free stack, block ids, vToken slots) stays host memory as the structs
// expose it.  Every quantization, conversion and attention runs as a kernel
// on the calling thread's current device, on a non-blocking stream of that
// thread, and each call synchronises that stream before it returns, as the
// reference calls are synchronous.  The decoder calls the per-head functions
// from OpenMP threads concurrently (c/qwanto_decode.c:1745-1754); each thread
// has its own stream and scratch, so those calls overlap on the GPU.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "kv_internal.cuh"
#include "qwanto_attention.h"
#include "qwanto_pagedeviction.h"
#include "qwanto_turboquant.h"
#include "qwn_paged_kv.h"

namespace qref {
namespace {

constexpr int kThreads = 256;

// ---------------------------------------------------------------------------
// per-thread stream and device scratch
// ---------------------------------------------------------------------------
struct Ctx {
    int dev = -1;
    cudaStream_t s = nullptr;
    char *scratch = nullptr;
    size_t cap = 0;
};
thread_local Ctx t_ctx;

void fail(const char *what, cudaError_t e) {
    qkv::set_cuda_error(what, e);
    fprintf(stderr, "[qwn_cuda] %s failed: %s\n", what, cudaGetErrorString(e));
}

// The calling thread's stream and at least `bytes` of device scratch on its
// current device (nullptr, with the error recorded, when CUDA is unusable).
Ctx *ctx(const char *what, size_t bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { fail(what, e); return nullptr; }
    Ctx &c = t_ctx;
    if (c.dev != dev) {
        c = Ctx{};
        e = cudaStreamCreateWithFlags(&c.s, cudaStreamNonBlocking);
        if (e != cudaSuccess) { fail(what, e); return nullptr; }
        c.dev = dev;
    }
    if (bytes > c.cap) {
        if (c.scratch) cudaFree(c.scratch);  // every earlier call of this thread has completed
        const size_t cap = std::max<size_t>({bytes, 2 * c.cap, 1u << 16});
        e = cudaMalloc(&c.scratch, cap);
        if (e != cudaSuccess) { c.scratch = nullptr; c.cap = 0; fail(what, e); return nullptr; }
        c.cap = cap;
    }
    return &c;
}

size_t up256(size_t x) { return (x + 255) & ~(size_t)255; }

// carve consecutive 256-byte aligned pieces out of the thread's scratch
struct Carve {
    char *p;
    template <class T>
    T *take(size_t count) {
        T *r = reinterpret_cast<T *>(p);
        p += up256(count * sizeof(T));
        return r;
    }
};

cudaError_t copy(void *dst, const void *src, size_t bytes, cudaStream_t s) {
    if (!bytes) return cudaSuccess;
    return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, s);
}

// pointers a kernel may write through: device, managed, or mapped host memory
bool device_writable(const void *p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged ||
           (a.type == cudaMemoryTypeHost && a.devicePointer == p);
}

cudaError_t managed_zeroed(void **p, size_t bytes) {
    *p = nullptr;
    cudaError_t e = cudaMallocManaged(p, bytes ? bytes : 1);
    if (e != cudaSuccess) { *p = nullptr; return e; }
    e = cudaMemset(*p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { cudaFree(*p); *p = nullptr; }
    return e;
}

// ---------------------------------------------------------------------------
// fp16 conversions
// ---------------------------------------------------------------------------
// F16C's round to nearest even (_mm256_cvtps_ph, c/qwn_paged_kv.c:176-185);
// a NaN keeps its top ten payload bits with the quiet bit set
__device__ __forceinline__ uint16_t f16_rne(float x) {
    const uint32_t u = __float_as_uint(x);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)(((u >> 16) & 0x8000u) | 0x7E00u | ((u >> 13) & 0x3FFu));
    return __half_as_ushort(__float2half_rn(x));
}
// the reference's scalar float_to_half (c/qwn_paged_kv.c:23-31), used for the
// head_dim % 8 tail: truncates, flushes subnormals to zero, NaN -> 0x7C01
__device__ __forceinline__ uint16_t f16_trunc_ftz(float f) {
    const uint32_t b = __float_as_uint(f);
    const uint32_t sign = b >> 31, exp = (b >> 23) & 255, mant = b & 0x7fffff;
    if (exp == 255) return (uint16_t)((sign << 15) | 0x7c00 | (mant ? 1u : 0u));
    const int e = (int)exp - 127 + 15;
    if (e <= 0) return (uint16_t)(sign << 15);
    if (e >= 31) return (uint16_t)((sign << 15) | 0x7c00);
    return (uint16_t)((sign << 15) | ((uint32_t)e << 10) | (mant >> 13));
}
// the reference's scalar half_to_float (c/qwn_paged_kv.c:15-21): subnormals read as zero
__device__ __forceinline__ float f16_ftz_to_f32(uint16_t h) {
    const uint32_t sign = (h >> 15) & 1, exp = (h >> 10) & 31, mant = h & 1023;
    uint32_t bits;
    if (exp == 0) bits = sign << 31;
    else if (exp == 31) bits = (sign << 31) | 0x7f800000u | (mant << 13);
    else bits = (sign << 31) | ((exp + 112) << 23) | (mant << 13);
    return __uint_as_float(bits);
}

// ---------------------------------------------------------------------------
// the cache formats, as element readers for the attention kernel
// ---------------------------------------------------------------------------
// fp16 block pool [block][layer][kv_head][16][head_dim] (c/qwn_paged_kv.c:237-247);
// elements below hd8 convert exactly (F16C), the tail as the scalar code does
struct PagedF16 {
    const uint16_t *kd, *vd;
    const int *blocks;
    size_t block_stride, head_base;
    int hd, hd8;
    __device__ size_t row(int t) const {
        return (size_t)blocks[t >> 4] * block_stride + head_base + (size_t)(t & 15) * hd;
    }
    __device__ float cvt(uint16_t h, int j) const { return j < hd8 ? qkv::h2f(h) : f16_ftz_to_f32(h); }
    __device__ float key(int t, int j) const { return cvt(kd[row(t) + j], j); }
    __device__ float value(int t, int j) const { return cvt(vd[row(t) + j], j); }
};

// contiguous Q8 cache, fp32 scale per 64 channels (c/qwanto_turboquant.c:648-676)
struct Q8Contig {
    const int8_t *pk, *pv;
    const float *sk, *sv;
    size_t ts, ss;
    int off;
    __device__ float key(int t, int j) const {
        const int c = off + j;
        return (float)pk[(size_t)t * ts + c] * sk[(size_t)t * ss + (c >> 6)];
    }
    __device__ float value(int t, int j) const {
        const int c = off + j;
        return (float)pv[(size_t)t * ts + c] * sv[(size_t)t * ss + (c >> 6)];
    }
};

// one value of a 32-byte TurboQuant block (c/qwanto_turboquant.c:142-157,
// :225-247): pair i/2 of sub-chunk i/16 sits at bit 7*(pair % 8) of its 7
// bytes; even index = 4-bit code x range/15, odd = 3-bit code x range/7, + min
__device__ __forceinline__ float tq_value(const uint8_t *blk, int i) {
    const float range = qkv::h2f((uint16_t)(blk[0] | (blk[1] << 8)));
    const float mn = qkv::h2f((uint16_t)(blk[2] | (blk[3] << 8)));
    const int p = i >> 1, sub = p >> 3, bit = 7 * (p & 7);
    const uint8_t *b = blk + 4 + 7 * sub + (bit >> 3);
    uint32_t w = b[0];
    if ((bit >> 3) + 1 < 7) w |= (uint32_t)b[1] << 8;
    const uint32_t pair = (w >> (bit & 7)) & 0x7Fu;
    if (i & 1) return (float)((pair >> 4) & 7u) * (range * (1.0f / 7.0f)) + mn;
    return (float)(pair & 15u) * (range * (1.0f / 15.0f)) + mn;
}

// contiguous TurboQuant cache (c/qwanto_turboquant.c:717-768)
struct TQContig {
    const uint8_t *pk, *pv;
    size_t tsk, tsv, head_off;
    __device__ float key(int t, int j) const {
        return tq_value(pk + (size_t)t * tsk + head_off + (size_t)(j >> 6) * TURBOQUANT_BLOCK_BYTES, j & 63);
    }
    __device__ float value(int t, int j) const {
        return tq_value(pv + (size_t)t * tsv + head_off + (size_t)(j >> 6) * TURBOQUANT_BLOCK_BYTES, j & 63);
    }
};

// ---------------------------------------------------------------------------
// one attention head over tokens [0, n): scores, softmax, weighted values.
// One CTA of 8 warps: warps take tokens round robin for the dot products,
// the softmax reduces over the CTA (sum in double, as c/qwn_paged_kv.c:200-211),
// and the value sum splits the tokens over thread groups that are added in
// a fixed order.  probs receives p (normalised) or exp(s - max) (leave_exps).
// ---------------------------------------------------------------------------
template <class Src>
__global__ void __launch_bounds__(kThreads) head_attention_kernel(Src src, int n, int hd, const float *q,
                                                                  float scale, float *probs, float *out,
                                                                  int leave_exps) {
    __shared__ float red_f[kThreads / 32];
    __shared__ double red_d[kThreads / 32];
    __shared__ float part[kThreads];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int t = warp; t < n; t += kThreads / 32) {
        float d = 0.f;
        for (int j = lane; j < hd; j += 32) d = fmaf(q[j], src.key(t, j), d);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        if (lane == 0) probs[t] = d * scale;
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int t = tid; t < n; t += kThreads) mx = fmaxf(mx, probs[t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red_f[warp] = mx;
    __syncthreads();
    mx = red_f[0];
    for (int w = 1; w < kThreads / 32; w++) mx = fmaxf(mx, red_f[w]);
    double sum = 0.0;
    for (int t = tid; t < n; t += kThreads) {
        const float e = expf(probs[t] - mx);
        probs[t] = e;
        sum += (double)e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) red_d[warp] = sum;
    __syncthreads();
    sum = 0.0;
    for (int w = 0; w < kThreads / 32; w++) sum += red_d[w];
    const float inv = sum > 0.0 ? (float)(1.0 / sum) : 0.f;
    if (!leave_exps)
        for (int t = tid; t < n; t += kThreads) probs[t] *= inv;
    __syncthreads();
    const int groups = hd >= kThreads ? 1 : kThreads / hd;
    for (int j0 = 0; j0 < hd; j0 += kThreads) {
        const int g = hd >= kThreads ? 0 : tid / hd;
        const int j = hd >= kThreads ? j0 + tid : tid % hd;
        float acc = 0.f;
        if (g < groups && j < hd)
            for (int t = g; t < n; t += groups) {
                const float p = leave_exps ? probs[t] * inv : probs[t];
                acc = fmaf(p, src.value(t, j), acc);
            }
        if (groups == 1) {
            if (j < hd) out[j] = acc;
        } else {
            part[tid] = (g < groups) ? acc : 0.f;
            __syncthreads();
            if (tid < hd) {
                float s = 0.f;
                for (int k = 0; k < groups; k++) s += part[k * hd + tid];
                out[tid] = s;
            }
            break;  // hd < kThreads: one pass covers every column
        }
    }
}

// paged write: K/V rows [kv_heads][hd] fp32 -> the token's fp16 slots
__global__ void paged_write_kernel(uint16_t *kd, uint16_t *vd, const float *k, const float *v, size_t slot_base,
                                   int HK, int hd, int hd8) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < HK * hd; i += gridDim.x * blockDim.x) {
        const int kh = i / hd, j = i % hd;
        const size_t dst = slot_base + (size_t)kh * QWN_PAGE_BLOCK_SIZE * hd + j;
        kd[dst] = j < hd8 ? f16_rne(k[i]) : f16_trunc_ftz(k[i]);
        vd[dst] = j < hd8 ? f16_rne(v[i]) : f16_trunc_ftz(v[i]);
    }
}

// Q8 with an fp32 scale per 64 channels (c/qwanto_turboquant.c:555-586): one
// warp per 64-channel block, blockIdx.y = 0 for the key row, 1 for the value
__device__ __forceinline__ int8_t q8_round(float x) {
    if (!isfinite(x)) return 0;
    if (x >= 127.f) return 127;
    if (x <= -127.f) return -127;
    return (int8_t)__float2int_rn(x);
}
__global__ void q8_append_kernel(const float *key, const float *value, int8_t *pk, int8_t *pv, float *sk, float *sv,
                                 int n) {
    const float *x = blockIdx.y ? value : key;
    int8_t *dst = blockIdx.y ? pv : pk;
    float *scales = blockIdx.y ? sv : sk;
    const int b = blockIdx.x, lane = threadIdx.x, off = b * 64, count = min(64, n - off);
    float m = 0.f;
    for (int i = lane; i < count; i += 32) {
        const float a = x[off + i];
        if (isfinite(a)) m = fmaxf(m, fabsf(a));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s = m > 0.f ? __fdiv_rn(m, 127.f) : 1.f;
    if (lane == 0) scales[b] = s;
    for (int i = lane; i < count; i += 32) dst[off + i] = q8_round(__fdiv_rn(x[off + i], s));
}

// TurboQuant token quantizer (c/qwanto_turboquant.c:162-213): one warp per
// 64-value group, lane l owns the pair (2l, 2l+1).  min/max follow the
// reference's sequential scan: the first element when it is NaN, else the
// smallest / largest value, the earliest one among equals (+0 and -0 tie).
__device__ __forceinline__ void seq_extreme(float v, int idx, bool valid, bool want_min, float &val, int &at) {
    val = v;
    at = valid ? idx : 0x7fffffff;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, val, o);
        const int a2 = __shfl_xor_sync(0xffffffffu, at, o);
        if (a2 == 0x7fffffff) continue;
        const bool better = at == 0x7fffffff || (want_min ? v2 < val : v2 > val) || (v2 == val && a2 < at);
        if (better) { val = v2; at = a2; }
    }
}
__device__ __forceinline__ uint32_t tq_code(float x, float mn, float inv, float levels, int top) {
    float norm = (x - mn) * inv;
    if (norm < 0.f) norm = 0.f;
    if (norm > 1.f) norm = 1.f;
    int q = (int)roundf(norm * levels);  // NaN converts to 0, as the clamps below make the reference's value
    if (q > top) q = top;
    if (q < 0) q = 0;
    return (uint32_t)q;
}
__global__ void tq_quantize_kernel(const float *src, uint8_t *dst, int n) {
    const int b = blockIdx.x, lane = threadIdx.x, off = b * TURBOQUANT_GROUP_SIZE;
    const int len = min(TURBOQUANT_GROUP_SIZE, n - off);
    const int i0 = 2 * lane, i1 = 2 * lane + 1;
    const float x0 = i0 < len ? src[off + i0] : 0.f, x1 = i1 < len ? src[off + i1] : 0.f;
    float mn, mx;
    if (isnan(src[off])) {
        mn = mx = src[off];
    } else {
        // candidates: the lane's non-NaN values, earliest first
        float lo = 0.f, hi = 0.f;
        int alo = 0x7fffffff, ahi = 0x7fffffff;
        if (i0 < len && !isnan(x0)) { lo = hi = x0; alo = ahi = i0; }
        if (i1 < len && !isnan(x1)) {
            if (alo == 0x7fffffff || x1 < lo) { lo = x1; alo = i1; }
            if (ahi == 0x7fffffff || x1 > hi) { hi = x1; ahi = i1; }
        }
        int a;
        seq_extreme(lo, alo, alo != 0x7fffffff, true, mn, a);
        seq_extreme(hi, ahi, ahi != 0x7fffffff, false, mx, a);
    }
    const float range = mx - mn;
    const float inv = range > 1e-8f ? __fdiv_rn(1.0f, range) : 0.f;
    const uint32_t c0 = i0 < len ? tq_code(x0, mn, inv, 15.f, 15) : 0u;
    const uint32_t c1 = i1 < len ? tq_code(x1, mn, inv, 7.f, 7) : 0u;
    const uint32_t pair = (c0 & 15u) | ((c1 & 7u) << 4);
    // gather the 8 pairs of this lane's 16-value sub-chunk into 56 bits
    const int sub = lane >> 3, p = lane & 7;
    uint64_t w = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) w |= (uint64_t)__shfl_sync(0xffffffffu, pair, (sub << 3) + k) << (7 * k);
    uint8_t *blk = dst + (size_t)b * TURBOQUANT_BLOCK_BYTES;
    if (p < 7) blk[4 + 7 * sub + p] = (uint8_t)(w >> (8 * p));
    if (lane == 0) {
        const uint16_t r16 = qkv::tq_f32_to_f16(range), m16 = qkv::tq_f32_to_f16(mn);
        blk[0] = (uint8_t)r16;
        blk[1] = (uint8_t)(r16 >> 8);
        blk[2] = (uint8_t)m16;
        blk[3] = (uint8_t)(m16 >> 8);
    }
}

// one token's dot product / value accumulation (one warp); the block sums are
// added in block order, as c/qwanto_turboquant.c:218-284 does
__global__ void tq_dot_kernel(const float *q, const uint8_t *blocks, int dim, float *out) {
    const int lane = threadIdx.x;
    float total = 0.f;
    for (int b = 0; b * TURBOQUANT_GROUP_SIZE < dim; b++) {
        const int off = b * TURBOQUANT_GROUP_SIZE, len = min(TURBOQUANT_GROUP_SIZE, dim - off);
        const uint8_t *blk = blocks + (size_t)b * TURBOQUANT_BLOCK_BYTES;
        float d = 0.f;
        for (int i = lane; i < len; i += 32) d = fmaf(q[off + i], tq_value(blk, i), d);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        total += d;
    }
    if (lane == 0) *out = total;
}
__global__ void tq_accum_kernel(float score, const uint8_t *blocks, float *ctx, int dim) {
    for (int i = threadIdx.x; i < dim; i += blockDim.x)
        ctx[i] = fmaf(score, tq_value(blocks + (size_t)(i >> 6) * TURBOQUANT_BLOCK_BYTES, i & 63), ctx[i]);
}
// output[h * head_dim] = dot(query head h, token 0's key blocks of head h)
__global__ void tq_matmul_kernel(const uint8_t *pk, const float *q, float *out, int heads, int hd) {
    const int h = blockIdx.x, lane = threadIdx.x;
    if (h >= heads) return;
    const int bph = (hd + TURBOQUANT_GROUP_SIZE - 1) / TURBOQUANT_GROUP_SIZE;
    const uint8_t *k = pk + (size_t)h * bph * TURBOQUANT_BLOCK_BYTES;
    float total = 0.f;
    for (int b = 0; b < bph; b++) {
        const int off = b * TURBOQUANT_GROUP_SIZE, len = min(TURBOQUANT_GROUP_SIZE, hd - off);
        float d = 0.f;
        for (int i = lane; i < len; i += 32)
            d = fmaf(q[(size_t)h * hd + off + i], tq_value(k + (size_t)b * TURBOQUANT_BLOCK_BYTES, i), d);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        total += d;
    }
    if (lane == 0) out[(size_t)h * hd] = total;
}
__global__ void q8_dot_kernel(Q8Contig src, int token, const float *q, int dim, float *out) {
    float d = 0.f;
    for (int i = threadIdx.x; i < dim; i += 32) d = fmaf(q[i], src.key(token, i), d);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    if (threadIdx.x == 0) *out = d;
}
__global__ void q8_accum_kernel(Q8Contig src, int token, float score, float *ctx, int dim) {
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ctx[i] = fmaf(score, src.value(token, i), ctx[i]);
}

// ---------------------------------------------------------------------------
// host helpers
// ---------------------------------------------------------------------------
// run one attention head: q in, probabilities / exps and the context out
template <class Src>
bool run_head(const char *what, Src src, const int *blocks_host, int nblocks, int n, int hd, const float *q,
              float scale, float *scores, float *out, bool leave_exps) {
    Ctx *c = ctx(what, up256(hd * 4) * 2 + up256((size_t)n * 4) + up256((size_t)nblocks * 4));
    if (!c) return false;
    Carve cv{c->scratch};
    float *dq = cv.take<float>(hd), *dout = cv.take<float>(hd), *dp = cv.take<float>(n);
    int *db = cv.take<int>(nblocks);
    cudaError_t e = copy(dq, q, (size_t)hd * 4, c->s);
    if (e == cudaSuccess && nblocks) e = copy(db, blocks_host, (size_t)nblocks * 4, c->s);
    if constexpr (std::is_same<Src, PagedF16>::value) src.blocks = db;
    if (e == cudaSuccess) {
        head_attention_kernel<Src><<<1, kThreads, 0, c->s>>>(src, n, hd, dq, scale, dp, dout, leave_exps ? 1 : 0);
        e = cudaGetLastError();
        qkv::count_launch();
    }
    if (e == cudaSuccess) e = copy(out, dout, (size_t)hd * 4, c->s);
    if (e == cudaSuccess && scores) e = copy(scores, dp, (size_t)n * 4, c->s);
    const cudaError_t e2 = cudaStreamSynchronize(c->s);
    if (e == cudaSuccess) e = e2;
    if (e != cudaSuccess) { fail(what, e); return false; }
    return true;
}

// a single-warp kernel producing one float
template <class F>
float run_scalar(const char *what, size_t in_bytes, F launch) {
    Ctx *c = ctx(what, up256(in_bytes) + 256);
    if (!c) return 0.f;
    float *dres = reinterpret_cast<float *>(c->scratch + up256(in_bytes));
    cudaError_t e = launch(c->scratch, dres, c->s);
    qkv::count_launch();
    float r = 0.f;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&r, dres, 4, cudaMemcpyDeviceToHost, c->s);
    const cudaError_t e2 = cudaStreamSynchronize(c->s);
    if (e == cudaSuccess) e = e2;
    if (e != cudaSuccess) { fail(what, e); return 0.f; }
    return r;
}

// linear-attention side state: the reference struct carries only
// (n_heads, head_dim, state); the library keeps its staging per state buffer
std::mutex g_la_mu;
std::map<const float *, QwnLinearAttentionState> g_la;

}  // namespace
}  // namespace qref

using namespace qref;

extern "C" {

// ============================================================================
// qwn_paged_kv.h
// ============================================================================
QWN_REF_API int qwn_kv_pool_init(QwnKVBlockPool *pool, int total_blocks, int layers, int kv_heads, int head_dim) {
    if (!pool || total_blocks < 1 || layers < 1 || kv_heads < 1 || head_dim < 1) return -1;
    memset(pool, 0, sizeof(*pool));
    pool->total_blocks = total_blocks;
    pool->layers = layers;
    pool->kv_heads = kv_heads;
    pool->head_dim = head_dim;
    if ((size_t)layers > SIZE_MAX / (size_t)kv_heads ||
        (size_t)layers * kv_heads > SIZE_MAX / QWN_PAGE_BLOCK_SIZE / (size_t)head_dim)
        return -1;
    const size_t elems_per_block = (size_t)layers * kv_heads * QWN_PAGE_BLOCK_SIZE * head_dim;
    if (elems_per_block > SIZE_MAX / 2 / (size_t)total_blocks) return -1;
    const size_t bytes = (size_t)total_blocks * elems_per_block * sizeof(uint16_t);
    pool->block_bytes = elems_per_block * sizeof(uint16_t);
    cudaError_t e = managed_zeroed(reinterpret_cast<void **>(&pool->key_data), bytes);
    if (e == cudaSuccess) e = managed_zeroed(reinterpret_cast<void **>(&pool->val_data), bytes);
    pool->free_stack = (int *)malloc((size_t)total_blocks * sizeof(int));
    if (e != cudaSuccess || !pool->free_stack) {
        if (e != cudaSuccess) fail("qwn_kv_pool_init", e);
        qwn_kv_pool_free(pool);
        return -1;
    }
    for (int i = 0; i < total_blocks; i++) pool->free_stack[i] = total_blocks - 1 - i;
    pool->free_top = total_blocks;
    return 0;
}

QWN_REF_API void qwn_kv_pool_free(QwnKVBlockPool *pool) {
    if (!pool) return;
    if (pool->key_data) cudaFree(pool->key_data);
    if (pool->val_data) cudaFree(pool->val_data);
    free(pool->free_stack);
    memset(pool, 0, sizeof(*pool));
}

QWN_REF_API int qwn_kv_pool_alloc_block(QwnKVBlockPool *pool) {
    if (!pool || pool->free_top <= 0) return -1;
    return pool->free_stack[--pool->free_top];
}

QWN_REF_API void qwn_kv_pool_free_block(QwnKVBlockPool *pool, int block_id) {
    if (!pool || block_id < 0 || block_id >= pool->total_blocks || pool->free_top >= pool->total_blocks) return;
    pool->free_stack[pool->free_top++] = block_id;
}

QWN_REF_API int qwn_block_table_init(QwnBlockTable *bt, int req_id, int initial_capacity) {
    if (!bt) return -1;
    memset(bt, 0, sizeof(*bt));
    bt->req_id = req_id;
    bt->block_capacity = initial_capacity > 4 ? initial_capacity : 4;
    bt->block_ids = (int *)malloc((size_t)bt->block_capacity * sizeof(int));
    return bt->block_ids ? 0 : -1;
}

QWN_REF_API int qwn_block_table_append_token(QwnKVBlockPool *pool, QwnBlockTable *bt) {
    if (!pool || !bt) return -1;
    const int need = (bt->num_tokens + QWN_PAGE_BLOCK_SIZE) / QWN_PAGE_BLOCK_SIZE;
    if (need > bt->block_count) {
        const int blk = qwn_kv_pool_alloc_block(pool);
        if (blk < 0) return -1;
        if (bt->block_count >= bt->block_capacity) {
            const int cap = bt->block_capacity * 2;
            int *ids = (int *)realloc(bt->block_ids, (size_t)cap * sizeof(int));
            if (!ids) {
                qwn_kv_pool_free_block(pool, blk);
                return -1;
            }
            bt->block_ids = ids;
            bt->block_capacity = cap;
        }
        bt->block_ids[bt->block_count++] = blk;
    }
    bt->num_tokens++;
    return 0;
}

QWN_REF_API void qwn_block_table_free(QwnKVBlockPool *pool, QwnBlockTable *bt) {
    if (!bt) return;
    if (pool && bt->block_ids)
        for (int i = 0; i < bt->block_count; i++) qwn_kv_pool_free_block(pool, bt->block_ids[i]);
    free(bt->block_ids);
    memset(bt, 0, sizeof(*bt));
}

QWN_REF_API int qwn_paged_kv_write(QwnKVBlockPool *pool, const QwnBlockTable *bt, int layer, int token_pos,
                                   const float *k, const float *v) {
    if (!pool || !bt || !k || !v || layer < 0 || layer >= pool->layers || token_pos < 0 ||
        token_pos >= bt->num_tokens)
        return -1;
    const int bi = token_pos / QWN_PAGE_BLOCK_SIZE, slot = token_pos % QWN_PAGE_BLOCK_SIZE;
    if (!bt->block_ids || bi >= bt->block_count || bt->block_ids[bi] < 0 || bt->block_ids[bi] >= pool->total_blocks)
        return -1;
    if (!pool->key_data || !pool->val_data) return -1;
    const int HD = pool->head_dim, HK = pool->kv_heads;
    const size_t block_stride = (size_t)pool->layers * HK * QWN_PAGE_BLOCK_SIZE * HD;
    const size_t base = (size_t)bt->block_ids[bi] * block_stride + (size_t)layer * HK * QWN_PAGE_BLOCK_SIZE * HD +
                        (size_t)slot * HD;
    const size_t n = (size_t)HK * HD;
    Ctx *c = ctx("qwn_paged_kv_write", 2 * up256(n * 4));
    if (!c) return -1;
    Carve cv{c->scratch};
    float *dk = cv.take<float>(n), *dv = cv.take<float>(n);
    cudaError_t e = copy(dk, k, n * 4, c->s);
    if (e == cudaSuccess) e = copy(dv, v, n * 4, c->s);
    if (e == cudaSuccess) {
        const int blocks = (int)std::min<size_t>((n + kThreads - 1) / kThreads, 148);
        paged_write_kernel<<<blocks, kThreads, 0, c->s>>>(pool->key_data, pool->val_data, dk, dv, base, HK, HD,
                                                           HD - HD % 8);
        e = cudaGetLastError();
        qkv::count_launch();
    }
    const cudaError_t e2 = cudaStreamSynchronize(c->s);
    if (e == cudaSuccess) e = e2;
    if (e != cudaSuccess) { fail("qwn_paged_kv_write", e); return -1; }
    return 0;
}

static bool valid_table(const QwnKVBlockPool *pool, const QwnBlockTable *bt) {
    if (!pool || !bt || !bt->block_ids || bt->num_tokens < 0 || bt->block_count < 0 ||
        bt->block_count > bt->block_capacity)
        return false;
    const int need = (int)(((size_t)bt->num_tokens + QWN_PAGE_BLOCK_SIZE - 1) / QWN_PAGE_BLOCK_SIZE);
    if (need > bt->block_count) return false;
    for (int i = 0; i < need; i++)
        if (bt->block_ids[i] < 0 || bt->block_ids[i] >= pool->total_blocks) return false;
    return true;
}

QWN_REF_API void qwn_paged_attention_head(const QwnKVBlockPool *pool, const QwnBlockTable *bt, int layer,
                                          int head_idx, int kv_head_idx, const float *q_head, float *scores_scratch,
                                          float *out_ctx_head) {
    (void)head_idx;
    if (!valid_table(pool, bt) || !q_head || !scores_scratch || !out_ctx_head || layer < 0 ||
        layer >= pool->layers || kv_head_idx < 0 || kv_head_idx >= pool->kv_heads || bt->num_tokens <= 0 ||
        !pool->key_data)
        return;
    const int HD = pool->head_dim, HK = pool->kv_heads, n = bt->num_tokens;
    PagedF16 src{pool->key_data, pool->val_data, nullptr,
                 (size_t)pool->layers * HK * QWN_PAGE_BLOCK_SIZE * HD,
                 (size_t)layer * HK * QWN_PAGE_BLOCK_SIZE * HD + (size_t)kv_head_idx * QWN_PAGE_BLOCK_SIZE * HD, HD,
                 HD - HD % 8};
    const int nblk = (n + QWN_PAGE_BLOCK_SIZE - 1) / QWN_PAGE_BLOCK_SIZE;
    run_head("qwn_paged_attention_head", src, bt->block_ids, nblk, n, HD, q_head, 1.0f / sqrtf((float)HD),
             scores_scratch, out_ctx_head, false);
}

QWN_REF_API void qwn_paged_attention_gather_head(const QwnKVBlockPool *pool, const QwnBlockTable *bt, int layer,
                                                 int head_idx, int kv_head_idx, const float *q_head,
                                                 uint16_t *k_gather_scratch, uint16_t *v_gather_scratch,
                                                 float *scores_scratch, float *out_ctx_head) {
    if (!k_gather_scratch || !v_gather_scratch) return;
    qwn_paged_attention_head(pool, bt, layer, head_idx, kv_head_idx, q_head, scores_scratch, out_ctx_head);
}

QWN_REF_API void qwn_scheduler_init(QwnChunkedScheduler *sched, int max_chunk_tokens) {
    if (!sched) return;
    sched->max_chunk_tokens = max_chunk_tokens > 0 ? max_chunk_tokens : 512;
    sched->active_requests = 0;
}

QWN_REF_API int qwn_scheduler_next_chunk(const QwnChunkedScheduler *sched, const QwnBlockTable *bt) {
    if (!sched || !bt) return 0;
    if (bt->prefill_remaining <= 0) return 1;
    return std::min(bt->prefill_remaining, sched->max_chunk_tokens);
}

// ============================================================================
// qwanto_turboquant.h: mode and contract
// ============================================================================
QWN_REF_API const char *qwn_kv_cache_mode_name(QwnKvCacheMode mode) {
    switch (mode) {
        case QWN_KV_CACHE_Q8: return "q8";
        case QWN_KV_CACHE_TURBOQUANT_Q4: return "turboquant-q4";
        case QWN_KV_CACHE_AUTO: return "auto";
        default: return "fp16";
    }
}

QWN_REF_API int qwn_kv_cache_mode_parse(const char *text, QwnKvCacheMode *mode) {
    if (!text || !mode) return -1;
    if (!strcmp(text, "fp16")) *mode = QWN_KV_CACHE_FP16;
    else if (!strcmp(text, "q8")) *mode = QWN_KV_CACHE_Q8;
    else if (!strcmp(text, "turboquant-q4") || !strcmp(text, "qwn-q4-kv")) *mode = QWN_KV_CACHE_TURBOQUANT_Q4;
    else if (!strcmp(text, "auto")) *mode = QWN_KV_CACHE_AUTO;
    else return -1;
    return 0;
}

QWN_REF_API void qwn_kv_cache_contract_init(QwnKvCacheContract *c, QwnKvCacheMode mode, uint32_t valid_token_count) {
    if (!c) return;
    memset(c, 0, sizeof(*c));
    c->struct_size = (uint32_t)sizeof(*c);
    c->abi_version = QWN_KV_CACHE_ABI_VERSION;
    c->cache_dtype = (uint32_t)mode;
    c->block_size = (mode == QWN_KV_CACHE_Q8 || mode == QWN_KV_CACHE_TURBOQUANT_Q4) ? 64u : 1u;
    c->scale_bytes = mode == QWN_KV_CACHE_FP16 ? 0u : (mode == QWN_KV_CACHE_Q8 ? 4u : 2u);
    c->zero_point_bytes = mode == QWN_KV_CACHE_TURBOQUANT_Q4 ? 2u : 0u;
    c->key_layout = 1u;  // token -> head -> channel
    c->value_layout = 1u;
    c->page_size = QWN_KV_CACHE_PAGE_SIZE;
    c->alignment = 64u;
    c->valid_token_count = valid_token_count;
}

// ============================================================================
// qwanto_turboquant.h: the Q8 cache
// ============================================================================
QWN_REF_API int qwn_q8_cache_init(QwnQ8Cache *cache, int max_tokens, int n_heads, int head_dim) {
    if (!cache || max_tokens <= 0 || n_heads <= 0 || head_dim <= 0) return -1;
    memset(cache, 0, sizeof(*cache));
    cache->max_tokens = max_tokens;
    cache->n_heads = n_heads;
    cache->head_dim = head_dim;
    cache->n_channels = n_heads * head_dim;
    cache->token_stride = (size_t)cache->n_channels;
    cache->scale_stride = ((size_t)cache->n_channels + 63) / 64u;
    const size_t tok = (size_t)max_tokens * cache->token_stride;
    const size_t sc = (size_t)max_tokens * cache->scale_stride * sizeof(float);
    cudaError_t e = managed_zeroed(reinterpret_cast<void **>(&cache->packed_k), tok);
    if (e == cudaSuccess) e = managed_zeroed(reinterpret_cast<void **>(&cache->packed_v), tok);
    if (e == cudaSuccess) e = managed_zeroed(reinterpret_cast<void **>(&cache->scales_k), sc);
    if (e == cudaSuccess) e = managed_zeroed(reinterpret_cast<void **>(&cache->scales_v), sc);
    if (e != cudaSuccess) {
        fail("qwn_q8_cache_init", e);
        qwn_q8_cache_free(cache);
        return -1;
    }
    cache->total_bytes = tok * 2u + sc * 2u;
    qwn_kv_cache_contract_init(&cache->contract, QWN_KV_CACHE_Q8, 0);
    return 0;
}

QWN_REF_API void qwn_q8_cache_free(QwnQ8Cache *cache) {
    if (!cache) return;
    if (cache->packed_k) cudaFree(cache->packed_k);
    if (cache->packed_v) cudaFree(cache->packed_v);
    if (cache->scales_k) cudaFree(cache->scales_k);
    if (cache->scales_v) cudaFree(cache->scales_v);
    memset(cache, 0, sizeof(*cache));
}

QWN_REF_API void qwn_q8_cache_reset(QwnQ8Cache *cache) {
    if (!cache) return;
    cache->n_tokens = 0;
    cache->contract.valid_token_count = 0;
}

QWN_REF_API int qwn_q8_cache_append(QwnQ8Cache *cache, const float *key, const float *value, int n_channels) {
    if (!cache || !key || !value || n_channels != cache->n_channels || cache->n_tokens >= cache->max_tokens ||
        !cache->packed_k)
        return -1;
    const size_t n = (size_t)n_channels, t = (size_t)cache->n_tokens;
    Ctx *c = ctx("qwn_q8_cache_append", 2 * up256(n * 4));
    if (!c) return -1;
    Carve cv{c->scratch};
    float *dk = cv.take<float>(n), *dv = cv.take<float>(n);
    cudaError_t e = copy(dk, key, n * 4, c->s);
    if (e == cudaSuccess) e = copy(dv, value, n * 4, c->s);
    if (e == cudaSuccess) {
        q8_append_kernel<<<dim3((unsigned)cache->scale_stride, 2), 32, 0, c->s>>>(
            dk, dv, cache->packed_k + t * cache->token_stride, cache->packed_v + t * cache->token_stride,
            cache->scales_k + t * cache->scale_stride, cache->scales_v + t * cache->scale_stride, n_channels);
        e = cudaGetLastError();
        qkv::count_launch();
    }
    const cudaError_t e2 = cudaStreamSynchronize(c->s);
    if (e == cudaSuccess) e = e2;
    if (e != cudaSuccess) { fail("qwn_q8_cache_append", e); return -1; }
    cache->n_tokens++;
    cache->contract.valid_token_count = (uint32_t)cache->n_tokens;
    return 0;
}

static Q8Contig q8_src(const QwnQ8Cache *c, int off) {
    return Q8Contig{c->packed_k, c->packed_v, c->scales_k, c->scales_v, c->token_stride, c->scale_stride, off};
}

QWN_REF_API float qwn_q8_cache_dot_key_scalar(const QwnQ8Cache *cache, int token, int channel_offset,
                                              const float *query, int dim) {
    if (!cache || !query || token < 0 || token >= cache->n_tokens || channel_offset < 0 || dim <= 0 ||
        channel_offset + dim > cache->n_channels)
        return 0.0f;
    const Q8Contig src = q8_src(cache, channel_offset);
    return run_scalar("qwn_q8_cache_dot_key_scalar", (size_t)dim * 4,
                      [&](char *scr, float *res, cudaStream_t s) {
                          cudaError_t e = copy(scr, query, (size_t)dim * 4, s);
                          if (e != cudaSuccess) return e;
                          q8_dot_kernel<<<1, 32, 0, s>>>(src, token, reinterpret_cast<float *>(scr), dim, res);
                          return cudaGetLastError();
                      });
}

QWN_REF_API void qwn_q8_cache_accum_value_scalar(const QwnQ8Cache *cache, int token, int channel_offset, float score,
                                                 float *ctx_io, int dim) {
    if (!cache || !ctx_io || token < 0 || token >= cache->n_tokens || channel_offset < 0 || dim <= 0 ||
        channel_offset + dim > cache->n_channels)
        return;
    Ctx *c = ctx("qwn_q8_cache_accum_value_scalar", up256((size_t)dim * 4));
    if (!c) return;
    float *d = reinterpret_cast<float *>(c->scratch);
    cudaError_t e = copy(d, ctx_io, (size_t)dim * 4, c->s);
    if (e == cudaSuccess) {
        q8_accum_kernel<<<1, 128, 0, c->s>>>(q8_src(cache, channel_offset), token, score, d, dim);
        e = cudaGetLastError();
        qkv::count_launch();
    }
    if (e == cudaSuccess) e = copy(ctx_io, d, (size_t)dim * 4, c->s);
    const cudaError_t e2 = cudaStreamSynchronize(c->s);
    if (e == cudaSuccess) e = e2;
    if (e != cudaSuccess) fail("qwn_q8_cache_accum_value_scalar", e);
}

QWN_REF_API void qwn_q8_cache_attention_head(const float *query, const QwnQ8Cache *cache, int kv_head_idx, int pos,
                                             float scale, float *scores_scratch, float *ctx_out) {
    if (!query || !cache || !scores_scratch || !ctx_out || pos < 0 || pos >= cache->n_tokens || kv_head_idx < 0 ||
        kv_head_idx >= cache->n_heads)
        return;
    run_head("qwn_q8_cache_attention_head", q8_src(cache, kv_head_idx * cache->head_dim), nullptr, 0, pos + 1,
             cache->head_dim, query, scale, scores_scratch, ctx_out, true);
}

// ============================================================================
// qwanto_turboquant.h: the TurboQuant cache
// ============================================================================
QWN_REF_API int qwn_turboquant_init(TurboQuantCache *cache, int max_tokens, int n_heads, int head_dim) {
    if (!cache || max_tokens <= 0 || n_heads <= 0 || head_dim <= 0) return -1;
    memset(cache, 0, sizeof(*cache));
    cache->max_tokens = max_tokens;
    cache->n_heads = n_heads;
    cache->head_dim = head_dim;
    cache->n_channels = n_heads * head_dim;
    const size_t blocks = (size_t)(cache->n_channels + TURBOQUANT_GROUP_SIZE - 1) / TURBOQUANT_GROUP_SIZE;
    cache->token_stride_k = blocks * TURBOQUANT_BLOCK_BYTES;
    cache->token_stride_v = blocks * TURBOQUANT_BLOCK_BYTES;
    const size_t bk = (size_t)max_tokens * cache->token_stride_k, bv = (size_t)max_tokens * cache->token_stride_v;
    cudaError_t e = managed_zeroed(reinterpret_cast<void **>(&cache->packed_k), bk);
    if (e == cudaSuccess) e = managed_zeroed(reinterpret_cast<void **>(&cache->packed_v), bv);
    if (e != cudaSuccess) {
        fail("qwn_turboquant_init", e);
        qwn_turboquant_free(cache);
        return -1;
    }
    cache->total_bytes = bk + bv;
    return 0;
}

QWN_REF_API void qwn_turboquant_free(TurboQuantCache *cache) {
    if (!cache) return;
    if (cache->packed_k) cudaFree(cache->packed_k);
    if (cache->packed_v) cudaFree(cache->packed_v);
    memset(cache, 0, sizeof(*cache));
}

QWN_REF_API void qwn_turboquant_quantize_token(const float *src, uint8_t *dst_blocks, int n_channels) {
    if (!src || !dst_blocks || n_channels <= 0) return;
    const size_t nb = (size_t)(n_channels + TURBOQUANT_GROUP_SIZE - 1) / TURBOQUANT_GROUP_SIZE;
    const size_t out_bytes = nb * TURBOQUANT_BLOCK_BYTES;
    const bool direct = device_writable(dst_blocks);
    Ctx *c = ctx("qwn_turboquant_quantize_token", up256((size_t)n_channels * 4) + up256(out_bytes));
    if (!c) return;
    Carve cv{c->scratch};
    float *dsrc = cv.take<float>(n_channels);
    uint8_t *dout = direct ? dst_blocks : cv.take<uint8_t>(out_bytes);
    cudaError_t e = copy(dsrc, src, (size_t)n_channels * 4, c->s);
    if (e == cudaSuccess) {
        tq_quantize_kernel<<<(unsigned)nb, 32, 0, c->s>>>(dsrc, dout, n_channels);
        e = cudaGetLastError();
        qkv::count_launch();
    }
    if (e == cudaSuccess && !direct) e = copy(dst_blocks, dout, out_bytes, c->s);
    const cudaError_t e2 = cudaStreamSynchronize(c->s);
    if (e == cudaSuccess) e = e2;
    if (e != cudaSuccess) fail("qwn_turboquant_quantize_token", e);
}

QWN_REF_API float qwn_turboquant_dot_key_scalar(const float *query, const uint8_t *key_blocks, int dim) {
    if (!query || !key_blocks || dim <= 0) return 0.0f;
    const size_t kb = (size_t)((dim + TURBOQUANT_GROUP_SIZE - 1) / TURBOQUANT_GROUP_SIZE) * TURBOQUANT_BLOCK_BYTES;
    return run_scalar("qwn_turboquant_dot_key", up256((size_t)dim * 4) + kb, [&](char *scr, float *res, cudaStream_t s) {
        float *dq = reinterpret_cast<float *>(scr);
        uint8_t *dk = reinterpret_cast<uint8_t *>(scr + up256((size_t)dim * 4));
        cudaError_t e = copy(dq, query, (size_t)dim * 4, s);
        if (e == cudaSuccess) e = copy(dk, key_blocks, kb, s);
        if (e != cudaSuccess) return e;
        tq_dot_kernel<<<1, 32, 0, s>>>(dq, dk, dim, res);
        return cudaGetLastError();
    });
}

QWN_REF_API void qwn_turboquant_accum_value_scalar(float score, const uint8_t *value_blocks, float *ctx_io, int dim) {
    if (!value_blocks || !ctx_io || dim <= 0) return;
    const size_t vb = (size_t)((dim + TURBOQUANT_GROUP_SIZE - 1) / TURBOQUANT_GROUP_SIZE) * TURBOQUANT_BLOCK_BYTES;
    Ctx *c = ctx("qwn_turboquant_accum_value", up256((size_t)dim * 4) + vb);
    if (!c) return;
    float *d = reinterpret_cast<float *>(c->scratch);
    uint8_t *dv = reinterpret_cast<uint8_t *>(c->scratch + up256((size_t)dim * 4));
    cudaError_t e = copy(d, ctx_io, (size_t)dim * 4, c->s);
    if (e == cudaSuccess) e = copy(dv, value_blocks, vb, c->s);
    if (e == cudaSuccess) {
        tq_accum_kernel<<<1, 128, 0, c->s>>>(score, dv, d, dim);
        e = cudaGetLastError();
        qkv::count_launch();
    }
    if (e == cudaSuccess) e = copy(ctx_io, d, (size_t)dim * 4, c->s);
    const cudaError_t e2 = cudaStreamSynchronize(c->s);
    if (e == cudaSuccess) e = e2;
    if (e != cudaSuccess) fail("qwn_turboquant_accum_value", e);
}

QWN_REF_API float qwn_turboquant_dot_key_avx2(const float *q, const uint8_t *k, int dim) {
    return qwn_turboquant_dot_key_scalar(q, k, dim);
}
QWN_REF_API void qwn_turboquant_accum_value_avx2(float s, const uint8_t *v, float *c, int dim) {
    qwn_turboquant_accum_value_scalar(s, v, c, dim);
}
QWN_REF_API float qwn_turboquant_dot_key_vnni(const float *q, const uint8_t *k, int dim) {
    return qwn_turboquant_dot_key_scalar(q, k, dim);
}
QWN_REF_API void qwn_turboquant_accum_value_vnni(float s, const uint8_t *v, float *c, int dim) {
    qwn_turboquant_accum_value_scalar(s, v, c, dim);
}
QWN_REF_API float qwn_turboquant_dot_key_avx512(const float *q, const uint8_t *k, int dim) {
    return qwn_turboquant_dot_key_scalar(q, k, dim);
}
QWN_REF_API void qwn_turboquant_accum_value_avx512(float s, const uint8_t *v, float *c, int dim) {
    qwn_turboquant_accum_value_scalar(s, v, c, dim);
}

QWN_REF_API void qwn_turboquant_attention_head(const float *query, const TurboQuantCache *cache, int layer,
                                               int head_idx, int kv_head_idx, int pos, float scale,
                                               float *scores_scratch, float *ctx_out) {
    (void)layer;
    (void)head_idx;
    if (!query || !cache || !cache->packed_k || !scores_scratch || !ctx_out || pos < 0 || pos >= cache->max_tokens ||
        kv_head_idx < 0 || kv_head_idx >= cache->n_heads)
        return;
    const int hd = cache->head_dim;
    const size_t bph = (size_t)(hd + TURBOQUANT_GROUP_SIZE - 1) / TURBOQUANT_GROUP_SIZE;
    TQContig src{cache->packed_k, cache->packed_v, cache->token_stride_k, cache->token_stride_v,
                 (size_t)kv_head_idx * bph * TURBOQUANT_BLOCK_BYTES};
    run_head("qwn_turboquant_attention_head", src, nullptr, 0, pos + 1, hd, query, scale, scores_scratch, ctx_out,
             false);
}

QWN_REF_API void qwn_turboquant_matmul_avx512(const TurboQuantCache *cache, const float *query, float *output,
                                              int n_heads, int head_dim) {
    if (!cache || !cache->packed_k || !query || !output || n_heads <= 0 || head_dim <= 0) return;
    const size_t n = (size_t)n_heads * head_dim;
    Ctx *c = ctx("qwn_turboquant_matmul_avx512", 2 * up256(n * 4));
    if (!c) return;
    Carve cv{c->scratch};
    float *dq = cv.take<float>(n), *dout = cv.take<float>(n);
    cudaError_t e = copy(dq, query, n * 4, c->s);
    if (e == cudaSuccess) e = copy(dout, output, n * 4, c->s);  // only [h * head_dim] changes
    if (e == cudaSuccess) {
        tq_matmul_kernel<<<n_heads, 32, 0, c->s>>>(cache->packed_k, dq, dout, n_heads, head_dim);
        e = cudaGetLastError();
        qkv::count_launch();
    }
    if (e == cudaSuccess) e = copy(output, dout, n * 4, c->s);
    const cudaError_t e2 = cudaStreamSynchronize(c->s);
    if (e == cudaSuccess) e = e2;
    if (e != cudaSuccess) fail("qwn_turboquant_matmul_avx512", e);
}

// ============================================================================
// qwanto_attention.h
// ============================================================================
QWN_REF_API int qwanto_linear_attention_init(QwantoLinearAttentionState *state, int n_heads, int head_dim) {
    if (!state || n_heads <= 0 || head_dim <= 0) return -1;
    state->n_heads = n_heads;
    state->head_dim = head_dim;
    state->state = nullptr;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { fail("qwanto_linear_attention_init", e); return -1; }
    if (head_dim > 512) {
        qkv::set_error("qwanto_linear_attention_init: head_dim above 512");
        return -1;
    }
    float *p = nullptr;
    e = managed_zeroed(reinterpret_cast<void **>(&p), (size_t)n_heads * head_dim * head_dim * sizeof(float));
    if (e != cudaSuccess) { fail("qwanto_linear_attention_init", e); return -1; }
    QwnLinearAttentionState st{};
    st.n_heads = n_heads;
    st.head_dim = head_dim;
    st.state = p;
    st.device_id = dev;
    {
        std::lock_guard<std::mutex> g(g_la_mu);
        g_la[p] = st;
    }
    state->state = p;
    return 0;
}

static QwnLinearAttentionState *la_of(QwantoLinearAttentionState *state) {
    if (!state || !state->state) return nullptr;
    std::lock_guard<std::mutex> g(g_la_mu);
    auto it = g_la.find(state->state);
    if (it == g_la.end()) return nullptr;
    if (it->second.n_heads != state->n_heads || it->second.head_dim != state->head_dim) return nullptr;
    return &it->second;
}

QWN_REF_API void qwanto_linear_attention_reset(QwantoLinearAttentionState *state) {
    QwnLinearAttentionState *st = la_of(state);
    if (!st) return;
    if (qwn_linear_attention_reset(st, nullptr) != QWN_CUDA_STATUS_OK || cudaStreamSynchronize(0) != cudaSuccess)
        fprintf(stderr, "[qwn_cuda] qwanto_linear_attention_reset failed: %s\n", qkv::last_error().c_str());
}

QWN_REF_API void qwanto_linear_attention_destroy(QwantoLinearAttentionState *state) {
    if (!state || !state->state) return;
    QwnLinearAttentionState st{};
    bool found = false;
    {
        std::lock_guard<std::mutex> g(g_la_mu);
        auto it = g_la.find(state->state);
        if (it != g_la.end()) {
            st = it->second;
            g_la.erase(it);
            found = true;
        }
    }
    if (found) qwn_linear_attention_destroy(&st);  // frees the state and the staging
    state->state = nullptr;
}

QWN_REF_API void qwanto_linear_attention_prefill(QwantoLinearAttentionState *state, const float *Q, const float *K,
                                                 const float *V, float decay, int seq_len, float *O) {
    QwnLinearAttentionState *st = la_of(state);
    if (!st || seq_len <= 0) return;
    if (qwn_linear_attention_prefill_host(st, Q, K, V, decay, seq_len, O) != QWN_CUDA_STATUS_OK)
        fprintf(stderr, "[qwn_cuda] qwanto_linear_attention_prefill failed: %s\n", qkv::last_error().c_str());
}

QWN_REF_API void qwanto_linear_attention_decode(QwantoLinearAttentionState *state, const float *Q, const float *K,
                                                const float *V, float decay, float *O) {
    qwanto_linear_attention_prefill(state, Q, K, V, decay, 1, O);
}

// ============================================================================
// qwanto_pagedeviction.h (host bookkeeping on the caller's struct)
// ============================================================================
QWN_REF_API int qwn_paged_eviction_init(QwnPagedEvictionPool *pool, uint32_t max_capacity,
                                        uint32_t physical_pool_size, float eviction_threshold) {
    if (!pool || max_capacity == 0 || physical_pool_size == 0) return -1;
    if (max_capacity > QWN_VTOKEN_MAX_CAPACITY) max_capacity = QWN_VTOKEN_MAX_CAPACITY;
    memset(pool, 0, sizeof(*pool));
    pool->max_capacity = max_capacity;
    pool->physical_pool_size = physical_pool_size;
    pool->eviction_threshold = eviction_threshold > 0.0f ? eviction_threshold : 0.05f;
    return 0;
}

QWN_REF_API int qwn_paged_eviction_insert(QwnPagedEvictionPool *pool, uint32_t token_id, float initial_importance,
                                          uint32_t *assigned_physical_slot) {
    if (!pool || !assigned_physical_slot) return -1;
    if (pool->active_count >= pool->physical_pool_size)
        qwn_paged_eviction_prune(pool, (uint32_t)((float)pool->physical_pool_size * 0.9f));
    const uint32_t slot = pool->active_count;
    if (slot >= pool->max_capacity) return -2;
    QwnVToken &t = pool->virtual_tokens[slot];
    t.token_id = token_id;
    t.importance_score = initial_importance > 0.0f ? initial_importance : 1.0f;
    t.physical_slot = slot;
    t.is_sink = token_id < QWN_VTOKEN_SINK_TOKENS;
    t.is_active = true;
    *assigned_physical_slot = slot;
    pool->active_count++;
    return 0;
}

QWN_REF_API void qwn_paged_eviction_update_scores(QwnPagedEvictionPool *pool, const float *attention_scores,
                                                  uint32_t sequence_length) {
    if (!pool || !attention_scores) return;
    const uint32_t n = std::min(sequence_length, pool->active_count);
    for (uint32_t i = 0; i < n; i++) {
        QwnVToken &t = pool->virtual_tokens[i];
        if (!t.is_sink)  // the reference's 0.8*old + 0.2*new, compiled as one fused multiply-add
            t.importance_score = fmaf(0.8f, t.importance_score, 0.2f * attention_scores[i]);
    }
}

QWN_REF_API uint32_t qwn_paged_eviction_prune(QwnPagedEvictionPool *pool, uint32_t target_retained_tokens) {
    if (!pool || pool->active_count <= target_retained_tokens) return 0;
    const uint32_t to_evict = pool->active_count - target_retained_tokens;
    uint32_t evicted = 0;
    // the reference evicts active non-sink slots in index order from slot 4
    // (its threshold test is or-ed with evicted < to_evict, which the loop
    // condition already guarantees)
    for (uint32_t i = QWN_VTOKEN_SINK_TOKENS; i < pool->active_count && evicted < to_evict; i++) {
        QwnVToken &t = pool->virtual_tokens[i];
        if (t.is_active && !t.is_sink) {
            t.is_active = false;
            evicted++;
        }
    }
    pool->total_evictions += evicted;
    return evicted;
}

QWN_REF_API float qwn_paged_eviction_memory_waste_pct(const QwnPagedEvictionPool *pool) {
    if (!pool || pool->physical_pool_size == 0) return 0.0f;
    return pool->active_count >= pool->physical_pool_size ? 4.8f : 5.2f;  // the reference's constants
}

}  // extern "C"
