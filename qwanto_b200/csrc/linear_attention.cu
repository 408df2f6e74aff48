// Linear-attention decode and prefill on a device-resident fp32 state.
//
// The reference keeps one [n_heads][d][d] fp32 state on the host and, per
// token, updates every row i (key dim) and column j (value dim) as
//     S[i][j] = fma(decay, S[i][j], RN(k_i * v_j))
// then forms O[j] = q_0*S[0][j] + q_1*S[1][j] + ... as a chain of fmas that
// starts from 0 and takes the rows in ascending order
// (c/qwanto_attention.c:57-140, the AVX2/AVX-512 paths; prefill runs decode
// once per token, :144-156).  Both kernels keep exactly that order and those
// roundings (__fmul_rn / __fmaf_rn, nothing left for the compiler to
// contract), so states and outputs are bit-identical to the reference.
//
// Work unit: (head, 32-column block); lane = column, so a warp's access to
// one state row is one 128-byte line and the state streams through HBM fully
// coalesced.
//
//   decode : HBM-bound -- the state is read and written once per token
//            (8 d^2 bytes per head).  Persistent CTAs; eight producer warps
//            stream units through registers while a ninth warp runs the
//            serial output chain of the previous unit from shared memory.
//   prefill: the state slice stays in registers for the whole sequence (read
//            and written once); eight warps form a systolic pipeline over the
//            rows, each handing a token's partial output sum to the next
//            warp, so several tokens are in flight and the chain order is
//            unchanged.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <utility>

#include "kv_internal.cuh"

namespace qkv {
namespace {

constexpr int kLaCols = 32;   // columns per work unit (one per lane)
constexpr int kLaWarps = 8;   // row stripes (decode producers, prefill stages)
constexpr int kLaThreads = kLaCols * kLaWarps;
constexpr int kLaMaxDim = 512;

struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceScope() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// ---------------------------------------------------------------------------
// Decode.  A persistent CTA walks units (head, 32-column block) with a stride
// of the grid.  Warps 0..7 produce: for their rows i = w, w+8, ... they load
// the state (kLaDecodeUnroll rows per thread per batch of loads), k_i and q_i
// (warp-uniform), write the updated state back to HBM and into the unit's
// shared slice, and publish q into the slice's q vector.  Warp 8 consumes: it
// runs the output chain over the slice.  Two slices alternate, handed over
// with named barriers (FULL: producers arrive, consumer syncs; EMPTY: the
// reverse), so the producers stream the next unit while the consumer finishes
// the last one.
// ---------------------------------------------------------------------------
constexpr int kLaDecodeUnroll = 8;
constexpr int kLaDecodeThreads = kLaThreads + 32;
constexpr int kBarFull = 1, kBarEmpty = 3;  // ids kBarFull + b, kBarEmpty + b for b in {0, 1}

template <int ID>
__device__ __forceinline__ void named_sync() {
    asm volatile("bar.sync %0, %1;" ::"n"(ID), "n"(kLaDecodeThreads) : "memory");
}
template <int ID>
__device__ __forceinline__ void named_arrive() {
    asm volatile("bar.arrive %0, %1;" ::"n"(ID), "n"(kLaDecodeThreads) : "memory");
}
__device__ __forceinline__ void sync_empty(int b) {
    if (b) named_sync<kBarEmpty + 1>();
    else named_sync<kBarEmpty>();
}

// FAST = head_dim a multiple of 8 x kLaDecodeUnroll: every row and column of a batch of loads exists.
template <bool FAST>
__global__ void __launch_bounds__(kLaDecodeThreads, 4) la_decode_kernel(float *__restrict__ state, int d,
                                                                        int col_blocks, int units,
                                                                        const float *__restrict__ q,
                                                                        const float *__restrict__ k,
                                                                        const float *__restrict__ v, float decay,
                                                                        float *__restrict__ o) {
    extern __shared__ __align__(16) float sm[];
    // buffer b: slice [d][32] then q [d]
    const int buf_floats = d * kLaCols + d;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int n = 0;
    if (w < kLaWarps) {
        for (int unit = blockIdx.x; unit < units; unit += gridDim.x, n++) {
            const int b = n & 1;
            float *slice = sm + b * buf_floats, *sq = slice + d * kLaCols;
            const int h = unit / col_blocks, cb = unit - h * col_blocks;
            const int j = cb * kLaCols + lane;
            const bool col = j < d;
            const size_t hd = (size_t)h * d;
            float *S = state + hd * d;
            const float *kh = k + hd;
            const float vj = col ? v[hd + j] : 0.f;
            bool free = n < 2;  // slice b was released by the consumer (unit n - 2)
            for (int i0 = w; i0 < d; i0 += kLaWarps * kLaDecodeUnroll) {
                float s[kLaDecodeUnroll], kk[kLaDecodeUnroll];
                float *Si = S + (i0 * d + j);  // row i0, column j; rows u apart are 8d floats apart
                const int rs = kLaWarps * d;
#pragma unroll
                for (int u = 0; u < kLaDecodeUnroll; u++) {
                    const int i = i0 + u * kLaWarps;
                    if (FAST) {
                        s[u] = Si[u * rs];
                        kk[u] = kh[i];
                    } else {
                        s[u] = (col && i < d) ? Si[u * rs] : 0.f;
                        kk[u] = i < d ? kh[i] : 0.f;
                    }
                }
                const int iq = i0 + lane * kLaWarps;
                const bool qlane = lane < kLaDecodeUnroll && (FAST || iq < d);
                const float qv = qlane ? q[hd + iq] : 0.f;
                if (!free) {  // wait only once the loads are in flight
                    sync_empty(b);
                    free = true;
                }
                if (qlane) sq[iq] = qv;
#pragma unroll
                for (int u = 0; u < kLaDecodeUnroll; u++) {
                    const int i = i0 + u * kLaWarps;
                    if (FAST || i < d) {
                        const float ns = __fmaf_rn(decay, s[u], __fmul_rn(kk[u], vj));
                        if (FAST || col) Si[u * rs] = ns;
                        slice[i * kLaCols + lane] = ns;
                    }
                }
            }
            if (!free) sync_empty(b);  // a warp without rows (head_dim < 8) still takes its turn
            if (b) named_arrive<kBarFull + 1>();
            else named_arrive<kBarFull>();
        }
        // take the consumer's last two EMPTY arrivals so both barriers end balanced
        for (int m = max(n - 2, 0); m < n; m++) sync_empty(m & 1);
    } else {
        for (int unit = blockIdx.x; unit < units; unit += gridDim.x, n++) {
            const int b = n & 1;
            const float *slice = sm + b * buf_floats, *sq = slice + d * kLaCols;
            const int h = unit / col_blocks, cb = unit - h * col_blocks;
            const int j = cb * kLaCols + lane;
            if (b) named_sync<kBarFull + 1>();
            else named_sync<kBarFull>();
            float acc = 0.f;
            if (FAST) {
#pragma unroll 4
                for (int i = 0; i < d; i += 4) {
                    const float4 qq = *reinterpret_cast<const float4 *>(sq + i);
                    acc = __fmaf_rn(qq.x, slice[(i + 0) * kLaCols + lane], acc);
                    acc = __fmaf_rn(qq.y, slice[(i + 1) * kLaCols + lane], acc);
                    acc = __fmaf_rn(qq.z, slice[(i + 2) * kLaCols + lane], acc);
                    acc = __fmaf_rn(qq.w, slice[(i + 3) * kLaCols + lane], acc);
                }
            } else {
#pragma unroll 8
                for (int i = 0; i < d; i++) acc = __fmaf_rn(sq[i], slice[i * kLaCols + lane], acc);
            }
            if (j < d) o[(size_t)h * d + j] = acc;
            if (b) named_arrive<kBarEmpty + 1>();
            else named_arrive<kBarEmpty>();
        }
    }
}

// ---------------------------------------------------------------------------
// Prefill: a systolic pipeline over the CTA's 8 warps.  Warp b holds rows
// [b*rpw, b*rpw + rpw) of the 32-column slice in registers for the whole
// sequence (rpw = ceil(d / 8) <= R).  Tokens go in groups of P; at step s warp
// b works on group g = s - b: for each token of the group it updates its rows
// with k_t and v_t and continues token t's output chain over its rows from the
// partial sum warp b-1 produced for the same token at step s-1 (0 for warp 0),
// then hands the P sums on (the last warp stores them).  The chain still
// visits rows 0..d-1 in ascending order, as in the reference, while 8 groups
// are in flight; the P chains of a group are independent, which hides the fma
// latency; no state slice passes through shared memory.  One barrier ends
// each step.
//
// k, q and the 32-column v slice arrive in chunks of 8 groups (8P tokens) by
// cp.async into three rotating buffers: chunk m is fetched at step
// 8(m-2) + 7 (when chunk m-3 has left the pipeline) and waited for at step 8m,
// so its global latency overlaps ~9 steps of arithmetic.
// ---------------------------------------------------------------------------
constexpr int kLaGroupsPerChunk = kLaWarps;  // >= the stage count (see the wait accounting above)
constexpr int kLaBuffers = 3;

// tokens per group: 4 while three chunks fit shared memory comfortably (head_dim <= 128)
template <int R>
__host__ __device__ constexpr int group_tokens() { return R <= 16 ? 4 : (R <= 32 ? 2 : 1); }

__device__ __forceinline__ void cp_async4(float *dst, const float *src) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(a), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(float *dst, const float *src) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(a), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// One group of P tokens for one warp of the prefill pipeline: update the
// warp's rows with each token's k and v, then continue each token's output
// chain over them, for each of the thread's CPT columns (lane, lane + 32, ...).
// FULL = all P tokens exist (no guards, so the independent chains interleave).
template <int R, bool EXACT, int P, int CPT, bool FULL>
__device__ __forceinline__ void la_group(float (&s)[CPT][R], float (&acc)[CPT][P], const float *gb, int np,
                                         int tok_floats, int d, int r0, int rpw, int lane, float decay) {
#pragma unroll
    for (int p = 0; p < P; p++) {
        if (FULL || p < np) {
            const float *tb = gb + p * tok_floats;
            float vj[CPT];
#pragma unroll
            for (int c = 0; c < CPT; c++) vj[c] = tb[2 * d + c * kLaCols + lane];
            if (EXACT) {
#pragma unroll
                for (int u = 0; u < R; u += 4) {
                    const float4 kk = *reinterpret_cast<const float4 *>(tb + r0 + u);
                    const float4 qq = *reinterpret_cast<const float4 *>(tb + d + r0 + u);
#pragma unroll
                    for (int c = 0; c < CPT; c++) {
                        s[c][u + 0] = __fmaf_rn(decay, s[c][u + 0], __fmul_rn(kk.x, vj[c]));
                        s[c][u + 1] = __fmaf_rn(decay, s[c][u + 1], __fmul_rn(kk.y, vj[c]));
                        s[c][u + 2] = __fmaf_rn(decay, s[c][u + 2], __fmul_rn(kk.z, vj[c]));
                        s[c][u + 3] = __fmaf_rn(decay, s[c][u + 3], __fmul_rn(kk.w, vj[c]));
                        acc[c][p] = __fmaf_rn(qq.x, s[c][u + 0], acc[c][p]);
                        acc[c][p] = __fmaf_rn(qq.y, s[c][u + 1], acc[c][p]);
                        acc[c][p] = __fmaf_rn(qq.z, s[c][u + 2], acc[c][p]);
                        acc[c][p] = __fmaf_rn(qq.w, s[c][u + 3], acc[c][p]);
                    }
                }
            } else {
#pragma unroll
                for (int u = 0; u < R; u++) {
                    const int i = r0 + u;
                    if (u < rpw && i < d) {
#pragma unroll
                        for (int c = 0; c < CPT; c++) {
                            s[c][u] = __fmaf_rn(decay, s[c][u], __fmul_rn(tb[i], vj[c]));
                            acc[c][p] = __fmaf_rn(tb[d + i], s[c][u], acc[c][p]);
                        }
                    }
                }
            }
        }
    }
}

// EXACT = (head_dim == 8R with R a multiple of 4) and q/k/v 16-byte aligned:
// whole rows per warp, float4 shared reads and 16-byte cp.async; otherwise
// every row is bounds-checked and staged with 4-byte copies.  CPT = columns
// per thread (a CTA covers 32 x CPT columns): 2 halves the warp-uniform k/q
// shared reads per fma, for launches with enough CTAs to fill the GPU.
template <int R, bool EXACT, int CPT>
__global__ void __launch_bounds__(kLaThreads, (R * CPT <= 16 ? 2 : 1)) la_prefill_kernel(
    float *__restrict__ state, int n_heads, int d_arg, int col_blocks, int seq_len, const float *__restrict__ q,
    const float *__restrict__ k, const float *__restrict__ v, float decay, float *__restrict__ o) {
    constexpr int P = group_tokens<R>();
    constexpr int C = kLaGroupsPerChunk * P;  // tokens per chunk
    constexpr int W = kLaCols * CPT;          // columns per CTA
    const int d = EXACT ? kLaWarps * R : d_arg;
    extern __shared__ __align__(16) float sm[];
    // buffer x: [C tokens][k d | q d | v W]; then the hand-off sums [2][8][P][W]
    const int tok_floats = 2 * d + W, buf_floats = C * tok_floats;
    float *hand = sm + kLaBuffers * buf_floats;
    const int h = blockIdx.x / col_blocks, cb = blockIdx.x - h * col_blocks;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int j0 = cb * W;
    const int rpw = EXACT ? R : (d + kLaWarps - 1) / kLaWarps;
    const int r0 = w * rpw;
    const size_t hd = (size_t)h * d, row_stride = (size_t)n_heads * d;  // token stride of q/k/v/o
    const int n_chunks = (seq_len + C - 1) / C, n_groups = (seq_len + P - 1) / P;

    auto fetch = [&](int m) {  // every thread issues its share of chunk m, then commits (possibly empty)
        if (m < n_chunks) {
            float *buf = sm + (m % kLaBuffers) * buf_floats;
            const int t0 = m * C, n = min(C, seq_len - t0);
            if (EXACT) {
                constexpr int KU = kLaWarps * R / 4;  // 16-byte units of a k (or q) row
                constexpr int U = 2 * KU + W / 4;     // per token: k, q, v slice
                for (int x = threadIdx.x; x < n * U; x += kLaThreads) {
                    const int c = x / U, r = x - c * U;
                    const size_t base = (size_t)(t0 + c) * row_stride + hd;
                    const float *src = r < KU ? k + base + 4 * r
                                     : r < 2 * KU ? q + base + 4 * (r - KU)
                                                  : v + base + j0 + 4 * (r - 2 * KU);
                    cp_async16(buf + c * tok_floats + 4 * r, src);
                }
            } else {
                for (int c = 0; c < n; c++) {
                    const size_t base = (size_t)(t0 + c) * row_stride + hd;
                    float *dst = buf + c * tok_floats;
                    for (int x = threadIdx.x; x < tok_floats; x += kLaThreads) {
                        if (x < d) cp_async4(dst + x, k + base + x);
                        else if (x < 2 * d) cp_async4(dst + x, q + base + (x - d));
                        else if (j0 + x - 2 * d < d) cp_async4(dst + x, v + base + j0 + (x - 2 * d));
                    }
                }
            }
        }
        cp_async_commit();
    };

    float *S = state + hd * d;
    float s[CPT][R];  // this warp's rows of the thread's columns, for the whole sequence
#pragma unroll
    for (int c = 0; c < CPT; c++) {
        const int j = j0 + c * kLaCols + lane;
#pragma unroll
        for (int u = 0; u < R; u++) {
            const int i = r0 + u;
            s[c][u] = (j < d && u < rpw && i < d) ? S[(size_t)i * d + j] : 0.f;
        }
    }
    fetch(0);
    fetch(1);
    const int steps = n_groups + kLaWarps - 1;
    for (int st = 0; st < steps; st++) {
        if (st % kLaGroupsPerChunk == 0) {  // chunk st / 8 is needed from this step on
            cp_async_wait1();
            __syncthreads();
        }
        if (st >= kLaWarps - 1 && (st - (kLaWarps - 1)) % kLaGroupsPerChunk == 0)
            fetch((st - (kLaWarps - 1)) / kLaGroupsPerChunk + 2);
        const int g = st - w;
        if (g >= 0 && g < n_groups) {
            const int t0 = g * P, np = min(P, seq_len - t0);
            const float *gb = sm + ((t0 / C) % kLaBuffers) * buf_floats + (t0 % C) * tok_floats;
            float acc[CPT][P];
            const float *hin = hand + (((st - 1) & 1) * kLaWarps + (w - 1)) * P * W + lane;
#pragma unroll
            for (int c = 0; c < CPT; c++)
#pragma unroll
                for (int p = 0; p < P; p++) acc[c][p] = w == 0 ? 0.f : hin[p * W + c * kLaCols];
            if (np == P) la_group<R, EXACT, P, CPT, true>(s, acc, gb, np, tok_floats, d, r0, rpw, lane, decay);
            else la_group<R, EXACT, P, CPT, false>(s, acc, gb, np, tok_floats, d, r0, rpw, lane, decay);
            if (w == kLaWarps - 1) {
#pragma unroll
                for (int c = 0; c < CPT; c++) {
                    const int j = j0 + c * kLaCols + lane;
#pragma unroll
                    for (int p = 0; p < P; p++)
                        if (p < np && j < d) o[(size_t)(t0 + p) * row_stride + hd + j] = acc[c][p];
                }
            } else {
                float *hout = hand + ((st & 1) * kLaWarps + w) * P * W + lane;
#pragma unroll
                for (int c = 0; c < CPT; c++)
#pragma unroll
                    for (int p = 0; p < P; p++) hout[p * W + c * kLaCols] = acc[c][p];
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int c = 0; c < CPT; c++) {
        const int j = j0 + c * kLaCols + lane;
#pragma unroll
        for (int u = 0; u < R; u++) {
            const int i = r0 + u;
            if (j < d && u < rpw && i < d) S[(size_t)i * d + j] = s[c][u];
        }
    }
}

bool state_ok(const QwnLinearAttentionState *st) {
    return st && st->state && st->n_heads > 0 && st->head_dim > 0 && st->head_dim <= kLaMaxDim;
}

// dynamic shared memory above 48 KB is opted into once per kernel and device
template <typename K>
cudaError_t allow_smem(K kernel, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    static std::mutex mu;
    static std::map<std::pair<const void *, int>, size_t> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    size_t &have = done[{(const void *)kernel, dev}];
    if (have >= bytes) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) have = bytes;
    return e;
}

// SM count of the current device, and resident CTAs per SM of a kernel at a
// shared-memory size, looked up once (launches are host-latency sensitive)
int current_sms() {
    static std::mutex mu;
    static std::map<int, int> sms;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    auto it = sms.find(dev);
    if (it != sms.end()) return it->second;
    int n = 148;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return sms[dev] = n;
}

template <typename K>
int resident_ctas(K kernel, int threads, size_t smem) {
    static std::mutex mu;
    static std::map<std::pair<const void *, size_t>, int> cache;
    std::lock_guard<std::mutex> g(mu);
    auto key = std::make_pair((const void *)kernel, smem);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    int per_sm = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess) per_sm = 1;
    return cache[key] = std::max(per_sm, 1);
}

template <int R, bool EXACT, int CPT = 1>
cudaError_t launch_prefill_r(const QwnLinearAttentionState *st, int seq_len, const float *q, const float *k,
                             const float *v, float decay, float *o, cudaStream_t stream) {
    const int d = st->head_dim, col_blocks = (d + kLaCols * CPT - 1) / (kLaCols * CPT);
    constexpr int P = group_tokens<R>();
    const size_t smem = ((size_t)kLaBuffers * kLaGroupsPerChunk * P * (2 * d + kLaCols * CPT) +
                         2 * kLaWarps * P * kLaCols * CPT) * sizeof(float);
    cudaError_t e = allow_smem(la_prefill_kernel<R, EXACT, CPT>, smem);
    if (e != cudaSuccess) return e;
    la_prefill_kernel<R, EXACT, CPT><<<(unsigned)(st->n_heads * col_blocks), kLaThreads, smem, stream>>>(
        st->state, st->n_heads, d, col_blocks, seq_len, q, k, v, decay, o);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_decode(const QwnLinearAttentionState *st, const float *q, const float *k, const float *v,
                          float decay, float *o, cudaStream_t stream) {
    const int d = st->head_dim, col_blocks = (d + kLaCols - 1) / kLaCols;
    const int units = st->n_heads * col_blocks;
    const size_t smem = 2 * ((size_t)d * kLaCols + d) * sizeof(float);
    const bool fast = d % (kLaWarps * kLaDecodeUnroll) == 0;
    auto kernel = fast ? la_decode_kernel<true> : la_decode_kernel<false>;
    cudaError_t e = allow_smem(kernel, smem);
    if (e != cudaSuccess) return e;
    const int grid = std::min(units, current_sms() * resident_ctas(kernel, kLaDecodeThreads, smem));
    kernel<<<(unsigned)grid, kLaDecodeThreads, smem, stream>>>(st->state, d, col_blocks, units, q, k, v, decay, o);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_step(const QwnLinearAttentionState *st, int seq_len, const float *q, const float *k,
                        const float *v, float decay, float *o, cudaStream_t stream) {
    if (seq_len == 1) return launch_decode(st, q, k, v, decay, o, stream);
    const int d = st->head_dim, r = (d + kLaWarps - 1) / kLaWarps;
    const bool aligned = ((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) % 16 == 0;
    if (aligned && d % (4 * kLaWarps) == 0) {  // whole rows per warp, 16-byte staging
        // two columns per thread once the one-column grid would be over 4 waves of SMs
        if ((long)st->n_heads * (d / kLaCols) >= 4L * current_sms() && d % (2 * kLaCols) == 0) {
            switch (d / kLaWarps) {
                case 8: return launch_prefill_r<8, true, 2>(st, seq_len, q, k, v, decay, o, stream);
                case 16: return launch_prefill_r<16, true, 2>(st, seq_len, q, k, v, decay, o, stream);
                case 32: return launch_prefill_r<32, true, 2>(st, seq_len, q, k, v, decay, o, stream);
                default: break;
            }
        }
        switch (d / kLaWarps) {
            case 4: return launch_prefill_r<4, true>(st, seq_len, q, k, v, decay, o, stream);
            case 8: return launch_prefill_r<8, true>(st, seq_len, q, k, v, decay, o, stream);
            case 16: return launch_prefill_r<16, true>(st, seq_len, q, k, v, decay, o, stream);
            case 32: return launch_prefill_r<32, true>(st, seq_len, q, k, v, decay, o, stream);
            default: break;
        }
    }
    if (r <= 2) return launch_prefill_r<2, false>(st, seq_len, q, k, v, decay, o, stream);
    if (r <= 4) return launch_prefill_r<4, false>(st, seq_len, q, k, v, decay, o, stream);
    if (r <= 8) return launch_prefill_r<8, false>(st, seq_len, q, k, v, decay, o, stream);
    if (r <= 16) return launch_prefill_r<16, false>(st, seq_len, q, k, v, decay, o, stream);
    if (r <= 32) return launch_prefill_r<32, false>(st, seq_len, q, k, v, decay, o, stream);
    return launch_prefill_r<64, false>(st, seq_len, q, k, v, decay, o, stream);
}

int finish(const char *what, cudaError_t e) {
    if (e == cudaSuccess) return QWN_CUDA_STATUS_OK;
    set_cuda_error(what, e);
    return QWN_CUDA_STATUS_RUNTIME_ERROR;
}

// Host-buffer prefill of a long sequence: chunks of kLaHostChunkBytes per
// input array go through two staging slots so that the copy of chunk c+1 in,
// the prefill of chunk c and the copy of chunk c-1 out overlap (three
// non-blocking streams per device, created once).  Prefilling the chunks one
// after another is the same computation as one prefill, so results do not
// change.
constexpr size_t kLaHostChunkBytes = 4u << 20;

struct HostPipe {
    std::mutex mu;  // one pipelined call per device at a time (the streams and events are shared)
    bool ok = false;
    cudaStream_t in = nullptr, comp = nullptr, out = nullptr;
    cudaEvent_t start = nullptr, in_done[2] = {}, comp_done[2] = {}, out_done[2] = {};
};

HostPipe *host_pipe(int dev) {
    static std::mutex mu;
    static std::map<int, HostPipe> pipes;
    std::lock_guard<std::mutex> g(mu);
    HostPipe &p = pipes[dev];
    if (!p.ok) {
        bool good = cudaStreamCreateWithFlags(&p.in, cudaStreamNonBlocking) == cudaSuccess &&
                    cudaStreamCreateWithFlags(&p.comp, cudaStreamNonBlocking) == cudaSuccess &&
                    cudaStreamCreateWithFlags(&p.out, cudaStreamNonBlocking) == cudaSuccess &&
                    cudaEventCreateWithFlags(&p.start, cudaEventDisableTiming) == cudaSuccess;
        for (int s = 0; s < 2 && good; s++)
            good = cudaEventCreateWithFlags(&p.in_done[s], cudaEventDisableTiming) == cudaSuccess &&
                   cudaEventCreateWithFlags(&p.comp_done[s], cudaEventDisableTiming) == cudaSuccess &&
                   cudaEventCreateWithFlags(&p.out_done[s], cudaEventDisableTiming) == cudaSuccess;
        p.ok = good;
    }
    return p.ok ? &p : nullptr;
}

int prefill_host_pipelined(QwnLinearAttentionState *st, const float *q, const float *k, const float *v, float decay,
                           int seq_len, float *o, int chunk) {
    const char *what = "qwn_linear_attention_prefill_host";
    int dev = 0;
    cudaGetDevice(&dev);
    HostPipe *p = host_pipe(dev);
    if (!p) return finish(what, cudaErrorUnknown);
    std::lock_guard<std::mutex> g(p->mu);
    const size_t tok_floats = (size_t)st->n_heads * st->head_dim, slot = 4 * (size_t)chunk * tok_floats;
    if (st->staging_bytes < 2 * slot * sizeof(float)) {
        if (st->staging) cudaFree(st->staging);
        st->staging = nullptr;
        st->staging_bytes = 0;
        cudaError_t e = cudaMalloc(&st->staging, 2 * slot * sizeof(float));
        if (e != cudaSuccess) {
            set_cuda_error("qwn_linear_attention_prefill_host: cudaMalloc", e);
            return QWN_CUDA_STATUS_OUT_OF_MEMORY;
        }
        st->staging_bytes = 2 * slot * sizeof(float);
    }
    // the state may have been written by work the caller queued on the legacy default stream
    cudaError_t e = cudaEventRecord(p->start, 0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(p->comp, p->start, 0);
    const int n_chunks = (seq_len + chunk - 1) / chunk;
    for (int c = 0; c < n_chunks && e == cudaSuccess; c++) {
        const int s = c & 1, n = std::min(chunk, seq_len - c * chunk);
        const size_t off = (size_t)c * chunk * tok_floats, bytes = (size_t)n * tok_floats * sizeof(float);
        float *dq = (float *)st->staging + s * slot, *dk = dq + (size_t)chunk * tok_floats,
              *dv = dk + (size_t)chunk * tok_floats, *dout = dv + (size_t)chunk * tok_floats;
        if (c >= 2) e = cudaStreamWaitEvent(p->in, p->out_done[s], 0);  // slot s is free again
        if (e == cudaSuccess) e = cudaMemcpyAsync(dq, q + off, bytes, cudaMemcpyDefault, p->in);
        if (e == cudaSuccess) e = cudaMemcpyAsync(dk, k + off, bytes, cudaMemcpyDefault, p->in);
        if (e == cudaSuccess) e = cudaMemcpyAsync(dv, v + off, bytes, cudaMemcpyDefault, p->in);
        if (e == cudaSuccess) e = cudaEventRecord(p->in_done[s], p->in);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(p->comp, p->in_done[s], 0);
        if (e == cudaSuccess) e = launch_step(st, n, dq, dk, dv, decay, dout, p->comp);
        if (e == cudaSuccess) e = cudaEventRecord(p->comp_done[s], p->comp);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(p->out, p->comp_done[s], 0);
        if (e == cudaSuccess) e = cudaMemcpyAsync(o + off, dout, bytes, cudaMemcpyDefault, p->out);
        if (e == cudaSuccess) e = cudaEventRecord(p->out_done[s], p->out);
    }
    // drain all three streams whatever happened, so no copy outlives the call
    cudaError_t e1 = cudaStreamSynchronize(p->in), e2 = cudaStreamSynchronize(p->comp),
                e3 = cudaStreamSynchronize(p->out);
    if (e == cudaSuccess) e = e1 != cudaSuccess ? e1 : (e2 != cudaSuccess ? e2 : e3);
    return finish(what, e);
}

}  // namespace
}  // namespace qkv

using namespace qkv;

QWN_CUDA_ABI_API int qwn_linear_attention_init(QwnLinearAttentionState *st, int32_t device_id, int32_t n_heads,
                                               int32_t head_dim) {
    if (!st || n_heads <= 0 || head_dim <= 0) {
        set_error("qwn_linear_attention_init: invalid argument");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    memset(st, 0, sizeof(*st));
    if (head_dim > kLaMaxDim) {
        set_error("qwn_linear_attention_init: head_dim above 512");
        return QWN_CUDA_STATUS_UNSUPPORTED;
    }
    DeviceScope scope(device_id);
    const size_t bytes = (size_t)n_heads * head_dim * head_dim * sizeof(float);
    float *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        set_cuda_error("qwn_linear_attention_init: cudaMalloc", e);
        return QWN_CUDA_STATUS_OUT_OF_MEMORY;
    }
    e = cudaMemset(p, 0, bytes);
    if (e != cudaSuccess) {
        cudaFree(p);
        return finish("qwn_linear_attention_init: cudaMemset", e);
    }
    st->n_heads = n_heads;
    st->head_dim = head_dim;
    st->state = p;
    st->device_id = device_id;
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_linear_attention_reset(QwnLinearAttentionState *st, void *stream) {
    if (!state_ok(st)) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    DeviceScope scope(st->device_id);
    const size_t bytes = (size_t)st->n_heads * st->head_dim * st->head_dim * sizeof(float);
    return finish("qwn_linear_attention_reset", cudaMemsetAsync(st->state, 0, bytes, (cudaStream_t)stream));
}

QWN_CUDA_ABI_API int qwn_linear_attention_destroy(QwnLinearAttentionState *st) {
    if (!st) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    DeviceScope scope(st->device_id);
    if (st->state) cudaFree(st->state);
    if (st->staging) cudaFree(st->staging);
    st->state = nullptr;
    st->staging = nullptr;
    st->staging_bytes = 0;
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_linear_attention_prefill(QwnLinearAttentionState *st, const float *q_dev,
                                                  const float *k_dev, const float *v_dev, float decay,
                                                  int32_t seq_len, float *o_dev, void *stream) {
    if (!state_ok(st) || seq_len < 0 || (seq_len > 0 && (!q_dev || !k_dev || !v_dev || !o_dev))) {
        set_error("qwn_linear_attention_prefill: invalid argument");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    if (seq_len == 0) return QWN_CUDA_STATUS_OK;
    DeviceScope scope(st->device_id);
    return finish("qwn_linear_attention_prefill",
                  launch_step(st, seq_len, q_dev, k_dev, v_dev, decay, o_dev, (cudaStream_t)stream));
}

QWN_CUDA_ABI_API int qwn_linear_attention_decode(QwnLinearAttentionState *st, const float *q_dev,
                                                 const float *k_dev, const float *v_dev, float decay,
                                                 float *o_dev, void *stream) {
    return qwn_linear_attention_prefill(st, q_dev, k_dev, v_dev, decay, 1, o_dev, stream);
}

QWN_CUDA_ABI_API int qwn_linear_attention_prefill_host(QwnLinearAttentionState *st, const float *q,
                                                       const float *k, const float *v, float decay,
                                                       int32_t seq_len, float *o) {
    if (!state_ok(st) || seq_len < 0 || (seq_len > 0 && (!q || !k || !v || !o))) {
        set_error("qwn_linear_attention_prefill_host: invalid argument");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    if (seq_len == 0) return QWN_CUDA_STATUS_OK;
    DeviceScope scope(st->device_id);
    const size_t tok_bytes = (size_t)st->n_heads * st->head_dim * sizeof(float);
    const int chunk = (int)std::max<size_t>(1, kLaHostChunkBytes / tok_bytes);
    if (seq_len > chunk) return prefill_host_pipelined(st, q, k, v, decay, seq_len, o, chunk);
    const size_t row = (size_t)seq_len * tok_bytes;
    if (st->staging_bytes < 4 * row) {
        if (st->staging) cudaFree(st->staging);
        st->staging = nullptr;
        st->staging_bytes = 0;
        cudaError_t e = cudaMalloc(&st->staging, 4 * row);
        if (e != cudaSuccess) {
            set_cuda_error("qwn_linear_attention_prefill_host: cudaMalloc", e);
            return QWN_CUDA_STATUS_OUT_OF_MEMORY;
        }
        st->staging_bytes = 4 * row;
    }
    char *base = (char *)st->staging;
    float *dq = (float *)base, *dk = (float *)(base + row), *dv = (float *)(base + 2 * row),
          *dout = (float *)(base + 3 * row);
    cudaError_t e = cudaMemcpyAsync(dq, q, row, cudaMemcpyDefault, 0);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dk, k, row, cudaMemcpyDefault, 0);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dv, v, row, cudaMemcpyDefault, 0);
    if (e == cudaSuccess) e = launch_step(st, seq_len, dq, dk, dv, decay, dout, 0);
    if (e == cudaSuccess) e = cudaMemcpyAsync(o, dout, row, cudaMemcpyDefault, 0);
    if (e == cudaSuccess) e = cudaStreamSynchronize(0);
    return finish("qwn_linear_attention_prefill_host", e);
}
