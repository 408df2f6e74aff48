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
// Layout: CTA = (head, 32-column block); lane = column, warp w = rows
// w, w+8, w+16, ...  A warp's row access is one 128-byte line, so the state
// streams through HBM fully coalesced.  The output chain is serial in the
// rows, so the updated 32-column slice goes to shared memory and one warp
// (decode) or one warp per buffered token (prefill) runs the chain from there.
//
//   decode : HBM-bound -- the state is read and written once per token
//            (8 d^2 bytes per head); loads are issued 16 rows per thread at a
//            time so each CTA has 16 KB in flight.
//   prefill: the state slice stays in registers for the whole sequence (read
//            and written once), tokens are processed in chunks of up to 8:
//            every warp updates its rows for all chunk tokens, then each warp
//            runs the output chain of one token of the chunk.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>

#include "kv_internal.cuh"

namespace qkv {
namespace {

constexpr int kLaCols = 32;   // columns per CTA
constexpr int kLaWarps = 8;   // row stripes per CTA
constexpr int kLaThreads = kLaCols * kLaWarps;
constexpr int kLaMaxDim = 512;
constexpr int kLaDecodeUnroll = 16;
constexpr int kLaMaxChunk = 8;
constexpr size_t kLaSmemBudget = 200 * 1024;

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

__global__ void __launch_bounds__(kLaThreads) la_decode_kernel(float *__restrict__ state, int d, int col_blocks,
                                                               const float *__restrict__ q,
                                                               const float *__restrict__ k,
                                                               const float *__restrict__ v, float decay,
                                                               float *__restrict__ o) {
    extern __shared__ float sm[];
    float *sk = sm, *sq = sm + d, *slice = sm + 2 * d;  // slice: [d][32]
    const int h = blockIdx.x / col_blocks, cb = blockIdx.x - h * col_blocks;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int j = cb * kLaCols + lane;
    const bool col = j < d;
    const size_t hd = (size_t)h * d;
    for (int i = threadIdx.x; i < d; i += kLaThreads) {
        sk[i] = k[hd + i];
        sq[i] = q[hd + i];
    }
    const float vj = col ? v[hd + j] : 0.f;
    __syncthreads();
    float *S = state + hd * d;
    for (int i0 = w; i0 < d; i0 += kLaWarps * kLaDecodeUnroll) {
        float s[kLaDecodeUnroll];
#pragma unroll
        for (int u = 0; u < kLaDecodeUnroll; u++) {
            const int i = i0 + u * kLaWarps;
            s[u] = (col && i < d) ? S[(size_t)i * d + j] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < kLaDecodeUnroll; u++) {
            const int i = i0 + u * kLaWarps;
            if (i < d) {
                const float ns = __fmaf_rn(decay, s[u], __fmul_rn(sk[i], vj));
                if (col) S[(size_t)i * d + j] = ns;
                slice[i * kLaCols + lane] = ns;
            }
        }
    }
    __syncthreads();
    if (w == 0 && col) {
        float acc = 0.f;
#pragma unroll 8
        for (int i = 0; i < d; i++) acc = __fmaf_rn(sq[i], slice[i * kLaCols + lane], acc);
        o[hd + j] = acc;
    }
}

// R = rows held per thread (>= ceil(d / 8)); chunk = tokens buffered per pass.
template <int R>
__global__ void __launch_bounds__(kLaThreads) la_prefill_kernel(float *__restrict__ state, int n_heads, int d,
                                                                int col_blocks, int seq_len, int chunk,
                                                                const float *__restrict__ q,
                                                                const float *__restrict__ k,
                                                                const float *__restrict__ v, float decay,
                                                                float *__restrict__ o) {
    extern __shared__ float sm[];
    // per buffered token c: k[d], q[d], v[32], then the slices [chunk][d][32]
    const int tok_stride = 2 * d + kLaCols;
    float *stage = sm, *slices = sm + (size_t)chunk * tok_stride;
    const int h = blockIdx.x / col_blocks, cb = blockIdx.x - h * col_blocks;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int j = cb * kLaCols + lane;
    const bool col = j < d;
    const size_t hd = (size_t)h * d, row_stride = (size_t)n_heads * d;  // token stride of q/k/v/o
    float *S = state + hd * d;
    float s[R];
#pragma unroll
    for (int u = 0; u < R; u++) {
        const int i = w + u * kLaWarps;
        s[u] = (col && i < d) ? S[(size_t)i * d + j] : 0.f;
    }
    for (int t0 = 0; t0 < seq_len; t0 += chunk) {
        const int n = min(chunk, seq_len - t0);
        for (int c = 0; c < n; c++) {
            const size_t base = (size_t)(t0 + c) * row_stride + hd;
            float *st = stage + c * tok_stride;
            for (int i = threadIdx.x; i < d; i += kLaThreads) {
                st[i] = k[base + i];
                st[d + i] = q[base + i];
            }
            if (threadIdx.x < kLaCols) st[2 * d + threadIdx.x] = col ? v[base + j] : 0.f;
        }
        __syncthreads();
        for (int c = 0; c < n; c++) {
            const float *st = stage + c * tok_stride;
            const float vj = st[2 * d + lane];
            float *sl = slices + (size_t)c * d * kLaCols;
#pragma unroll
            for (int u = 0; u < R; u++) {
                const int i = w + u * kLaWarps;
                if (i < d) {
                    s[u] = __fmaf_rn(decay, s[u], __fmul_rn(st[i], vj));
                    sl[i * kLaCols + lane] = s[u];
                }
            }
        }
        __syncthreads();
        for (int c = w; c < n; c += kLaWarps) {
            if (col) {
                const float *qc = stage + c * tok_stride + d;
                const float *sl = slices + (size_t)c * d * kLaCols;
                float acc = 0.f;
#pragma unroll 8
                for (int i = 0; i < d; i++) acc = __fmaf_rn(qc[i], sl[i * kLaCols + lane], acc);
                o[(size_t)(t0 + c) * row_stride + hd + j] = acc;
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int u = 0; u < R; u++) {
        const int i = w + u * kLaWarps;
        if (col && i < d) S[(size_t)i * d + j] = s[u];
    }
}

bool state_ok(const QwnLinearAttentionState *st) {
    return st && st->state && st->n_heads > 0 && st->head_dim > 0 && st->head_dim <= kLaMaxDim;
}

int prefill_chunk(int d) {
    const size_t per_tok = ((size_t)d * kLaCols + 2 * d + kLaCols) * sizeof(float);
    return (int)std::max<size_t>(1, std::min<size_t>(kLaMaxChunk, kLaSmemBudget / per_tok));
}

template <int R>
cudaError_t launch_prefill_r(const QwnLinearAttentionState *st, int seq_len, const float *q, const float *k,
                             const float *v, float decay, float *o, cudaStream_t stream) {
    const int d = st->head_dim, col_blocks = (d + kLaCols - 1) / kLaCols;
    const int chunk = prefill_chunk(d);
    const size_t smem = ((size_t)chunk * (2 * d + kLaCols) + (size_t)chunk * d * kLaCols) * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(la_prefill_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    la_prefill_kernel<R><<<(unsigned)(st->n_heads * col_blocks), kLaThreads, smem, stream>>>(
        st->state, st->n_heads, d, col_blocks, seq_len, chunk, q, k, v, decay, o);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_decode(const QwnLinearAttentionState *st, const float *q, const float *k, const float *v,
                          float decay, float *o, cudaStream_t stream) {
    const int d = st->head_dim, col_blocks = (d + kLaCols - 1) / kLaCols;
    const size_t smem = ((size_t)2 * d + (size_t)d * kLaCols) * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(la_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    la_decode_kernel<<<(unsigned)(st->n_heads * col_blocks), kLaThreads, smem, stream>>>(st->state, d, col_blocks,
                                                                                        q, k, v, decay, o);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_step(const QwnLinearAttentionState *st, int seq_len, const float *q, const float *k,
                        const float *v, float decay, float *o, cudaStream_t stream) {
    if (seq_len == 1) return launch_decode(st, q, k, v, decay, o, stream);
    const int r = (st->head_dim + kLaWarps - 1) / kLaWarps;
    if (r <= 4) return launch_prefill_r<4>(st, seq_len, q, k, v, decay, o, stream);
    if (r <= 8) return launch_prefill_r<8>(st, seq_len, q, k, v, decay, o, stream);
    if (r <= 16) return launch_prefill_r<16>(st, seq_len, q, k, v, decay, o, stream);
    if (r <= 32) return launch_prefill_r<32>(st, seq_len, q, k, v, decay, o, stream);
    return launch_prefill_r<64>(st, seq_len, q, k, v, decay, o, stream);
}

int finish(const char *what, cudaError_t e) {
    if (e == cudaSuccess) return QWN_CUDA_STATUS_OK;
    set_cuda_error(what, e);
    return QWN_CUDA_STATUS_RUNTIME_ERROR;
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
    const size_t row = (size_t)seq_len * st->n_heads * st->head_dim * sizeof(float);
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
    cudaError_t e = cudaMemcpyAsync(dq, q, row, cudaMemcpyHostToDevice, 0);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dk, k, row, cudaMemcpyHostToDevice, 0);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dv, v, row, cudaMemcpyHostToDevice, 0);
    if (e == cudaSuccess) e = launch_step(st, seq_len, dq, dk, dv, decay, dout, 0);
    if (e == cudaSuccess) e = cudaMemcpyAsync(o, dout, row, cudaMemcpyDeviceToHost, 0);
    if (e == cudaSuccess) e = cudaStreamSynchronize(0);
    return finish("qwn_linear_attention_prefill_host", e);
}
