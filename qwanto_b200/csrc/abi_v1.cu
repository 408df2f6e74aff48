// qwnrun-facing ABI version 1 (include/qwn_cuda_abi.h).
//
// Behaviour follows the reference contract c/cuda/qwn_hypervsq2_cuda_abi.cu:
// header checks accept struct_size >= the known size; a process-wide mutex
// serialises entry points; every call is synchronous on return; errors set
// a last-error string; telemetry is copied out on each KV call.
//
// A KV cache created with head_dim 128 is a one-sequence, one-layer paged
// pool with the reference Q8 codec (int8 + fp32 scale per 64 channels,
// c/qwanto_turboquant.c:562-586), so appends and attention run on the same
// B200 kernels as the batched path.  Other head dims keep the reference's
// contiguous [max_tokens][channels] layout with a generic split-KV kernel.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "kv_internal.cuh"

namespace qkv {
namespace {

std::mutex g_abi_mu;

// A HyperVSQ-2 tensor, repacked at upload: the 64 code bytes of every block
// in [rows][blocks][64] (16-byte aligned for vector loads), then the block
// headers (fp16 base, fp16 offset, four sub-scale bytes; the two reserved
// bytes dropped) in [rows][blocks][8]: 72 bytes per block instead of 74.
struct Tensor {
    void *dev = nullptr;
    uint64_t bytes = 0;
    uint32_t rows = 0, cols = 0, nblk = 0;
    const uint8_t *codes() const { return static_cast<const uint8_t *>(dev); }
    const uint8_t *hdr() const { return codes() + (uint64_t)rows * nblk * 64; }
};

struct KvCache {
    // paged fast path (head_dim == 128)
    QwnKvPoolHandle pool{};
    // generic path
    int8_t *key = nullptr, *value = nullptr;
    float *key_scales = nullptr, *value_scales = nullptr;
    float *part = nullptr;  // generic split-KV partials
    size_t part_cap = 0;
    uint32_t max_tokens = 0, kv_heads = 0, head_dim = 0, channels = 0, blocks = 0, tokens = 0;
    uint64_t bytes = 0;
    bool paged = false;
};

struct Context {
    int device = -1;
    uint64_t budget = 0, resident = 0;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    std::vector<Tensor *> tensors;
    std::vector<KvCache *> caches;
    // staging
    float *d_k = nullptr, *d_v = nullptr, *d_q = nullptr, *d_o = nullptr;
    size_t k_cap = 0, v_cap = 0, q_cap = 0, o_cap = 0;
    int8_t *d_in = nullptr;
    float *d_out = nullptr, *d_scales = nullptr;
    size_t in_cap = 0, out_cap = 0, sc_cap = 0;
    QwnCudaTelemetry tel{};
    // paged attention with a query-to-kv-head map that is not uniform: the
    // query and output rows in the padded kv_heads x G' layout (host side)
    std::vector<float> pad_q, pad_o;
};

Context *ctx_from(const QwnCudaContextHandle *h) {
    if (!h || !header_ok(h->header, sizeof(*h)) || !h->opaque) return nullptr;
    return static_cast<Context *>(h->opaque);
}
KvCache *kv_from(const QwnCudaKvCacheHandle &h) {
    if (!header_ok(h.header, sizeof(h)) || !h.opaque) return nullptr;
    return static_cast<KvCache *>(h.opaque);
}
Tensor *tensor_from(const QwnCudaTensorHandle &h) {
    if (!header_ok(h.header, sizeof(h)) || !h.opaque) return nullptr;
    return static_cast<Tensor *>(h.opaque);
}

void init_tel(QwnCudaTelemetry *t, int device) {
    std::memset(t, 0, sizeof(*t));
    qwn_cuda_abi_header_init(&t->header, sizeof(*t));
    t->device_id = device;
    std::snprintf(t->kernel_type, sizeof(t->kernel_type), "hypervsq2-74-q8-b200");
    std::snprintf(t->kv_cache_kernel_type, sizeof(t->kv_cache_kernel_type), "Unavailable");
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, device) == cudaSuccess)
        std::snprintf(t->device_name, sizeof(t->device_name), "%s", prop.name);
}

bool grow(void **p, size_t *cap, size_t bytes) {
    if (bytes <= *cap) return true;
    cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    if (cudaMalloc(p, bytes) != cudaSuccess) return false;
    *cap = bytes;
    return true;
}

// ---------------------------------------------------------------------------
// generic contiguous Q8 path (head_dim != 128)
// ---------------------------------------------------------------------------
__device__ __forceinline__ int q8_round_g(float x) {
    if (!isfinite(x)) return 0;
    if (x >= 127.f) return 127;
    if (x <= -127.f) return -127;
    return __float2int_rn(x);
}
// one warp per 64-channel block, c/qwanto_turboquant.c:573-586
__global__ void q8_quantize_generic(const float *in, int8_t *out, float *scales, uint32_t channels,
                                    uint32_t blocks) {
    const uint32_t b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (b >= blocks) return;
    const uint32_t c0 = b * 64 + lane, c1 = c0 + 32;
    const float x0 = c0 < channels ? in[c0] : 0.f, x1 = c1 < channels ? in[c1] : 0.f;
    float m = 0.f;
    if (c0 < channels && isfinite(x0)) m = fmaxf(m, fabsf(x0));
    if (c1 < channels && isfinite(x1)) m = fmaxf(m, fabsf(x1));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s = m > 0.f ? __fdiv_rn(m, 127.f) : 1.f;
    if (lane == 0) scales[b] = s;
    if (c0 < channels) out[c0] = (int8_t)q8_round_g(__fdiv_rn(x0, s));
    if (c1 < channels) out[c1] = (int8_t)q8_round_g(__fdiv_rn(x1, s));
}

constexpr int kGenChunk = 256;  // tokens per CTA
// grid (query_heads, chunks), 4 warps; per CTA partial (m, l, o[head_dim])
__global__ void q8_attention_generic(const int8_t *keys, const int8_t *values, const float *ks,
                                     const float *vs, const float *q, float *part, uint32_t H, uint32_t HK,
                                     uint32_t hd, uint32_t channels, uint32_t blocks, uint32_t ntok,
                                     float scale_log2) {
    const uint32_t head = blockIdx.x, chunk = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t kvh = (head * HK) / H, off = kvh * hd;
    const uint32_t t0 = chunk * kGenChunk, t1 = min(ntok, t0 + kGenChunk);
    extern __shared__ float sh[];  // [4][hd] o, [4] m, [4] l
    float *so = sh, *sm = sh + 4 * hd, *sl = sm + 4;
    float m = -INFINITY, l = 0.f;
    float o[32];
    const int per = (int)((hd + 31) / 32);
#pragma unroll
    for (int k = 0; k < 32; k++) o[k] = 0.f;
    const float *qh = q + (size_t)head * hd;
    for (uint32_t t = t0 + warp; t < t1; t += 4) {
        float dot = 0.f;
        for (uint32_t c = lane; c < hd; c += 32) {
            const uint32_t ch = off + c;
            dot += qh[c] * ((float)keys[(size_t)t * channels + ch] * ks[(size_t)t * blocks + ch / 64]);
        }
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, s);
        const float sc = dot * scale_log2;
        const float mn = fmaxf(m, sc);
        const float alpha = exp2f(m - mn), p = exp2f(sc - mn);
        l = l * alpha + p;
        for (int k = 0; k < per && k < 32; k++) {
            const uint32_t c = lane + 32 * k;
            float v = 0.f;
            if (c < hd) {
                const uint32_t ch = off + c;
                v = (float)values[(size_t)t * channels + ch] * vs[(size_t)t * blocks + ch / 64];
            }
            o[k] = o[k] * alpha + p * v;
        }
        m = mn;
    }
    for (int k = 0; k < per && k < 32; k++) {
        const uint32_t c = lane + 32 * k;
        if (c < hd) so[warp * hd + c] = o[k];
    }
    if (lane == 0) { sm[warp] = m; sl[warp] = l; }
    __syncthreads();
    if (warp == 0) {
        float ms = -INFINITY;
        for (int w = 0; w < 4; w++) ms = fmaxf(ms, sm[w]);
        float ls = 0.f;
        float wgt[4];
        for (int w = 0; w < 4; w++) {
            wgt[w] = sm[w] == -INFINITY ? 0.f : exp2f(sm[w] - ms);
            ls += sl[w] * wgt[w];
        }
        float *dst = part + ((size_t)chunk * H + head) * (hd + 2);
        for (uint32_t c = lane; c < hd; c += 32) {
            float acc = 0.f;
            for (int w = 0; w < 4; w++) acc += so[w * hd + c] * wgt[w];
            dst[c] = acc;
        }
        if (lane == 0) { dst[hd] = ms; dst[hd + 1] = ls; }
    }
}

__global__ void merge_generic(const float *part, float *out, uint32_t H, uint32_t hd, uint32_t chunks) {
    const uint32_t head = blockIdx.x;
    float ms = -INFINITY;
    for (uint32_t c = 0; c < chunks; c++) ms = fmaxf(ms, part[((size_t)c * H + head) * (hd + 2) + hd]);
    float ls = 0.f;
    for (uint32_t c = 0; c < chunks; c++) {
        const float *pc = part + ((size_t)c * H + head) * (hd + 2);
        ls += pc[hd + 1] * (pc[hd] == -INFINITY ? 0.f : exp2f(pc[hd] - ms));
    }
    for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x) {
        float acc = 0.f;
        for (uint32_t c = 0; c < chunks; c++) {
            const float *pc = part + ((size_t)c * H + head) * (hd + 2);
            acc += pc[d] * (pc[hd] == -INFINITY ? 0.f : exp2f(pc[hd] - ms));
        }
        out[(size_t)head * hd + d] = ls > 0.f ? acc / ls : 0.f;
    }
}

// ---------------------------------------------------------------------------
// HyperVSQ-2 GEMV: 74-byte blocks of 256 weights (fp16 base, fp16 offset,
// eight 4-bit sub-scales, 2 reserved bytes, 64 bytes of 2-bit codes) times
// int8 activations; the block format of c/cuda/qwn_hypervsq2_cuda_abi.cu:225-289.
// One warp per output row; lane l handles weights 8l..8l+7 of every block
// (octant l/4), summing (q-1)*a exactly in integers before scaling.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float half_ftz(const uint8_t *b) {
    // the reference decodes these fp16 fields with subnormals flushed to zero
    const uint32_t raw = (uint32_t)b[0] | ((uint32_t)b[1] << 8);
    const uint32_t sign = (raw >> 15) & 1u, ex = (raw >> 10) & 31u, mant = raw & 1023u;
    uint32_t bits;
    if (ex == 0) bits = sign << 31;
    else if (ex == 31) bits = (sign << 31) | 0x7F800000u | (mant << 13);
    else bits = (sign << 31) | ((ex + 112u) << 23) | (mant << 13);
    return __uint_as_float(bits);
}

// Activations of up to kGemvTokens tokens are staged per CTA in shared
// memory: block b of token t at t*nblk*320 + b*320, its quarter qd (weights
// 64qd..64qd+63) at +80qd (the padding keeps the quarters of eight blocks on
// distinct banks), and inside a quarter each group of 16 weights permuted so
// that word i holds weights i, 4+i, 8+i, 12+i -- the order in which one
// masked shift of a code word yields them.  Past cols the activations are 0.
// osum[t][8b+o] is the sum of octant o's activations (the offset term and
// the -1 of the codes).  A lane takes one quarter block (two octants), loads
// its 16 code bytes once and applies them to every staged token with dp4a:
// sum (q-1)*a = dp4a(q, a) - sum a, exact in integers, then the octant's
// scale base*sub/8 and the block offset in fp32.
constexpr int kGemvWarps = 8, kGemvTokens = 8, kGemvBlockSmem = 320 + 8 * 4;

template <int TOKS, int ROWS>
__global__ void __launch_bounds__(kGemvWarps * 32)
    hypervsq2_gemv_kernel(const uint8_t *codes, const uint8_t *hdr, const int8_t *in, float in_scale,
                          const float *in_scales, float *out, uint32_t batch, uint32_t rows, uint32_t cols,
                          uint32_t nblk, uint32_t in_stride, uint32_t out_stride, uint32_t tokens_per_pass) {
    extern __shared__ __align__(16) uint8_t gsm[];
    const uint32_t tok_bytes = nblk * 320u;
    int8_t *act = reinterpret_cast<int8_t *>(gsm);
    int *osum = reinterpret_cast<int *>(gsm + (size_t)tokens_per_pass * tok_bytes);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t wglob = blockIdx.x * kGemvWarps + warp, wtot = gridDim.x * kGemvWarps;
    const int qd = lane & 3;
    for (uint32_t t0 = 0; t0 < batch; t0 += tokens_per_pass) {
        const uint32_t nt = min(tokens_per_pass, batch - t0);
        __syncthreads();  // the previous pass is done with the staged tokens
        // stage one octant (32 activations) per thread: its two groups of 16
        // permuted (a 4x4 byte transpose) and its sum; zero past cols
        const bool vec = (in_stride & 15u) == 0;
        for (uint32_t idx = threadIdx.x; idx < nt * nblk * 8u; idx += blockDim.x) {
            const uint32_t tt = idx / (nblk * 8u), og = idx % (nblk * 8u);
            const uint32_t c0 = og * 32u;
            const int8_t *ip = in + (uint64_t)(t0 + tt) * in_stride + c0;
            uint32_t wv[8];
            if (vec && c0 + 32u <= cols) {
                const uint4 x0 = *reinterpret_cast<const uint4 *>(ip);
                const uint4 x1 = *reinterpret_cast<const uint4 *>(ip + 16);
                wv[0] = x0.x; wv[1] = x0.y; wv[2] = x0.z; wv[3] = x0.w;
                wv[4] = x1.x; wv[5] = x1.y; wv[6] = x1.z; wv[7] = x1.w;
            } else {
#pragma unroll
                for (int m = 0; m < 8; m++) {
                    uint32_t v = 0;
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const uint32_t c = c0 + 4u * m + k;
                        v |= (uint32_t)(uint8_t)(c < cols ? ip[4 * m + k] : 0) << (8 * k);
                    }
                    wv[m] = v;
                }
            }
            int s = 0;
#pragma unroll
            for (int m = 0; m < 8; m++) s = __dp4a((int)wv[m], 0x01010101, s);
            osum[tt * nblk * 8u + og] = s;
            const uint32_t blk = og >> 3, ol = og & 7u;
            int8_t *dst = act + (size_t)tt * tok_bytes + blk * 320u + (ol >> 1) * 80u + (ol & 1u) * 32u;
#pragma unroll
            for (int gg = 0; gg < 2; gg++) {
                const uint32_t *W = wv + 4 * gg;
                const uint32_t p0 = __byte_perm(W[0], W[1], 0x5140), p1 = __byte_perm(W[2], W[3], 0x5140);
                const uint32_t p2 = __byte_perm(W[0], W[1], 0x7362), p3 = __byte_perm(W[2], W[3], 0x7362);
                *reinterpret_cast<uint4 *>(dst + 16 * gg) =
                    make_uint4(__byte_perm(p0, p1, 0x5410), __byte_perm(p0, p1, 0x7632), __byte_perm(p2, p3, 0x5410),
                               __byte_perm(p2, p3, 0x7632));
            }
        }
        __syncthreads();
        // ROWS rows per iteration (rows row, row + wtot, ...): all their code
        // and header loads are in flight before any is used
        for (uint32_t row = wglob; row < rows; row += ROWS * wtot) {
            uint32_t rr[ROWS];
            float acc[ROWS][TOKS];
            const uint8_t *rc[ROWS], *rh[ROWS];
#pragma unroll
            for (int r = 0; r < ROWS; r++) {
                rr[r] = row + r * wtot < rows ? row + r * wtot : row;
                rc[r] = codes + (uint64_t)rr[r] * nblk * 64u;
                rh[r] = hdr + (uint64_t)rr[r] * nblk * 8u;
#pragma unroll
                for (int k = 0; k < TOKS; k++) acc[r][k] = 0.f;
            }
            for (uint32_t b = lane >> 2; b < nblk; b += 8) {
                uint4 cw[ROWS];
                uint2 h[ROWS];
#pragma unroll
                for (int r = 0; r < ROWS; r++) {
                    cw[r] = *reinterpret_cast<const uint4 *>(rc[r] + b * 64u + qd * 16u);
                    h[r] = *reinterpret_cast<const uint2 *>(rh[r] + b * 8u);
                }
#pragma unroll
                for (int r = 0; r < ROWS; r++) {
                    const float base = half_ftz(reinterpret_cast<const uint8_t *>(&h[r]));
                    const float offs = half_ftz(reinterpret_cast<const uint8_t *>(&h[r]) + 2);
                    const uint32_t sb = (h[r].y >> (8 * qd)) & 0xFFu;  // octants 2qd (low nibble), 2qd+1 (high)
                    const float eff0 = base * ((float)(sb & 15u) * (1.0f / 8.0f));
                    const float eff1 = base * ((float)(sb >> 4) * (1.0f / 8.0f));
                    const uint32_t cwa[4] = {cw[r].x, cw[r].y, cw[r].z, cw[r].w};
                    int e[4][4];
#pragma unroll
                    for (int j = 0; j < 4; j++)
#pragma unroll
                        for (int i = 0; i < 4; i++) e[j][i] = (int)((cwa[j] >> (2 * i)) & 0x03030303u);
#pragma unroll
                    for (int k = 0; k < TOKS; k++) {
                        if ((uint32_t)k >= nt) break;
                        const int8_t *ta = act + (size_t)k * tok_bytes + b * 320u + qd * 80u;
                        int d[2] = {0, 0};
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const int4 a = *reinterpret_cast<const int4 *>(ta + 16 * j);
                            d[j >> 1] = __dp4a(e[j][0], a.x, d[j >> 1]);
                            d[j >> 1] = __dp4a(e[j][1], a.y, d[j >> 1]);
                            d[j >> 1] = __dp4a(e[j][2], a.z, d[j >> 1]);
                            d[j >> 1] = __dp4a(e[j][3], a.w, d[j >> 1]);
                        }
                        const int *os = osum + k * nblk * 8u + b * 8u + 2 * qd;
                        const int s0 = os[0], s1 = os[1];
                        acc[r][k] += eff0 * (float)(d[0] - s0) + eff1 * (float)(d[1] - s1) + offs * (float)(s0 + s1);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < ROWS; r++) {
                if (r > 0 && rr[r] == row) break;
#pragma unroll
                for (int k = 0; k < TOKS; k++) {
                    if ((uint32_t)k >= nt) break;
                    float v = acc[r][k];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    if (lane == 0)
                        out[(uint64_t)(t0 + k) * out_stride + rr[r]] =
                            v * (in_scales ? in_scales[t0 + k] : in_scale);
                }
            }
        }
    }
}

int gemv_execute(Context *c, const QwnCudaGemmRequest *r, QwnCudaTelemetry *tel) {
    if (!r || !header_ok(r->header, sizeof(*r)) || r->input_mode != QWN_CUDA_INPUT_Q8 || !r->input_q8 ||
        !r->output || r->batch == 0 || r->rows == 0 || r->cols == 0) {
        set_error("invalid HyperVSQ-2 GEMV/GEMM request");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    Tensor *t = tensor_from(r->tensor);
    if (!t || t->rows != r->rows || t->cols != r->cols) {
        set_error("tensor dimensions do not match the HyperVSQ-2 request");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    cudaSetDevice(c->device);
    const uint32_t ist = r->input_stride ? r->input_stride : r->cols;
    const uint32_t ost = r->output_stride ? r->output_stride : r->rows;
    const size_t in_b = (size_t)r->batch * ist, out_b = (size_t)r->batch * ost * sizeof(float);
    if (!grow((void **)&c->d_in, &c->in_cap, in_b) || !grow((void **)&c->d_out, &c->out_cap, out_b) ||
        !grow((void **)&c->d_scales, &c->sc_cap, r->batch * sizeof(float))) {
        set_error("CUDA activation workspace allocation failed");
        return QWN_CUDA_STATUS_OUT_OF_MEMORY;
    }
    auto t0 = std::chrono::steady_clock::now();
    cudaError_t e = cudaMemcpyAsync(c->d_in, r->input_q8, in_b, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess && r->input_scales)
        e = cudaMemcpyAsync(c->d_scales, r->input_scales, r->batch * sizeof(float), cudaMemcpyHostToDevice,
                            c->stream);
    auto t1 = std::chrono::steady_clock::now();
    if (e == cudaSuccess) e = cudaEventRecord(c->ev0, c->stream);
    // tokens staged per pass: as many as ~96 KB of shared memory holds (two
    // CTAs per SM), at least one (up to the opt-in limit set below)
    const uint64_t per_tok = (uint64_t)t->nblk * kGemvBlockSmem;
    uint32_t tpp = (uint32_t)std::min<uint64_t>(kGemvTokens, std::max<uint64_t>(1, (96u << 10) / per_tok));
    tpp = std::min<uint32_t>(tpp, r->batch);
    const size_t smem = (size_t)tpp * per_tok;
    if (smem > (200u << 10)) {
        set_error("HyperVSQ-2 GEMV: cols too large for one token's activations in shared memory");
        return QWN_CUDA_STATUS_UNSUPPORTED;
    }
    // one token (decode): four rows per warp iteration; more tokens: two
    const bool single = r->batch == 1;
    const void *kern = single ? (const void *)hypervsq2_gemv_kernel<1, 4> : (const void *)hypervsq2_gemv_kernel<kGemvTokens, 2>;
    const uint32_t rows_per = single ? 4u : 2u;
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 << 10);
    if (e == cudaSuccess) {
        int sms = 0, per_sm = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c->device);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGemvWarps * 32, smem);
        // every resident warp streams rows: the GEMV is bound by the loads in flight
        const uint32_t grid = std::min<uint32_t>((r->rows + rows_per * kGemvWarps - 1) / (rows_per * kGemvWarps),
                                                 (uint32_t)std::max(1, sms) * (uint32_t)std::max(1, per_sm));
        const float *isc = r->input_scales ? c->d_scales : nullptr;
        if (single)
            hypervsq2_gemv_kernel<1, 4><<<grid, kGemvWarps * 32, smem, c->stream>>>(
                t->codes(), t->hdr(), c->d_in, r->input_scale, isc, c->d_out, r->batch, r->rows, r->cols, t->nblk,
                ist, ost, tpp);
        else
            hypervsq2_gemv_kernel<kGemvTokens, 2><<<grid, kGemvWarps * 32, smem, c->stream>>>(
                t->codes(), t->hdr(), c->d_in, r->input_scale, isc, c->d_out, r->batch, r->rows, r->cols, t->nblk,
                ist, ost, tpp);
        count_launch();
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaEventRecord(c->ev1, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(r->output, c->d_out, out_b, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) { set_cuda_error("HyperVSQ-2 GEMV", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    float ms = 0.f;
    cudaEventElapsedTime(&ms, c->ev0, c->ev1);
    c->tel.gpu_matmul_count++;
    c->tel.gpu_kernel_launch_count++;
    c->tel.gpu_projection_count++;
    c->tel.gpu_kernel_ms += ms;
    c->tel.gpu_transfer_ms += std::chrono::duration<double, std::milli>(t1 - t0).count();
    c->tel.gpu_resident_bytes = c->resident;
    if (tel) *tel = c->tel;
    return QWN_CUDA_STATUS_OK;
}

}  // namespace
}  // namespace qkv

using namespace qkv;

extern "C" {

QWN_CUDA_ABI_API int qwn_cuda_abi_query(QwnCudaAbiInfo *info) {
    if (!info || !header_ok(info->header, sizeof(*info))) {
        set_error("invalid ABI query structure");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    std::memset(info, 0, sizeof(*info));
    qwn_cuda_abi_header_init(&info->header, sizeof(*info));
    info->capability_bits = QWN_CUDA_CAP_HYPERVSQ2_GEMV | QWN_CUDA_CAP_HYPERVSQ2_GEMM |
                            QWN_CUDA_CAP_RESIDENT_WEIGHTS | QWN_CUDA_CAP_TELEMETRY |
                            QWN_CUDA_CAP_DEVICE_ENUMERATION | QWN_CUDA_CAP_Q8_KV | QWN_CUDA_CAP_PAGED_KV |
                            QWN_CUDA_CAP_TQ_KV | QWN_CUDA_CAP_BATCHED_DEVICE | QWN_CUDA_CAP_SPLIT_KV_MERGE |
                            QWN_CUDA_CAP_PAGE_EVICTION | QWN_CUDA_CAP_LINEAR_ATTENTION;
    info->max_devices = 16;
    info->max_resident_tensors = QWN_CUDA_MAX_RESIDENT_TENSORS;
    info->hypervsq2_block_bytes = QWN_CUDA_HYPERVSQ2_BLOCK_BYTES;
    info->hypervsq2_block_elements = QWN_CUDA_HYPERVSQ2_BLOCK_ELEMENTS;
    std::snprintf(info->abi_name, sizeof(info->abi_name), "%s", QWN_CUDA_ABI_NAME);
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_cuda_abi_get_capabilities(QwnCudaAbiInfo *info) { return qwn_cuda_abi_query(info); }

QWN_CUDA_ABI_API int qwn_cuda_abi_enumerate_devices(QwnCudaDeviceInfo *devices, uint32_t capacity,
                                                     uint32_t *count) {
    if (!count) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        set_cuda_error("cudaGetDeviceCount", e);
        *count = 0;
        return QWN_CUDA_STATUS_UNAVAILABLE;
    }
    *count = (uint32_t)n;
    if (!devices || capacity == 0) return QWN_CUDA_STATUS_OK;
    int drv = 0;
    cudaDriverGetVersion(&drv);
    int cur = 0;
    cudaGetDevice(&cur);
    for (uint32_t i = 0; i < std::min<uint32_t>(capacity, (uint32_t)n); i++) {
        std::memset(&devices[i], 0, sizeof(devices[i]));
        qwn_cuda_abi_header_init(&devices[i].header, sizeof(devices[i]));
        cudaDeviceProp prop{};
        if (cudaGetDeviceProperties(&prop, (int)i) != cudaSuccess) continue;
        devices[i].device_id = (int32_t)i;
        devices[i].compute_major = prop.major;
        devices[i].compute_minor = prop.minor;
        devices[i].total_vram_bytes = prop.totalGlobalMem;
        size_t fb = 0, tb = 0;
        if (cudaSetDevice((int)i) == cudaSuccess && cudaMemGetInfo(&fb, &tb) == cudaSuccess)
            devices[i].free_vram_bytes = fb;
        std::snprintf(devices[i].name, sizeof(devices[i].name), "%s", prop.name);
        std::snprintf(devices[i].driver, sizeof(devices[i].driver), "%d", drv);
    }
    cudaSetDevice(cur);
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_cuda_abi_context_create(const QwnCudaContextOptions *o, QwnCudaContextHandle *h) {
    if (!o || !h || !header_ok(o->header, sizeof(*o)) || !header_ok(h->header, sizeof(*h)) || o->device_id < 0) {
        set_error("invalid CUDA context options");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    std::lock_guard<std::mutex> lk(g_abi_mu);
    Context *c = new (std::nothrow) Context();
    if (!c) return QWN_CUDA_STATUS_OUT_OF_MEMORY;
    c->device = o->device_id;
    c->budget = o->memory_budget_bytes;
    if (cudaSetDevice(c->device) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete c;
        set_cuda_error("CUDA context creation", cudaGetLastError());
        return QWN_CUDA_STATUS_UNAVAILABLE;
    }
    cudaEventCreate(&c->ev0);
    cudaEventCreate(&c->ev1);
    init_tel(&c->tel, c->device);
    std::memset(h, 0, sizeof(*h));
    qwn_cuda_abi_header_init(&h->header, sizeof(*h));
    h->opaque = c;
    return QWN_CUDA_STATUS_OK;
}

static void free_cache(KvCache *k) {
    if (k->paged) qwn_kv_pool_destroy(&k->pool);
    cudaFree(k->key); cudaFree(k->value); cudaFree(k->key_scales); cudaFree(k->value_scales); cudaFree(k->part);
    delete k;
}

QWN_CUDA_ABI_API int qwn_cuda_abi_context_destroy(QwnCudaContextHandle *h) {
    Context *c = ctx_from(h);
    if (!c) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lk(g_abi_mu);
    cudaSetDevice(c->device);
    for (Tensor *t : c->tensors) { cudaFree(t->dev); delete t; }
    for (KvCache *k : c->caches) free_cache(k);
    cudaFree(c->d_k); cudaFree(c->d_v); cudaFree(c->d_q); cudaFree(c->d_o);
    cudaFree(c->d_in); cudaFree(c->d_out); cudaFree(c->d_scales);
    cudaEventDestroy(c->ev0);
    cudaEventDestroy(c->ev1);
    cudaStreamDestroy(c->stream);
    delete c;
    h->opaque = nullptr;
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_cuda_abi_upload_tensor(QwnCudaContextHandle *h, const QwnCudaTensorUpload *u,
                                                QwnCudaTensorHandle *out) {
    Context *c = ctx_from(h);
    if (!c || !u || !out || !header_ok(u->header, sizeof(*u)) || !header_ok(out->header, sizeof(*out)) ||
        !u->host_data || u->dtype != QWN_CUDA_TENSOR_HYPERVSQ2_74 || u->rows == 0 || u->cols == 0 ||
        u->block_bytes != QWN_CUDA_HYPERVSQ2_BLOCK_BYTES) {
        set_error("invalid HyperVSQ-2 tensor upload request");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    const uint32_t nblk = (u->cols + 255u) / 256u;
    if (u->data_bytes < (uint64_t)u->rows * nblk * u->block_bytes) {
        set_error("HyperVSQ-2 tensor upload is shorter than its validated shape");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    const uint64_t need = (uint64_t)u->rows * nblk * 72u;  // the repacked layout (struct Tensor)
    std::lock_guard<std::mutex> lk(g_abi_mu);
    cudaSetDevice(c->device);
    size_t fb = 0, tb = 0;
    if (cudaMemGetInfo(&fb, &tb) != cudaSuccess || (c->budget && c->resident + need > c->budget) || need > fb) {
        set_error("HyperVSQ-2 tensor does not fit the configured CUDA memory budget");
        return QWN_CUDA_STATUS_OUT_OF_MEMORY;
    }
    Tensor *t = new (std::nothrow) Tensor();
    if (!t) return QWN_CUDA_STATUS_OUT_OF_MEMORY;
    t->bytes = need;
    t->rows = u->rows;
    t->cols = u->cols;
    t->nblk = nblk;
    // repack on the host: codes [rows][blocks][64], then headers [rows][blocks][8]
    std::vector<uint8_t> packed;
    try {
        packed.resize(need);
    } catch (...) {
        delete t;
        set_error("HyperVSQ-2 tensor upload: host staging allocation failed");
        return QWN_CUDA_STATUS_OUT_OF_MEMORY;
    }
    const uint8_t *src = static_cast<const uint8_t *>(u->host_data);
    const uint64_t nb = (uint64_t)u->rows * nblk;
    for (uint64_t i = 0; i < nb; i++) {
        const uint8_t *blk = src + i * QWN_CUDA_HYPERVSQ2_BLOCK_BYTES;
        std::memcpy(packed.data() + i * 64, blk + 10, 64);
        std::memcpy(packed.data() + nb * 64 + i * 8, blk, 8);
    }
    if (cudaMalloc(&t->dev, need) != cudaSuccess ||
        cudaMemcpy(t->dev, packed.data(), need, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(t->dev);
        delete t;
        set_cuda_error("HyperVSQ-2 tensor upload", cudaGetLastError());
        return QWN_CUDA_STATUS_RUNTIME_ERROR;
    }
    c->tensors.push_back(t);
    c->resident += need;
    c->tel.gpu_upload_count++;
    c->tel.gpu_upload_bytes += need;
    c->tel.gpu_resident_bytes = c->resident;
    std::memset(out, 0, sizeof(*out));
    qwn_cuda_abi_header_init(&out->header, sizeof(*out));
    out->opaque = t;
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_cuda_abi_release_tensor(QwnCudaContextHandle *h, QwnCudaTensorHandle *th) {
    Context *c = ctx_from(h);
    Tensor *t = th ? tensor_from(*th) : nullptr;
    if (!c || !t) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lk(g_abi_mu);
    auto it = std::find(c->tensors.begin(), c->tensors.end(), t);
    if (it == c->tensors.end()) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    cudaSetDevice(c->device);
    cudaFree(t->dev);
    c->resident -= std::min(c->resident, t->bytes);
    delete t;
    c->tensors.erase(it);
    th->opaque = nullptr;
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_cuda_abi_kv_cache_create(QwnCudaContextHandle *h, const QwnCudaKvCacheOptions *o,
                                                  QwnCudaKvCacheHandle *out) {
    Context *c = ctx_from(h);
    if (!c || !o || !out || !header_ok(o->header, sizeof(*o)) || !header_ok(out->header, sizeof(*out)) ||
        o->max_tokens == 0 || o->kv_heads == 0 || o->head_dim == 0) {
        set_error("invalid Q8 KV-cache options");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    std::lock_guard<std::mutex> lk(g_abi_mu);
    cudaSetDevice(c->device);
    KvCache *k = new (std::nothrow) KvCache();
    if (!k) return QWN_CUDA_STATUS_OUT_OF_MEMORY;
    k->max_tokens = o->max_tokens;
    k->kv_heads = o->kv_heads;
    k->head_dim = o->head_dim;
    k->channels = o->kv_heads * o->head_dim;
    k->blocks = (k->channels + 63) / 64;
    k->paged = o->head_dim == (uint32_t)kHeadDim;
    size_t fb = 0, tb = 0;
    cudaMemGetInfo(&fb, &tb);
    if (k->paged) {
        QwnKvPoolOptions po{};
        qwn_cuda_abi_header_init(&po.header, sizeof(po));
        po.device_id = c->device;
        po.codec = QWN_KV_CODEC_Q8_B64_F32;
        po.layers = 1;
        po.kv_heads = o->kv_heads;
        po.head_dim = kHeadDim;
        po.page_tokens = 16;
        po.total_pages = (o->max_tokens + 15) / 16;
        po.max_seqs = 1;
        po.max_pages_per_seq = po.total_pages;
        po.max_query_heads = o->kv_heads * kMaxGroup;
        po.memory_budget_bytes = c->budget ? (c->budget > c->resident ? c->budget - c->resident : 1) : 0;
        qwn_cuda_abi_header_init(&k->pool.header, sizeof(k->pool));
        int rc = qwn_kv_pool_create(&po, &k->pool);
        if (rc != QWN_CUDA_STATUS_OK) {
            delete k;
            return rc;
        }
        QwnKvPoolInfo info{};
        qwn_cuda_abi_header_init(&info.header, sizeof(info));
        qwn_kv_pool_get_info(&k->pool, &info);
        k->bytes = info.pool_bytes;
    } else {
        const size_t vb = (size_t)k->max_tokens * k->channels, sb = (size_t)k->max_tokens * k->blocks * 4;
        k->bytes = 2 * vb + 2 * sb;
        if (o->head_dim > 1024) {
            delete k;
            set_error("Q8 KV-cache: head_dim above 1024 is not supported");
            return QWN_CUDA_STATUS_UNSUPPORTED;
        }
        if ((c->budget && c->resident + k->bytes > c->budget) || k->bytes > fb) {
            delete k;
            set_error("Q8 KV-cache does not fit the configured CUDA memory budget");
            return QWN_CUDA_STATUS_OUT_OF_MEMORY;
        }
        if (cudaMalloc(&k->key, vb) != cudaSuccess || cudaMalloc(&k->value, vb) != cudaSuccess ||
            cudaMalloc(&k->key_scales, sb) != cudaSuccess || cudaMalloc(&k->value_scales, sb) != cudaSuccess) {
            free_cache(k);
            set_cuda_error("Q8 KV-cache allocation", cudaGetLastError());
            return QWN_CUDA_STATUS_OUT_OF_MEMORY;
        }
    }
    c->caches.push_back(k);
    c->resident += k->bytes;
    c->tel.kv_cache_resident_bytes += k->bytes;
    std::memset(out, 0, sizeof(*out));
    qwn_cuda_abi_header_init(&out->header, sizeof(*out));
    out->opaque = k;
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_cuda_abi_kv_cache_append(QwnCudaContextHandle *h, const QwnCudaKvAppendRequest *r,
                                                  QwnCudaTelemetry *tel) {
    Context *c = ctx_from(h);
    KvCache *k = r ? kv_from(r->cache) : nullptr;
    if (!c || !r || !k || !header_ok(r->header, sizeof(*r)) || !r->host_key || !r->host_value ||
        r->n_channels != k->channels || r->token != k->tokens || r->token >= k->max_tokens) {
        set_error("invalid Q8 KV-cache append request");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    std::lock_guard<std::mutex> lk(g_abi_mu);
    cudaSetDevice(c->device);
    if (!grow((void **)&c->d_k, &c->k_cap, (size_t)k->channels * 4) ||
        !grow((void **)&c->d_v, &c->v_cap, (size_t)k->channels * 4)) {
        set_error("Q8 KV append: staging allocation failed");
        return QWN_CUDA_STATUS_OUT_OF_MEMORY;
    }
    const auto t0 = std::chrono::steady_clock::now();
    cudaError_t e = cudaMemcpyAsync(c->d_k, r->host_key, (size_t)k->channels * 4, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(c->d_v, r->host_value, (size_t)k->channels * 4, cudaMemcpyHostToDevice, c->stream);
    uint64_t launches = 0;
    if (e == cudaSuccess) e = cudaEventRecord(c->ev0, c->stream);
    if (e == cudaSuccess) {
        if (k->paged) {
            Pool *p = pool_from(&k->pool);
            e = launch_seq_append(p, 1, nullptr, nullptr, c->stream);
            if (e == cudaSuccess) e = launch_append(p, 0, 1, nullptr, c->d_k, c->d_v, c->stream);
            launches = 2;
        } else {
            const uint32_t warps = k->blocks;
            q8_quantize_generic<<<(warps + 3) / 4, 128, 0, c->stream>>>(
                c->d_k, k->key + (size_t)k->tokens * k->channels, k->key_scales + (size_t)k->tokens * k->blocks,
                k->channels, k->blocks);
            q8_quantize_generic<<<(warps + 3) / 4, 128, 0, c->stream>>>(
                c->d_v, k->value + (size_t)k->tokens * k->channels,
                k->value_scales + (size_t)k->tokens * k->blocks, k->channels, k->blocks);
            count_launch(2);
            e = cudaGetLastError();
            launches = 2;
        }
    }
    if (e == cudaSuccess) e = cudaEventRecord(c->ev1, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) { set_cuda_error("Q8 KV quantize", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    if (k->paged) {
        uint32_t st = 0;
        qwn_kv_pool_check(&k->pool, &st);
        if (st) { set_error("Q8 KV append: device status error"); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    }
    float ms = 0.f;
    cudaEventElapsedTime(&ms, c->ev0, c->ev1);
    k->tokens++;
    c->tel.kv_cache_kernel_count += launches;
    c->tel.kv_cache_upload_bytes += (uint64_t)k->channels * 8u;
    c->tel.kv_cache_kernel_ms += ms;
    c->tel.kv_cache_transfer_ms +=
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count() - ms;
    std::snprintf(c->tel.kv_cache_kernel_type, sizeof(c->tel.kv_cache_kernel_type),
                  k->paged ? "q8-paged-b200" : "q8-generic-b200");
    if (tel) *tel = c->tel;
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_cuda_abi_kv_cache_attention(QwnCudaContextHandle *h, const QwnCudaKvAttentionRequest *r,
                                                     QwnCudaTelemetry *tel) {
    Context *c = ctx_from(h);
    KvCache *k = r ? kv_from(r->cache) : nullptr;
    if (!c || !r || !k || !header_ok(r->header, sizeof(*r)) || !r->host_query || !r->host_output ||
        r->query_heads == 0 || r->kv_heads != k->kv_heads || r->head_dim != k->head_dim ||
        r->position >= k->tokens) {
        set_error("invalid Q8 KV-cache attention request");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    // Query head h reads kv head (h * kv_heads) / query_heads, as in the
    // reference (c/cuda/qwn_hypervsq2_cuda_abi.cu:184).  The paged kernel
    // takes G query heads per kv head; when the map is not uniform, the rows
    // go through a padded kv_heads x G' layout (G' = the largest group, the
    // spare rows zero and their outputs dropped).
    const uint32_t Hq = r->query_heads, HK = r->kv_heads;
    const bool uniform = Hq % HK == 0;
    uint32_t Gp = uniform ? Hq / HK : 0;
    std::vector<uint32_t> slot;  // padded row of query head h (non-uniform map)
    if (!uniform) {
        std::vector<uint32_t> cnt(HK, 0);
        slot.resize(Hq);
        for (uint32_t h = 0; h < Hq; h++) {
            const uint32_t kv = (uint32_t)(((uint64_t)h * HK) / Hq);
            slot[h] = cnt[kv]++;  // index within its group; the group base is added below
        }
        for (uint32_t j = 0; j < HK; j++) Gp = cnt[j] > Gp ? cnt[j] : Gp;
        for (uint32_t h = 0; h < Hq; h++) slot[h] += (uint32_t)(((uint64_t)h * HK) / Hq) * Gp;
    }
    if (k->paged && Gp > (uint32_t)kMaxGroup) {
        set_error("paged Q8 attention takes at most 8 query heads per kv head");
        return QWN_CUDA_STATUS_UNSUPPORTED;
    }
    const bool padded = k->paged && !uniform;
    std::lock_guard<std::mutex> lk(g_abi_mu);
    cudaSetDevice(c->device);
    const uint32_t Hrows = padded ? HK * Gp : Hq;  // query rows the device sees
    const size_t qn = (size_t)Hrows * k->head_dim;
    const float *q_src = r->host_query;
    if (padded) {
        c->pad_q.assign(qn, 0.f);
        c->pad_o.resize(qn);
        for (uint32_t h = 0; h < Hq; h++)
            std::memcpy(&c->pad_q[(size_t)slot[h] * k->head_dim], r->host_query + (size_t)h * k->head_dim,
                        k->head_dim * sizeof(float));
        q_src = c->pad_q.data();
    }
    if (!grow((void **)&c->d_q, &c->q_cap, qn * 4) || !grow((void **)&c->d_o, &c->o_cap, qn * 4)) {
        set_error("Q8 KV attention: staging allocation failed");
        return QWN_CUDA_STATUS_OUT_OF_MEMORY;
    }
    float *d_o = c->d_o;
    const auto t0 = std::chrono::steady_clock::now();
    cudaError_t e = cudaMemcpyAsync(c->d_q, q_src, qn * 4, cudaMemcpyHostToDevice, c->stream);
    uint64_t launches = 0;
    if (e == cudaSuccess) e = cudaEventRecord(c->ev0, c->stream);
    if (e == cudaSuccess) {
        if (k->paged) {
            Pool *p = pool_from(&k->pool);
            AttnLaunch a{};
            a.layer = 0;
            a.num_seqs = 1;
            a.query_heads = Hrows;
            a.attend_limit = r->position + 1;
            a.query = c->d_q;
            a.output = d_o;
            a.scale = r->scale;
            e = launch_attention(p, a, c->stream);
            launches = 1;
        } else {
            const uint32_t ntok = r->position + 1, chunks = (ntok + kGenChunk - 1) / kGenChunk;
            if (!grow((void **)&k->part, &k->part_cap, (size_t)chunks * r->query_heads * (k->head_dim + 2) * 4))
                e = cudaErrorMemoryAllocation;
            if (e == cudaSuccess) {
                const size_t sm = (4 * (size_t)k->head_dim + 8) * 4;
                q8_attention_generic<<<dim3(r->query_heads, chunks), 128, sm, c->stream>>>(
                    k->key, k->value, k->key_scales, k->value_scales, c->d_q, k->part, r->query_heads,
                    r->kv_heads, k->head_dim, k->channels, k->blocks, ntok, r->scale * 1.4426950408889634f);
                merge_generic<<<r->query_heads, 128, 0, c->stream>>>(k->part, d_o, r->query_heads, k->head_dim,
                                                                    chunks);
                count_launch(2);
                e = cudaGetLastError();
                launches = 2;
            }
        }
    }
    if (e == cudaSuccess) e = cudaEventRecord(c->ev1, c->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(padded ? c->pad_o.data() : r->host_output, d_o, qn * 4, cudaMemcpyDeviceToHost,
                            c->stream);
    // the paged pool's status word, read on this stream (no device-wide sync)
    uint32_t st = 0;
    Pool *pp = k->paged ? pool_from(&k->pool) : nullptr;
    if (e == cudaSuccess && pp) e = cudaMemcpyAsync(&st, pp->status, sizeof(st), cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) { set_cuda_error("Q8 KV attention", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    if (st) {  // clear it, as qwn_kv_pool_check does, and fail this call
        cudaMemsetAsync(pp->status, 0, sizeof(uint32_t), c->stream);
        if (st & QWN_KV_STATUS_WAIT_TIMEOUT) cudaMemsetAsync(pp->counters, 0, sizeof(uint32_t) * counter_count(pp), c->stream);
        cudaStreamSynchronize(c->stream);
        set_error("Q8 KV attention: device status error");
        return QWN_CUDA_STATUS_RUNTIME_ERROR;
    }
    if (padded)
        for (uint32_t h = 0; h < Hq; h++)
            std::memcpy(r->host_output + (size_t)h * k->head_dim, &c->pad_o[(size_t)slot[h] * k->head_dim],
                        k->head_dim * sizeof(float));
    float ms = 0.f;
    cudaEventElapsedTime(&ms, c->ev0, c->ev1);
    c->tel.kv_cache_kernel_count += launches;
    c->tel.kv_cache_kernel_ms += ms;
    c->tel.kv_cache_transfer_ms +=
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count() - ms;
    std::snprintf(c->tel.kv_cache_kernel_type, sizeof(c->tel.kv_cache_kernel_type),
                  k->paged ? "q8-paged-b200" : "q8-generic-b200");
    if (tel) *tel = c->tel;
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_cuda_abi_kv_cache_reset(QwnCudaContextHandle *h, QwnCudaKvCacheHandle *kh) {
    Context *c = ctx_from(h);
    KvCache *k = kh ? kv_from(*kh) : nullptr;
    if (!c || !k) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lk(g_abi_mu);
    k->tokens = 0;
    if (k->paged) return qwn_kv_pool_reset(&k->pool);
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_cuda_abi_kv_cache_destroy(QwnCudaContextHandle *h, QwnCudaKvCacheHandle *kh) {
    Context *c = ctx_from(h);
    KvCache *k = kh ? kv_from(*kh) : nullptr;
    if (!c || !k) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lk(g_abi_mu);
    auto it = std::find(c->caches.begin(), c->caches.end(), k);
    if (it == c->caches.end()) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    cudaSetDevice(c->device);
    const uint64_t b = k->bytes;
    free_cache(k);
    c->caches.erase(it);
    c->resident -= std::min(c->resident, b);
    c->tel.kv_cache_resident_bytes -= std::min(c->tel.kv_cache_resident_bytes, b);
    kh->opaque = nullptr;
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_cuda_abi_hypervsq2_gemv(QwnCudaContextHandle *h, const QwnCudaGemmRequest *r,
                                                 QwnCudaTelemetry *tel) {
    Context *c = ctx_from(h);
    if (!c || !r || r->batch != 1) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lk(g_abi_mu);
    return gemv_execute(c, r, tel);
}

QWN_CUDA_ABI_API int qwn_cuda_abi_hypervsq2_gemm(QwnCudaContextHandle *h, const QwnCudaGemmRequest *r,
                                                 QwnCudaTelemetry *tel) {
    Context *c = ctx_from(h);
    if (!c) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lk(g_abi_mu);
    return gemv_execute(c, r, tel);
}

QWN_CUDA_ABI_API int qwn_cuda_abi_synchronize(QwnCudaContextHandle *h) {
    Context *c = ctx_from(h);
    if (!c) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    cudaError_t e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) { set_cuda_error("CUDA stream synchronize", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_cuda_abi_get_telemetry(QwnCudaContextHandle *h, QwnCudaTelemetry *tel) {
    Context *c = ctx_from(h);
    if (!c || !tel || !header_ok(tel->header, sizeof(*tel))) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    *tel = c->tel;
    return QWN_CUDA_STATUS_OK;
}

QWN_CUDA_ABI_API int qwn_cuda_abi_last_error(char *buf, uint32_t size) {
    if (!buf || size == 0) return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    std::snprintf(buf, size, "%s", last_error().c_str());
    return QWN_CUDA_STATUS_OK;
}

}  // extern "C"
