// Internal declarations shared by the qwn_cuda.so translation units.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>
#include <string>

#include "qwn_cuda_abi.h"
#include "qwn_kv_b200.h"

namespace qkv {

constexpr int kHeadDim = 128;
constexpr int kTileTokens = 16;
constexpr int kMaxGroup = 8;          // query heads per kv head handled by one warp
constexpr int kWarpsPerCta = 4;       // attention CTA = 4 independent warps
constexpr uint32_t kWaitLimit = 1u << 22;  // bounded mbarrier polls before giving up

// ----------------------------------------------------------------------------
// host-side error state and launch accounting
// ----------------------------------------------------------------------------
void set_error(const char *msg);
void set_cuda_error(const char *what, cudaError_t e);
std::string last_error();
extern std::atomic<uint64_t> g_launches;
inline void count_launch(uint64_t n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

inline bool header_ok(const QwnCudaAbiHeader &h, size_t expected) {
    return h.abi_version == QWN_CUDA_ABI_VERSION && h.struct_size >= expected;
}

inline size_t tile_bytes_of(uint32_t codec) {
    switch (codec) {
        case QWN_KV_CODEC_Q8_B64_F32: return 4352;
        case QWN_KV_CODEC_Q8_HEAD_F16: return 4160;
        case QWN_KV_CODEC_TQ35_G64: return 2048;
        case QWN_KV_CODEC_Q4_G32: return 2560;
        case QWN_KV_CODEC_F16: return 8192;
        default: return 0;
    }
}

// ----------------------------------------------------------------------------
// the pool (device state behind QwnKvPoolHandle)
// ----------------------------------------------------------------------------
struct Pool {
    int device = 0;
    uint32_t codec = 0, layers = 0, kv_heads = 0, page_tokens = 0, tiles_per_page = 0;
    uint32_t total_pages = 0, max_seqs = 0, max_pages_per_seq = 0, max_query_heads = 0;
    uint64_t perm_seed = 0;
    size_t tile_bytes = 0, page_bytes = 0, pool_bytes = 0, scratch_bytes = 0;
    cudaStream_t stream = nullptr;      // default stream of the pool
    cudaStream_t copy_stream = nullptr; // host-step copies in
    cudaStream_t out_stream = nullptr;  // host-step copies out (both copy directions at once)
    // device state
    uint8_t *pages = nullptr;
    int32_t *page_table = nullptr, *seq_lens = nullptr, *seq_pages = nullptr;
    int32_t *free_stack = nullptr, *free_top = nullptr;
    float *page_scores = nullptr;
    uint32_t *status = nullptr;
    // attention scratch
    float *partials = nullptr;          // [warps + segments][kPartialFloats]
    uint32_t *counters = nullptr;       // [segments] then [warps + segments] (merge groups)
    // per-step launch plans of the attention kernel: word 0 is the epoch that
    // every change of lengths or page tables increments, then kPlanWords per
    // warp (see kv_attention.cu)
    uint32_t *plans = nullptr;
    float2 *tile_mass = nullptr;        // [units][kMaxGroup] (u, m) per tile and row
    float2 *seg_ml = nullptr;           // [segments][kMaxGroup] final (m, l)
    uint8_t *evict_dead = nullptr;      // [max_seqs][max_pages_per_seq]
    int32_t *evict_count = nullptr;     // [max_seqs]
    int32_t *ident = nullptr;           // [max_seqs] 0..max_seqs-1
    uint32_t attn_ctas = 0, attn_ctas2 = 0, attn_warps = 0;  // grids of the 1- and 2-head-group kernels
    uint64_t max_units = 0, max_segments = 0;
    // host-step staging
    float *stage_q = nullptr, *stage_k = nullptr, *stage_v = nullptr, *stage_o = nullptr;
    size_t stage_q_elems = 0, stage_kv_elems = 0;
    cudaEvent_t *layer_in_ev = nullptr, *layer_out_ev = nullptr;
    uint32_t layer_events = 0;
    cudaEvent_t step_t0 = nullptr, step_t1 = nullptr;  // host-step timing (created on first use)
    uint32_t *status_host = nullptr;                    // pinned copy of the status word for the host step
    std::mutex mu;
    // the pool's last attention launch, for the next launch's early start
    // (AttnArgs::early): its stream, layer and output range
    struct LastAttention {
        bool valid = false;
        bool recorded = false;  // it (re)wrote the plan records
        cudaStream_t stream = nullptr;
        uint32_t layer = 0;
        uintptr_t out_lo = 0, out_hi = 0;
    } last_attn;
    // host mirror of the plan records' key: plan_valid is cleared by every
    // launch that changes lengths or tables (the device epoch moves)
    bool plan_valid = false;
    uint32_t plan_key[6] = {};
    std::mutex last_mu;
};
// a launch that changes lengths or page tables (the plans' epoch) was queued
inline void plans_invalidated(Pool *p) {
    std::lock_guard<std::mutex> lk(p->last_mu);
    p->plan_valid = false;
}

constexpr int kPartialFloats = kMaxGroup * kHeadDim + 2 * kMaxGroup;  // room for o[G][128], m[G], l[G]
// launch plans: a 32-word header (word 0 = epoch), then kPlanWords per warp
constexpr uint32_t kPlanWords = 128;
inline size_t plan_words(const Pool *p) { return 32 + (size_t)p->attn_warps * kPlanWords; }
// merge counters of a pool: one per segment, then one per partial slot
// (the counter of a merge group sits at its first part's slot index)
inline size_t counter_count(const Pool *p) { return (size_t)p->max_segments * 2 + p->attn_warps; }

inline Pool *pool_from(const QwnKvPoolHandle *h) {
    if (!h || !header_ok(h->header, sizeof(*h)) || !h->opaque) return nullptr;
    return static_cast<Pool *>(h->opaque);
}
// NULL is the CUDA default stream of the calling thread (as for any CUDA
// API), so callers on the default stream -- torch's current stream by
// default -- are ordered with this library's launches.
inline cudaStream_t stream_of(Pool *, void *s) { return static_cast<cudaStream_t>(s); }

// launchers implemented in the .cu files (return cudaError_t of the launch)
cudaError_t launch_seq_append(Pool *p, uint32_t n, const int32_t *seq_ids, const int32_t *counts,
                              cudaStream_t s);
cudaError_t launch_append(Pool *p, uint32_t layer, uint32_t n, const int32_t *seq_ids,
                          const float *key, const float *value, cudaStream_t s);
cudaError_t launch_store_tokens(Pool *p, int32_t seq, uint32_t layer, uint32_t first,
                                uint32_t n, const float *key, const float *value, cudaStream_t s);
cudaError_t launch_prefill_synthetic(Pool *p, uint32_t n, const int32_t *seq_ids_dev,
                                     uint32_t max_len, uint64_t seed, const uint8_t *mask_dev,
                                     cudaStream_t s);
cudaError_t launch_generate(float *out, uint32_t rows, uint32_t width, uint32_t kind,
                            uint64_t seed, uint32_t layer, const int32_t *seq_ids,
                            const int32_t *pos, const uint8_t *mask, cudaStream_t s);
struct AttnLaunch {
    uint32_t layer, num_seqs, query_heads, attend_limit;
    const int32_t *seq_ids;
    const float *query;
    float *output;
    float scale;
    float *page_mass;
    // partial mode (split-KV across devices)
    float *part_m, *part_l, *part_o;
    uint32_t t_begin, t_end;
    // fused quantize-on-append of the newest token ([num_seqs][kv_heads][128])
    const float *new_k, *new_v;
    // split-KV over ranks: exchange of the segments' partials, merged in-kernel
    const QwnKvPeerSet *peers;
    uint32_t epoch;
};
cudaError_t launch_attention(Pool *p, const AttnLaunch &a, cudaStream_t s);
cudaError_t launch_merge(uint32_t parts, uint32_t rows, const float *m, const float *l,
                         const float *o, float *out, size_t stride_ml, size_t stride_o, cudaStream_t s);
cudaError_t launch_evict(Pool *p, uint32_t n, const int32_t *seq_ids, const float *mass,
                         const uint8_t *flags, uint32_t budget, cudaStream_t s);
cudaError_t launch_pool_init_state(Pool *p, cudaStream_t s);
cudaError_t launch_page_mass(Pool *p, uint32_t n, const int32_t *seq_ids, uint32_t query_heads,
                             float *page_mass, cudaStream_t s);
cudaError_t launch_fill_f32(float *p, float v, size_t n, cudaStream_t s);

}  // namespace qkv

// ============================================================================
// device helpers
// ============================================================================
#ifdef __CUDACC__
namespace qkv {

__device__ __forceinline__ uint64_t mix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t gen_key(uint64_t seed, uint32_t kind, uint32_t seq,
                                            uint32_t layer) {
    uint64_t stream = ((uint64_t)kind << 56) ^ ((uint64_t)layer << 32) ^ (uint64_t)seq;
    return mix64(seed ^ mix64(stream));
}
// Irwin-Hall(12) of 16-bit uniforms; exact integer sum, exact fp32 result
__device__ __forceinline__ float gen_normal(uint64_t key, uint64_t index) {
    int64_t sum = 0;
#pragma unroll
    for (int j = 0; j < 3; j++) {
        uint64_t h = mix64(key + 3ull * index + (uint64_t)j);
        sum += (int64_t)(h & 0xFFFF) + (int64_t)((h >> 16) & 0xFFFF) +
               (int64_t)((h >> 32) & 0xFFFF) + (int64_t)(h >> 48);
    }
    return (float)(sum - 393210) * (1.0f / 65536.0f);
}

__device__ __forceinline__ void latch(uint32_t *status, uint32_t bits) {
    if (status) atomicOr(status, bits);
}

// fp16 with the reference's truncating rounding (c/qwanto_turboquant.c:106-120)
__device__ __forceinline__ uint16_t tq_f32_to_f16(float f) {
    uint32_t x = __float_as_uint(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    int32_t e = (int32_t)((x >> 23) & 0xFF) - 127 + 15;
    uint32_t mant = x & 0x7FFFFFu;
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant = (mant | 0x800000u) >> (1 - e);
        return (uint16_t)(sign | (mant >> 13));
    }
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | ((uint32_t)e << 10) | (mant >> 13));
}
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// ---- PTX wrappers ----------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ uint32_t mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok;
}
// bounded wait: returns false after kWaitLimit unsuccessful polls
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
    for (uint32_t it = 0; it < kWaitLimit; ++it)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t *p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
// 1-D bulk copy global -> this CTA's shared memory, completion counted on an mbarrier
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
template <uint32_t LUT>
__device__ __forceinline__ uint32_t lop3(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(d) : "r"(a), "r"(b), "r"(c), "n"(LUT));
    return d;
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}
// D = A(16x16 f16, row) * B(16x8 f16, col) + D, fp32 accumulators
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// biased int8 (code+128) bytes 0,1 / 2,3 of w -> exact f16 pairs
// integer tensor-core product: D(16x8 s32) += A(16x32 u8, row) x B(32x8 s8, col)
__device__ __forceinline__ void imma16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D = A x B with a zero accumulator input
__device__ __forceinline__ void imma16832_z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
// four 8x8 matrices of 16-bit values from shared memory (lane l gives the
// address of row l&7 of matrix l>>3); .trans delivers them transposed
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void *row) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(row)));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void *row) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(row)));
}
// fp16 tile element (t, d) of the K (is_value 0) or V half: rows of 256
// bytes, 16-byte chunk d>>3 at position (d>>3) xor (t&7)
__device__ __forceinline__ uint32_t f16_off(int is_value, int t, int d) {
    return (uint32_t)(is_value * 4096 + t * 256 + ((((d >> 3) ^ (t & 7))) << 4) + (d & 7) * 2);
}
// transpose of an 8x8 matrix of 16-bit values held one row pair per lane
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}
// exact int32 -> fp32 for |x| < 2^22: the integer is added to the mantissa of
// 1.5*2^23 (whose bit pattern is 0x4B400000) and that float is subtracted
__device__ __forceinline__ float small_int_to_float(int x, uint32_t magic) {
    return __uint_as_float((uint32_t)x + magic) - 12582912.0f;
}
__device__ __forceinline__ void u8x4_to_h2x2(uint32_t w, uint32_t &b01, uint32_t &b23) {
    const uint32_t k1152 = 0x64806480u;  // 1152.0 in both halves
    b01 = hsub2(prmt(w, 0x64646464u, 0x4140u), k1152);
    b23 = hsub2(prmt(w, 0x64646464u, 0x4342u), k1152);
}
// 8 nibbles of w -> four exact f16 pairs (n0,n4) (n1,n5) (n2,n6) (n3,n7)
__device__ __forceinline__ void nib8_to_h2x4(uint32_t w, uint32_t (&r)[4]) {
    const uint32_t k1024 = 0x64006400u, k64 = 0x54005400u;
    uint32_t ws = w >> 8;
    r[0] = hsub2(lop3<0xEA>(w, 0x000F000Fu, k1024), k1024);
    r[1] = hsub2(lop3<0xEA>(w, 0x00F000F0u, k64), k64);
    r[2] = hsub2(lop3<0xEA>(ws, 0x000F000Fu, k1024), k1024);
    r[3] = hsub2(lop3<0xEA>(ws, 0x00F000F0u, k64), k64);
}
// 3-bit fields in the low bits of each nibble (mask 7) -> f16 pairs
__device__ __forceinline__ void nib8_low3_to_h2x4(uint32_t w, uint32_t (&r)[4]) {
    const uint32_t k1024 = 0x64006400u, k64 = 0x54005400u;
    uint32_t ws = w >> 8;
    r[0] = hsub2(lop3<0xEA>(w, 0x00070007u, k1024), k1024);
    r[1] = hsub2(lop3<0xEA>(w, 0x00700070u, k64), k64);
    r[2] = hsub2(lop3<0xEA>(ws, 0x00070007u, k1024), k1024);
    r[3] = hsub2(lop3<0xEA>(ws, 0x00700070u, k64), k64);
}

// ---- paged tile layout (head_dim 128, 16 tokens per tile) ------------------
// int8 K: token rows of 128 bytes, 16-byte chunk (d>>4) at (d>>4) ^ ((t&1)<<2)
__device__ __forceinline__ uint32_t k8_off(int t, int d) {
    return (uint32_t)(t * 128 + (((d >> 4) ^ ((t & 1) << 2)) << 4) + (d & 15));
}
// int8 V: the PV A operand (dims x tokens); lane ((r&7)<<2)|((t&7)>>1) of
// m-block d>>4, 8 bytes per m-block in the lane's 64 (16-byte chunks swizzled)
__device__ __forceinline__ uint32_t v8_off(int t, int d) {
    const int mb = d >> 4, r = d & 15, lane = ((r & 7) << 2) | ((t & 7) >> 1);
    const int chunk = (mb >> 1) ^ ((lane >> 1) & 3);
    return (uint32_t)(2048 + lane * 64 + chunk * 16 + 8 * (mb & 1) + 4 * (t >> 3) + 2 * (r >> 3) + (t & 1));
}
// int8 scales: tokens t and t+8 adjacent
__device__ __forceinline__ uint32_t s16_off(int t) { return (uint32_t)(4 * (t & 7) + 2 * (t >> 3)); }
__device__ __forceinline__ uint32_t s32_off(int t, int x) { return (uint32_t)(16 * (t & 7) + 8 * x + 4 * (t >> 3)); }

}  // namespace qkv
#endif
