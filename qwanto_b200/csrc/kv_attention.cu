// GQA decode attention over the quantized paged pool, split-KV.
//
// Work decomposition ("stream-K" over tiles): the units of work are
// (sequence, kv head, 16-token tile).  A persistent grid of warps splits the
// T units of the batch into W equal contiguous ranges, so every warp streams
// the same number of tiles whatever the mix of context lengths.  A warp
// keeps the online-softmax state (m, l, o) of the segment (sequence, kv head)
// it is in; at a segment boundary it either writes the final output (when it
// covered the whole segment) or a partial, and the last warp to finish a
// segment merges the partials in warp order (deterministic).
//
// Each warp owns a private pipeline of kStages shared-memory stages filled by
// 1-D cp.async.bulk copies (no multicast) completed on per-stage mbarriers.
// The tile layout in HBM is arranged so that each lane's mma.sync fragments
// are a few conflict-free 128-bit shared loads.  Dequantisation happens in
// registers: biased int8 / 4-bit codes become exact f16 by byte permutes, the
// query is split hi+lo into f16 rows 0-7 / 8-15 of the m16n8k16 A operand (the
// GQA group of G<=8 query heads uses rows 0..G-1), scales and zero points are
// applied in fp32 outside the MMA, so the result tracks the reference's fp32
// arithmetic (c/qwanto_turboquant.c:648-705, :218-288) within ~1e-6.
//
// When the caller passes the newest token's K/V, the warp that owns the last
// tile of a segment quantizes and stores that token into the page (the
// append of c/qwanto_turboquant.c:632-646) just before it issues the bulk
// copy of that tile, so append and attention are one launch.
#include "kv_internal.cuh"
#include "kv_store.cuh"

#include <float.h>

namespace qkv {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNuFloor = 7.888609052210118e-31f;  // 2^-100
constexpr float kNuHeadroom = 16384.0f;            // rescale only when a scale exceeds nu * 2^14

struct AttnArgs {
    const uint8_t *pages;
    uint64_t page_bytes;
    uint32_t tile_bytes, tpp, page_tokens;
    const int32_t *page_table;
    uint32_t mp, total_pages, max_seqs;
    const int32_t *seq_lens;
    const int32_t *seq_ids;
    uint32_t num_seqs, kv_heads, group, layer;
    uint32_t attend_limit, t_begin, t_end;
    const float *query;
    float *output;
    float scale_log2;
    float *partials;
    uint32_t *counters;
    float2 *tile_mass;
    float2 *seg_ml;
    float *part_m, *part_l, *part_o;  // non-null: export unnormalised (m, l, o)
    const float *new_k, *new_v;       // non-null: fused append of the newest token
    uint32_t *status;
};

__device__ __forceinline__ float pow2ceil(float x) {
    uint32_t b = __float_as_uint(x);
    if (b & 0x7FFFFFu) b = (b & 0x7F800000u) + 0x00800000u;
    return __uint_as_float(b);
}
__device__ __forceinline__ float2 h2x2f(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2 *>(&w));
}

// A-operand rows gid (hi) and gid+8 (lo) for four values at k-positions
// (2tig, 2tig+1) and (2tig+8, 2tig+9); packed conversions
__device__ __forceinline__ void make_a(const float (&v)[4], uint32_t (&a)[4]) {
    const __half2 h01 = __floats2half2_rn(v[0], v[1]);
    const __half2 h23 = __floats2half2_rn(v[2], v[3]);
    const float2 b01 = __half22float2(h01), b23 = __half22float2(h23);
    const __half2 l01 = __floats2half2_rn(v[0] - b01.x, v[1] - b01.y);
    const __half2 l23 = __floats2half2_rn(v[2] - b23.x, v[3] - b23.y);
    a[0] = *reinterpret_cast<const uint32_t *>(&h01);
    a[1] = *reinterpret_cast<const uint32_t *>(&l01);
    a[2] = *reinterpret_cast<const uint32_t *>(&h23);
    a[3] = *reinterpret_cast<const uint32_t *>(&l23);
}

// ---------------------------------------------------------------------------
// softmax bookkeeping shared by the codecs.  s[i]: base-2 scores of this
// lane's four tokens (4tig+i) for row gid, -inf when masked.  Returns the
// probabilities p[i] after rescaling the accumulators when the max grows.
// ---------------------------------------------------------------------------
template <class Acc>
__device__ __forceinline__ void online_softmax(const float (&s)[4], float (&p)[4], float &m, float &l,
                                               Acc &acc) {
    float tmax = fmaxf(fmaxf(s[0], s[1]), fmaxf(s[2], s[3]));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
    const float m_new = fmaxf(m, tmax);
    if (__any_sync(0xffffffffu, m_new > m)) {
        const float alpha = ex2(m - m_new);
        l *= alpha;
        acc.rescale_all(alpha);
        m = m_new;
    }
#pragma unroll
    for (int i = 0; i < 4; i++) p[i] = ex2(s[i] - m);
    l += (p[0] + p[1]) + (p[2] + p[3]);
}

// Value normaliser: nu is a power of two set from the first tile of the
// segment; p*scale/nu is then an f16 of moderate size.  It is raised (with
// an exact power-of-two rescale of the accumulators) only when a later scale
// exceeds nu*2^14, which keeps p*scale/nu < 2^15 inside the f16 range.
template <class Acc>
__device__ __forceinline__ void update_nu(const float (&vs)[4], int x, Acc &acc) {
    const float lmax = fmaxf(fmaxf(vs[0], vs[1]), fmaxf(vs[2], vs[3]));
    const bool first = acc.nu[x] == 0.f;
    if (__any_sync(0xffffffffu, first || lmax > acc.nu[x] * kNuHeadroom)) {
        float vmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, 1));
        vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 2));
        const float nn = fmaxf(pow2ceil(vmax), kNuFloor);
        if (first) {
            acc.nu[x] = nn;
        } else if (nn > acc.nu[x]) {
            acc.rescale_part(x, acc.nu[x] / nn);
            acc.nu[x] = nn;
        }
        acc.inv_nu[x] = 1.0f / acc.nu[x];
    }
}

// ---------------------------------------------------------------------------
// codecs
// ---------------------------------------------------------------------------
template <int CODEC> struct Codec;

// int8 codes, per-token-head fp16 scale (4160-byte tile)
template <> struct Codec<QWN_KV_CODEC_Q8_HEAD_F16> {
    static constexpr int kBytes = 4160, kStages = 4, kNu = 1;
    struct Frag { uint32_t a[8][4]; };
    struct Acc {
        float o[16][4];
        float nu[kNu], inv_nu[kNu];
        __device__ void reset() {
#pragma unroll
            for (int j = 0; j < 16; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
            nu[0] = 0.f; inv_nu[0] = 0.f;
        }
        __device__ void rescale_all(float f) {
#pragma unroll
            for (int j = 0; j < 16; j++) { o[j][0] *= f; o[j][1] *= f; o[j][2] *= f; o[j][3] *= f; }
        }
        __device__ void rescale_part(int, float f) { rescale_all(f); }
    };
    __device__ static int dim_of(int j, int tig, int c) { return 8 * j + 2 * tig + c; }
    // k-step s covers dims 64(s>>2) + 16tig + 4(s&3) + {0,1 | 2,3}
    __device__ static void load_q(Frag &f, const float *q, int tig) {
#pragma unroll
        for (int s = 0; s < 8; s++) {
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (q) {
                const float4 x = *reinterpret_cast<const float4 *>(q + 64 * (s >> 2) + 16 * tig + 4 * (s & 3));
                v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
            }
            make_a(v, f.a[s]);
        }
    }
    __device__ static float out_value(const Acc &acc, int j, int c, float) {
        return (acc.o[j][c] + acc.o[j][c + 2]) * acc.nu[0];
    }
    // K: per half h (token columns), two accumulator chains (even / odd
    // k-steps) so consecutive MMAs are independent
    __device__ static void qk(const uint8_t *tile, const Frag &f, float (&raw)[4]) {
        const int lane = threadIdx.x & 31, sw = (lane >> 2) & 1;
        const uint2 ksr = *reinterpret_cast<const uint2 *>(tile + 4096 + 8 * (lane & 3));
        const float2 k01 = h2x2f(ksr.x), k23 = h2x2f(ksr.y);
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint4 *kp = reinterpret_cast<const uint4 *>(tile + h * 1024 + lane * 32);
            const uint4 x0 = kp[sw], x1 = kp[sw ^ 1];
            const uint32_t w[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            float ce[4] = {0.f, 0.f, 0.f, 0.f}, co[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int st = 0; st < 8; st += 2) {
                uint32_t b0, b1;
                u8x4_to_h2x2(w[st], b0, b1);
                mma16816(ce, f.a[st], b0, b1);
                u8x4_to_h2x2(w[st + 1], b0, b1);
                mma16816(co, f.a[st + 1], b0, b1);
            }
            const float sa = h ? k23.x : k01.x, sb = h ? k23.y : k01.y;
            raw[2 * h] = ((ce[0] + co[0]) + (ce[2] + co[2])) * sa;
            raw[2 * h + 1] = ((ce[1] + co[1]) + (ce[3] + co[3])) * sb;
        }
    }
    __device__ static void pv(const uint8_t *tile, Acc &acc, const float (&p)[4], const bool (&ok)[4]) {
        const int lane = threadIdx.x & 31, tig = lane & 3;
        const uint2 vsr = *reinterpret_cast<const uint2 *>(tile + 4128 + 8 * tig);
        const float2 v01 = h2x2f(vsr.x), v23 = h2x2f(vsr.y);
        float vs[4] = {v01.x, v01.y, v23.x, v23.y};
#pragma unroll
        for (int i = 0; i < 4; i++) vs[i] = ok[i] ? vs[i] : 0.f;
        update_nu(vs, 0, acc);
        float pt[4];
#pragma unroll
        for (int i = 0; i < 4; i++) pt[i] = p[i] * vs[i] * acc.inv_nu[0];
        uint32_t a[4];
        make_a(pt, a);
        const uint8_t *vt = tile + 2048 + lane * 64;
        const int sw = (lane >> 1) & 3;
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const uint4 c = *reinterpret_cast<const uint4 *>(vt + ((q ^ sw) << 4));
            const uint32_t wv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
            for (int r = 0; r < 4; r++) {
                uint32_t b0, b1;
                u8x4_to_h2x2(wv[r], b0, b1);
                mma16816(acc.o[4 * q + r], a, b0, b1);
            }
        }
    }
};

// int8 codes, fp32 scale per 64 channels: the reference Q8 (4352-byte tile)
template <> struct Codec<QWN_KV_CODEC_Q8_B64_F32> {
    static constexpr int kBytes = 4352, kStages = 4, kNu = 2;
    using Frag = Codec<QWN_KV_CODEC_Q8_HEAD_F16>::Frag;
    struct Acc {
        float o[16][4];
        float nu[kNu], inv_nu[kNu];
        __device__ void reset() {
#pragma unroll
            for (int j = 0; j < 16; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
            nu[0] = nu[1] = 0.f; inv_nu[0] = inv_nu[1] = 0.f;
        }
        __device__ void rescale_all(float f) {
#pragma unroll
            for (int j = 0; j < 16; j++) { o[j][0] *= f; o[j][1] *= f; o[j][2] *= f; o[j][3] *= f; }
        }
        __device__ void rescale_part(int x, float f) {
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int jj = 8 * x + j;
                o[jj][0] *= f; o[jj][1] *= f; o[jj][2] *= f; o[jj][3] *= f;
            }
        }
    };
    __device__ static int dim_of(int j, int tig, int c) { return 8 * j + 2 * tig + c; }
    __device__ static void load_q(Frag &f, const float *q, int tig) {
        Codec<QWN_KV_CODEC_Q8_HEAD_F16>::load_q(f, q, tig);
    }
    __device__ static float out_value(const Acc &acc, int j, int c, float) {
        return (acc.o[j][c] + acc.o[j][c + 2]) * acc.nu[j >> 3];
    }
    // k-steps 0-3 cover dims 0..63 (scale 0), 4-7 dims 64..127 (scale 1)
    __device__ static void qk(const uint8_t *tile, const Frag &f, float (&raw)[4]) {
        const int lane = threadIdx.x & 31, sw = (lane >> 2) & 1, tig = lane & 3;
        const float4 ka = *reinterpret_cast<const float4 *>(tile + 4096 + 16 * tig);
        const float4 kb = *reinterpret_cast<const float4 *>(tile + 4096 + 64 + 16 * tig);
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint4 *kp = reinterpret_cast<const uint4 *>(tile + h * 1024 + lane * 32);
            const uint4 x0 = kp[sw], x1 = kp[sw ^ 1];
            const uint32_t w[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            float ca[4] = {0.f, 0.f, 0.f, 0.f}, cb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int st = 0; st < 4; st++) {
                uint32_t b0, b1;
                u8x4_to_h2x2(w[st], b0, b1);
                mma16816(ca, f.a[st], b0, b1);
                u8x4_to_h2x2(w[st + 4], b0, b1);
                mma16816(cb, f.a[st + 4], b0, b1);
            }
            const float sa0 = h ? ka.z : ka.x, sa1 = h ? ka.w : ka.y;
            const float sb0 = h ? kb.z : kb.x, sb1 = h ? kb.w : kb.y;
            raw[2 * h] = (ca[0] + ca[2]) * sa0 + (cb[0] + cb[2]) * sb0;
            raw[2 * h + 1] = (ca[1] + ca[3]) * sa1 + (cb[1] + cb[3]) * sb1;
        }
    }
    __device__ static void pv(const uint8_t *tile, Acc &acc, const float (&p)[4], const bool (&ok)[4]) {
        const int lane = threadIdx.x & 31, tig = lane & 3;
        uint32_t a[2][4];
#pragma unroll
        for (int x = 0; x < 2; x++) {
            const float4 v4 = *reinterpret_cast<const float4 *>(tile + 4224 + 64 * x + 16 * tig);
            float vs[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
            for (int i = 0; i < 4; i++) vs[i] = ok[i] ? vs[i] : 0.f;
            update_nu(vs, x, acc);
            float pt[4];
#pragma unroll
            for (int i = 0; i < 4; i++) pt[i] = p[i] * vs[i] * acc.inv_nu[x];
            make_a(pt, a[x]);
        }
        const uint8_t *vt = tile + 2048 + lane * 64;
        const int sw = (lane >> 1) & 3;
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const uint4 c = *reinterpret_cast<const uint4 *>(vt + ((q ^ sw) << 4));
            const uint32_t wv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
            for (int r = 0; r < 4; r++) {
                uint32_t b0, b1;
                u8x4_to_h2x2(wv[r], b0, b1);
                mma16816(acc.o[4 * q + r], a[q >> 1], b0, b1);
            }
        }
    }
};

// 4-bit codes, groups of 32 with fp16 range + fp16 min (2560-byte tile)
template <> struct Codec<QWN_KV_CODEC_Q4_G32> {
    static constexpr int kBytes = 2560, kStages = 6, kNu = 4;
    struct Frag { uint32_t a[8][4]; float qsum[4]; };
    struct Acc {
        float o[16][4];
        float z[4];  // sum_t p_t * min_t,g (this lane's tokens, row gid)
        float nu[kNu], inv_nu[kNu];
        __device__ void reset() {
#pragma unroll
            for (int j = 0; j < 16; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
#pragma unroll
            for (int g = 0; g < 4; g++) { z[g] = 0.f; nu[g] = 0.f; inv_nu[g] = 0.f; }
        }
        __device__ void rescale_all(float f) {
#pragma unroll
            for (int j = 0; j < 16; j++) { o[j][0] *= f; o[j][1] *= f; o[j][2] *= f; o[j][3] *= f; }
#pragma unroll
            for (int g = 0; g < 4; g++) z[g] *= f;
        }
        __device__ void rescale_part(int g, float f) {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int jj = 4 * g + j;
                o[jj][0] *= f; o[jj][1] *= f; o[jj][2] *= f; o[jj][3] *= f;
            }
        }
    };
    __device__ static int dim_of(int j, int tig, int c) { return 8 * j + 2 * tig + c; }
    // k-step s: group g = s>>1, dims 32g + 16(s&1) + 4tig + {0,1 | 2,3}
    __device__ static void load_q(Frag &f, const float *q, int tig) {
#pragma unroll
        for (int g = 0; g < 4; g++) {
            float part = 0.f;
#pragma unroll
            for (int e = 0; e < 2; e++) {
                float v[4] = {0.f, 0.f, 0.f, 0.f};
                if (q) {
                    const float4 x = *reinterpret_cast<const float4 *>(q + 32 * g + 16 * e + 4 * tig);
                    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
                }
                part += (v[0] + v[1]) + (v[2] + v[3]);
                make_a(v, f.a[2 * g + e]);
            }
            part += __shfl_xor_sync(0xffffffffu, part, 1);
            part += __shfl_xor_sync(0xffffffffu, part, 2);
            f.qsum[g] = part;
        }
    }
    // z[] must be reduced across the four lanes of a row before this is used
    __device__ static float out_value(const Acc &acc, int j, int c, float zsum) {
        return (acc.o[j][c] + acc.o[j][c + 2]) * acc.nu[j >> 2] + zsum;
    }
    __device__ static void qk(const uint8_t *tile, const Frag &f, float (&raw)[4]) {
        const int lane = threadIdx.x & 31, tig = lane & 3;
        const uint4 kw0 = *reinterpret_cast<const uint4 *>(tile + lane * 16);
        const uint4 kw1 = *reinterpret_cast<const uint4 *>(tile + 512 + lane * 16);
        const uint32_t w0[4] = {kw0.x, kw0.y, kw0.z, kw0.w}, w1[4] = {kw1.x, kw1.y, kw1.z, kw1.w};
        raw[0] = raw[1] = raw[2] = raw[3] = 0.f;
#pragma unroll
        for (int g = 0; g < 4; g++) {
            float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t r[4], u[4];
            nib8_to_h2x4(w0[g], r);
            nib8_to_h2x4(w1[g], u);
            mma16816(c0, f.a[2 * g], r[0], r[1]);
            mma16816(c1, f.a[2 * g], u[0], u[1]);
            mma16816(c0, f.a[2 * g + 1], r[2], r[3]);
            mma16816(c1, f.a[2 * g + 1], u[2], u[3]);
            const uint4 kp = *reinterpret_cast<const uint4 *>(tile + 2048 + 64 * g + 16 * tig);
            const float2 p0 = h2x2f(kp.x), p1 = h2x2f(kp.y), p2 = h2x2f(kp.z), p3 = h2x2f(kp.w);
            const float zq = f.qsum[g];
            raw[0] += p0.x * (1.0f / 15.0f) * (c0[0] + c0[2]) + p0.y * zq;
            raw[1] += p1.x * (1.0f / 15.0f) * (c0[1] + c0[3]) + p1.y * zq;
            raw[2] += p2.x * (1.0f / 15.0f) * (c1[0] + c1[2]) + p2.y * zq;
            raw[3] += p3.x * (1.0f / 15.0f) * (c1[1] + c1[3]) + p3.y * zq;
        }
    }
    __device__ static void pv(const uint8_t *tile, Acc &acc, const float (&p)[4], const bool (&ok)[4]) {
        const int lane = threadIdx.x & 31, tig = lane & 3;
        uint32_t a[4][4];
#pragma unroll
        for (int g = 0; g < 4; g++) {
            const uint4 vp = *reinterpret_cast<const uint4 *>(tile + 2304 + 64 * g + 16 * tig);
            const float2 p0 = h2x2f(vp.x), p1 = h2x2f(vp.y), p2 = h2x2f(vp.z), p3 = h2x2f(vp.w);
            float vs[4] = {p0.x * (1.0f / 15.0f), p1.x * (1.0f / 15.0f), p2.x * (1.0f / 15.0f),
                           p3.x * (1.0f / 15.0f)};
            const float mn[4] = {p0.y, p1.y, p2.y, p3.y};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                vs[i] = ok[i] ? vs[i] : 0.f;
                acc.z[g] += ok[i] ? p[i] * mn[i] : 0.f;
            }
            update_nu(vs, g, acc);
            float pt[4];
#pragma unroll
            for (int i = 0; i < 4; i++) pt[i] = p[i] * vs[i] * acc.inv_nu[g];
            make_a(pt, a[g]);
        }
        const uint8_t *vt = tile + 1024 + lane * 32;
        const int sw = (lane >> 2) & 1;
#pragma unroll
        for (int cc = 0; cc < 2; cc++) {
            const uint4 c = *reinterpret_cast<const uint4 *>(vt + ((cc ^ sw) << 4));
            const uint32_t wv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const int wi = 4 * cc + r;  // n-tiles 2wi, 2wi+1 (group wi>>1)
                uint32_t b[4];
                nib8_to_h2x4(wv[r], b);
                mma16816(acc.o[2 * wi], a[wi >> 1], b[0], b[1]);
                mma16816(acc.o[2 * wi + 1], a[wi >> 1], b[2], b[3]);
            }
        }
    }
};

// one tile: scores, online softmax, P x V.  Returns the tile's probability
// mass of this lane's tokens (for eviction scores).
template <int CODEC>
__device__ __forceinline__ float tile_step(const uint8_t *tile, const typename Codec<CODEC>::Frag &f,
                                           typename Codec<CODEC>::Acc &acc, float &m, float &l, int t_lo,
                                           int t_hi, float scale_log2) {
    using CD = Codec<CODEC>;
    const int tig = threadIdx.x & 3;
    float raw[4];
    CD::qk(tile, f, raw);
    float s[4];
    bool ok[4];
    if (t_lo == 0 && t_hi == 16) {  // warp-uniform: full tile
#pragma unroll
        for (int i = 0; i < 4; i++) { s[i] = raw[i] * scale_log2; ok[i] = true; }
    } else {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int t = 4 * tig + i;
            ok[i] = t >= t_lo && t < t_hi;
            s[i] = ok[i] ? raw[i] * scale_log2 : -INFINITY;
        }
    }
    float p[4];
    online_softmax(s, p, m, l, acc);
    CD::pv(tile, acc, p, ok);
    return (p[0] + p[1]) + (p[2] + p[3]);
}

// ---------------------------------------------------------------------------
// batch geometry
// ---------------------------------------------------------------------------
struct Geo {
    int32_t seq, tok_lo, tok_hi;
    uint32_t tile0, ntiles;
};

__device__ __forceinline__ Geo geo_of(const AttnArgs &A, uint32_t i) {
    Geo g;
    g.seq = A.seq_ids ? A.seq_ids[i] : (int32_t)i;
    g.tok_lo = g.tok_hi = 0;
    g.tile0 = g.ntiles = 0;
    if (g.seq < 0 || (uint32_t)g.seq >= A.max_seqs) {
        latch(A.status, QWN_KV_STATUS_BAD_SEQUENCE);
        return g;
    }
    int32_t hi = A.seq_lens[g.seq];
    if (A.attend_limit && hi > (int32_t)A.attend_limit) hi = (int32_t)A.attend_limit;
    if (A.t_end && hi > (int32_t)A.t_end) hi = (int32_t)A.t_end;
    const int32_t lo = (int32_t)A.t_begin;
    if (hi > (int32_t)(A.mp * A.page_tokens)) {
        latch(A.status, QWN_KV_STATUS_BAD_LENGTH);
        hi = (int32_t)(A.mp * A.page_tokens);
    }
    if (hi > lo) {
        g.tok_lo = lo;
        g.tok_hi = hi;
        g.tile0 = (uint32_t)lo / 16u;
        g.ntiles = ((uint32_t)hi + 15u) / 16u - g.tile0;
    }
    return g;
}

// position of a unit: batch entry i, kv head h, tile within the entry
struct Walk {
    uint32_t i, h, tile;
    uint64_t seg_base;  // global unit index of (i, h, tile 0)
    Geo geo;
};

__device__ __forceinline__ void walk_next_segment(const AttnArgs &A, Walk &w) {
    w.seg_base += w.geo.ntiles;
    w.tile = 0;
    if (++w.h == A.kv_heads) {
        w.h = 0;
        do {
            ++w.i;
            if (w.i >= A.num_seqs) { w.geo.ntiles = 0; return; }
            w.geo = geo_of(A, w.i);
        } while (w.geo.ntiles == 0);
    }
}
__device__ __forceinline__ void walk_advance(const AttnArgs &A, Walk &w, uint32_t k) {
    while (k > 0) {
        const uint32_t rem = w.geo.ntiles - w.tile;
        if (k < rem) { w.tile += k; return; }
        k -= rem;
        walk_next_segment(A, w);
        if (w.i >= A.num_seqs) return;
    }
}
__device__ __forceinline__ const uint8_t *unit_addr(const AttnArgs &A, const Walk &w) {
    const uint32_t tg = w.geo.tile0 + w.tile;
    const uint32_t lp = tg / A.tpp, tin = tg % A.tpp;
    int32_t pg = -1;
    if (lp < A.mp) pg = A.page_table[(size_t)w.geo.seq * A.mp + lp];
    if (pg < 0 || (uint32_t)pg >= A.total_pages) {
        latch(A.status, QWN_KV_STATUS_BAD_PAGE);
        pg = 0;  // stay in bounds; the latched status marks the result invalid
    }
    return A.pages + (size_t)pg * A.page_bytes +
           ((size_t)(A.layer * A.kv_heads + w.h) * A.tpp + tin) * A.tile_bytes;
}

__device__ __forceinline__ uint32_t warp_incl_scan(uint32_t v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

// per-warp shared-memory window: sources of the next 32 units and, for the
// fused append, the segment whose newest token lives in that unit (-1: none)
struct WarpWindow {
    const uint8_t *src[32];
    int32_t append_seg[32];
};

// Fill the window with units [base, base+32) of this warp, lane L taking unit
// base+L, walking forward `skip` units from `from`.
__device__ __forceinline__ void fill_window(const AttnArgs &A, const Walk &from, uint32_t skip, uint64_t base,
                                            uint64_t u1, WarpWindow *win) {
    const int lane = threadIdx.x & 31;
    const uint8_t *src = nullptr;
    int32_t app = -1;
    if (base + lane < u1) {
        Walk t = from;
        walk_advance(A, t, skip + lane);
        src = unit_addr(A, t);
        if (A.new_k && t.tile + 1 == t.geo.ntiles) app = (int32_t)(t.i * A.kv_heads + t.h);
    }
    win->src[lane] = src;
    win->append_seg[lane] = app;
    __syncwarp();
}

// quantize and store the newest token of segment `seg` into `tile`
template <int CODEC>
__device__ __noinline__ void fused_append(const float *new_k, const float *new_v, const int32_t *seq_ids,
                                          const int32_t *seq_lens, uint32_t kv_heads, int32_t seg,
                                          const uint8_t *tile) {
    const int lane = threadIdx.x & 31;
    const uint32_t i = (uint32_t)seg / kv_heads, h = (uint32_t)seg % kv_heads;
    const int32_t seq = seq_ids ? seq_ids[i] : (int32_t)i;
    const int32_t pos = seq_lens[seq] - 1;
    const size_t row = ((size_t)i * kv_heads + h) * kHeadDim;
    const float4 k = reinterpret_cast<const float4 *>(new_k + row)[lane];
    const float4 v = reinterpret_cast<const float4 *>(new_v + row)[lane];
    store_token<CODEC>(const_cast<uint8_t *>(tile), pos & 15, k, v, lane);
    // the bulk copy that follows reads this tile through the async proxy
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __syncwarp();
}

// Merge the nparts partial slots of segment s_idx into its output rows
// (row0 = s_idx * G).  The slots were written by other warps, so every read
// is an L2 round trip; they are batched so that a handful of round trips
// cover a segment: lane pp % 32 reads (m, l) of part pp while all lanes
// already load the o rows of the first kBatch parts, and the remaining parts
// follow kBatch at a time.  GG >= G is the compile-time row count.
template <int GG>
__device__ __forceinline__ void merge_rows(const AttnArgs &A, uint32_t s_idx, uint32_t nparts, uint64_t Us,
                                           uint64_t T, uint64_t W) {
    constexpr int kBatch = 16 / GG;  // float4 loads in flight per lane
    const int lane = threadIdx.x & 31;
    const uint32_t G = A.group;
    const uint64_t wa = ((Us + 1) * W - 1) / T;
    auto slot_of = [&](uint32_t pp) -> const float * {
        const uint64_t w = T >= W ? wa + pp : ((Us + pp + 1) * W - 1) / T;
        return A.partials + (size_t)(w + s_idx) * kPartialFloats;
    };
    float M[GG], ls[GG];
    float4 acc[GG];
#pragma unroll
    for (int g = 0; g < GG; g++) { M[g] = -INFINITY; ls[g] = 0.f; acc[g] = make_float4(0.f, 0.f, 0.f, 0.f); }
    for (uint32_t c = 0; c < nparts; c += 32) {
        const uint32_t nq = nparts - c < 32u ? nparts - c : 32u;
        float m[GG], l[GG];
#pragma unroll
        for (int g = 0; g < GG; g++) { m[g] = -INFINITY; l[g] = 0.f; }
        if ((uint32_t)lane < nq) {
            const float *ml = slot_of(c + lane) + kMaxGroup * kHeadDim;
#pragma unroll
            for (int g = 0; g < GG; g++)
                if ((uint32_t)g < G) { m[g] = __ldcg(ml + g); l[g] = __ldcg(ml + kMaxGroup + g); }
        }
        float4 v[kBatch][GG];
        auto load_batch = [&](uint32_t q0) {
#pragma unroll
            for (int b = 0; b < kBatch; b++) {
                const float *sl = slot_of(c + q0 + b);
#pragma unroll
                for (int g = 0; g < GG; g++)
                    v[b][g] = (q0 + b < nq && (uint32_t)g < G)
                                  ? __ldcg(reinterpret_cast<const float4 *>(sl + g * kHeadDim) + lane)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        };
        load_batch(0);
        float w[GG];
#pragma unroll
        for (int g = 0; g < GG; g++) {
            float cm = m[g];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
            const float nm = fmaxf(M[g], cm);
            const float alpha = M[g] == -INFINITY ? 0.f : ex2(M[g] - nm);
            M[g] = nm;
            ls[g] *= alpha;
            acc[g].x *= alpha; acc[g].y *= alpha; acc[g].z *= alpha; acc[g].w *= alpha;
            w[g] = (uint32_t)lane < nq && (uint32_t)g < G ? ex2(m[g] - nm) : 0.f;
            ls[g] += l[g] * w[g];
        }
        for (uint32_t q0 = 0; q0 < nq; q0 += kBatch) {
            if (q0) load_batch(q0);
#pragma unroll
            for (int b = 0; b < kBatch; b++) {
#pragma unroll
                for (int g = 0; g < GG; g++) {
                    const float wg = __shfl_sync(0xffffffffu, w[g], (q0 + b) & 31);
                    acc[g].x += v[b][g].x * wg; acc[g].y += v[b][g].y * wg;
                    acc[g].z += v[b][g].z * wg; acc[g].w += v[b][g].w * wg;
                }
            }
        }
    }
    const size_t row0 = (size_t)s_idx * G;
#pragma unroll
    for (int g = 0; g < GG; g++) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ls[g] += __shfl_xor_sync(0xffffffffu, ls[g], o);
        if ((uint32_t)g >= G) continue;
        const size_t row = row0 + g;
        if (A.part_o) {
            reinterpret_cast<float4 *>(A.part_o + row * kHeadDim)[lane] = acc[g];
            if (lane == 0) { A.part_m[row] = M[g]; A.part_l[row] = ls[g]; }
        } else {
            const float inv = ls[g] > 0.f ? 1.0f / ls[g] : 0.f;
            reinterpret_cast<float4 *>(A.output + row * kHeadDim)[lane] =
                make_float4(acc[g].x * inv, acc[g].y * inv, acc[g].z * inv, acc[g].w * inv);
        }
        if (A.seg_ml && lane == 0) A.seg_ml[(size_t)s_idx * kMaxGroup + g] = make_float2(M[g], ls[g]);
    }
    if (lane == 0) A.counters[s_idx] = 0u;  // ready for the next launch
}

__device__ __forceinline__ void merge_segment(const AttnArgs &A, uint32_t s_idx, uint32_t nparts, uint64_t Us,
                                              uint64_t T, uint64_t W) {
    if (A.group <= 2) merge_rows<2>(A, s_idx, nparts, Us, T, W);
    else if (A.group <= 4) merge_rows<4>(A, s_idx, nparts, Us, T, W);
    else merge_rows<8>(A, s_idx, nparts, Us, T, W);
}

// End of a warp's share of segment s_idx (batch entry i, kv head h, first
// unit Us, ns units).  A warp that saw the whole segment writes the output;
// otherwise it writes its partial (m, l, o) to slot wid + s_idx and counts
// itself on the segment's counter.  Returns the number of parts when this
// warp arrived last and must merge them, else 0.  The merge itself runs after
// the warp's streaming loop, where the loop's registers are free.
template <int CODEC>
__device__ __forceinline__ uint32_t finish_segment(const AttnArgs &A, const typename Codec<CODEC>::Acc &acc,
                                                   float m, float l, uint32_t s_idx, uint64_t Us, uint64_t ns,
                                                   uint64_t T, uint64_t W, uint64_t wid) {
    using CD = Codec<CODEC>;
    const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
    const uint32_t G = A.group;
    // warps whose (non-empty) range meets the segment: warp of unit u is
    // ((u+1)W-1)/T.  With T >= W every warp between the first and the last
    // is non-empty; with T < W each unit is a warp of its own.
    const uint64_t wa = ((Us + 1) * W - 1) / T, wb = ((Us + ns) * W - 1) / T;
    const uint32_t nparts = T >= W ? (uint32_t)(wb - wa + 1) : (uint32_t)ns;
    float lr = l;
    lr += __shfl_xor_sync(0xffffffffu, lr, 1);
    lr += __shfl_xor_sync(0xffffffffu, lr, 2);
    float zs[4] = {0.f, 0.f, 0.f, 0.f};
    if constexpr (CODEC == QWN_KV_CODEC_Q4_G32) {
#pragma unroll
        for (int g = 0; g < 4; g++) {
            float z = acc.z[g];
            z += __shfl_xor_sync(0xffffffffu, z, 1);
            z += __shfl_xor_sync(0xffffffffu, z, 2);
            zs[g] = z;
        }
    }
    const size_t row = (size_t)s_idx * G + gid;
    if (nparts == 1) {
        if ((uint32_t)gid < G) {
            if (A.part_o) {
                float *o = A.part_o + row * kHeadDim;
#pragma unroll
                for (int jn = 0; jn < 16; jn++)
                    *reinterpret_cast<float2 *>(o + CD::dim_of(jn, tig, 0)) =
                        make_float2(CD::out_value(acc, jn, 0, zs[jn >> 2]), CD::out_value(acc, jn, 1, zs[jn >> 2]));
                if (tig == 0) { A.part_m[row] = m; A.part_l[row] = lr; }
            } else {
                const float inv = lr > 0.f ? 1.0f / lr : 0.f;
                float *o = A.output + row * kHeadDim;
#pragma unroll
                for (int jn = 0; jn < 16; jn++)
                    *reinterpret_cast<float2 *>(o + CD::dim_of(jn, tig, 0)) =
                        make_float2(CD::out_value(acc, jn, 0, zs[jn >> 2]) * inv,
                                    CD::out_value(acc, jn, 1, zs[jn >> 2]) * inv);
            }
            if (A.seg_ml && tig == 0) A.seg_ml[(size_t)s_idx * kMaxGroup + gid] = make_float2(m, lr);
        }
        return 0;
    }
    float *slot = A.partials + (size_t)(wid + s_idx) * kPartialFloats;
    if ((uint32_t)gid < G) {
#pragma unroll
        for (int jn = 0; jn < 16; jn++)
            *reinterpret_cast<float2 *>(slot + gid * kHeadDim + CD::dim_of(jn, tig, 0)) =
                make_float2(CD::out_value(acc, jn, 0, zs[jn >> 2]), CD::out_value(acc, jn, 1, zs[jn >> 2]));
        if (tig == 0) {
            slot[kMaxGroup * kHeadDim + gid] = m;
            slot[kMaxGroup * kHeadDim + kMaxGroup + gid] = lr;
        }
    }
    // the warp barrier orders the lanes' slot stores before lane 0's release;
    // the acquire side orders the last arriver's reads of the other slots
    __syncwarp();
    uint32_t old = 0;
    if (lane == 0) old = atom_add_acq_rel_gpu(&A.counters[s_idx], 1u);
    old = __shfl_sync(0xffffffffu, old, 0);
    __syncwarp();
    return old == nparts - 1 ? nparts : 0u;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int CODEC>
__global__ void __launch_bounds__(kWarpsPerCta * 32, 3) attn_kernel(const AttnArgs A) {
    using CD = Codec<CODEC>;
    constexpr int S = CD::kStages, B = CD::kBytes;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
    uint8_t *wsm = smem + (size_t)warp * S * B;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + (size_t)kWarpsPerCta * S * B) + warp * S;
    WarpWindow *win = reinterpret_cast<WarpWindow *>(smem + (size_t)kWarpsPerCta * S * (B + 8)) + warp;
    if (lane == 0) {
#pragma unroll
        for (int st = 0; st < S; st++) mbar_init(&bars[st], 1);
        fence_barrier_init();
    }
    __syncwarp();

    const uint32_t HK = A.kv_heads, G = A.group, Hq = HK * G;
    const uint64_t W = (uint64_t)gridDim.x * kWarpsPerCta;
    const uint64_t wid = (uint64_t)blockIdx.x * kWarpsPerCta + warp;

    // total units of the batch
    uint64_t T = 0;
    for (uint32_t base = 0; base < A.num_seqs; base += 32) {
        const uint32_t i = base + lane;
        uint32_t u = i < A.num_seqs ? geo_of(A, i).ntiles * HK : 0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) u += __shfl_xor_sync(0xffffffffu, u, o);
        T += u;
    }
    if (T == 0) return;
    const uint64_t u0 = wid * T / W, u1 = (wid + 1) * T / W;
    if (u0 >= u1) return;
    const uint32_t n = (uint32_t)(u1 - u0);

    // locate u0
    Walk cons;
    {
        uint64_t acc = 0;
        for (uint32_t base = 0; base < A.num_seqs; base += 32) {
            const uint32_t i = base + lane;
            const uint32_t u = i < A.num_seqs ? geo_of(A, i).ntiles * HK : 0;
            const uint32_t incl = warp_incl_scan(u);
            const uint32_t tot = __shfl_sync(0xffffffffu, incl, 31);
            if (u0 < acc + tot) {
                const uint32_t ball = __ballot_sync(0xffffffffu, acc + incl > u0);
                const int L = __ffs(ball) - 1;
                const uint32_t excl = __shfl_sync(0xffffffffu, incl - u, L);
                cons.i = base + L;
                cons.geo = geo_of(A, cons.i);
                const uint64_t rem = u0 - (acc + excl);
                cons.h = (uint32_t)(rem / cons.geo.ntiles);
                cons.tile = (uint32_t)(rem % cons.geo.ntiles);
                cons.seg_base = acc + excl + (uint64_t)cons.h * cons.geo.ntiles;
                break;
            }
            acc += tot;
        }
    }

    // window of unit sources: units [wbase, wbase+32) of this warp's range
    uint32_t wbase = 0;
    fill_window(A, cons, 0, u0, u1, win);
    const uint32_t npro = n < (uint32_t)S ? n : (uint32_t)S;
    for (uint32_t j = 0; j < npro; j++) {
        const int32_t seg = win->append_seg[j];
        if (seg >= 0) fused_append<CODEC>(A.new_k, A.new_v, A.seq_ids, A.seq_lens, A.kv_heads, seg, win->src[j]);
        if (lane == 0) {
            mbar_expect_tx(&bars[j], B);
            bulk_g2s(wsm + j * B, win->src[j], B, &bars[j]);
        }
    }

    typename CD::Frag frag;
    typename CD::Acc acc;
    float m = -INFINITY, l = 0.f;
    uint32_t st = 0, par = 0;
    // merges this warp owes (it arrived last at a shared segment), run after the loop
    uint32_t pend_n = 0, pend_s0 = 0, pend_n0 = 0, pend_s1 = 0, pend_n1 = 0;
    uint64_t pend_u0 = 0, pend_u1 = 0;

    for (uint32_t k = 0; k < n; ++k) {
        if (cons.tile == 0 || k == 0) {
            const float *q = nullptr;
            if ((uint32_t)gid < G) q = A.query + ((size_t)cons.i * Hq + (size_t)cons.h * G + gid) * kHeadDim;
            CD::load_q(frag, q, tig);
            acc.reset();
            m = -INFINITY;
            l = 0.f;
        }
        if (!mbar_wait_bounded(&bars[st], par)) {
            if (lane == 0) latch(A.status, QWN_KV_STATUS_WAIT_TIMEOUT);
            // wait (bounded) for the copies still in flight into this warp's stages
            uint32_t s2 = st, p2 = par;
            for (uint32_t d = k + 1; d < n && d < k + (uint32_t)S; ++d) {
                if (++s2 == (uint32_t)S) { s2 = 0; p2 ^= 1u; }
                mbar_wait_bounded(&bars[s2], p2);
            }
            return;
        }
        const int tile_tok0 = (int)(cons.geo.tile0 + cons.tile) * 16;
        const int t_lo = max(cons.geo.tok_lo - tile_tok0, 0);
        const int t_hi = min(cons.geo.tok_hi - tile_tok0, 16);
        float tile_u = tile_step<CODEC>(wsm + st * B, frag, acc, m, l, t_lo, t_hi, A.scale_log2);
        if (A.tile_mass) {
            tile_u += __shfl_xor_sync(0xffffffffu, tile_u, 1);
            tile_u += __shfl_xor_sync(0xffffffffu, tile_u, 2);
            if (tig == 0 && (uint32_t)gid < G)
                A.tile_mass[(u0 + k) * kMaxGroup + gid] = make_float2(tile_u, m);
        }
        __syncwarp();

        // refill this stage with unit k + S
        const uint32_t j = k + (uint32_t)S;
        if (j < n) {
            if (j - wbase == 32u) {
                wbase = j;
                fill_window(A, cons, (uint32_t)S, u0 + wbase, u1, win);
            }
            const int32_t seg = win->append_seg[j - wbase];
            const uint8_t *src = win->src[j - wbase];
            if (seg >= 0) fused_append<CODEC>(A.new_k, A.new_v, A.seq_ids, A.seq_lens, A.kv_heads, seg, src);
            if (lane == 0) {
                fence_proxy_async_shared();
                mbar_expect_tx(&bars[st], B);
                bulk_g2s(wsm + st * B, src, B, &bars[st]);
            }
        }
        if (++st == (uint32_t)S) { st = 0; par ^= 1u; }

        // end of this warp's share of the segment?
        if (cons.tile + 1 == cons.geo.ntiles || k + 1 == n) {
            const uint32_t s_idx = cons.i * HK + cons.h;
            const uint32_t np = finish_segment<CODEC>(A, acc, m, l, s_idx, cons.seg_base, cons.geo.ntiles, T, W, wid);
            if (np) {
                const int e = pend_n++;  // at most two: the segment the range starts in and the one it ends in
                if (e == 0) { pend_s0 = s_idx; pend_n0 = np; pend_u0 = cons.seg_base; }
                else { pend_s1 = s_idx; pend_n1 = np; pend_u1 = cons.seg_base; }
            }
        }
        // next unit
        if (k + 1 < n) {
            if (++cons.tile == cons.geo.ntiles) walk_next_segment(A, cons);
        }
    }
    for (uint32_t e = 0; e < pend_n; e++) {
        merge_segment(A, e ? pend_s1 : pend_s0, e ? pend_n1 : pend_n0, e ? pend_u1 : pend_u0, T, W);
    }
}

// merge of partial states produced on several devices (base-2 domain)
__global__ void merge_kernel(uint32_t parts, uint32_t rows, const float *m, const float *l,
                             const float *o, float *out) {
    const uint32_t row = blockIdx.x;
    const uint32_t d = threadIdx.x;
    if (row >= rows || d >= kHeadDim) return;
    float ms = -INFINITY;
    for (uint32_t p = 0; p < parts; p++) ms = fmaxf(ms, m[(size_t)p * rows + row]);
    float ls = 0.f, acc = 0.f;
    for (uint32_t p = 0; p < parts; p++) {
        const float mp = m[(size_t)p * rows + row];
        const float w = mp == -INFINITY ? 0.f : ex2(mp - ms);
        ls += l[(size_t)p * rows + row] * w;
        acc += o[((size_t)p * rows + row) * kHeadDim + d] * w;
    }
    out[(size_t)row * kHeadDim + d] = ls > 0.f ? acc / ls : 0.f;
}

template <int CODEC>
constexpr size_t codec_smem() {
    return (size_t)kWarpsPerCta * Codec<CODEC>::kStages * (Codec<CODEC>::kBytes + 8) +
           (size_t)kWarpsPerCta * sizeof(WarpWindow);
}

template <int CODEC>
cudaError_t launch_codec(Pool *p, const AttnArgs &A, cudaStream_t s) {
    const size_t smem = codec_smem<CODEC>();
    static bool configured[64] = {false};
    if (!configured[p->device & 63]) {
        cudaError_t e = cudaFuncSetAttribute(attn_kernel<CODEC>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured[p->device & 63] = true;
    }
    attn_kernel<CODEC><<<p->attn_ctas, kWarpsPerCta * 32, smem, s>>>(A);
    count_launch();
    return cudaGetLastError();
}

}  // namespace

size_t attention_smem_bytes(uint32_t codec) {
    switch (codec) {
        case QWN_KV_CODEC_Q8_HEAD_F16: return codec_smem<QWN_KV_CODEC_Q8_HEAD_F16>();
        case QWN_KV_CODEC_Q8_B64_F32: return codec_smem<QWN_KV_CODEC_Q8_B64_F32>();
        case QWN_KV_CODEC_Q4_G32: return codec_smem<QWN_KV_CODEC_Q4_G32>();
        default: return 0;
    }
}

const void *attention_kernel_ptr(uint32_t codec) {
    switch (codec) {
        case QWN_KV_CODEC_Q8_HEAD_F16: return (const void *)attn_kernel<QWN_KV_CODEC_Q8_HEAD_F16>;
        case QWN_KV_CODEC_Q8_B64_F32: return (const void *)attn_kernel<QWN_KV_CODEC_Q8_B64_F32>;
        case QWN_KV_CODEC_Q4_G32: return (const void *)attn_kernel<QWN_KV_CODEC_Q4_G32>;
        default: return nullptr;
    }
}

cudaError_t launch_attention(Pool *p, const AttnLaunch &a, cudaStream_t s) {
    if (a.num_seqs == 0) return cudaSuccess;
    AttnArgs A{};
    A.pages = p->pages;
    A.page_bytes = p->page_bytes;
    A.tile_bytes = (uint32_t)p->tile_bytes;
    A.tpp = p->tiles_per_page;
    A.page_tokens = p->page_tokens;
    A.page_table = p->page_table;
    A.mp = p->max_pages_per_seq;
    A.total_pages = p->total_pages;
    A.max_seqs = p->max_seqs;
    A.seq_lens = p->seq_lens;
    A.seq_ids = a.seq_ids;
    A.num_seqs = a.num_seqs;
    A.kv_heads = p->kv_heads;
    A.group = a.query_heads / p->kv_heads;
    A.layer = a.layer;
    A.attend_limit = a.attend_limit;
    A.t_begin = a.t_begin;
    A.t_end = a.t_end;
    A.query = a.query;
    A.output = a.output;
    A.scale_log2 = a.scale * kLog2e;
    A.partials = p->partials;
    A.counters = p->counters;
    A.tile_mass = a.page_mass ? p->tile_mass : nullptr;
    A.seg_ml = a.page_mass ? p->seg_ml : nullptr;
    A.part_m = a.part_m;
    A.part_l = a.part_l;
    A.part_o = a.part_o;
    A.new_k = a.new_k;
    A.new_v = a.new_v;
    A.status = p->status;
    switch (p->codec) {
        case QWN_KV_CODEC_Q8_HEAD_F16: return launch_codec<QWN_KV_CODEC_Q8_HEAD_F16>(p, A, s);
        case QWN_KV_CODEC_Q8_B64_F32: return launch_codec<QWN_KV_CODEC_Q8_B64_F32>(p, A, s);
        case QWN_KV_CODEC_Q4_G32: return launch_codec<QWN_KV_CODEC_Q4_G32>(p, A, s);
        default: return cudaErrorNotSupported;
    }
}

cudaError_t launch_merge(uint32_t parts, uint32_t rows, const float *m, const float *l,
                         const float *o, float *out, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    merge_kernel<<<rows, kHeadDim, 0, s>>>(parts, rows, m, l, o, out);
    count_launch();
    return cudaGetLastError();
}

}  // namespace qkv

// ===========================================================================
// Decode attention that allocates nothing.
//
// Some callers cannot allocate device memory when they need attention: a
// serving process that handed all free HBM to its own arena at start-up (a
// cudaMalloc here would fail, or fragment the arena), a latency-critical loop
// where cudaMalloc/cudaFree would synchronise the device and stall other
// streams, and FFI callers that hold only raw device pointers to a KV pool and
// no qwn_kv_pool handle (whose scratch was allocated with the pool).  This
// entry point runs the same split-KV kernel with its scratch -- the partial
// (m, l, o) slots and the merge counters -- in a file-scope device array.
//
// Limits: at most kStaticSegments (sequence x kv head) segments per call and
// kStaticSlots partial slots (warps of the grid + segments); larger requests
// are rejected.  The array is shared by every call on a device and keeps the
// last call's contents: the counters are cleared on the stream at the start
// of each call, so calls whose work overlaps on the GPU (different streams,
// no ordering between them) race on the array and must not be issued.
// The first call on a device looks up the array's device address and sets
// the kernel's shared-memory attribute; make that first call before any
// stream capture.  Every GPU that loads the library holds the array
// (kStaticBytes) until the process exits.
// ===========================================================================
namespace qkv {
namespace {
constexpr int kStaticSlots = 1024;
constexpr int kStaticSegments = 256;
constexpr size_t kStaticFloats = (size_t)kStaticSlots * kPartialFloats + kStaticSegments;
static __device__ __align__(256) float g_static_scratch[kStaticFloats];
constexpr int kStaticMaxDevices = 64;
std::mutex g_static_mu;
float *g_static_addr[kStaticMaxDevices] = {};
uint32_t g_static_ctas[kStaticMaxDevices][5] = {};

template <int CODEC>
cudaError_t static_setup(int dev) {
    const size_t smem = codec_smem<CODEC>();
    cudaError_t e = cudaFuncSetAttribute(attn_kernel<CODEC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int sms = 0, per_sm = 0;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_kernel<CODEC>, kWarpsPerCta * 32, smem)) !=
        cudaSuccess)
        return e;
    g_static_ctas[dev][CODEC] = (uint32_t)(sms * (per_sm > 0 ? per_sm : 1));
    return cudaSuccess;
}
}  // namespace
}  // namespace qkv

extern "C" QWN_CUDA_ABI_API int qwn_kv_attention_static(const QwnKvStaticAttentionRequest *r) {
    using namespace qkv;
    if (!r || !header_ok(r->header, sizeof(*r))) return QWN_CUDA_STATUS_ABI_MISMATCH;
    const size_t tb = tile_bytes_of(r->codec);
    if (!tb || r->codec == QWN_KV_CODEC_TQ35_G64 || r->head_dim != (uint32_t)kHeadDim || r->kv_heads == 0 ||
        r->page_tokens == 0 || r->page_tokens % 16 || r->layer >= r->layers || r->query_heads == 0 ||
        r->query_heads % r->kv_heads || r->query_heads / r->kv_heads > (uint32_t)kMaxGroup || !r->pages_dev ||
        !r->page_table_dev || !r->seq_lens_dev || !r->query_dev || !r->output_dev || r->total_pages == 0 ||
        r->max_seqs == 0 || r->max_pages_per_seq == 0 || r->num_seqs > r->max_seqs) {
        set_error("qwn_kv_attention_static: invalid request");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    if ((uint64_t)r->num_seqs * r->kv_heads > (uint64_t)kStaticSegments) {
        set_error("qwn_kv_attention_static: num_seqs x kv_heads exceeds the static scratch limit of 256 segments");
        return QWN_CUDA_STATUS_UNSUPPORTED;
    }
    if (r->device_id < 0 || r->device_id >= kStaticMaxDevices) {
        set_error("qwn_kv_attention_static: device id out of range");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    cudaError_t e = cudaSetDevice(r->device_id);
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_attention_static: cudaSetDevice", e); return QWN_CUDA_STATUS_UNAVAILABLE; }
    const int dev = r->device_id;
    {
        std::lock_guard<std::mutex> lk(g_static_mu);
        if (!g_static_addr[dev]) {
            float *ptr = nullptr;
            e = cudaGetSymbolAddress(reinterpret_cast<void **>(&ptr), g_static_scratch);
            if (e != cudaSuccess || !ptr) {
                set_cuda_error("qwn_kv_attention_static: cudaGetSymbolAddress", e);
                return QWN_CUDA_STATUS_RUNTIME_ERROR;
            }
            if ((e = static_setup<QWN_KV_CODEC_Q8_B64_F32>(dev)) != cudaSuccess ||
                (e = static_setup<QWN_KV_CODEC_Q8_HEAD_F16>(dev)) != cudaSuccess ||
                (e = static_setup<QWN_KV_CODEC_Q4_G32>(dev)) != cudaSuccess) {
                set_cuda_error("qwn_kv_attention_static: kernel set-up", e);
                return QWN_CUDA_STATUS_RUNTIME_ERROR;
            }
            g_static_addr[dev] = ptr;
        }
    }
    if (r->num_seqs == 0) return QWN_CUDA_STATUS_OK;
    float *scratch = g_static_addr[dev];
    uint32_t *counters = reinterpret_cast<uint32_t *>(scratch + (size_t)kStaticSlots * kPartialFloats);
    cudaStream_t s = static_cast<cudaStream_t>(r->stream);
    // the merge counters must start at zero; the slots are written before read
    e = cudaMemsetAsync(counters, 0, sizeof(uint32_t) * kStaticSegments, s);
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_attention_static: clear", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    const uint32_t segs = r->num_seqs * r->kv_heads;
    uint32_t ctas = g_static_ctas[dev][r->codec];
    const uint32_t max_ctas = (kStaticSlots - segs) / kWarpsPerCta;  // warps + segments <= slots
    if (ctas > max_ctas) ctas = max_ctas;
    AttnArgs A{};
    A.pages = static_cast<const uint8_t *>(r->pages_dev);
    A.tile_bytes = (uint32_t)tb;
    A.tpp = r->page_tokens / 16;
    A.page_tokens = r->page_tokens;
    A.page_bytes = tb * A.tpp * (uint64_t)r->layers * r->kv_heads;
    A.page_table = r->page_table_dev;
    A.mp = r->max_pages_per_seq;
    A.total_pages = r->total_pages;
    A.max_seqs = r->max_seqs;
    A.seq_lens = r->seq_lens_dev;
    A.seq_ids = r->seq_ids_dev;
    A.num_seqs = r->num_seqs;
    A.kv_heads = r->kv_heads;
    A.group = r->query_heads / r->kv_heads;
    A.layer = r->layer;
    A.query = r->query_dev;
    A.output = r->output_dev;
    A.scale_log2 = (r->scale > 0.f ? r->scale : 1.0f / sqrtf((float)kHeadDim)) * kLog2e;
    A.partials = scratch;
    A.counters = counters;
    A.status = r->status_dev;
    switch (r->codec) {
        case QWN_KV_CODEC_Q8_HEAD_F16: {
            attn_kernel<QWN_KV_CODEC_Q8_HEAD_F16><<<ctas, kWarpsPerCta * 32, codec_smem<QWN_KV_CODEC_Q8_HEAD_F16>(), s>>>(A);
            break;
        }
        case QWN_KV_CODEC_Q8_B64_F32: {
            attn_kernel<QWN_KV_CODEC_Q8_B64_F32><<<ctas, kWarpsPerCta * 32, codec_smem<QWN_KV_CODEC_Q8_B64_F32>(), s>>>(A);
            break;
        }
        default: {
            attn_kernel<QWN_KV_CODEC_Q4_G32><<<ctas, kWarpsPerCta * 32, codec_smem<QWN_KV_CODEC_Q4_G32>(), s>>>(A);
            break;
        }
    }
    count_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) {
        set_cuda_error("qwn_kv_attention_static: launch", e);
        return QWN_CUDA_STATUS_RUNTIME_ERROR;
    }
    return QWN_CUDA_STATUS_OK;
}
