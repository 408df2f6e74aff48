// Quantize-on-append device code shared by the append, prefill and fused
// attention kernels.  One warp stores one token-head; lane l holds dims
// 4l..4l+3 of K and of V.  The rules are the reference quantizers'
// (c/qwanto_turboquant.c:555-586 for Q8, :162-213 for TurboQuant); the byte
// positions are this library's tile layout (see qwn_oracle.c for the
// independent restatement used by the tests).
#pragma once

#include "kv_internal.cuh"

namespace qkv {
namespace {

// ---------------------------------------------------------------------------
// quantize-on-append: one warp stores one token-head; lane holds dims
// 4*lane .. 4*lane+3 of K and of V.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float absmax4(float4 v) {
    float m = 0.f;
    if (isfinite(v.x)) m = fmaxf(m, fabsf(v.x));
    if (isfinite(v.y)) m = fmaxf(m, fabsf(v.y));
    if (isfinite(v.z)) m = fmaxf(m, fabsf(v.z));
    if (isfinite(v.w)) m = fmaxf(m, fabsf(v.w));
    return m;
}
// c/qwanto_turboquant.c:555-560
__device__ __forceinline__ int q8_round(float x) {
    if (!isfinite(x)) return 0;
    if (x >= 127.f) return 127;
    if (x <= -127.f) return -127;
    return __float2int_rn(x);
}
__device__ __forceinline__ uint32_t q8_pack4(float4 v, float s) {
    const uint32_t b0 = (uint32_t)(q8_round(__fdiv_rn(v.x, s)) + 128);
    const uint32_t b1 = (uint32_t)(q8_round(__fdiv_rn(v.y, s)) + 128);
    const uint32_t b2 = (uint32_t)(q8_round(__fdiv_rn(v.z, s)) + 128);
    const uint32_t b3 = (uint32_t)(q8_round(__fdiv_rn(v.w, s)) + 128);
    return b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
}
__device__ __forceinline__ uint16_t head_scale16(float m) {
    const float s = m > 0.f ? __fdiv_rn(m, 127.f) : 1.f;
    uint16_t h = __half_as_ushort(__float2half_rn(s));
    if ((h & 0x7FFFu) == 0) h = 0x0001u;
    if ((h & 0x7FFFu) >= 0x7C00u) h = 0x7BFFu;
    return h;
}
// the lane's four dims 4*lane..4*lane+3 are consecutive bytes of the K row
__device__ __forceinline__ uint32_t k8_lane_off(int t, int lane) { return k8_off(t, 4 * lane); }
__device__ __forceinline__ void store_v8(uint8_t *tile, int t, int lane, uint32_t packed) {
#pragma unroll
    for (int i = 0; i < 4; i++) tile[v8_off(t, 4 * lane + i)] = (uint8_t)(packed >> (8 * i));
}

// min / max with the reference's first-occurrence tie rule over `width`
// lanes (4 values per lane, index 4*lane+i): c/qwanto_turboquant.c:171-177
__device__ __forceinline__ void minmax_first(float4 v, int lane, int width, float &mn, float &mx) {
    float a[4] = {v.x, v.y, v.z, v.w};
    float lo = a[0], hi = a[0];
    int ilo = 4 * lane, ihi = 4 * lane;
#pragma unroll
    for (int i = 1; i < 4; i++) {
        if (a[i] < lo) { lo = a[i]; ilo = 4 * lane + i; }
        if (a[i] > hi) { hi = a[i]; ihi = 4 * lane + i; }
    }
    for (int o = 1; o < width; o <<= 1) {
        const float lo2 = __shfl_xor_sync(0xffffffffu, lo, o);
        const int il2 = __shfl_xor_sync(0xffffffffu, ilo, o);
        const float hi2 = __shfl_xor_sync(0xffffffffu, hi, o);
        const int ih2 = __shfl_xor_sync(0xffffffffu, ihi, o);
        if (lo2 < lo || (lo2 == lo && il2 < ilo)) { lo = lo2; ilo = il2; }
        if (hi2 > hi || (hi2 == hi && ih2 < ihi)) { hi = hi2; ihi = ih2; }
    }
    mn = lo;
    mx = hi;
}
// one TurboQuant-style code: c/qwanto_turboquant.c:188-206
__device__ __forceinline__ uint32_t tq_code(float x, float mn, float inv, float levels) {
    float norm = __fmul_rn(__fsub_rn(x, mn), inv);
    if (norm < 0.f) norm = 0.f;
    if (norm > 1.f) norm = 1.f;
    int q = (int)roundf(__fmul_rn(norm, levels));
    const int top = (int)levels;
    if (q > top) q = top;
    if (q < 0) q = 0;
    return (uint32_t)q;
}
__device__ __forceinline__ void put_bits(uint8_t *tile, uint32_t byte, uint32_t shift_in_byte,
                                         uint32_t mask, uint32_t val) {
    uint32_t *word = reinterpret_cast<uint32_t *>(tile + (byte & ~3u));
    const uint32_t sh = (byte & 3u) * 8u + shift_in_byte;
    atomicAnd(word, ~(mask << sh));
    atomicOr(word, (val & mask) << sh);
}

template <int CODEC>
__device__ void store_token(uint8_t *tile, int t, float4 k, float4 v, int lane);

// fp32 -> fp16 round to nearest even (c/qwn_paged_kv.c:151-198, F16C); a NaN
// stays a quiet NaN with the top ten payload bits, as F16C keeps them
__device__ __forceinline__ uint32_t f16_bits(float x) {
    const uint32_t u = __float_as_uint(x);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return ((u >> 16) & 0x8000u) | 0x7E00u | ((u >> 13) & 0x3FFu);
    return __half_as_ushort(__float2half_rn(x));
}
template <>
__device__ void store_token<QWN_KV_CODEC_F16>(uint8_t *tile, int t, float4 k, float4 v, int lane) {
    // the lane's dims 4*lane..4*lane+3: half of one 16-byte chunk
    const uint2 kk = make_uint2(f16_bits(k.x) | (f16_bits(k.y) << 16), f16_bits(k.z) | (f16_bits(k.w) << 16));
    const uint2 vv = make_uint2(f16_bits(v.x) | (f16_bits(v.y) << 16), f16_bits(v.z) | (f16_bits(v.w) << 16));
    *reinterpret_cast<uint2 *>(tile + f16_off(0, t, 4 * lane)) = kk;
    *reinterpret_cast<uint2 *>(tile + f16_off(1, t, 4 * lane)) = vv;
}
template <>
__device__ void store_token<QWN_KV_CODEC_Q8_HEAD_F16>(uint8_t *tile, int t, float4 k, float4 v, int lane) {
    const uint16_t sk = head_scale16(warp_max(absmax4(k)));
    const uint16_t sv = head_scale16(warp_max(absmax4(v)));
    const float fk = h2f(sk), fv = h2f(sv);
    *reinterpret_cast<uint32_t *>(tile + k8_lane_off(t, lane)) = q8_pack4(k, fk);
    store_v8(tile, t, lane, q8_pack4(v, fv));
    if (lane == 0) {
        *reinterpret_cast<uint16_t *>(tile + 4096 + s16_off(t)) = sk;
        *reinterpret_cast<uint16_t *>(tile + 4128 + s16_off(t)) = sv;
    }
}

template <>
__device__ void store_token<QWN_KV_CODEC_Q8_B64_F32>(uint8_t *tile, int t, float4 k, float4 v, int lane) {
    float mk = absmax4(k), mv = absmax4(v);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {  // within each half-warp (64 channels)
        mk = fmaxf(mk, __shfl_xor_sync(0xffffffffu, mk, o));
        mv = fmaxf(mv, __shfl_xor_sync(0xffffffffu, mv, o));
    }
    const float sk = mk > 0.f ? __fdiv_rn(mk, 127.f) : 1.f;
    const float sv = mv > 0.f ? __fdiv_rn(mv, 127.f) : 1.f;
    *reinterpret_cast<uint32_t *>(tile + k8_lane_off(t, lane)) = q8_pack4(k, sk);
    store_v8(tile, t, lane, q8_pack4(v, sv));
    if ((lane & 15) == 0) {
        const int x = lane >> 4;
        *reinterpret_cast<float *>(tile + 4096 + s32_off(t, x)) = sk;
        *reinterpret_cast<float *>(tile + 4224 + s32_off(t, x)) = sv;
    }
}

// 4-bit groups of 32: lane L holds dims 4L..4L+3, group c = L>>3.  K word
// (t, tig = (L&7)>>1, c) at 64t + 16tig + 4c takes dim i of lane L in the low
// nibble of byte i (L even) or the high nibble (L odd).  V: the byte for
// (t, m-block, row gid) holds rows gid (lanes with L&2 == 0) and gid+8 (L+2).
template <>
__device__ void store_token<QWN_KV_CODEC_Q4_G32>(uint8_t *tile, int t, float4 k, float4 v, int lane) {
    const int c = lane >> 3;
#pragma unroll
    for (int which = 0; which < 2; which++) {
        const float4 x4 = which ? v : k;
        float mn, mx;
        minmax_first(x4, lane, 8, mn, mx);
        const float range = __fsub_rn(mx, mn);
        const float inv = range > 1e-8f ? __fdiv_rn(1.0f, range) : 0.f;
        const uint32_t q[4] = {tq_code(x4.x, mn, inv, 15.f), tq_code(x4.y, mn, inv, 15.f),
                               tq_code(x4.z, mn, inv, 15.f), tq_code(x4.w, mn, inv, 15.f)};
        if (!which) {
            uint32_t word = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t hi = __shfl_down_sync(0xffffffffu, q[i], 1);
                word |= (q[i] | (hi << 4)) << (8 * i);
            }
            if (!(lane & 1))
                *reinterpret_cast<uint32_t *>(tile + 64 * t + 16 * ((lane & 7) >> 1) + 4 * c) = word;
        } else {
            const int mb = 2 * c + ((lane & 7) >> 2);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t hi = __shfl_down_sync(0xffffffffu, q[i], 2);
                if (!(lane & 2)) {
                    const int lv = 4 * (4 * (lane & 1) + i) + ((t & 7) >> 1);
                    const int chunk = (mb >> 2) ^ ((lv >> 2) & 1);
                    tile[1024 + 32 * lv + 16 * chunk + 4 * (mb & 3) + (t >> 3) + 2 * (t & 1)] =
                        (uint8_t)(q[i] | (hi << 4));
                }
            }
        }
        if ((lane & 7) == 0)
            *reinterpret_cast<uint32_t *>(tile + (which ? 2304 : 2048) + 32 * (t & 7) + 8 * c + 4 * (t >> 3)) =
                (uint32_t)tq_f32_to_f16(range) | ((uint32_t)tq_f32_to_f16(mn) << 16);
    }
}

// 3.5-bit reference TurboQuant codes in the tile layout (restated in
// qwn_oracle.c): class c = 2*(d>>6) + (d&1), index m = (d&63)>>1
__device__ __forceinline__ int lb_k_nibble(int m) { return 2 * (m & 3) + ((m >> 2) & 1); }
__device__ void tq35_put(uint8_t *half, int is_value, int t, int d, uint32_t code) {
    const int x = d >> 6, m = (d & 63) >> 1;
    uint32_t eb, ob, pb, n;
    if (!is_value) {
        const int tig = m >> 3;
        n = (uint32_t)lb_k_nibble(m);
        eb = 32 * t + 8 * tig + 4 * x;
        ob = 512 + 16 * t + 4 * tig;
        pb = 768 + 8 * t + 2 * tig;
    } else {
        const int c = 2 * x + (d & 1), r = m & 15, mb = 2 * c + (m >> 4);
        const int lv = ((r & 7) << 2) | ((t & 7) >> 1);
        n = (uint32_t)((r >> 3) + 2 * (t >> 3) + 4 * (t & 1));
        eb = 16 * lv + 4 * (2 * x + (mb & 1));
        ob = 512 + 8 * lv + 4 * (mb & 1);
        pb = 768 + 4 * lv + 2 * (mb & 1);
    }
    if (!(d & 1)) {
        put_bits(half, eb + (n >> 1), (n & 1) * 4, 0xFu, code);
    } else if (x == 0) {
        put_bits(half, ob + (n >> 1), (n & 1) * 4, 0x7u, code);
    } else {
        put_bits(half, ob + (n >> 1), (n & 1) * 4 + 3, 0x1u, code & 1u);
        put_bits(half, pb + ((2 * n) >> 3), (2 * n) & 7, 0x3u, code >> 1);
    }
}

template <>
__device__ void store_token<QWN_KV_CODEC_TQ35_G64>(uint8_t *tile, int t, float4 k, float4 v, int lane) {
#pragma unroll
    for (int which = 0; which < 2; which++) {
        const float4 x4 = which ? v : k;
        uint8_t *half = tile + which * 1024;
        float mn, mx;
        minmax_first(x4, lane, 16, mn, mx);  // groups of 64 = 16 lanes
        const float range = __fsub_rn(mx, mn);
        const float inv = range > 1e-8f ? __fdiv_rn(1.0f, range) : 0.f;
        const float xv[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int d = 4 * lane + i;
            const uint32_t code = tq_code(xv[i], mn, inv, (i & 1) ? 7.f : 15.f);
            tq35_put(half, which, t, d, code);
        }
        if ((lane & 15) == 0) {
            const int x = lane >> 4;
            *reinterpret_cast<uint32_t *>(half + 896 + 16 * (t & 7) + 8 * x + 4 * (t >> 3)) =
                (uint32_t)tq_f32_to_f16(range) | ((uint32_t)tq_f32_to_f16(mn) << 16);
        }
    }
}

}  // namespace
}  // namespace qkv
