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

template <>
__device__ void store_token<QWN_KV_CODEC_Q4_G32>(uint8_t *tile, int t, float4 k, float4 v, int lane) {
    // K
    {
        float mn, mx;
        minmax_first(k, lane, 8, mn, mx);
        const float range = __fsub_rn(mx, mn);
        const float inv = range > 1e-8f ? __fdiv_rn(1.0f, range) : 0.f;
        const uint32_t c0 = tq_code(k.x, mn, inv, 15.f), c1 = tq_code(k.y, mn, inv, 15.f);
        const uint32_t c2 = tq_code(k.z, mn, inv, 15.f), c3 = tq_code(k.w, mn, inv, 15.f);
        const int n = 2 * (t >> 2) + (t & 1), h = (t >> 1) & 1;
        const int g = lane >> 3, e = (lane >> 2) & 1, tg = lane & 3;
        uint8_t *base = tile + h * 512 + (n * 4 + tg) * 16 + g * 4;
        base[e] = (uint8_t)(c0 | (c2 << 4));
        base[2 + e] = (uint8_t)(c1 | (c3 << 4));
        if ((lane & 7) == 0)
            *reinterpret_cast<uint32_t *>(tile + 2048 + 64 * g + 4 * t) =
                (uint32_t)tq_f32_to_f16(range) | ((uint32_t)tq_f32_to_f16(mn) << 16);
    }
    // V
    {
        float mn, mx;
        minmax_first(v, lane, 8, mn, mx);
        const float range = __fsub_rn(mx, mn);
        const float inv = range > 1e-8f ? __fdiv_rn(1.0f, range) : 0.f;
        const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int d = 4 * lane + i;
            const uint32_t code = tq_code(vv[i], mn, inv, 15.f);
            const int gidd = d & 7, j = d >> 3, lv = gidd * 4 + (t >> 2), b = t & 3;
            const int w = j >> 1, e = j & 1;
            const int pos = (b & 1) * 4 + e * 2 + (b >> 1);
            const int chunk = (w >> 2) ^ ((lv >> 2) & 1);
            const uint32_t byte = 1024 + lv * 32 + chunk * 16 + (w & 3) * 4 + (pos >> 1);
            put_bits(tile, byte, (pos & 1) * 4, 0xFu, code);
        }
        if ((lane & 7) == 0) {
            const int g = lane >> 3;
            *reinterpret_cast<uint32_t *>(tile + 2304 + 64 * g + 4 * t) =
                (uint32_t)tq_f32_to_f16(range) | ((uint32_t)tq_f32_to_f16(mn) << 16);
        }
    }
}

// 3.5-bit reference TurboQuant codes in the tile layout (see qwn_oracle.c)
__device__ void tq35_put(uint8_t *half, int is_value, int t, int d, uint32_t code) {
    if (!is_value) {
        const int h = (t >> 1) & 1, n = 2 * (t >> 2) + (t & 1);
        const int x = d >> 6, tg = (d >> 4) & 3, k = d & 15;
        const int slot = h * 32 + n * 4 + tg;
        const int e = k >> 1, np = (e & 1) * 4 + (e >> 1);
        if (!(k & 1)) {
            put_bits(half, slot * 8 + x * 4 + (np >> 1), (np & 1) * 4, 0xFu, code);
        } else {
            const uint32_t byte = 512 + slot * 4 + (np >> 1), sh = (np & 1) * 4;
            if (x == 0) {
                put_bits(half, byte, sh, 0x7u, code);
            } else {
                put_bits(half, byte, sh + 3, 0x1u, code & 1u);
                const uint32_t hb = 768 + slot * 2;  // 16-bit field, bits 2*np
                put_bits(half, hb + ((2 * np) >> 3), (2 * np) & 7, 0x3u, code >> 1);
            }
        }
    } else {
        const int x = d >> 6, r = d & 63, par = r & 1, q = r >> 1, gidd = q & 7, jl = q >> 3;
        const int lv = gidd * 4 + (t >> 2), b = t & 3;
        if (!par) {
            const int col = x * 4 + jl, np = (b & 1) * 4 + (col & 1) * 2 + (b >> 1);
            put_bits(half, lv * 16 + (col >> 1) * 4 + (np >> 1), (np & 1) * 4, 0xFu, code);
        } else {
            const int npos = (b & 1) * 4 + (jl & 1) * 2 + (b >> 1);
            const uint32_t byte = 512 + lv * 8 + (jl >> 1) * 4 + (npos >> 1), sh = (npos & 1) * 4;
            if (x == 0) {
                put_bits(half, byte, sh, 0x7u, code);
            } else {
                put_bits(half, byte, sh + 3, 0x1u, code & 1u);
                const int bitpos = 2 * ((jl >> 1) * 8 + npos);
                put_bits(half, 768 + lv * 4 + (bitpos >> 3), bitpos & 7, 0x3u, code >> 1);
            }
        }
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
            *reinterpret_cast<uint32_t *>(half + 896 + 64 * x + 4 * t) =
                (uint32_t)tq_f32_to_f16(range) | ((uint32_t)tq_f32_to_f16(mn) << 16);
        }
    }
}

}  // namespace
}  // namespace qkv
