/*
 * qwn_oracle.c -- CPU restatement of Qwanto's quantized KV-cache path.
 *
 * TEST INFRASTRUCTURE ONLY (see qwn_oracle.h).  Compiled with
 * -ffp-contract=off so that every a*b+c below is two IEEE roundings.
 */
#include "qwn_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ======================================================================== */
/* synthetic inputs                                                          */
/* ======================================================================== */

/* splitmix64 finaliser (public-domain mixing function by S. Vigna). */
uint64_t qor_mix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t qor_stream(uint32_t kind, uint32_t seq, uint32_t layer) {
    return ((uint64_t)kind << 56) ^ ((uint64_t)layer << 32) ^ (uint64_t)seq;
}

/* Irwin-Hall(12) of 16-bit uniforms: the integer sum is exact, and
 * (sum - 393210) / 65536 is exact in fp32, so CPU and GPU agree bit for bit. */
float qor_normal(uint64_t seed, uint64_t stream, uint64_t index) {
    uint64_t key = qor_mix64(seed ^ qor_mix64(stream));
    int64_t sum = 0;
    for (int j = 0; j < 3; j++) {
        uint64_t h = qor_mix64(key + 3u * index + (uint64_t)j);
        sum += (int64_t)(h & 0xFFFF) + (int64_t)((h >> 16) & 0xFFFF) +
               (int64_t)((h >> 32) & 0xFFFF) + (int64_t)(h >> 48);
    }
    return (float)(sum - 393210) * (1.0f / 65536.0f);
}

static float normal_keyed(uint64_t key, uint64_t index);

void qor_fill_normal(uint64_t seed, uint64_t stream, uint64_t first_index, float *out,
                     size_t n) {
    const uint64_t key = qor_mix64(seed ^ qor_mix64(stream));  /* qor_normal's key, once per row */
    for (size_t i = 0; i < n; i++) out[i] = normal_keyed(key, first_index + i);
}

void qor_permuted_free_stack(uint64_t seed, int total, int32_t *stack) {
    for (int i = 0; i < total; i++) stack[i] = total - 1 - i;
    if (seed == 0) return;
    uint64_t key = qor_mix64(seed ^ 0x5045524Dull);
    for (int i = total - 1; i > 0; i--) {
        uint64_t j = qor_mix64(key + (uint64_t)i) % (uint64_t)(i + 1);
        int32_t t = stack[i];
        stack[i] = stack[j];
        stack[j] = t;
    }
}

void qor_outlier_channels(uint64_t seed, uint32_t layer, int channels, int count,
                          uint8_t *mask) {
    int32_t *idx = (int32_t *)malloc(sizeof(int32_t) * (size_t)channels);
    for (int i = 0; i < channels; i++) idx[i] = i;
    uint64_t key = qor_mix64(seed ^ qor_mix64(0x4F55544Cull + layer));
    if (channels > 0) memset(mask, 0, (size_t)channels);
    for (int i = 0; i < count && i < channels; i++) {
        uint64_t j = (uint64_t)i + qor_mix64(key + (uint64_t)i) % (uint64_t)(channels - i);
        int32_t t = idx[i];
        idx[i] = idx[j];
        idx[j] = t;
        mask[idx[i]] = 1;
    }
    free(idx);
}

/* ======================================================================== */
/* fp16                                                                      */
/* ======================================================================== */

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* IEEE binary32 -> binary16, round to nearest even, with subnormals; a NaN
 * stays a quiet NaN with the top ten payload bits, as the F16C conversion
 * the reference's fp16 pool write uses (_mm256_cvtps_ph). */
uint16_t qor_f32_to_f16_rne(float f) {
    uint32_t x = f2u(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7FFFFFFFu;
    if (absx >= 0x7F800000u) /* inf or nan */
        return (uint16_t)(sign | 0x7C00u | (absx > 0x7F800000u ? (0x200u | ((absx >> 13) & 0x3FFu)) : 0u));
    if (absx >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* >= 65520 */
    if (absx < 0x33000001u) return (uint16_t)sign;              /* <= 2^-25 */
    int e = (int)(absx >> 23) - 127;
    uint32_t mant = (absx & 0x7FFFFFu) | 0x800000u;
    int shift;
    uint32_t base;
    if (e < -14) { /* subnormal half: m = mant * 2^(e+1) with mant 24-bit */
        shift = -e - 1;
        base = 0;
    } else {
        shift = 13;
        base = (uint32_t)(e + 15) << 10;
        mant &= 0x7FFFFFu;
    }
    uint32_t q = mant >> shift;
    uint32_t rem = mant & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    uint32_t h = base + q; /* carry from mantissa into exponent is correct */
    if (rem > half || (rem == half && (q & 1u))) h += 1u;
    return (uint16_t)(sign | h);
}

float qor_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    if (e == 0) {
        float v = (float)m * (1.0f / 16777216.0f); /* m * 2^-24, exact */
        return sign ? -v : v;
    }
    if (e == 31) return u2f(sign | 0x7F800000u | (m << 13));
    return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

/* restates tq_float_to_half, c/qwanto_turboquant.c:106-120 (truncating,
 * NaN -> inf) */
uint16_t qor_tq_f32_to_f16(float f) {
    uint32_t x = f2u(f);
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

/* restates tq_half_to_float, c/qwanto_turboquant.c:84-104 */
float qor_tq_f16_to_f32(uint16_t h) { return qor_f16_to_f32(h); }

/* ======================================================================== */
/* codecs on logical rows                                                     */
/* ======================================================================== */

/* c/qwanto_turboquant.c:555-560 */
static int8_t q8_round(float v) {
    if (!isfinite(v)) return 0;
    if (v >= 127.0f) return 127;
    if (v <= -127.0f) return -127;
    return (int8_t)lrintf(v);
}

/* c/qwanto_turboquant.c:562-571 */
static float q8_absmax(const float *v, int n) {
    float m = 0.0f;
    for (int i = 0; i < n; i++)
        if (isfinite(v[i])) {
            float a = fabsf(v[i]);
            if (a > m) m = a;
        }
    return m;
}

/* c/qwanto_turboquant.c:573-586.  The reference also zero-fills the tail of
 * a partial 64-block past n (writing beyond the row); only n codes here. */
void qor_q8_b64_quantize(const float *src, int n, int8_t *codes, float *scales) {
    int blocks = (n + 63) / 64;
    for (int b = 0; b < blocks; b++) {
        int off = b * 64, cnt = n - off > 64 ? 64 : n - off;
        float m = q8_absmax(src + off, cnt);
        float s = m > 0.0f ? m / 127.0f : 1.0f;
        scales[b] = s;
        for (int i = 0; i < cnt; i++) codes[off + i] = q8_round(src[off + i] / s);
    }
}

/* Per token-head Q8 with an fp16 scale: the reference's rules with the
 * block widened to the head and the scale rounded to fp16 before use.
 * The scale is clamped to the finite fp16 range [2^-24, 65504]. */
void qor_q8_head_quantize(const float *src, int n, int8_t *codes, uint16_t *scale16) {
    float m = q8_absmax(src, n);
    float s = m > 0.0f ? m / 127.0f : 1.0f;
    uint16_t h = qor_f32_to_f16_rne(s);
    if ((h & 0x7FFFu) == 0) h = 0x0001u;
    if ((h & 0x7FFFu) >= 0x7C00u) h = 0x7BFFu;
    *scale16 = h;
    float sf = qor_f16_to_f32(h);
    for (int i = 0; i < n; i++) codes[i] = q8_round(src[i] / sf);
}

/* c/qwanto_turboquant.c:125-140 */
static void tq_pack16(const uint8_t *c, uint8_t *o) {
    uint8_t p[8];
    for (int i = 0; i < 8; i++) p[i] = (uint8_t)((c[2 * i] & 0x0F) | ((c[2 * i + 1] & 0x07) << 4));
    o[0] = (uint8_t)(p[0] | ((p[1] & 0x01) << 7));
    o[1] = (uint8_t)((p[1] >> 1) | ((p[2] & 0x03) << 6));
    o[2] = (uint8_t)((p[2] >> 2) | ((p[3] & 0x07) << 5));
    o[3] = (uint8_t)((p[3] >> 3) | ((p[4] & 0x0F) << 4));
    o[4] = (uint8_t)((p[4] >> 4) | ((p[5] & 0x1F) << 3));
    o[5] = (uint8_t)((p[5] >> 5) | ((p[6] & 0x3F) << 2));
    o[6] = (uint8_t)((p[6] >> 6) | (p[7] << 1));
}

/* c/qwanto_turboquant.c:142-157 */
static void tq_unpack16(const uint8_t *in, uint8_t *c) {
    uint8_t p[8];
    p[0] = in[0] & 0x7F;
    p[1] = ((in[0] >> 7) | (in[1] << 1)) & 0x7F;
    p[2] = ((in[1] >> 6) | (in[2] << 2)) & 0x7F;
    p[3] = ((in[2] >> 5) | (in[3] << 3)) & 0x7F;
    p[4] = ((in[3] >> 4) | (in[4] << 4)) & 0x7F;
    p[5] = ((in[4] >> 3) | (in[5] << 5)) & 0x7F;
    p[6] = ((in[5] >> 2) | (in[6] << 6)) & 0x7F;
    p[7] = (in[6] >> 1) & 0x7F;
    for (int i = 0; i < 8; i++) {
        c[2 * i] = p[i] & 0x0F;
        c[2 * i + 1] = (p[i] >> 4) & 0x07;
    }
}

/* min/max/range/inverse and the rounding of c/qwanto_turboquant.c:171-206,
 * for one group of `len` values, `odd_bits3` selecting the alternating
 * 4-bit/3-bit code widths of the reference (else every code is 4-bit). */
static void tq_group(const float *src, int len, int odd_bits3, uint8_t *codes,
                     uint16_t *range16, uint16_t *min16) {
    float mn = src[0], mx = src[0];
    for (int i = 1; i < len; i++) {
        float v = src[i];
        if (v < mn) mn = v;
        if (v > mx) mx = v;
    }
    float range = mx - mn;
    float inv = (range > 1e-8f) ? (1.0f / range) : 0.0f;
    *range16 = qor_tq_f32_to_f16(range);
    *min16 = qor_tq_f32_to_f16(mn);
    for (int i = 0; i < len; i++) {
        float norm = (src[i] - mn) * inv;
        if (norm < 0.0f) norm = 0.0f;
        if (norm > 1.0f) norm = 1.0f;
        int q;
        if (odd_bits3 && (i & 1)) {
            q = (int)roundf(norm * 7.0f);
            if (q > 7) q = 7;
        } else {
            q = (int)roundf(norm * 15.0f);
            if (q > 15) q = 15;
        }
        if (q < 0) q = 0;
        codes[i] = (uint8_t)q;
    }
}

/* c/qwanto_turboquant.c:162-213 */
void qor_tq35_quantize(const float *src, int n, uint8_t *blocks) {
    int nb = (n + 63) / 64;
    for (int b = 0; b < nb; b++) {
        uint8_t *blk = blocks + (size_t)b * 32;
        int off = b * 64, len = n - off > 64 ? 64 : n - off;
        uint8_t codes[64];
        uint16_t r16, m16;
        memset(codes, 0, sizeof(codes));
        tq_group(src + off, len, 1, codes, &r16, &m16);
        blk[0] = (uint8_t)(r16 & 0xFF);
        blk[1] = (uint8_t)(r16 >> 8);
        blk[2] = (uint8_t)(m16 & 0xFF);
        blk[3] = (uint8_t)(m16 >> 8);
        for (int sc = 0; sc < 4; sc++) tq_pack16(codes + sc * 16, blk + 4 + sc * 7);
    }
}

void qor_tq35_unpack(const uint8_t *block, uint8_t codes[64], uint16_t *range16,
                     uint16_t *min16) {
    *range16 = (uint16_t)(block[0] | (block[1] << 8));
    *min16 = (uint16_t)(block[2] | (block[3] << 8));
    for (int sc = 0; sc < 4; sc++) tq_unpack16(block + 4 + sc * 7, codes + sc * 16);
}

void qor_q4g32_quantize(const float *src, int n, uint8_t *codes, uint16_t *range16,
                        uint16_t *min16) {
    int ng = (n + 31) / 32;
    for (int g = 0; g < ng; g++) {
        int off = g * 32, len = n - off > 32 ? 32 : n - off;
        tq_group(src + off, len, 0, codes + off, &range16[g], &min16[g]);
    }
}

/* ======================================================================== */
/* paged tile layout (this project's format, head_dim 128, 16 tokens)         */
/* ======================================================================== */
/*
 * A tile holds 16 tokens of one (page, layer, kv head).  Byte positions are
 * chosen so that each lane of a warp loads its mma.sync fragments with a few
 * 128-bit shared-memory loads and no bank conflicts:
 *  - int8 K (bytes 0..2047), token t, dim d: row t of 128 bytes (the A
 *    operand rows of the integer QK^T product), 16-byte chunk (d>>4) stored
 *    at position (d>>4) xor ((t&1)<<2), byte d&15; stored biased (code+128).
 *  - int8 V (bytes 2048..4095), token t, dim d: m-block mb=d>>4, row
 *    r=d&15, lane ((r&7)<<2)|((t&7)>>1); the lane's 64 bytes hold 8 bytes
 *    per m-block, 16-byte chunk (mb>>1) stored at position
 *    (mb>>1) xor ((lane>>1)&3), byte 8*(mb&1) + 4*(t>>3) + 2*(r>>3) + (t&1):
 *    the A operand (dims x tokens) of the PV product; biased.
 *  - int8 scales: tokens t and t+8 adjacent.  Q8_HEAD: fp16 K scale at
 *    4096 + 4*(t&7) + 2*(t>>3), V scale at 4128 + same.  Q8_B64: fp32 K
 *    scale of channel block x at 4096 + 16*(t&7) + 8*x + 4*(t>>3), V at
 *    4224 + same.
 *  - low-bit codecs (4-bit groups of 32, 3.5-bit TurboQuant) are organised
 *    in classes of 32 dims with one scale each: codec 4 class c = d>>5 (the
 *    group), index m = d&31; TurboQuant class c = 2*(d>>6) + (d&1) (group,
 *    parity), index m = (d&63)>>1.  K codes are the A rows of the integer
 *    QK^T product: the "K word" of (token t, tig = m>>3, class c) holds the
 *    8 codes m = 8*tig+i in byte i&3, low nibble for i<4, high for i>=4.
 *    V codes are the A operand of P x V: m-block mb = 2c + (m>>4), row
 *    r = m&15, lane ((r&7)<<2)|((t&7)>>1), nibble (r>>3) + 2*(t>>3) + 4*(t&1)
 *    of the lane's word for mb.
 *    codec 4 (2560 B): K word at 64t + 16tig + 4c; V word at 1024 + 32*lane
 *    + 16*((mb>>2) ^ ((lane>>2)&1)) + 4*(mb&3); params (range16, min16) at
 *    2048 (K) / 2304 (V) + 32*(t&7) + 8c + 4*(t>>3).
 *    codec 3 (2048 B): K half [0,1024), V half [1024,2048), each: 4-bit even
 *    codes, 3-bit odd codes (group 0 in the low 3 bits of a nibble, bit 0
 *    of group 1 in its top bit), a plane of the group-1 odd codes' bits 1-2
 *    (two bits per nibble position n at bit 2n), params (range16, min16) at
 *    896 + 16*(t&7) + 8*group + 4*(t>>3).  K: even word at 32t + 8tig +
 *    4*group, odd word at 512 + 16t + 4tig, plane u16 at 768 + 8t + 2tig.
 *    V: even word e = 2*group + (mb&1) at 16*lane + 4e, odd word k = mb&1 at
 *    512 + 8*lane + 4k, plane u16 at 768 + 4*lane + 2k.
 *  - fp16 (codec 5, 8192 B): K [0,4096), V [4096,8192), each row t of 256
 *    bytes holds dims 0..127 as fp16 (RNE), 16-byte chunk c = d>>3 stored
 *    at position c xor (t&7), so that ldmatrix reads eight rows without bank
 *    conflicts.
 */

size_t qor_tile_bytes(int codec) {
    switch (codec) {
        case QOR_CODEC_Q8_B64_F32: return 4352;
        case QOR_CODEC_Q8_HEAD_F16: return 4160;
        case QOR_CODEC_TQ35_G64: return 2048;
        case QOR_CODEC_Q4_G32: return 2560;
        case QOR_CODEC_F16: return 8192;
        default: return 0;
    }
}

static size_t k8_off(int t, int d) {
    return (size_t)t * 128 + (size_t)(((d >> 4) ^ ((t & 1) << 2)) << 4) + (size_t)(d & 15);
}

static size_t v8_off(int t, int d) {
    int mb = d >> 4, r = d & 15, lane = ((r & 7) << 2) | ((t & 7) >> 1);
    int chunk = (mb >> 1) ^ ((lane >> 1) & 3);
    int e = 4 * (t >> 3) + 2 * (r >> 3) + (t & 1);
    return 2048 + (size_t)lane * 64 + (size_t)chunk * 16 + (size_t)(8 * (mb & 1) + e);
}

/* fp16 element (t, d) of the K (is_value 0) or V half */
static size_t f16_off(int is_value, int t, int d) {
    return (size_t)is_value * 4096 + (size_t)t * 256 + (size_t)((((d >> 3) ^ (t & 7))) << 4) + (size_t)(d & 7) * 2;
}

/* int8 scale positions (see the layout notes above) */
static size_t s16_off(int t) { return (size_t)(4 * (t & 7) + 2 * (t >> 3)); }
static size_t s32_off(int t, int x) { return (size_t)(16 * (t & 7) + 8 * x + 4 * (t >> 3)); }

/* low-bit class structure: class and index within the class of dim d */
static void lb_class(int codec, int d, int *c, int *m) {
    if (codec == QOR_CODEC_Q4_G32) { *c = d >> 5; *m = d & 31; }
    else { *c = 2 * (d >> 6) + (d & 1); *m = (d & 63) >> 1; }
}
/* K word position: (t, tig, c) and the nibble n (0..7, bit 4n) of code m */
static int lb_k_nibble(int m) { int i = m & 7; return 2 * (i & 3) + (i >> 2); }
/* V: lane, m-block and nibble of (t, d) */
static void lb_v(int codec, int t, int d, int *lane, int *mb, int *nib) {
    int c, m;
    lb_class(codec, d, &c, &m);
    int r = m & 15;
    *mb = 2 * c + (m >> 4);
    *lane = ((r & 7) << 2) | ((t & 7) >> 1);
    *nib = (r >> 3) + 2 * (t >> 3) + 4 * (t & 1);
}
/* nibble address: byte offset and high(1)/low(0) nibble (codec 4) */
static void k4_pos(int t, int d, size_t *byte, int *hi) {
    int c, m;
    lb_class(QOR_CODEC_Q4_G32, d, &c, &m);
    int n = lb_k_nibble(m);
    *byte = (size_t)t * 64 + (size_t)(m >> 3) * 16 + (size_t)c * 4 + (size_t)(n >> 1);
    *hi = n & 1;
}

static void v4_pos(int t, int d, size_t *byte, int *hi) {
    int lane, mb, n;
    lb_v(QOR_CODEC_Q4_G32, t, d, &lane, &mb, &n);
    int chunk = (mb >> 2) ^ ((lane >> 2) & 1);
    *byte = 1024 + (size_t)lane * 32 + (size_t)chunk * 16 + (size_t)(mb & 3) * 4 + (size_t)(n >> 1);
    *hi = n & 1;
}
/* low-bit params: (range16, min16) of (t, class c) for codec 4, (t, group x) for codec 3 */
static size_t q4_param_off(int t, int c) { return (size_t)(32 * (t & 7) + 8 * c + 4 * (t >> 3)); }
static size_t tq_param_off(int t, int x) { return (size_t)(896 + 16 * (t & 7) + 8 * x + 4 * (t >> 3)); }

static void put_nib(uint8_t *tile, size_t byte, int hi, uint8_t v) {
    if (hi) tile[byte] = (uint8_t)((tile[byte] & 0x0F) | ((v & 0x0F) << 4));
    else tile[byte] = (uint8_t)((tile[byte] & 0xF0) | (v & 0x0F));
}
static uint8_t get_nib(const uint8_t *tile, size_t byte, int hi) {
    return hi ? (uint8_t)(tile[byte] >> 4) : (uint8_t)(tile[byte] & 0x0F);
}
static void put_u16(uint8_t *p, uint16_t v) { p[0] = (uint8_t)(v & 0xFF); p[1] = (uint8_t)(v >> 8); }
static uint16_t get_u16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static void put_f32(uint8_t *p, float v) { memcpy(p, &v, 4); }
static float get_f32(const uint8_t *p) { float v; memcpy(&v, p, 4); return v; }

/* 3.5-bit TurboQuant codes: see the layout notes above.  Odd codes of group
 * 0 fill bits 0-2 of a nibble; bit 0 of the group-1 odd code sits in bit 3
 * of the same nibble and its bits 1-2 in the plane at bit 2n. */
static void tq_pos(int is_value, int t, int d, size_t *even_byte, int *even_hi, size_t *odd_byte,
                   int *odd_hi, size_t *plane_byte, int *plane_shift) {
    int c, m;
    lb_class(QOR_CODEC_TQ35_G64, d, &c, &m);
    int x = c >> 1;
    if (!is_value) {
        int tig = m >> 3, n = lb_k_nibble(m);
        *even_byte = (size_t)(32 * t + 8 * tig + 4 * x + (n >> 1));
        *odd_byte = (size_t)(512 + 16 * t + 4 * tig + (n >> 1));
        *even_hi = *odd_hi = n & 1;
        *plane_byte = (size_t)(768 + 8 * t + 2 * tig + ((2 * n) >> 3));
        *plane_shift = (2 * n) & 7;
    } else {
        int lane, mb, n;
        lb_v(QOR_CODEC_TQ35_G64, t, d, &lane, &mb, &n);
        int e = 2 * x + (mb & 1), k = mb & 1;
        *even_byte = (size_t)(16 * lane + 4 * e + (n >> 1));
        *odd_byte = (size_t)(512 + 8 * lane + 4 * k + (n >> 1));
        *even_hi = *odd_hi = n & 1;
        *plane_byte = (size_t)(768 + 4 * lane + 2 * k + ((2 * n) >> 3));
        *plane_shift = (2 * n) & 7;
    }
}

static void tq_store_codes(uint8_t *half, int is_value, int t, int d, uint8_t code) {
    size_t eb, ob, pb; int eh, oh, ps;
    tq_pos(is_value, t, d, &eb, &eh, &ob, &oh, &pb, &ps);
    int x = d >> 6;
    if (!(d & 1)) {
        put_nib(half, eb, eh, code);
    } else {
        uint8_t nib = get_nib(half, ob, oh);
        if (x == 0) nib = (uint8_t)((nib & 0x8) | (code & 0x7));
        else nib = (uint8_t)((nib & 0x7) | ((code & 1) << 3));
        put_nib(half, ob, oh, nib);
        if (x == 1) half[pb] = (uint8_t)((half[pb] & ~(3u << ps)) | (((code >> 1) & 3u) << ps));
    }
}

static uint8_t tq_load_code(const uint8_t *half, int is_value, int t, int d) {
    size_t eb, ob, pb; int eh, oh, ps;
    tq_pos(is_value, t, d, &eb, &eh, &ob, &oh, &pb, &ps);
    if (!(d & 1)) return get_nib(half, eb, eh);
    uint8_t nib = get_nib(half, ob, oh);
    if ((d >> 6) == 0) return nib & 0x7;
    return (uint8_t)((nib >> 3) | (((half[pb] >> ps) & 3u) << 1));
}

void qor_tile_store(int codec, uint8_t *tile, int t, const float *k, const float *v) {
    const int HD = QOR_HEAD_DIM;
    if (codec == QOR_CODEC_F16) { /* c/qwn_paged_kv.c:151-198: fp32 -> fp16 RNE */
        for (int d = 0; d < HD; d++) {
            put_u16(tile + f16_off(0, t, d), qor_f32_to_f16_rne(k[d]));
            put_u16(tile + f16_off(1, t, d), qor_f32_to_f16_rne(v[d]));
        }
        return;
    }
    if (codec == QOR_CODEC_Q8_B64_F32 || codec == QOR_CODEC_Q8_HEAD_F16) {
        int8_t ck[HD], cv[HD];
        if (codec == QOR_CODEC_Q8_B64_F32) {
            float sk[2], sv[2];
            qor_q8_b64_quantize(k, HD, ck, sk);
            qor_q8_b64_quantize(v, HD, cv, sv);
            for (int x = 0; x < 2; x++) {
                put_f32(tile + 4096 + s32_off(t, x), sk[x]);
                put_f32(tile + 4224 + s32_off(t, x), sv[x]);
            }
        } else {
            uint16_t sk, sv;
            qor_q8_head_quantize(k, HD, ck, &sk);
            qor_q8_head_quantize(v, HD, cv, &sv);
            put_u16(tile + 4096 + s16_off(t), sk);
            put_u16(tile + 4128 + s16_off(t), sv);
        }
        for (int d = 0; d < HD; d++) {
            tile[k8_off(t, d)] = (uint8_t)((int)ck[d] + 128);
            tile[v8_off(t, d)] = (uint8_t)((int)cv[d] + 128);
        }
    } else if (codec == QOR_CODEC_Q4_G32) {
        uint8_t ck[HD], cv[HD];
        uint16_t rk[4], mk[4], rv[4], mv[4];
        qor_q4g32_quantize(k, HD, ck, rk, mk);
        qor_q4g32_quantize(v, HD, cv, rv, mv);
        for (int d = 0; d < HD; d++) {
            size_t byte; int hi;
            k4_pos(t, d, &byte, &hi); put_nib(tile, byte, hi, ck[d]);
            v4_pos(t, d, &byte, &hi); put_nib(tile, byte, hi, cv[d]);
        }
        for (int g = 0; g < 4; g++) {
            put_u16(tile + 2048 + q4_param_off(t, g), rk[g]);
            put_u16(tile + 2048 + q4_param_off(t, g) + 2, mk[g]);
            put_u16(tile + 2304 + q4_param_off(t, g), rv[g]);
            put_u16(tile + 2304 + q4_param_off(t, g) + 2, mv[g]);
        }
    } else if (codec == QOR_CODEC_TQ35_G64) {
        uint8_t bk[64], bv[64];
        qor_tq35_quantize(k, HD, bk);
        qor_tq35_quantize(v, HD, bv);
        for (int x = 0; x < 2; x++) {
            uint8_t codes_k[64], codes_v[64];
            uint16_t r, m;
            qor_tq35_unpack(bk + x * 32, codes_k, &r, &m);
            put_u16(tile + tq_param_off(t, x), r);
            put_u16(tile + tq_param_off(t, x) + 2, m);
            qor_tq35_unpack(bv + x * 32, codes_v, &r, &m);
            put_u16(tile + 1024 + tq_param_off(t, x), r);
            put_u16(tile + 1024 + tq_param_off(t, x) + 2, m);
            for (int i = 0; i < 64; i++) {
                tq_store_codes(tile, 0, t, x * 64 + i, codes_k[i]);
                tq_store_codes(tile + 1024, 1, t, x * 64 + i, codes_v[i]);
            }
        }
    }
}

void qor_tile_load(int codec, const uint8_t *tile, int t, int is_value, int16_t codes[128],
                   float *params) {
    const int HD = QOR_HEAD_DIM;
    if (codec == QOR_CODEC_Q8_B64_F32 || codec == QOR_CODEC_Q8_HEAD_F16) {
        for (int d = 0; d < HD; d++)
            codes[d] = (int16_t)((int)tile[is_value ? v8_off(t, d) : k8_off(t, d)] - 128);
        if (codec == QOR_CODEC_Q8_B64_F32) {
            for (int x = 0; x < 2; x++)
                params[x] = get_f32(tile + (is_value ? 4224 : 4096) + s32_off(t, x));
        } else {
            params[0] = qor_f16_to_f32(get_u16(tile + (is_value ? 4128 : 4096) + s16_off(t)));
        }
    } else if (codec == QOR_CODEC_Q4_G32) {
        for (int d = 0; d < HD; d++) {
            size_t byte; int hi;
            if (is_value) v4_pos(t, d, &byte, &hi); else k4_pos(t, d, &byte, &hi);
            codes[d] = get_nib(tile, byte, hi);
        }
        for (int g = 0; g < 4; g++) {
            const uint8_t *p = tile + (is_value ? 2304 : 2048) + q4_param_off(t, g);
            params[2 * g] = qor_tq_f16_to_f32(get_u16(p));
            params[2 * g + 1] = qor_tq_f16_to_f32(get_u16(p + 2));
        }
    } else if (codec == QOR_CODEC_TQ35_G64) {
        const uint8_t *half = tile + (is_value ? 1024 : 0);
        for (int d = 0; d < HD; d++) codes[d] = tq_load_code(half, is_value, t, d);
        for (int x = 0; x < 2; x++) {
            params[2 * x] = qor_tq_f16_to_f32(get_u16(half + tq_param_off(t, x)));
            params[2 * x + 1] = qor_tq_f16_to_f32(get_u16(half + tq_param_off(t, x) + 2));
        }
    }
}

float qor_tile_dequant(int codec, const uint8_t *tile, int t, int is_value, int d) {
    if (codec == QOR_CODEC_F16) return qor_f16_to_f32(get_u16(tile + f16_off(is_value, t, d)));
    int16_t codes[128];
    float params[8];
    qor_tile_load(codec, tile, t, is_value, codes, params);
    switch (codec) {
        case QOR_CODEC_Q8_B64_F32: return (float)codes[d] * params[d >> 6];
        case QOR_CODEC_Q8_HEAD_F16: return (float)codes[d] * params[0];
        case QOR_CODEC_Q4_G32: {
            int g = d >> 5;
            float s = params[2 * g] * (1.0f / 15.0f);
            return (float)codes[d] * s + params[2 * g + 1];
        }
        case QOR_CODEC_TQ35_G64: {
            int x = d >> 6;
            float s = (d & 1) ? params[2 * x] * (1.0f / 7.0f) : params[2 * x] * (1.0f / 15.0f);
            return (float)codes[d] * s + params[2 * x + 1];
        }
    }
    return 0.0f;
}

/* ======================================================================== */
/* pool / block table                                                         */
/* ======================================================================== */

int qor_pool_init(QorPool *p, int codec, int layers, int kv_heads, int page_tokens,
                  int total_pages, int max_seqs, int max_pages_per_seq, uint64_t perm_seed) {
    return qor_pool_init_ex(p, codec, layers, kv_heads, page_tokens, total_pages, max_seqs,
                            max_pages_per_seq, perm_seed, 1);
}

int qor_pool_init_ex(QorPool *p, int codec, int layers, int kv_heads, int page_tokens,
                     int total_pages, int max_seqs, int max_pages_per_seq, uint64_t perm_seed,
                     int with_pages) {
    memset(p, 0, sizeof(*p));
    if (qor_tile_bytes(codec) == 0 || page_tokens <= 0 || page_tokens % 16) return -1;
    p->codec = codec; p->layers = layers; p->kv_heads = kv_heads; p->page_tokens = page_tokens;
    p->total_pages = total_pages; p->max_seqs = max_seqs; p->max_pages_per_seq = max_pages_per_seq;
    p->tile_bytes = qor_tile_bytes(codec);
    p->page_bytes = p->tile_bytes * (size_t)(page_tokens / 16) * (size_t)layers * (size_t)kv_heads;
    p->pages = with_pages ? (uint8_t *)calloc((size_t)total_pages, p->page_bytes) : NULL;
    p->free_stack = (int32_t *)malloc(sizeof(int32_t) * (size_t)total_pages);
    p->page_table = (int32_t *)malloc(sizeof(int32_t) * (size_t)max_seqs * (size_t)max_pages_per_seq);
    p->lens = (int32_t *)calloc((size_t)max_seqs, sizeof(int32_t));
    p->npages = (int32_t *)calloc((size_t)max_seqs, sizeof(int32_t));
    p->page_score = (float *)calloc((size_t)max_seqs * (size_t)max_pages_per_seq, sizeof(float));
    if ((with_pages && !p->pages) || !p->free_stack || !p->page_table || !p->lens || !p->npages || !p->page_score) {
        qor_pool_free(p);
        return -1;
    }
    for (size_t i = 0; i < (size_t)max_seqs * (size_t)max_pages_per_seq; i++) p->page_table[i] = -1;
    qor_permuted_free_stack(perm_seed, total_pages, p->free_stack);
    p->free_top = total_pages;
    return 0;
}

void qor_pool_free(QorPool *p) {
    free(p->pages); free(p->free_stack); free(p->page_table); free(p->lens);
    free(p->npages); free(p->page_score);
    memset(p, 0, sizeof(*p));
}

/* qwn_block_table_append_token applied counts[i] times per sequence, in
 * order; pages popped from the top of the free stack (c/qwn_paged_kv.c:95-98,
 * :115-138).  All-or-nothing, like the device allocator. */
int qor_pool_append(QorPool *p, int n, const int32_t *seq_ids, const int32_t *counts) {
    int P = p->page_tokens;
    long need = 0;
    for (int i = 0; i < n; i++) {
        int s = seq_ids[i];
        int np = (p->lens[s] + counts[i] + P - 1) / P;
        int add = np - p->npages[s];
        if (np > p->max_pages_per_seq) return -1;
        need += add > 0 ? add : 0;
    }
    if (need > p->free_top) return -1;
    for (int i = 0; i < n; i++) {
        int s = seq_ids[i];
        int np = (p->lens[s] + counts[i] + P - 1) / P;
        while (p->npages[s] < np) {
            int32_t pg = p->free_stack[--p->free_top];
            p->page_table[(size_t)s * p->max_pages_per_seq + p->npages[s]] = pg;
            p->page_score[(size_t)s * p->max_pages_per_seq + p->npages[s]] = 1.0f;
            p->npages[s]++;
        }
        p->lens[s] += counts[i];
    }
    return 0;
}

uint8_t *qor_pool_tile(QorPool *p, int seq, int layer, int kv_head, int pos) {
    int P = p->page_tokens, tiles = P / 16;
    int lp = pos / P, tile = (pos % P) / 16;
    int32_t pg = p->page_table[(size_t)seq * p->max_pages_per_seq + lp];
    if (pg < 0 || !p->pages) return NULL;
    size_t off = (size_t)pg * p->page_bytes +
                 (((size_t)layer * p->kv_heads + kv_head) * tiles + tile) * p->tile_bytes;
    return p->pages + off;
}

int qor_pool_write_token(QorPool *p, int seq, int layer, int pos, const float *k,
                         const float *v) {
    if (pos < 0 || pos >= p->lens[seq]) return -1;
    for (int h = 0; h < p->kv_heads; h++) {
        uint8_t *tile = qor_pool_tile(p, seq, layer, h, pos);
        if (!tile) return -1;
        qor_tile_store(p->codec, tile, pos % 16, k + h * 128, v + h * 128);
    }
    return 0;
}

/* The synthetic K/V rows of (seed, seq, gen_layer) for positions
 * [first, last), stored into `layer`: K = normal(kind 2) x 8 on the channels
 * k_outlier_mask marks, V = normal(kind 3) -- the values qwn_kv_prefill_synthetic
 * and qwn_kv_generate_rows produce on the device. */
static float normal_keyed(uint64_t key, uint64_t index) {
    int64_t sum = 0;
    for (int j = 0; j < 3; j++) {
        uint64_t h = qor_mix64(key + 3u * index + (uint64_t)j);
        sum += (int64_t)(h & 0xFFFF) + (int64_t)((h >> 16) & 0xFFFF) +
               (int64_t)((h >> 32) & 0xFFFF) + (int64_t)(h >> 48);
    }
    return (float)(sum - 393210) * (1.0f / 65536.0f);
}

int qor_pool_fill_synthetic(QorPool *p, int seq, int layer, int gen_layer, int first, int last,
                            uint64_t seed, const uint8_t *k_outlier_mask) {
    if (!p->pages || first < 0 || last > p->lens[seq] || layer < 0 || layer >= p->layers) return -1;
    const int W = p->kv_heads * 128;
    float *k = (float *)malloc(sizeof(float) * (size_t)W);
    float *v = (float *)malloc(sizeof(float) * (size_t)W);
    if (!k || !v) { free(k); free(v); return -1; }
    const uint64_t kk = qor_mix64(seed ^ qor_mix64(qor_stream(2, (uint32_t)seq, (uint32_t)gen_layer)));
    const uint64_t kv = qor_mix64(seed ^ qor_mix64(qor_stream(3, (uint32_t)seq, (uint32_t)gen_layer)));
    int rc = 0;
    for (int t = first; t < last && rc == 0; t++) {
        for (int c = 0; c < W; c++) {
            float x = normal_keyed(kk, (uint64_t)t * (uint64_t)W + (uint64_t)c);
            k[c] = (k_outlier_mask && k_outlier_mask[c]) ? x * 8.0f : x;
            v[c] = normal_keyed(kv, (uint64_t)t * (uint64_t)W + (uint64_t)c);
        }
        rc = qor_pool_write_token(p, seq, layer, t, k, v);
    }
    free(k);
    free(v);
    return rc;
}

static const uint8_t *ctile(const QorPool *p, int seq, int layer, int kv, int pos) {
    return qor_pool_tile((QorPool *)p, seq, layer, kv, pos);
}

/* one token's dot product in the reference's order:
 *  Q8 (c/qwanto_turboquant.c:648-662): total += q[i] * (code * scale)
 *  TurboQuant scalar (:218-252): per group block_dot += q*(code*s+zp); total += block_dot */
static float token_dot(const QorPool *p, const uint8_t *tile, int t, const float *q) {
    if (p->codec == QOR_CODEC_F16) { /* c/qwn_paged_kv.c:338-355: dot of q with the fp16 row */
        float total = 0.0f;
        for (int i = 0; i < 128; i++) total += q[i] * qor_f16_to_f32(get_u16(tile + f16_off(0, t, i)));
        return total;
    }
    int16_t c[128];
    float par[8];
    qor_tile_load(p->codec, tile, t, 0, c, par);
    float total = 0.0f;
    if (p->codec == QOR_CODEC_Q8_B64_F32) {
        for (int i = 0; i < 128; i++) total += q[i] * ((float)c[i] * par[i >> 6]);
    } else if (p->codec == QOR_CODEC_Q8_HEAD_F16) {
        for (int i = 0; i < 128; i++) total += q[i] * ((float)c[i] * par[0]);
    } else {
        int gs = p->codec == QOR_CODEC_Q4_G32 ? 32 : 64;
        for (int g = 0; g < 128 / gs; g++) {
            float scale = par[2 * g], zp = par[2 * g + 1];
            float s_even = scale * (1.0f / 15.0f);
            float s_odd = p->codec == QOR_CODEC_Q4_G32 ? s_even : scale * (1.0f / 7.0f);
            float bd = 0.0f;
            for (int i = 0; i < gs; i++) {
                float kv = (i & 1) ? (float)c[g * gs + i] * s_odd + zp : (float)c[g * gs + i] * s_even + zp;
                bd += q[g * gs + i] * kv;
            }
            total += bd;
        }
    }
    return total;
}

static void token_value(const QorPool *p, const uint8_t *tile, int t, float *v) {
    if (p->codec == QOR_CODEC_F16) {
        for (int i = 0; i < 128; i++) v[i] = qor_f16_to_f32(get_u16(tile + f16_off(1, t, i)));
        return;
    }
    int16_t c[128];
    float par[8];
    qor_tile_load(p->codec, tile, t, 1, c, par);
    for (int i = 0; i < 128; i++) {
        if (p->codec == QOR_CODEC_Q8_B64_F32) v[i] = (float)c[i] * par[i >> 6];
        else if (p->codec == QOR_CODEC_Q8_HEAD_F16) v[i] = (float)c[i] * par[0];
        else {
            int gs = p->codec == QOR_CODEC_Q4_G32 ? 32 : 64, g = i / gs;
            float scale = par[2 * g], zp = par[2 * g + 1];
            float s = (p->codec == QOR_CODEC_TQ35_G64 && (i & 1)) ? scale * (1.0f / 7.0f)
                                                                   : scale * (1.0f / 15.0f);
            v[i] = (float)c[i] * s + zp;
        }
    }
}

/* c/qwanto_turboquant.c:678-705 (Q8) and :739-768 (TurboQuant): scores,
 * max, expf, fp32 sum, inv = 1/sum, ctx += (p*inv) * value. */
void qor_pool_attention(const QorPool *p, int seq, int layer, int len, const float *q,
                        int H, float scale, float *out, float *token_probs) {
    int HK = p->kv_heads;
    if (!p->pages) { memset(out, 0, sizeof(float) * (size_t)H * 128); return; }
    float *scores = (float *)malloc(sizeof(float) * (size_t)(len > 0 ? len : 1));
    float vrow[128];
    for (int h = 0; h < H; h++) {
        int kv = (h * HK) / H;
        const float *qh = q + (size_t)h * 128;
        float *o = out + (size_t)h * 128;
        memset(o, 0, sizeof(float) * 128);
        if (len <= 0) continue;
        for (int t = 0; t < len; t++)
            scores[t] = token_dot(p, ctile(p, seq, layer, kv, t), t % 16, qh) * scale;
        float mx = scores[0];
        for (int t = 1; t < len; t++) if (scores[t] > mx) mx = scores[t];
        float sum = 0.0f;
        for (int t = 0; t < len; t++) { scores[t] = expf(scores[t] - mx); sum += scores[t]; }
        float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
        for (int t = 0; t < len; t++) {
            float pt = scores[t] * inv;
            if (token_probs) token_probs[(size_t)h * len + t] = pt;
            token_value(p, ctile(p, seq, layer, kv, t), t % 16, vrow);
            for (int i = 0; i < 128; i++) o[i] += pt * vrow[i];
        }
    }
    free(scores);
}

void qor_partial_attention(const QorPool *p, int seq, int layer, int t0, int t1,
                           const float *q, int H, float scale, float *m, float *l, float *o) {
    const float log2e = 1.4426950408889634f;
    int HK = p->kv_heads;
    float vrow[128];
    for (int h = 0; h < H; h++) {
        int kv = (h * HK) / H;
        const float *qh = q + (size_t)h * 128;
        float mx = -INFINITY;
        for (int t = t0; t < t1; t++) {
            float s = token_dot(p, ctile(p, seq, layer, kv, t), t % 16, qh) * scale * log2e;
            if (s > mx) mx = s;
        }
        float sum = 0.0f;
        float *oh = o + (size_t)h * 128;
        memset(oh, 0, sizeof(float) * 128);
        for (int t = t0; t < t1; t++) {
            float s = token_dot(p, ctile(p, seq, layer, kv, t), t % 16, qh) * scale * log2e;
            float e = exp2f(s - mx);
            sum += e;
            token_value(p, ctile(p, seq, layer, kv, t), t % 16, vrow);
            for (int i = 0; i < 128; i++) oh[i] += e * vrow[i];
        }
        m[h] = mx;
        l[h] = sum;
    }
}

void qor_merge_partials(int nparts, int H, const float *m, const float *l, const float *o,
                        float *out) {
    for (int h = 0; h < H; h++) {
        float ms = -INFINITY;
        for (int i = 0; i < nparts; i++) if (m[(size_t)i * H + h] > ms) ms = m[(size_t)i * H + h];
        float ls = 0.0f;
        for (int i = 0; i < nparts; i++) ls += l[(size_t)i * H + h] * exp2f(m[(size_t)i * H + h] - ms);
        for (int d = 0; d < 128; d++) {
            float acc = 0.0f;
            for (int i = 0; i < nparts; i++)
                acc += o[((size_t)i * H + h) * 128 + d] * exp2f(m[(size_t)i * H + h] - ms);
            out[(size_t)h * 128 + d] = ls > 0.0f ? acc / ls : 0.0f;
        }
    }
}

/* ======================================================================== */
/* eviction                                                                   */
/* ======================================================================== */

/* c/qwanto_pagedeviction.c:7-21 */
int qor_vtoken_init(QorEvictionPool *p, uint32_t max_capacity, uint32_t physical,
                    float threshold) {
    if (!p || max_capacity == 0 || physical == 0) return -1;
    if (max_capacity > QOR_VTOKEN_MAX_CAPACITY) max_capacity = QOR_VTOKEN_MAX_CAPACITY;
    memset(p, 0, sizeof(*p));
    p->max_capacity = max_capacity;
    p->physical_pool_size = physical;
    p->eviction_threshold = threshold > 0.0f ? threshold : 0.05f;
    return 0;
}

/* c/qwanto_pagedeviction.c:24-52 */
int qor_vtoken_insert(QorEvictionPool *p, uint32_t token_id, float importance, uint32_t *slot) {
    if (!p || !slot) return -1;
    if (p->active_count >= p->physical_pool_size) {
        uint32_t target = (uint32_t)((float)p->physical_pool_size * 0.9f);
        qor_vtoken_prune(p, target);
    }
    uint32_t s = p->active_count;
    if (s >= p->max_capacity) return -2;
    QorVToken *t = &p->tokens[s];
    t->token_id = token_id;
    t->importance_score = importance > 0.0f ? importance : 1.0f;
    t->physical_slot = s;
    t->is_sink = token_id < QOR_VTOKEN_SINK_TOKENS;
    t->is_active = 1;
    *slot = s;
    p->active_count++;
    return 0;
}

/* c/qwanto_pagedeviction.c:54-70.  `fused` selects fmaf(0.8,old,0.2*new),
 * the form gcc emits for the reference's -mfma -ffp-contract=fast build. */
void qor_vtoken_update_scores(QorEvictionPool *p, const float *scores, uint32_t n, int fused) {
    if (!p || !scores) return;
    uint32_t count = n < p->active_count ? n : p->active_count;
    for (uint32_t i = 0; i < count; i++) {
        if (p->tokens[i].is_sink) continue;
        float old = p->tokens[i].importance_score, nw = scores[i];
        p->tokens[i].importance_score = fused ? fmaf(0.8f, old, 0.2f * nw) : 0.8f * old + 0.2f * nw;
    }
}

/* c/qwanto_pagedeviction.c:72-93: while evicted < to_evict the condition
 * `score < thr || evicted < to_evict` holds, so the first non-sink active
 * slots from index 4 are evicted in index order; active_count unchanged. */
uint32_t qor_vtoken_prune(QorEvictionPool *p, uint32_t target) {
    if (!p || p->active_count <= target) return 0;
    uint32_t to_evict = p->active_count - target, evicted = 0;
    for (uint32_t i = QOR_VTOKEN_SINK_TOKENS; i < p->active_count && evicted < to_evict; i++) {
        if (p->tokens[i].is_active && !p->tokens[i].is_sink) {
            if (p->tokens[i].importance_score < p->eviction_threshold || evicted < to_evict) {
                p->tokens[i].is_active = 0;
                evicted++;
            }
        }
    }
    p->total_evictions += evicted;
    return evicted;
}

/* c/qwanto_pagedeviction.c:95-103 */
float qor_vtoken_waste_pct(const QorEvictionPool *p) {
    if (!p || p->physical_pool_size == 0) return 0.0f;
    if (p->active_count >= p->physical_pool_size) return 4.8f;
    return 5.2f;
}

int qor_evict_trigger(uint64_t seed, uint32_t step, uint32_t seq, double prob) {
    uint64_t h = qor_mix64(qor_mix64(seed ^ 0x45564943ull) + ((uint64_t)step << 32) + seq);
    double u = (double)(h >> 11) * (1.0 / 9007199254740992.0);
    return u < prob;
}

int qor_pool_evict(QorPool *p, int nseqs, const int32_t *seq_ids, const float *mass,
                   const uint8_t *flags, int budget) {
    int P = p->page_tokens, MP = p->max_pages_per_seq;
    int total = 0;
    /* EMA on every live page of the listed sequences */
    for (int i = 0; i < nseqs; i++) {
        int s = seq_ids[i];
        for (int pg = 0; pg < p->npages[s]; pg++) {
            float *sc = &p->page_score[(size_t)s * MP + pg];
            float a = 0.8f * *sc;
            float b = 0.2f * mass[(size_t)s * MP + pg];
            *sc = a + b;
        }
    }
    int32_t *order = (int32_t *)malloc(sizeof(int32_t) * (size_t)MP);
    uint8_t *dead = (uint8_t *)malloc((size_t)MP);
    for (int i = 0; i < nseqs; i++) {
        int s = seq_ids[i];
        if (!flags[i] || p->lens[s] <= budget) continue;
        int np = p->npages[s];
        if (np < 3) continue;
        int want = (p->lens[s] - budget + P - 1) / P;
        int cand = np - 2;
        int ne = want < cand ? want : cand;
        /* rank candidates 1..np-2 by (score, index) */
        int nc = 0;
        for (int pg = 1; pg <= np - 2; pg++) order[nc++] = pg;
        const float *sc = p->page_score + (size_t)s * MP;
        for (int a = 1; a < nc; a++) { /* stable insertion sort: ties keep index order */
            int32_t x = order[a];
            int b = a - 1;
            while (b >= 0 && sc[order[b]] > sc[x]) { order[b + 1] = order[b]; b--; }
            order[b + 1] = x;
        }
        memset(dead, 0, (size_t)np);
        for (int e = 0; e < ne; e++) dead[order[e]] = 1;
        int32_t *pt = p->page_table + (size_t)s * MP;
        float *ps = p->page_score + (size_t)s * MP;
        for (int pg = 0; pg < np; pg++) /* freed pages, ascending logical order */
            if (dead[pg]) p->free_stack[p->free_top++] = pt[pg];
        int w = 0;
        for (int pg = 0; pg < np; pg++) {
            if (dead[pg]) continue;
            pt[w] = pt[pg];
            ps[w] = ps[pg];
            w++;
        }
        for (int pg = w; pg < np; pg++) { pt[pg] = -1; ps[pg] = 0.0f; }
        p->npages[s] = w;
        p->lens[s] -= ne * P;
        total += ne;
    }
    free(order);
    free(dead);
    return total;
}

/* ======================================================================== */
/* linear attention (c/qwanto_attention.c:34-156)                            */
/* ======================================================================== */
void qor_linear_attention_decode(float *state, int n_heads, int head_dim, const float *q,
                                 const float *k, const float *v, float decay, float *o) {
    const int d = head_dim;
    for (int h = 0; h < n_heads; h++) {
        float *s = state + (size_t)h * d * d;
        const float *qh = q + (size_t)h * d, *kh = k + (size_t)h * d, *vh = v + (size_t)h * d;
        float *oh = o + (size_t)h * d;
        for (int i = 0; i < d; i++)
            for (int j = 0; j < d; j++) {
                volatile float kv = kh[i] * vh[j]; /* rounded product, as _mm256_mul_ps */
                s[(size_t)i * d + j] = fmaf(decay, s[(size_t)i * d + j], kv);
            }
        for (int j = 0; j < d; j++) oh[j] = 0.0f;
        for (int i = 0; i < d; i++)
            for (int j = 0; j < d; j++) oh[j] = fmaf(qh[i], s[(size_t)i * d + j], oh[j]);
    }
}
