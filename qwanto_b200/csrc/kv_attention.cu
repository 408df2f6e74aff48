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
// 1-D cp.async.bulk copies into its own shared memory, completed on per-stage
// mbarriers.
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
#include <cstring>

namespace qkv {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
// a warp range holds at least this many units (small batches use fewer warps)
constexpr uint64_t kMinUnitsPerWarp = 2;
// the even split counts each segment as its tiles plus this many virtual
// units at its start: a warp that starts a new segment (query slicing, a
// partial written) gets correspondingly fewer tiles; when the launch stores
// the newest token, kVirtualEnd more at the segment's end charge that store
constexpr uint32_t kVirtualUnits = 2;
constexpr uint32_t kVirtualEnd = 2;
// segments split into more parts merge in two levels: groups of this many
// parts first, then the group results
constexpr uint32_t kMergeGroup = 16;
// a small launch (one short sequence, say) whose longest segment would be
// split into more than kMergeGroup parts uses fewer warps -- every segment
// then merges in one level -- as long as a warp streams at most this many
// tiles: a second merge level costs more than streaming these serially
constexpr uint64_t kOneLevelTilesPerWarp = 24;
// ... namely at most this many warp ranges start inside the longest segment:
// with the CTA-level merge (four interior warps count as one part) that
// keeps a segment within kMergeGroup parts
constexpr uint64_t kOneLevelWarps = 32;
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
    uint32_t *counters;   // [segments]: parts (or merged groups) counted per segment
    uint32_t *gcounters;  // [warps + segments]: parts counted per merge group (slot index of its first part)
    uint32_t *plans;      // launch plans ([0] = epoch); null: compute the setup every launch
    float2 *tile_mass;
    float2 *seg_ml;
    float *part_m, *part_l, *part_o;  // non-null: export unnormalised (m, l, o)
    const float *new_k, *new_v;       // non-null: fused append of the newest token
    uint32_t *status;
    // 1: the host found that the kernel before this one on the stream (an
    // attention launch of the same pool, on another layer, whose outputs this
    // launch does not read) writes nothing this launch reads, so the setup,
    // the tile stream and the fused append start before that kernel ends;
    // the launch waits for it only before its first write to memory that
    // kernel also writes (plans, partial slots, counters, outputs)
    uint32_t early;
    // split-KV over ranks (xworld > 0): every segment's partial goes to each
    // rank's exchange buffer (xbuf[p] as mapped here) and the ranks' partials
    // of the segment merge into the output
    uint8_t *xbuf[QWN_KV_MAX_RANKS];
    uint32_t xrank, xworld, xepoch, xrows;
    uint64_t xtimeout_ns;
};

__device__ __forceinline__ float pow2ceil(float x) {
    uint32_t b = __float_as_uint(x);
    if (b & 0x7FFFFFu) b = (b & 0x7F800000u) + 0x00800000u;
    return __uint_as_float(b);
}
__device__ __forceinline__ float2 h2x2f(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2 *>(&w));
}

// ---------------------------------------------------------------------------
// int8 codecs (Q8_HEAD_F16, Q8_B64_F32): products with the tile as the A
// operand.  The query heads of the GQA group fill the N columns, so one
// m16n8 product covers 16 tokens x 4 heads:
//  * QK^T on the integer tensor cores (m16n8k32 u8 x s8 -> s32): the K codes
//    (stored biased, 1..255) are used as they are; each query row is split
//    into three int8 slices q = s0*c0 + s1*c1 + s2*c2 (s_{j+1} = s_j/254,
//    residual below 2^-23 of max|q|), columns (head, slice): 4 heads x 3
//    slices in 2 n-blocks, 8 heads x 3 slices in 3.  The sums are exact
//    integers; 128*sum(c_j) removes the code bias, and the slices
//    recombine in fp32 with the token's K scale.
//  * P x V on the f16 tensor cores with V^T as the A operand (dims x
//    tokens) and P^T (tokens x (head, hi/lo)) as B: the probabilities of a
//    lane's two tokens become f16 hi+lo pairs, and movmatrix transposes them
//    into the B fragment.  V codes become exact f16 by byte permutes; the
//    V scale is folded into P with the power-of-two normaliser nu.
// HG head groups of 4 (G <= 4: HG = 1; G <= 8: HG = 2).
// Lane (gid, tig): scores of tokens gid and gid+8 for head 4*hg + tig.
// ---------------------------------------------------------------------------
template <int CODEC, int HG>
struct Int8T {
    static constexpr bool kB64 = CODEC == QWN_KV_CODEC_Q8_B64_F32;
    static constexpr int kX = kB64 ? 2 : 1;  // scale groups along head_dim
    // every variant fits 3 CTAs per SM (168 registers; two head groups too)
    static constexpr int kBytes = kB64 ? 4352 : 4160, kStages = 4;
    static constexpr int kTilesPerStep = 1;
    // QK^T n-blocks: columns (head, slice), three query slices per head.
    // C column e (0, 1) of n-block nb held by a lane belongs to head group
    // col_hg and slice col_slice of the lane's head tig (-1: unused):
    //   HG = 1: nb0 = slices 0, 1; nb1 = slice 2 | unused
    //   HG = 2: nb0 = group 0 slices 0, 1; nb1 = group 1 slices 0, 1;
    //           nb2 = slice 2 of group 0 | of group 1
    static constexpr int kNB = HG == 1 ? 2 : 3;
    __device__ static constexpr int col_hg(int nb, int e) { return HG == 1 ? 0 : (nb < 2 ? nb : e); }
    __device__ static constexpr int col_slice(int nb, int e) {
        return HG == 1 ? (nb == 0 ? e : (e == 0 ? 2 : -1)) : (nb < 2 ? e : 2);
    }
    struct Frag {
        uint32_t b[kNB][4][2];        // IMMA B: [n-block][k-block][reg]
        uint32_t magic[kX][2 * kNB];  // per (scale group, C column 2nb+e of this lane)
        float sc[2 * kNB];            // slice scale x log2(e) x softmax scale per C column
    };
    struct State {
        float o[HG][8][4];  // (dims x (head, hi/lo)) accumulators per m-block
        float m[HG], l[HG];
        float nu[kX], inv_nu[kX];
    };

    // dims of the lane's 32 query values: 16*tig + i (i < 16), 64 + 16*tig + i-16
    __device__ static void begin(Frag &f, State &st, const AttnArgs &A, uint32_t s_idx) {
        const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
        const uint32_t G = A.group;
        uint32_t packed[HG][3][8];  // B words of the lane's head of each group, per slice
        int colsum[HG][3][kX];      // sum of the slice codes over the head's dims, per scale group
        float s0[HG];
        int bad[HG];
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            const uint32_t hq = 4 * hg + (gid >> 1);
            float v[32];
            if (hq < G) {
                const float *q = A.query + ((size_t)s_idx * G + hq) * kHeadDim;
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    const float4 x = *reinterpret_cast<const float4 *>(q + (c >> 2) * 64 + 16 * tig + 4 * (c & 3));
                    v[4 * c] = x.x; v[4 * c + 1] = x.y; v[4 * c + 2] = x.z; v[4 * c + 3] = x.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++) v[i] = 0.f;
            }
            float mx = 0.f;
            int bd = 0;
#pragma unroll
            for (int i = 0; i < 32; i++) {
                if (isfinite(v[i])) mx = fmaxf(mx, fabsf(v[i]));
                else bd = 1;
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            bd |= __shfl_xor_sync(0xffffffffu, bd, 1);
            bd |= __shfl_xor_sync(0xffffffffu, bd, 2);
            bad[hg] = bd;
            // slice scales s_j = s_0 / 254^j (the C side repeats these steps)
            float s = mx > 0.f ? mx * (1.0f / 127.0f) : 1.0f;
            float inv = mx > 0.f ? 127.0f / mx : 1.0f;
            s0[hg] = s;
            // slice j: c = round(v / s_j) with |v / s_j| <= 127 by construction
            // (|v| <= max|q| for j = 0, |residual| <= s_{j-1}/2 = 127 s_j after);
            // the residual after three slices is below 2^-23 of max|q|.  Adding
            // 1.5*2^23 rounds to an integer held in the low mantissa bits,
            // whose low byte is the two's-complement code
            constexpr float kRound = 12582912.0f;
#pragma unroll
            for (int j = 0; j < 3; j++) {
                float sum[kX];
#pragma unroll
                for (int x = 0; x < kX; x++) sum[x] = 0.f;
#pragma unroll
                for (int w = 0; w < 8; w++) {
                    uint32_t bits[4];
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int i = 4 * w + e;
                        const float r = fmaf(v[i], inv, kRound);
                        const float c = r - kRound;
                        v[i] = fmaf(-c, s, v[i]);
                        sum[kB64 ? (i >> 4) : 0] += c;
                        bits[e] = __float_as_uint(r);
                    }
                    packed[hg][j][w] = prmt(prmt(bits[0], bits[1], 0x0040u), prmt(bits[2], bits[3], 0x0040u), 0x5410u);
                }
#pragma unroll
                for (int x = 0; x < kX; x++) {
                    int cs = (int)sum[x];
                    // over the head's 128 dims (the four tig lanes)
                    cs += __shfl_xor_sync(0xffffffffu, cs, 1);
                    cs += __shfl_xor_sync(0xffffffffu, cs, 2);
                    colsum[hg][j][x] = cs;
                }
                s = s * (1.0f / 254.0f);
                inv = inv * 254.0f;
            }
        }
        // B column gid of n-block nb = C column e' = gid & 1 of the lanes with tig = gid >> 1
        const int ep = gid & 1;
        int cs_b[kNB][kX];
#pragma unroll
        for (int nb = 0; nb < kNB; nb++) {
            const int hgb = ep ? col_hg(nb, 1) : col_hg(nb, 0);
            const int slb = ep ? col_slice(nb, 1) : col_slice(nb, 0);
#pragma unroll
            for (int kb = 0; kb < 4; kb++) {
                const int base = 4 * (kb >> 1) + 2 * (kb & 1);  // word index of dims base..base+7
                uint32_t w0 = 0u, w1 = 0u;
#pragma unroll
                for (int hg = 0; hg < HG; hg++)
#pragma unroll
                    for (int j = 0; j < 3; j++)
                        if (hg == hgb && j == slb) { w0 = packed[hg][j][base]; w1 = packed[hg][j][base + 1]; }
                f.b[nb][kb][0] = w0;
                f.b[nb][kb][1] = w1;
            }
#pragma unroll
            for (int x = 0; x < kX; x++) {
                int cs = 0;
#pragma unroll
                for (int hg = 0; hg < HG; hg++)
#pragma unroll
                    for (int j = 0; j < 3; j++)
                        if (hg == hgb && j == slb) cs = colsum[hg][j][x];
                cs_b[nb][x] = cs;
            }
        }
        // C side: column 2tig+e of n-block nb comes from the lanes with gid = 2tig + e
#pragma unroll
        for (int nb = 0; nb < kNB; nb++)
#pragma unroll
            for (int e = 0; e < 2; e++)
#pragma unroll
                for (int x = 0; x < kX; x++) {
                    const int cs = __shfl_sync(0xffffffffu, cs_b[nb][x], 8 * tig + 4 * e);
                    f.magic[x][2 * nb + e] = 0x4B400000u - (uint32_t)(128 * cs);
                }
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            const float hs0 = __shfl_sync(0xffffffffu, s0[hg], 8 * tig);
            const int hbad = __shfl_sync(0xffffffffu, bad[hg], 8 * tig);
#pragma unroll
            for (int nb = 0; nb < kNB; nb++)
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    if (col_hg(nb, e) != hg || col_slice(nb, e) < 0) continue;
                    const float sj = col_slice(nb, e) == 0 ? hs0
                                     : col_slice(nb, e) == 1 ? hs0 * (1.0f / 254.0f)
                                                             : hs0 * (1.0f / 254.0f) * (1.0f / 254.0f);
                    f.sc[2 * nb + e] = hbad ? __int_as_float(0x7fffffff) : sj * A.scale_log2;
                }
        }
        if constexpr (HG == 1) f.sc[3] = 0.f;
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            st.m[hg] = -INFINITY;
            st.l[hg] = 0.f;
#pragma unroll
            for (int mb = 0; mb < 8; mb++) st.o[hg][mb][0] = st.o[hg][mb][1] = st.o[hg][mb][2] = st.o[hg][mb][3] = 0.f;
        }
#pragma unroll
        for (int x = 0; x < kX; x++) { st.nu[x] = 0.f; st.inv_nu[x] = 0.f; }
    }

    // scores of one tile (base 2, masked to -inf outside [t_lo, t_hi)) and
    // the V scales of its tokens gid, gid+8 (zero outside the range)
    __device__ static void scores(const uint8_t *tile, const Frag &f, int t_lo, int t_hi, float (&s)[HG][2],
                                  float (&vs)[kX][2]) {
        const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
        (void)tig;
        // ---- K fragments: token rows gid and gid+8
        const int sw = (gid & 1) << 2;
        const uint8_t *r0 = tile + 128 * gid, *r1 = tile + 128 * (gid + 8);
        const uint4 k00 = *reinterpret_cast<const uint4 *>(r0 + ((tig ^ sw) << 4));
        const uint4 k01 = *reinterpret_cast<const uint4 *>(r0 + (((4 + tig) ^ sw) << 4));
        const uint4 k10 = *reinterpret_cast<const uint4 *>(r1 + ((tig ^ sw) << 4));
        const uint4 k11 = *reinterpret_cast<const uint4 *>(r1 + (((4 + tig) ^ sw) << 4));
        const uint32_t ka[4][4] = {{k00.x, k10.x, k00.y, k10.y},
                                   {k00.z, k10.z, k00.w, k10.w},
                                   {k01.x, k11.x, k01.y, k11.y},
                                   {k01.z, k11.z, k01.w, k11.w}};
        // ---- scales of tokens gid, gid+8
        float ks[kX][2];
        if constexpr (kB64) {
            const float4 k4 = *reinterpret_cast<const float4 *>(tile + 4096 + 16 * gid);
            const float4 v4 = *reinterpret_cast<const float4 *>(tile + 4224 + 16 * gid);
            ks[0][0] = k4.x; ks[0][1] = k4.y; ks[kX - 1][0] = k4.z; ks[kX - 1][1] = k4.w;
            vs[0][0] = v4.x; vs[0][1] = v4.y; vs[kX - 1][0] = v4.z; vs[kX - 1][1] = v4.w;
        } else {
            const float2 k2 = h2x2f(*reinterpret_cast<const uint32_t *>(tile + 4096 + 4 * gid));
            const float2 v2 = h2x2f(*reinterpret_cast<const uint32_t *>(tile + 4128 + 4 * gid));
            ks[0][0] = k2.x; ks[0][1] = k2.y;
            vs[0][0] = v2.x; vs[0][1] = v2.y;
        }
        const bool full = t_lo == 0 && t_hi == 16;  // warp-uniform
        const bool ok0 = full || (gid >= t_lo && gid < t_hi);
        const bool ok1 = full || (gid + 8 >= t_lo && gid + 8 < t_hi);
        // ---- scores: kNB x 4 integer MMAs for all head groups
        int acc[kNB][2][4];  // [n-block][k-block pair][c]
#pragma unroll
        for (int kb = 0; kb < 4; kb++)
#pragma unroll
            for (int nb = 0; nb < kNB; nb++) {
                // per 64-channel scales (codec 1): one sum per half of the
                // head; per-head scale (codec 2): one chain over all 128 dims
                const int half = kB64 ? (kb >> 1) : 0;
                if (kB64 ? (kb & 1) : kb != 0)
                    imma16832(acc[nb][half], ka[kb][0], ka[kb][1], ka[kb][2], ka[kb][3], f.b[nb][kb][0],
                              f.b[nb][kb][1]);
                else
                    imma16832_z(acc[nb][half], ka[kb][0], ka[kb][1], ka[kb][2], ka[kb][3], f.b[nb][kb][0],
                                f.b[nb][kb][1]);
            }
#pragma unroll
        for (int tk = 0; tk < 2; tk++) {
            float raw[HG][kX];
#pragma unroll
            for (int hg = 0; hg < HG; hg++)
#pragma unroll
                for (int x = 0; x < kX; x++) raw[hg][x] = 0.f;
#pragma unroll
            for (int nb = 0; nb < kNB; nb++)
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    if (col_slice(nb, e) < 0) continue;
                    const int hg = col_hg(nb, e), j = 2 * nb + e, c = 2 * tk + e;
                    if constexpr (kB64) {
                        raw[hg][0] = fmaf(small_int_to_float(acc[nb][0][c], f.magic[0][j]), f.sc[j], raw[hg][0]);
                        raw[hg][kX - 1] =
                            fmaf(small_int_to_float(acc[nb][1][c], f.magic[kX - 1][j]), f.sc[j], raw[hg][kX - 1]);
                    } else {
                        raw[hg][0] = fmaf(small_int_to_float(acc[nb][0][c], f.magic[0][j]), f.sc[j],
                                          raw[hg][0]);
                    }
                }
#pragma unroll
            for (int hg = 0; hg < HG; hg++) {
                float sc = raw[hg][0] * ks[0][tk];
                if constexpr (kB64) sc = fmaf(raw[hg][kX - 1], ks[kX - 1][tk], sc);
                s[hg][tk] = (tk ? ok1 : ok0) ? sc : -INFINITY;
            }
        }

#pragma unroll
        for (int x = 0; x < kX; x++) {
            vs[x][0] = ok0 ? vs[x][0] : 0.f;
            vs[x][1] = ok1 ? vs[x][1] : 0.f;
        }
    }

    // P x V of one tile: P' = p * vs / nu as f16 hi+lo, transposed into the
    // B operand; V codes -> exact f16 A fragments
    __device__ static void pv(const uint8_t *tile, State &st, const float (&p)[HG][2], const float (&vs)[kX][2]) {
        const int lane = threadIdx.x & 31;
        // ---- P' = p * vs / nu as f16 hi+lo, transposed into the PV B operand
        uint32_t bp[HG][kX][2];
#pragma unroll
        for (int hg = 0; hg < HG; hg++)
#pragma unroll
            for (int x = 0; x < kX; x++) {
                const float pt0 = p[hg][0] * vs[x][0] * st.inv_nu[x];
                const float pt1 = p[hg][1] * vs[x][1] * st.inv_nu[x];
                const __half2 hi = __floats2half2_rn(pt0, pt1);
                const float2 hf = __half22float2(hi);
                const __half2 lo = __floats2half2_rn(pt0 - hf.x, pt1 - hf.y);
                const uint32_t hu = *reinterpret_cast<const uint32_t *>(&hi);
                const uint32_t lu = *reinterpret_cast<const uint32_t *>(&lo);
                bp[hg][x][0] = movmatrix_trans(prmt(hu, lu, 0x5410u));  // (hi, lo) of token gid
                bp[hg][x][1] = movmatrix_trans(prmt(hu, lu, 0x7632u));  // (hi, lo) of token gid+8
            }
        // ---- P x V
        const uint8_t *vt = tile + 2048 + lane * 64;
        const int vsw = (lane >> 1) & 3;
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const uint4 c = *reinterpret_cast<const uint4 *>(vt + ((q ^ vsw) << 4));
#pragma unroll
            for (int hm = 0; hm < 2; hm++) {
                const int mb = 2 * q + hm;
                uint32_t a[4];
                u8x4_to_h2x2(hm ? c.z : c.x, a[0], a[1]);
                u8x4_to_h2x2(hm ? c.w : c.y, a[2], a[3]);
                const int x = kB64 ? (mb >> 2) : 0;
#pragma unroll
                for (int hg = 0; hg < HG; hg++) mma16816(st.o[hg][mb], a, bp[hg][x][0], bp[hg][x][1]);
            }
        }
    }

    // NT consecutive tiles of one segment: their scores, one online-softmax
    // update and one normaliser check for all of them, then P x V per tile
    template <int NT>
    __device__ static void stepn(const uint8_t *const (&tiles)[NT], const Frag &f, State &st,
                                 const int (&t_lo)[NT], const int (&t_hi)[NT], float (&psum)[NT][HG]) {
        float s[NT][HG][2], vs[NT][kX][2];
#pragma unroll
        for (int u = 0; u < NT; u++) scores(tiles[u], f, t_lo[u], t_hi[u], s[u], vs[u]);
        // ---- online softmax per head (reduction over the 8 token lanes gid)
        float p[NT][HG][2];
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            float tmax = fmaxf(s[0][hg][0], s[0][hg][1]);
#pragma unroll
            for (int u = 1; u < NT; u++) tmax = fmaxf(tmax, fmaxf(s[u][hg][0], s[u][hg][1]));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 8));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
            const float m_new = fmaxf(st.m[hg], tmax);
            if (__any_sync(0xffffffffu, m_new > st.m[hg])) {
                const float alpha = ex2(st.m[hg] - m_new);
                st.l[hg] *= alpha;
#pragma unroll
                for (int mb = 0; mb < 8; mb++) {
                    st.o[hg][mb][0] *= alpha; st.o[hg][mb][1] *= alpha;
                    st.o[hg][mb][2] *= alpha; st.o[hg][mb][3] *= alpha;
                }
                st.m[hg] = m_new;
            }
#pragma unroll
            for (int u = 0; u < NT; u++) {
                p[u][hg][0] = ex2(s[u][hg][0] - st.m[hg]);
                p[u][hg][1] = ex2(s[u][hg][1] - st.m[hg]);
                psum[u][hg] = p[u][hg][0] + p[u][hg][1];
                st.l[hg] += psum[u][hg];
            }
        }
        // ---- V scales -> normaliser nu (shared by all heads)
#pragma unroll
        for (int x = 0; x < kX; x++) {
            float lmax = fmaxf(vs[0][x][0], vs[0][x][1]);
#pragma unroll
            for (int u = 1; u < NT; u++) lmax = fmaxf(lmax, fmaxf(vs[u][x][0], vs[u][x][1]));
            const bool first = st.nu[x] == 0.f;
            if (__any_sync(0xffffffffu, first || lmax > st.nu[x] * kNuHeadroom)) {
                float vmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, 4));
                vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 8));
                vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 16));
                const float nn = fmaxf(pow2ceil(vmax), kNuFloor);
                if (first) {
                    st.nu[x] = nn;
                } else if (nn > st.nu[x]) {
                    const float r = st.nu[x] / nn;
#pragma unroll
                    for (int hg = 0; hg < HG; hg++)
#pragma unroll
                        for (int mb = 0; mb < 8; mb++) {
                            if (kB64 && (mb >> 2) != x) continue;
                            st.o[hg][mb][0] *= r; st.o[hg][mb][1] *= r;
                            st.o[hg][mb][2] *= r; st.o[hg][mb][3] *= r;
                        }
                    st.nu[x] = nn;
                }
                st.inv_nu[x] = 1.0f / st.nu[x];
            }
        }
#pragma unroll
        for (int u = 0; u < NT; u++) pv(tiles[u], st, p[u], vs[u]);
    }

    __device__ static void step(const uint8_t *tile, const Frag &f, State &st, int t_lo, int t_hi,
                                float (&psum)[HG]) {
        const uint8_t *const tiles[1] = {tile};
        const int lo[1] = {t_lo}, hi[1] = {t_hi};
        float ps[1][HG];
        stepn<1>(tiles, f, st, lo, hi, ps);
#pragma unroll
        for (int hg = 0; hg < HG; hg++) psum[hg] = ps[0][hg];
    }

    // tile probability mass and running max per head (eviction scores)
    __device__ static void mass(const AttnArgs &A, uint64_t unit, const State &st, float (&psum)[HG]) {
        const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            float u = psum[hg];
            u += __shfl_xor_sync(0xffffffffu, u, 4);
            u += __shfl_xor_sync(0xffffffffu, u, 8);
            u += __shfl_xor_sync(0xffffffffu, u, 16);
            const uint32_t h = 4 * hg + tig;
            if (gid == 0 && h < A.group) A.tile_mass[unit * kMaxGroup + h] = make_float2(u, st.m[hg]);
        }
    }

    // rows of the G query heads at o_base (stride 128), optionally normalised;
    // m_out / l_out / seg_ml per head when non-null
    __device__ static void store_rows(const AttnArgs &A, const State &st, float *o_base, float *m_out, float *l_out,
                                      bool normalize, float2 *seg_ml) {
        const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            float lt = st.l[hg];
            lt += __shfl_xor_sync(0xffffffffu, lt, 4);
            lt += __shfl_xor_sync(0xffffffffu, lt, 8);
            lt += __shfl_xor_sync(0xffffffffu, lt, 16);
            const uint32_t h = 4 * hg + tig;
            if (h >= A.group) continue;
            const float inv = normalize ? (lt > 0.f ? 1.0f / lt : 0.f) : 1.0f;
            float *row = o_base + (size_t)h * kHeadDim;
#pragma unroll
            for (int mb = 0; mb < 8; mb++) {
                const float f = st.nu[kB64 ? (mb >> 2) : 0] * inv;
                row[16 * mb + gid] = (st.o[hg][mb][0] + st.o[hg][mb][1]) * f;
                row[16 * mb + gid + 8] = (st.o[hg][mb][2] + st.o[hg][mb][3]) * f;
            }
            if (gid == 0) {
                if (m_out) { m_out[h] = st.m[hg]; l_out[h] = lt; }
                if (seg_ml) seg_ml[h] = make_float2(st.m[hg], lt);
            }
        }
    }
};

// ---------------------------------------------------------------------------
// low-bit codecs (Q4_G32, TQ35_G64): the same products as Int8T with the
// codes in classes of 32 dims that share one scale -- codec 4 class = group
// of 32; TurboQuant class = (group of 64, parity), even dims 4-bit codes
// scaled by range/15, odd dims 3-bit codes by range/7.  Each class is one
// k-block of the integer QK^T (codes 0..15 as u8, no bias) and two m-blocks
// of P x V.  The query splits into three int8 slices at ratio 2^7
// (q ~ s2 * (16384 c0 + 128 c1 + c2)), so the slice sums combine exactly in
// int32 and each class needs one conversion; the class scale multiplies in
// fp32 and the group minimum enters through the query sum (K) and through
// z = sum_t p_t * min_t (V).
// ---------------------------------------------------------------------------
template <int CODEC, int HG>
struct LowBitT {
    static constexpr bool kTQ = CODEC == QWN_KV_CODEC_TQ35_G64;
    static constexpr int kC = 4;               // classes of 32 dims
    static constexpr int kG = kTQ ? 2 : 4;     // groups (min values)
    static constexpr int kBytes = kTQ ? 2048 : 2560, kStages = kTQ ? 8 : 6;
    // tiles per loop iteration: pairs for the 4-bit single-head-group kernel
    // (long contexts gain ~3%; TurboQuant's larger step does not)
    static constexpr int kTilesPerStep = (HG == 1 && !kTQ) ? 2 : 1;
    struct Frag {
        uint32_t b[HG][2][kC][2];  // [head group][n-block][class][reg]
        float s2l[HG][2];          // unit slice scale x log2(e) x softmax scale x code scale
                                   // (1/15; TurboQuant odd classes [1]: 1/7)
        float qs[HG][kG];          // query sum per group x log2(e) x softmax scale
    };
    struct State {
        float o[HG][8][4];
        float z[HG][kG];  // sum_t p_t * min (this lane's tokens)
        float m[HG], l[HG];
        float nu[kC], inv_nu[kC], nu_lim[kC];  // normaliser of each class's raw ranges
    };
    // the code scale of class c: range/15 (4-bit codes), range/7 (3-bit odd TurboQuant codes)
    __device__ static constexpr float code_scale(int c) { return (kTQ && (c & 1)) ? 1.0f / 7.0f : 1.0f / 15.0f; }
    // dim of (class c, index m)
    __device__ static int dim_of(int c, int m) { return kTQ ? 64 * (c >> 1) + 2 * m + (c & 1) : 32 * c + m; }
    __device__ static int group_of_class(int c) { return kTQ ? (c >> 1) : c; }

    __device__ static void begin(Frag &f, State &st, const AttnArgs &A, uint32_t s_idx) {
        const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
        const uint32_t G = A.group;
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            const uint32_t hq = 4 * hg + (gid >> 1);
            // v[8c + i] = q[dim_of(c, 8 tig + i)]
            float v[32];
            if (hq < G) {
                const float *q = A.query + ((size_t)s_idx * G + hq) * kHeadDim;
                if constexpr (kTQ) {
                    // dims 64x + 16tig + j: even j -> class 2x, odd -> 2x+1
#pragma unroll
                    for (int x = 0; x < 2; x++)
#pragma unroll
                        for (int c4 = 0; c4 < 4; c4++) {
                            const float4 w = *reinterpret_cast<const float4 *>(q + 64 * x + 16 * tig + 4 * c4);
                            v[8 * (2 * x) + 2 * c4] = w.x;
                            v[8 * (2 * x + 1) + 2 * c4] = w.y;
                            v[8 * (2 * x) + 2 * c4 + 1] = w.z;
                            v[8 * (2 * x + 1) + 2 * c4 + 1] = w.w;
                        }
                } else {
#pragma unroll
                    for (int c = 0; c < 4; c++)
#pragma unroll
                        for (int h2 = 0; h2 < 2; h2++) {
                            const float4 w = *reinterpret_cast<const float4 *>(q + 32 * c + 8 * tig + 4 * h2);
                            v[8 * c + 4 * h2] = w.x; v[8 * c + 4 * h2 + 1] = w.y;
                            v[8 * c + 4 * h2 + 2] = w.z; v[8 * c + 4 * h2 + 3] = w.w;
                        }
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++) v[i] = 0.f;
            }
            float mx = 0.f;
            int bad = 0;
            float qs[kG];
#pragma unroll
            for (int g = 0; g < kG; g++) qs[g] = 0.f;
#pragma unroll
            for (int i = 0; i < 32; i++) {
                if (isfinite(v[i])) mx = fmaxf(mx, fabsf(v[i]));
                else bad = 1;
                qs[group_of_class(i >> 3)] += v[i];
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            bad |= __shfl_xor_sync(0xffffffffu, bad, 1);
            bad |= __shfl_xor_sync(0xffffffffu, bad, 2);
#pragma unroll
            for (int g = 0; g < kG; g++) {
                qs[g] += __shfl_xor_sync(0xffffffffu, qs[g], 1);
                qs[g] += __shfl_xor_sync(0xffffffffu, qs[g], 2);
            }
            // slices: s1 = s0/128, s2 = s0/16384 exactly; |c1|, |c2| <= 64
            const float s0 = mx > 0.f ? mx * (1.0f / 127.0f) : 1.0f;
            const float inv0 = mx > 0.f ? 127.0f / mx : 1.0f;
            constexpr float kRound = 12582912.0f;
            uint32_t packed[3][8];
            {
                float s = s0, inv = inv0;
#pragma unroll
                for (int j = 0; j < 3; j++) {
#pragma unroll
                    for (int w = 0; w < 8; w++) {
                        uint32_t bits[4];
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const int i = 4 * w + e;
                            const float r = fmaf(v[i], inv, kRound);
                            v[i] = fmaf(-(r - kRound), s, v[i]);
                            bits[e] = __float_as_uint(r);
                        }
                        packed[j][w] = prmt(prmt(bits[0], bits[1], 0x0040u), prmt(bits[2], bits[3], 0x0040u), 0x5410u);
                    }
                    s = s * (1.0f / 128.0f);
                    inv = inv * 128.0f;
                }
            }
            // B columns: n-block 0 col gid = (head gid>>1, slice gid&1);
            // n-block 1 col gid = (head gid>>1, slice 2) when gid even, else 0
#pragma unroll
            for (int c = 0; c < kC; c++) {
                f.b[hg][0][c][0] = (gid & 1) ? packed[1][2 * c] : packed[0][2 * c];
                f.b[hg][0][c][1] = (gid & 1) ? packed[1][2 * c + 1] : packed[0][2 * c + 1];
                f.b[hg][1][c][0] = (gid & 1) ? 0u : packed[2][2 * c];
                f.b[hg][1][c][1] = (gid & 1) ? 0u : packed[2][2 * c + 1];
            }
            // C side: this lane's head is 4hg + tig, held by the lanes gid = 2tig
            const float hs0 = __shfl_sync(0xffffffffu, s0, 8 * tig);
            const int hbad = __shfl_sync(0xffffffffu, bad, 8 * tig);
            const float s2 = hbad ? __int_as_float(0x7fffffff) : hs0 * (1.0f / 16384.0f) * A.scale_log2;
            f.s2l[hg][0] = s2 * code_scale(0);
            f.s2l[hg][1] = s2 * code_scale(1);
#pragma unroll
            for (int g = 0; g < kG; g++) f.qs[hg][g] = __shfl_sync(0xffffffffu, qs[g], 8 * tig) * A.scale_log2;
        }
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            st.m[hg] = -INFINITY;
            st.l[hg] = 0.f;
#pragma unroll
            for (int g = 0; g < kG; g++) st.z[hg][g] = 0.f;
#pragma unroll
            for (int mb = 0; mb < 8; mb++) st.o[hg][mb][0] = st.o[hg][mb][1] = st.o[hg][mb][2] = st.o[hg][mb][3] = 0.f;
        }
#pragma unroll
        for (int c = 0; c < kC; c++) { st.nu[c] = 0.f; st.inv_nu[c] = 0.f; st.nu_lim[c] = 0.f; }
    }

    // the three group-1 TurboQuant odd-code bits: bit 0 in bit 3 of each nibble
    // of `odd`, bits 1-2 in the 2-bit fields of `plane` (field n -> nibble n)
    __device__ static uint32_t tq_hi_codes(uint32_t odd, uint32_t plane) {
        uint32_t s = plane & 0xFFFFu;
        s = (s | (s << 8)) & 0x00FF00FFu;
        s = (s | (s << 4)) & 0x0F0F0F0Fu;
        s = (s | (s << 2)) & 0x33333333u;
        return ((odd >> 3) & 0x11111111u) | (s << 1);
    }

    // K code words (u8-expanded per class), class ranges and group minima of
    // tokens gid (tk 0) and gid+8 (tk 1) of one tile
    __device__ static void kload(const uint8_t *tile, uint32_t (&kw)[2][kC], float (&kp)[2][kC], float (&km)[2][kG]) {
        const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
        const uint8_t *kpar;
        if constexpr (kTQ) {
#pragma unroll
            for (int tk = 0; tk < 2; tk++) {
                const int t = gid + 8 * tk;
                const uint2 ev = *reinterpret_cast<const uint2 *>(tile + 32 * t + 8 * tig);
                const uint32_t od = *reinterpret_cast<const uint32_t *>(tile + 512 + 16 * t + 4 * tig);
                const uint32_t pl = *reinterpret_cast<const uint16_t *>(tile + 768 + 8 * t + 2 * tig);
                kw[tk][0] = ev.x;
                kw[tk][1] = od & 0x77777777u;
                kw[tk][2] = ev.y;
                kw[tk][3] = tq_hi_codes(od, pl);
            }
            kpar = tile + 896;
        } else {
#pragma unroll
            for (int tk = 0; tk < 2; tk++) {
                const uint4 w = *reinterpret_cast<const uint4 *>(tile + 64 * (gid + 8 * tk) + 16 * tig);
                kw[tk][0] = w.x; kw[tk][1] = w.y; kw[tk][2] = w.z; kw[tk][3] = w.w;
            }
            kpar = tile + 2048;
        }
        // params of tokens gid, gid+8: (range16, min16) words [class or group][token]
        uint32_t pw[kG][2];
        if constexpr (kTQ) {
            const uint4 p = *reinterpret_cast<const uint4 *>(kpar + 16 * gid);
            pw[0][0] = p.x; pw[0][1] = p.y; pw[kG - 1][0] = p.z; pw[kG - 1][1] = p.w;
        } else {
            const uint4 p0 = *reinterpret_cast<const uint4 *>(kpar + 32 * gid);
            const uint4 p1 = *reinterpret_cast<const uint4 *>(kpar + 32 * gid + 16);
            pw[0][0] = p0.x; pw[0][1] = p0.y; pw[1][0] = p0.z; pw[1][1] = p0.w;
            pw[kG - 2][0] = p1.x; pw[kG - 2][1] = p1.y; pw[kG - 1][0] = p1.z; pw[kG - 1][1] = p1.w;
        }
#pragma unroll
        for (int g = 0; g < kG; g++)
#pragma unroll
            for (int tk = 0; tk < 2; tk++) {
                const float2 rm = h2x2f(pw[g][tk]);
                km[tk][g] = rm.y;
                if constexpr (kTQ) {
                    kp[tk][2 * g] = rm.x;
                    kp[tk][2 * g + 1] = rm.x;
                } else {
                    kp[tk][g] = rm.x;
                }
            }
    }

    // base-2 scores of NT tiles, the tiles' integer products interleaved
    template <int NT>
    __device__ static void scores(const uint8_t *const (&tiles)[NT], const Frag &f, const int (&t_lo)[NT],
                                  const int (&t_hi)[NT], float (&s)[NT][HG][2], bool (&ok0)[NT], bool (&ok1)[NT],
                                  bool (&full)[NT]) {
        const int gid = (threadIdx.x & 31) >> 2;
        uint32_t kw[NT][2][kC];
        float kp[NT][2][kC], km[NT][2][kG];
#pragma unroll
        for (int u = 0; u < NT; u++) {
            kload(tiles[u], kw[u], kp[u], km[u]);
            full[u] = t_lo[u] == 0 && t_hi[u] == 16;  // warp-uniform
            ok0[u] = full[u] || (gid >= t_lo[u] && gid < t_hi[u]);
            ok1[u] = full[u] || (gid + 8 >= t_lo[u] && gid + 8 < t_hi[u]);
        }
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            float raw[NT][2][2];  // [tile][token][odd TurboQuant class]
#pragma unroll
            for (int u = 0; u < NT; u++) raw[u][0][0] = raw[u][0][1] = raw[u][1][0] = raw[u][1][1] = 0.f;
#pragma unroll
            for (int c = 0; c < kC; c++) {
                int acc[NT][2][4];
#pragma unroll
                for (int u = 0; u < NT; u++) {
                    const uint32_t a0 = kw[u][0][c] & 0x0F0F0F0Fu, a1 = kw[u][1][c] & 0x0F0F0F0Fu;
                    const uint32_t a2 = (kw[u][0][c] >> 4) & 0x0F0F0F0Fu, a3 = (kw[u][1][c] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                    for (int nb = 0; nb < 2; nb++)
                        imma16832_z(acc[u][nb], a0, a1, a2, a3, f.b[hg][nb][c][0], f.b[hg][nb][c][1]);
                }
#pragma unroll
                for (int u = 0; u < NT; u++)
#pragma unroll
                    for (int tk = 0; tk < 2; tk++) {
                        // columns 2tig (slice 0 | slice 2) and 2tig+1 (slice 1)
                        const int I = (acc[u][0][2 * tk] * 128 + acc[u][0][2 * tk + 1]) * 128 + acc[u][1][2 * tk];
                        const int o = kTQ ? (c & 1) : 0;
                        raw[u][tk][o] = fmaf(__int2float_rn(I), kp[u][tk][c], raw[u][tk][o]);
                    }
            }
#pragma unroll
            for (int u = 0; u < NT; u++)
#pragma unroll
                for (int tk = 0; tk < 2; tk++) {
                    float sc = raw[u][tk][0] * f.s2l[hg][0];
                    if constexpr (kTQ) sc = fmaf(raw[u][tk][1], f.s2l[hg][1], sc);
#pragma unroll
                    for (int g = 0; g < kG; g++) sc = fmaf(km[u][tk][g], f.qs[hg][g], sc);
                    s[u][hg][tk] = (tk ? ok1[u] : ok0[u]) ? sc : -INFINITY;
                }
        }
    }

    // V class ranges and group minima of tokens gid, gid+8 (zero for masked tokens)
    __device__ static void vparams(const uint8_t *tile, bool ok0, bool ok1, bool full, float (&vp)[2][kC],
                                   float (&vm)[2][kG]) {
        const int gid = (threadIdx.x & 31) >> 2;
        const uint8_t *vpar = kTQ ? tile + 1024 + 896 : tile + 2304;
        uint32_t pw[kG][2];
        if constexpr (kTQ) {
            const uint4 q4 = *reinterpret_cast<const uint4 *>(vpar + 16 * gid);
            pw[0][0] = q4.x; pw[0][1] = q4.y; pw[kG - 1][0] = q4.z; pw[kG - 1][1] = q4.w;
        } else {
            const uint4 p0 = *reinterpret_cast<const uint4 *>(vpar + 32 * gid);
            const uint4 p1 = *reinterpret_cast<const uint4 *>(vpar + 32 * gid + 16);
            pw[0][0] = p0.x; pw[0][1] = p0.y; pw[1][0] = p0.z; pw[1][1] = p0.w;
            pw[kG - 2][0] = p1.x; pw[kG - 2][1] = p1.y; pw[kG - 1][0] = p1.z; pw[kG - 1][1] = p1.w;
        }
        if (!full) {  // masked tokens contribute nothing (their slots may hold anything)
#pragma unroll
            for (int g = 0; g < kG; g++) {
                if (!ok0) pw[g][0] = 0u;
                if (!ok1) pw[g][1] = 0u;
            }
        }
#pragma unroll
        for (int g = 0; g < kG; g++)
#pragma unroll
            for (int tk = 0; tk < 2; tk++) {
                const float2 rm = h2x2f(pw[g][tk]);
                vm[tk][g] = rm.y;
                if constexpr (kTQ) {
                    vp[tk][2 * g] = rm.x;
                    vp[tk][2 * g + 1] = rm.x;
                } else {
                    vp[tk][g] = rm.x;
                }
            }
    }

    // V code words of one tile per m-block
    __device__ static void vload(const uint8_t *tile, uint32_t (&vw)[8]) {
        const int lane = threadIdx.x & 31;
        if constexpr (kTQ) {
            const uint8_t *vh = tile + 1024;
            const uint4 ev = *reinterpret_cast<const uint4 *>(vh + 16 * lane);
            const uint2 od = *reinterpret_cast<const uint2 *>(vh + 512 + 8 * lane);
            const uint32_t pl = *reinterpret_cast<const uint32_t *>(vh + 768 + 4 * lane);
            vw[0] = ev.x; vw[1] = ev.y;                    // class 0 (group 0, even)
            vw[2] = od.x & 0x77777777u; vw[3] = od.y & 0x77777777u;  // class 1 (group 0, odd)
            vw[4] = ev.z; vw[5] = ev.w;                    // class 2 (group 1, even)
            vw[6] = tq_hi_codes(od.x, pl); vw[7] = tq_hi_codes(od.y, pl >> 16);  // class 3
        } else {
            const uint8_t *vt = tile + 1024 + lane * 32;
            const int sw = (lane >> 2) & 1;
            const uint4 c0 = *reinterpret_cast<const uint4 *>(vt + ((0 ^ sw) << 4));
            const uint4 c1 = *reinterpret_cast<const uint4 *>(vt + ((1 ^ sw) << 4));
            vw[0] = c0.x; vw[1] = c0.y; vw[2] = c0.z; vw[3] = c0.w;
            vw[4] = c1.x; vw[5] = c1.y; vw[6] = c1.z; vw[7] = c1.w;
        }
    }

    // P' = p * range / nu per class as f16 hi+lo, transposed into the PV B
    // operand; V codes per m-block -> exact f16 A fragments; P x V for NT
    // tiles, interleaved
    template <int NT>
    __device__ static void pv(const uint8_t *const (&tiles)[NT], State &st, const float (&p)[NT][HG][2],
                              const float (&vp)[NT][2][kC]) {
        uint32_t bp[NT][HG][kC][2];
#pragma unroll
        for (int u = 0; u < NT; u++)
#pragma unroll
            for (int hg = 0; hg < HG; hg++)
#pragma unroll
                for (int c = 0; c < kC; c++) {
                    const float pt0 = p[u][hg][0] * vp[u][0][c] * st.inv_nu[c];
                    const float pt1 = p[u][hg][1] * vp[u][1][c] * st.inv_nu[c];
                    const __half2 hi = __floats2half2_rn(pt0, pt1);
                    const float2 hf = __half22float2(hi);
                    const __half2 lo = __floats2half2_rn(pt0 - hf.x, pt1 - hf.y);
                    const uint32_t hu = *reinterpret_cast<const uint32_t *>(&hi);
                    const uint32_t lu = *reinterpret_cast<const uint32_t *>(&lo);
                    bp[u][hg][c][0] = movmatrix_trans(prmt(hu, lu, 0x5410u));
                    bp[u][hg][c][1] = movmatrix_trans(prmt(hu, lu, 0x7632u));
                }
        uint32_t vw[NT][8];
#pragma unroll
        for (int u = 0; u < NT; u++) vload(tiles[u], vw[u]);
#pragma unroll
        for (int mb = 0; mb < 8; mb++)
#pragma unroll
            for (int u = 0; u < NT; u++) {
                uint32_t a[4];
                nib8_to_h2x4(vw[u][mb], a);
#pragma unroll
                for (int hg = 0; hg < HG; hg++) mma16816(st.o[hg][mb], a, bp[u][hg][mb >> 1][0], bp[u][hg][mb >> 1][1]);
            }
    }

    // NT consecutive tiles of one segment: their scores, one online-softmax
    // update and one normaliser check for all of them, then P x V per tile
    template <int NT>
    __device__ static void stepn(const uint8_t *const (&tiles)[NT], const Frag &f, State &st,
                                 const int (&t_lo)[NT], const int (&t_hi)[NT], float (&psum)[NT][HG]) {
        float s[NT][HG][2];
        bool ok0[NT], ok1[NT], full[NT];
        scores<NT>(tiles, f, t_lo, t_hi, s, ok0, ok1, full);
        // ---- online softmax per head
        float p[NT][HG][2];
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            float tmax = fmaxf(s[0][hg][0], s[0][hg][1]);
#pragma unroll
            for (int u = 1; u < NT; u++) tmax = fmaxf(tmax, fmaxf(s[u][hg][0], s[u][hg][1]));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 8));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
            const float m_new = fmaxf(st.m[hg], tmax);
            if (__any_sync(0xffffffffu, m_new > st.m[hg])) {
                const float alpha = ex2(st.m[hg] - m_new);
                st.l[hg] *= alpha;
#pragma unroll
                for (int g = 0; g < kG; g++) st.z[hg][g] *= alpha;
#pragma unroll
                for (int mb = 0; mb < 8; mb++) {
                    st.o[hg][mb][0] *= alpha; st.o[hg][mb][1] *= alpha;
                    st.o[hg][mb][2] *= alpha; st.o[hg][mb][3] *= alpha;
                }
                st.m[hg] = m_new;
            }
#pragma unroll
            for (int u = 0; u < NT; u++) {
                p[u][hg][0] = ex2(s[u][hg][0] - st.m[hg]);
                p[u][hg][1] = ex2(s[u][hg][1] - st.m[hg]);
                psum[u][hg] = p[u][hg][0] + p[u][hg][1];
                st.l[hg] += psum[u][hg];
            }
        }
        // ---- V params; z = sum_t p_t * min_t
        float vp[NT][2][kC], vm[NT][2][kG];
#pragma unroll
        for (int u = 0; u < NT; u++) vparams(tiles[u], ok0[u], ok1[u], full[u], vp[u], vm[u]);
#pragma unroll
        for (int u = 0; u < NT; u++)
#pragma unroll
            for (int hg = 0; hg < HG; hg++)
#pragma unroll
                for (int g = 0; g < kG; g++)
                    st.z[hg][g] = fmaf(p[u][hg][0], vm[u][0][g], fmaf(p[u][hg][1], vm[u][1][g], st.z[hg][g]));
        // ---- normalisers per class (shared by all heads)
        {
            float lmax[kC];
            bool need = false;
#pragma unroll
            for (int c = 0; c < kC; c++) {
                lmax[c] = fmaxf(vp[0][0][c], vp[0][1][c]);
#pragma unroll
                for (int u = 1; u < NT; u++) lmax[c] = fmaxf(lmax[c], fmaxf(vp[u][0][c], vp[u][1][c]));
                need |= lmax[c] > st.nu_lim[c];
            }
            if (__any_sync(0xffffffffu, need)) {
#pragma unroll
                for (int c = 0; c < kC; c++) {
                    float vmax = fmaxf(lmax[c], __shfl_xor_sync(0xffffffffu, lmax[c], 4));
                    vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 8));
                    vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 16));
                    const float nn = fmaxf(pow2ceil(vmax), kNuFloor);
                    if (st.nu[c] == 0.f) {
                        st.nu[c] = nn;
                    } else if (nn > st.nu[c]) {
                        const float r = st.nu[c] / nn;
#pragma unroll
                        for (int hg = 0; hg < HG; hg++)
#pragma unroll
                            for (int h2 = 0; h2 < 2; h2++) {
                                float *o = st.o[hg][2 * c + h2];
                                o[0] *= r; o[1] *= r; o[2] *= r; o[3] *= r;
                            }
                        st.nu[c] = nn;
                    }
                    st.inv_nu[c] = 1.0f / st.nu[c];
                    st.nu_lim[c] = st.nu[c] * kNuHeadroom;
                }
            }
        }
        pv<NT>(tiles, st, p, vp);
    }

    __device__ static void step(const uint8_t *tile, const Frag &f, State &st, int t_lo, int t_hi,
                                float (&psum)[HG]) {
        const uint8_t *const tiles[1] = {tile};
        const int lo[1] = {t_lo}, hi[1] = {t_hi};
        float ps[1][HG];
        stepn<1>(tiles, f, st, lo, hi, ps);
#pragma unroll
        for (int hg = 0; hg < HG; hg++) psum[hg] = ps[0][hg];
    }

    __device__ static void mass(const AttnArgs &A, uint64_t unit, const State &st, float (&psum)[HG]) {
        const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            float u = psum[hg];
            u += __shfl_xor_sync(0xffffffffu, u, 4);
            u += __shfl_xor_sync(0xffffffffu, u, 8);
            u += __shfl_xor_sync(0xffffffffu, u, 16);
            const uint32_t h = 4 * hg + tig;
            if (gid == 0 && h < A.group) A.tile_mass[unit * kMaxGroup + h] = make_float2(u, st.m[hg]);
        }
    }

    __device__ static void store_rows(const AttnArgs &A, const State &st, float *o_base, float *m_out, float *l_out,
                                      bool normalize, float2 *seg_ml) {
        const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            float lt = st.l[hg];
            lt += __shfl_xor_sync(0xffffffffu, lt, 4);
            lt += __shfl_xor_sync(0xffffffffu, lt, 8);
            lt += __shfl_xor_sync(0xffffffffu, lt, 16);
            float zt[kG];
#pragma unroll
            for (int g = 0; g < kG; g++) {
                float z = st.z[hg][g];
                z += __shfl_xor_sync(0xffffffffu, z, 4);
                z += __shfl_xor_sync(0xffffffffu, z, 8);
                z += __shfl_xor_sync(0xffffffffu, z, 16);
                zt[g] = z;
            }
            const uint32_t h = 4 * hg + tig;
            if (h >= A.group) continue;
            const float inv = normalize ? (lt > 0.f ? 1.0f / lt : 0.f) : 1.0f;
            float *row = o_base + (size_t)h * kHeadDim;
#pragma unroll
            for (int mb = 0; mb < 8; mb++) {
                const int c = mb >> 1, g = group_of_class(c);
                const int m0 = 16 * (mb & 1) + gid;
                const float sc = st.nu[c] * code_scale(c);
                row[dim_of(c, m0)] = ((st.o[hg][mb][0] + st.o[hg][mb][1]) * sc + zt[g]) * inv;
                row[dim_of(c, m0 + 8)] = ((st.o[hg][mb][2] + st.o[hg][mb][3]) * sc + zt[g]) * inv;
            }
            if (gid == 0) {
                if (m_out) { m_out[h] = st.m[hg]; l_out[h] = lt; }
                if (seg_ml) seg_ml[h] = make_float2(st.m[hg], lt);
            }
        }
    }
};

// ---------------------------------------------------------------------------
// fp16 codec (F16, the reference's paged pool format): the int8 structure
// without quantisation.  QK^T on the f16 tensor cores (m16n8k16) with the K
// rows as A, loaded by ldmatrix from the swizzled tile, and the query as B in
// two f16 parts per head (hi + lo of the query pre-scaled by log2(e) x the
// softmax scale and by a power of two that keeps it within [-1, 1]):
// columns (head, part), products exact in fp32, 8 MMAs per tile and head
// group.  P x V as in Int8T with V^T loaded by ldmatrix.trans and P^T as
// f16 hi/lo pairs through movmatrix; V needs no scale.
// ---------------------------------------------------------------------------
template <int HG>
struct F16T {
    static constexpr int kBytes = 8192, kStages = 2;
    static constexpr int kTilesPerStep = 1;
    struct Frag {
        uint32_t b[HG][8][2];  // B: [head group][k-block of 16 dims][reg]
        float sq[HG];          // the power of two of the lane's head (C side)
    };
    struct State {
        float o[HG][8][4];  // (dims x (head, hi/lo)) accumulators per m-block
        float m[HG], l[HG];
    };

    __device__ static void begin(Frag &f, State &st, const AttnArgs &A, uint32_t s_idx) {
        const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
        const uint32_t G = A.group;
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            const uint32_t hq = 4 * hg + (gid >> 1);
            // dims 16kb + 2tig + {0, 1, 8, 9} of the lane's head
            float v[32];
            if (hq < G) {
                const float *q = A.query + ((size_t)s_idx * G + hq) * kHeadDim;
#pragma unroll
                for (int kb = 0; kb < 8; kb++) {
                    const float2 x0 = *reinterpret_cast<const float2 *>(q + 16 * kb + 2 * tig);
                    const float2 x1 = *reinterpret_cast<const float2 *>(q + 16 * kb + 8 + 2 * tig);
                    v[4 * kb] = x0.x; v[4 * kb + 1] = x0.y; v[4 * kb + 2] = x1.x; v[4 * kb + 3] = x1.y;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++) v[i] = 0.f;
            }
            float mx = 0.f;
#pragma unroll
            for (int i = 0; i < 32; i++) {
                v[i] *= A.scale_log2;
                if (isfinite(v[i])) mx = fmaxf(mx, fabsf(v[i]));
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float sq = mx > 0.f ? pow2ceil(mx) : 1.0f;
            const float inv = 1.0f / sq;  // a power of two: exact
            const bool lo = gid & 1;      // B column gid = (head gid>>1, part gid&1)
#pragma unroll
            for (int kb = 0; kb < 8; kb++) {
                uint32_t w[2];
#pragma unroll
                for (int r = 0; r < 2; r++) {
                    const float y0 = v[4 * kb + 2 * r] * inv, y1 = v[4 * kb + 2 * r + 1] * inv;
                    const __half2 h = __floats2half2_rn(y0, y1);
                    const float2 hf = __half22float2(h);
                    const __half2 l2 = __floats2half2_rn(y0 - hf.x, y1 - hf.y);
                    w[r] = lo ? *reinterpret_cast<const uint32_t *>(&l2) : *reinterpret_cast<const uint32_t *>(&h);
                }
                f.b[hg][kb][0] = w[0];
                f.b[hg][kb][1] = w[1];
            }
            // C side: this lane's head 4hg + tig is held by the lanes gid = 2tig
            f.sq[hg] = __shfl_sync(0xffffffffu, sq, 8 * tig);
            st.m[hg] = -INFINITY;
            st.l[hg] = 0.f;
#pragma unroll
            for (int mb = 0; mb < 8; mb++) st.o[hg][mb][0] = st.o[hg][mb][1] = st.o[hg][mb][2] = st.o[hg][mb][3] = 0.f;
        }
    }

    __device__ static void step(const uint8_t *tile, const Frag &f, State &st, int t_lo, int t_hi,
                                float (&psum)[HG]) {
        const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
        // ---- scores: A = K rows; ldmatrix lane l gives row (l&7) of matrix
        // l>>3 = (tokens 8*(m&1).., dims 8*(2kb + (m>>1))..)
        const int krow = (lane & 7) + 8 * ((lane >> 3) & 1), kch = lane >> 4;
        float acc[HG][4];
#pragma unroll
        for (int hg = 0; hg < HG; hg++) acc[hg][0] = acc[hg][1] = acc[hg][2] = acc[hg][3] = 0.f;
#pragma unroll
        for (int kb = 0; kb < 8; kb++) {
            uint32_t a[4];
            ldmatrix_x4(a, tile + krow * 256 + ((((2 * kb + kch) ^ (krow & 7))) << 4));
#pragma unroll
            for (int hg = 0; hg < HG; hg++) mma16816(acc[hg], a, f.b[hg][kb][0], f.b[hg][kb][1]);
        }
        const bool full = t_lo == 0 && t_hi == 16;  // warp-uniform
        const bool ok0 = full || (gid >= t_lo && gid < t_hi);
        const bool ok1 = full || (gid + 8 >= t_lo && gid + 8 < t_hi);
        float s[HG][2];
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            // columns 2tig (hi part) and 2tig+1 (lo part) of head 4hg + tig
            s[hg][0] = ok0 ? (acc[hg][0] + acc[hg][1]) * f.sq[hg] : -INFINITY;
            s[hg][1] = ok1 ? (acc[hg][2] + acc[hg][3]) * f.sq[hg] : -INFINITY;
        }
        // ---- online softmax per head (reduction over the 8 token lanes gid)
        float p[HG][2];
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            float tmax = fmaxf(s[hg][0], s[hg][1]);
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 8));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
            const float m_new = fmaxf(st.m[hg], tmax);
            if (__any_sync(0xffffffffu, m_new > st.m[hg])) {
                const float alpha = ex2(st.m[hg] - m_new);
                st.l[hg] *= alpha;
#pragma unroll
                for (int mb = 0; mb < 8; mb++) {
                    st.o[hg][mb][0] *= alpha; st.o[hg][mb][1] *= alpha;
                    st.o[hg][mb][2] *= alpha; st.o[hg][mb][3] *= alpha;
                }
                st.m[hg] = m_new;
            }
            p[hg][0] = ex2(s[hg][0] - st.m[hg]);
            p[hg][1] = ex2(s[hg][1] - st.m[hg]);
            st.l[hg] += p[hg][0] + p[hg][1];
            psum[hg] = p[hg][0] + p[hg][1];
        }
        // ---- P as f16 hi+lo, transposed into the PV B operand
        uint32_t bp[HG][2];
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            const __half2 hi = __floats2half2_rn(p[hg][0], p[hg][1]);
            const float2 hf = __half22float2(hi);
            const __half2 lo = __floats2half2_rn(p[hg][0] - hf.x, p[hg][1] - hf.y);
            const uint32_t hu = *reinterpret_cast<const uint32_t *>(&hi);
            const uint32_t lu = *reinterpret_cast<const uint32_t *>(&lo);
            bp[hg][0] = movmatrix_trans(prmt(hu, lu, 0x5410u));  // (hi, lo) of token gid
            bp[hg][1] = movmatrix_trans(prmt(hu, lu, 0x7632u));  // (hi, lo) of token gid+8
        }
        // ---- P x V: A = V^T; ldmatrix.trans lane l gives row (l&7) of matrix
        // l>>3 = (tokens 8*(m>>1).., dims 8*(2mb + (m&1))..)
        const int vrow = (lane & 7) + 8 * (lane >> 4), vch = (lane >> 3) & 1;
        const uint8_t *vt = tile + 4096 + vrow * 256;
        // a partial tile's masked slots may hold anything (even non-finite
        // values): zero their V entries, tokens 2tig, 2tig+1 (+8) of this lane
        uint32_t vmask[2] = {0xFFFFFFFFu, 0xFFFFFFFFu};
        if (!full) {
#pragma unroll
            for (int hk = 0; hk < 2; hk++) {
                const int t0 = 2 * tig + 8 * hk;
                vmask[hk] = (t0 >= t_lo && t0 < t_hi ? 0x0000FFFFu : 0u) |
                            (t0 + 1 >= t_lo && t0 + 1 < t_hi ? 0xFFFF0000u : 0u);
            }
        }
#pragma unroll
        for (int mb = 0; mb < 8; mb++) {
            uint32_t a[4];
            ldmatrix_x4_trans(a, vt + ((((2 * mb + vch) ^ (vrow & 7))) << 4));
            a[0] &= vmask[0]; a[1] &= vmask[0]; a[2] &= vmask[1]; a[3] &= vmask[1];
#pragma unroll
            for (int hg = 0; hg < HG; hg++) mma16816(st.o[hg][mb], a, bp[hg][0], bp[hg][1]);
        }
    }

    // tile probability mass and running max per head (eviction scores)
    __device__ static void mass(const AttnArgs &A, uint64_t unit, const State &st, float (&psum)[HG]) {
        const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            float u = psum[hg];
            u += __shfl_xor_sync(0xffffffffu, u, 4);
            u += __shfl_xor_sync(0xffffffffu, u, 8);
            u += __shfl_xor_sync(0xffffffffu, u, 16);
            const uint32_t h = 4 * hg + tig;
            if (gid == 0 && h < A.group) A.tile_mass[unit * kMaxGroup + h] = make_float2(u, st.m[hg]);
        }
    }

    // rows of the G query heads at o_base (stride 128), optionally normalised;
    // m_out / l_out / seg_ml per head when non-null
    __device__ static void store_rows(const AttnArgs &A, const State &st, float *o_base, float *m_out, float *l_out,
                                      bool normalize, float2 *seg_ml) {
        const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
#pragma unroll
        for (int hg = 0; hg < HG; hg++) {
            float lt = st.l[hg];
            lt += __shfl_xor_sync(0xffffffffu, lt, 4);
            lt += __shfl_xor_sync(0xffffffffu, lt, 8);
            lt += __shfl_xor_sync(0xffffffffu, lt, 16);
            const uint32_t h = 4 * hg + tig;
            if (h >= A.group) continue;
            const float inv = normalize ? (lt > 0.f ? 1.0f / lt : 0.f) : 1.0f;
            float *row = o_base + (size_t)h * kHeadDim;
#pragma unroll
            for (int mb = 0; mb < 8; mb++) {
                row[16 * mb + gid] = (st.o[hg][mb][0] + st.o[hg][mb][1]) * inv;
                row[16 * mb + gid + 8] = (st.o[hg][mb][2] + st.o[hg][mb][3]) * inv;
            }
            if (gid == 0) {
                if (m_out) { m_out[h] = st.m[hg]; l_out[h] = lt; }
                if (seg_ml) seg_ml[h] = make_float2(st.m[hg], lt);
            }
        }
    }
};

// ---------------------------------------------------------------------------
// per-codec operations used by the kernel: begin (load the query rows of a
// segment, reset the state), step (one tile), mass (eviction scores of the
// tile), store_rows (the segment's G output rows, or a partial)
// ---------------------------------------------------------------------------
template <int CODEC, int HG>
struct Ops : Int8T<CODEC, HG> {};

template <int HG>
struct Ops<QWN_KV_CODEC_Q4_G32, HG> : LowBitT<QWN_KV_CODEC_Q4_G32, HG> {};
template <int HG>
struct Ops<QWN_KV_CODEC_TQ35_G64, HG> : LowBitT<QWN_KV_CODEC_TQ35_G64, HG> {};
template <int HG>
struct Ops<QWN_KV_CODEC_F16, HG> : F16T<HG> {};

// ---------------------------------------------------------------------------
// batch geometry
// ---------------------------------------------------------------------------
struct Geo {
    int32_t seq, tok_lo, tok_hi;
    uint32_t tile0, ntiles;
};

// (sequence id, length) of the first kLenCache batch entries, filled once per
// CTA at launch start: every warp's setup walks these, and the CTA reads the
// sequence table once instead of once per warp
constexpr uint32_t kLenCache = 256;
__device__ __forceinline__ int2 *len_cache() {
    __shared__ int2 cache[kLenCache];
    return cache;
}
__device__ __forceinline__ void fill_len_cache(const AttnArgs &A) {
    const uint32_t n = A.num_seqs < kLenCache ? A.num_seqs : kLenCache;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const int32_t seq = A.seq_ids ? A.seq_ids[i] : (int32_t)i;
        const int32_t len = (seq >= 0 && (uint32_t)seq < A.max_seqs) ? A.seq_lens[seq] : 0;
        len_cache()[i] = make_int2(seq, len);
    }
    __syncthreads();
}

__device__ __forceinline__ Geo geo_of(const AttnArgs &A, uint32_t i) {
    Geo g;
    int32_t len = 0;
    if (i < kLenCache) {
        const int2 c = len_cache()[i];
        g.seq = c.x;
        len = c.y;
    } else {
        g.seq = A.seq_ids ? A.seq_ids[i] : (int32_t)i;
    }
    g.tok_lo = g.tok_hi = 0;
    g.tile0 = g.ntiles = 0;
    if (g.seq < 0 || (uint32_t)g.seq >= A.max_seqs) {
        latch(A.status, QWN_KV_STATUS_BAD_SEQUENCE);
        return g;
    }
    if (i >= kLenCache) len = A.seq_lens[g.seq];
    int32_t hi = len;
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

// virtual units at a segment's end: the newest token's store, when the launch appends
__device__ __forceinline__ uint32_t virtual_tail(const AttnArgs &A) { return A.new_k ? kVirtualEnd : 0u; }

// floor(x / c) for x < 2^53: a double quotient (off by at most one)
// corrected to the exact integer, instead of a 64-bit integer division
__device__ __forceinline__ uint64_t floor_div(uint64_t x, uint64_t c) {
    uint64_t q = (uint64_t)((double)x / (double)c);
    if (q * c > x) --q;
    else if ((q + 1) * c <= x) ++q;
    return q;
}
__device__ __forceinline__ uint64_t muldiv_floor(uint64_t a, uint64_t b, uint64_t c) { return floor_div(a * b, c); }

// the warp whose range [w*T/W, (w+1)*T/W) holds unit u: ((u+1)W - 1) / T
__device__ __forceinline__ uint64_t warp_of_unit(uint64_t u, uint64_t T, uint64_t W) {
    return floor_div((u + 1) * W - 1, T);
}

// position of a unit: batch entry i, kv head h, tile within the entry
struct Walk {
    uint32_t i, h, tile;
    uint64_t seg_base;  // global unit index of (i, h, tile 0)
    uint64_t vbase;     // virtual index of the segment's start (kVirtualUnits before tile 0)
    Geo geo;
};

__device__ __forceinline__ void walk_next_segment(const AttnArgs &A, Walk &w) {
    w.seg_base += w.geo.ntiles;
    w.vbase += w.geo.ntiles + kVirtualUnits + virtual_tail(A);
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
__device__ __forceinline__ uint32_t warp_incl_scan(uint32_t v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

// per-warp shared-memory windows over the warp's units, double buffered: for
// unit base+L of window w, pg = the page id (copied from the page table by
// cp.async, so the warp never waits on it), off = the tile's byte offset in
// its page, app = the segment whose newest token lives in that unit when the
// launch appends (-1: none).  The next window is requested 16 units before it
// is needed.
struct WarpWindow {
    int32_t pg[2][32];    // page id (kNoUnit past the warp's last unit)
    uint32_t off[2][32];  // tile offset in its page; after window_resolve the
                          // tile's address in 64-byte units from the pool base
    int32_t app[2][32];
    uint32_t hv[2][32];  // h * tiles_per_page + tile in page (layer-free part of off)
};
constexpr int32_t kNoUnit = INT32_MIN;

// the newest token's K and V rows (512 B each) of segment `app` into L1 for its store
__device__ __forceinline__ void prefetch_new_rows(const AttnArgs &A, int32_t app) {
    const float *rk = A.new_k + (size_t)app * kHeadDim, *rv = A.new_v + (size_t)app * kHeadDim;
#pragma unroll
    for (int c = 0; c < 4; c++) {
        asm volatile("prefetch.global.L1 [%0];" ::"l"(rk + 32 * c));
        asm volatile("prefetch.global.L1 [%0];" ::"l"(rv + 32 * c));
    }
}

// Request window w for the warp's units [base, base+32) (of n), lane L taking
// unit base+L, walking forward `skip` units from `from`.
__device__ __forceinline__ void fill_window(const AttnArgs &A, const Walk &from, uint32_t skip, uint32_t base,
                                            uint32_t n, WarpWindow *win, int w) {
    const int lane = threadIdx.x & 31;
    int32_t app = -1;
    uint32_t off = 0, hv = 0;
    bool copied = false;
    if (base + lane < n) {
        Walk t = from;
        walk_advance(A, t, skip + lane);
        const uint32_t tg = t.geo.tile0 + t.tile;
        const uint32_t lp = tg / A.tpp, tin = tg % A.tpp;
        hv = t.h * A.tpp + tin;
        off = (A.layer * A.kv_heads * A.tpp + hv) * A.tile_bytes;
        if (lp < A.mp) {
            const int32_t *src = A.page_table + (size_t)t.geo.seq * A.mp + lp;
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(&win->pg[w][lane])), "l"(src)
                         : "memory");
            copied = true;
        }
        if (A.new_k && t.tile + 1 == t.geo.ntiles) {
            app = (int32_t)(t.i * A.kv_heads + t.h);
            prefetch_new_rows(A, app);
        }
    }
    if (!copied) win->pg[w][lane] = base + lane < n ? -1 : kNoUnit;
    win->off[w][lane] = off;
    win->app[w][lane] = app;
    win->hv[w][lane] = hv;
    asm volatile("cp.async.commit_group;" ::: "memory");
}
// wait for this warp's window requests
__device__ __forceinline__ void window_ready() {
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncwarp();
}
// tile addresses of window w's units, one lane each, once its page ids have
// landed (out-of-range page ids of real units latch BAD_PAGE and read page
// 0).  Pages and tiles are multiples of 64 bytes, so the address fits 32 bits
// in 64-byte units for pools up to 256 GB.
__device__ __forceinline__ void window_resolve(const AttnArgs &A, WarpWindow *win, int w) {
    const int lane = threadIdx.x & 31;
    int32_t pg = win->pg[w][lane];
    if (pg != kNoUnit && (pg < 0 || (uint32_t)pg >= A.total_pages)) {
        latch(A.status, QWN_KV_STATUS_BAD_PAGE);
        pg = 0;  // stay in bounds; the latched status marks the result invalid
    }
    if (pg == kNoUnit) pg = 0;
    win->off[w][lane] = (uint32_t)(((uint64_t)pg * A.page_bytes + win->off[w][lane]) >> 6);
    __syncwarp();
}
__device__ __forceinline__ const uint8_t *window_src(const AttnArgs &A, const WarpWindow *win, int w, uint32_t L) {
    return A.pages + ((size_t)win->off[w][L] << 6);
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

// Partial slot of a (warp, segment): the G rows of unnormalised o, then m[G]
// and l[G]; one bulk copy of slot_bytes(G) moves it.
__device__ __forceinline__ uint32_t slot_bytes(uint32_t G) { return (G * (kHeadDim + 2) * 4 + 15u) & ~15u; }

// The parts of a segment: the warps wa..wb whose ranges meet its tiles
// (warp of virtual unit u is ((u+1)W-1)/T, T the virtual total; the kernel
// caps W so that every warp range holds real units), except that the four
// warps of an "interior" CTA -- all of them strictly between wa and wb, so
// their ranges hold this segment's tiles and nothing else -- merge in shared
// memory first and count as one part.  Warps are numbered CTA by CTA (warp w
// is warp w % 4 of CTA w / 4).  Part order: the warps before the first
// interior CTA, the interior CTAs, the warps after; the slot of a part is
// the one of its (first) warp.
struct Parts {
    uint64_t wa, c0;          // first warp; first interior CTA
    uint32_t pre, ncta, n;    // parts before the interior CTAs; interior CTAs; all parts
};
__device__ __forceinline__ Parts parts_of(uint64_t Us, uint64_t ns, uint64_t T, uint64_t W) {
    Parts P;
    P.wa = warp_of_unit(Us + kVirtualUnits, T, W);
    const uint64_t wb = warp_of_unit(Us + kVirtualUnits + ns - 1, T, W);
    P.c0 = P.wa / kWarpsPerCta + 1;
    const uint64_t c_end = wb / kWarpsPerCta;  // CTAs c < c_end have 4c + 3 < wb
    P.ncta = c_end > P.c0 ? (uint32_t)(c_end - P.c0) : 0u;
    if (P.ncta == 0) {
        P.pre = P.n = (uint32_t)(wb - P.wa + 1);
    } else {
        P.pre = (uint32_t)(kWarpsPerCta * P.c0 - P.wa);
        P.n = P.pre + P.ncta + (uint32_t)(wb - kWarpsPerCta * c_end + 1);
    }
    return P;
}
// the warp whose slot holds part i
__device__ __forceinline__ uint64_t part_warp(const Parts &P, uint32_t i) {
    if (i < P.pre) return P.wa + i;
    if (i < P.pre + P.ncta) return kWarpsPerCta * (P.c0 + (i - P.pre));
    return kWarpsPerCta * (P.c0 + P.ncta) + (i - P.pre - P.ncta);
}
__device__ __forceinline__ bool interior_warp(const Parts &P, uint64_t w) {
    return P.ncta != 0 && w >= kWarpsPerCta * P.c0 && w < kWarpsPerCta * (P.c0 + P.ncta);
}
// part index of warp w (for an interior warp: of its CTA)
__device__ __forceinline__ uint32_t part_index(const Parts &P, uint64_t w) {
    if (w < P.wa + P.pre) return (uint32_t)(w - P.wa);
    const uint64_t cend = kWarpsPerCta * (P.c0 + P.ncta);
    if (w < cend) return P.pre + (uint32_t)(w / kWarpsPerCta - P.c0);
    return P.pre + P.ncta + (uint32_t)(w - cend);
}

// ---------------------------------------------------------------------------
// split-KV exchange between ranks (peer memory over NVLink)
// ---------------------------------------------------------------------------
constexpr size_t kXFlagBytes = 2ull * QWN_KV_MAX_RANKS * QWN_KV_EXCHANGE_SEGMENTS * 4;
__device__ __forceinline__ uint32_t *xflag(uint8_t *buf, uint32_t parity, uint32_t sender, uint32_t seg) {
    return reinterpret_cast<uint32_t *>(buf) + (parity * QWN_KV_MAX_RANKS + sender) * QWN_KV_EXCHANGE_SEGMENTS + seg;
}
// block of (parity, sender): o[xrows][128], m[xrows], l[xrows]
__device__ __forceinline__ float *xblock(uint8_t *buf, uint32_t parity, uint32_t sender, uint32_t xrows) {
    return reinterpret_cast<float *>(buf + kXFlagBytes) +
           (size_t)(parity * QWN_KV_MAX_RANKS + sender) * xrows * (kHeadDim + 2);
}
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// copy this warp's partial slot of segment s_idx (written by the warp itself)
// into every rank's block
__device__ __forceinline__ void publish_slot(const AttnArgs &A, uint32_t s_idx, const float *slot) {
    const int lane = threadIdx.x & 31;
    const uint32_t G = A.group;
    const size_t row0 = (size_t)s_idx * G;
    __syncwarp();  // the lanes' slot stores are visible to the whole warp
    for (uint32_t g = 0; g < G; g++) {
        const float4 v = reinterpret_cast<const float4 *>(slot + g * kHeadDim)[lane];
        const float m = slot[G * kHeadDim + g], l = slot[G * kHeadDim + G + g];
        for (uint32_t r = 0; r < A.xworld; r++) {
            float *blk = xblock(A.xbuf[r], A.xepoch & 1u, A.xrank, A.xrows);
            reinterpret_cast<float4 *>(blk + (row0 + g) * kHeadDim)[lane] = v;
            if (lane == 0) {
                blk[(size_t)A.xrows * kHeadDim + row0 + g] = m;
                blk[(size_t)A.xrows * (kHeadDim + 1) + row0 + g] = l;
            }
        }
    }
}

// This rank's partial of segment s_idx (rows row0..row0+G) has been stored
// into every rank's block by the calling warp: raise the segment's flag on
// every rank (lane r releases to rank r; the warp barrier before it orders the
// other lanes' block stores), wait -- lane r for rank r's flag in this rank's
// buffer, bounded by xtimeout_ns -- and merge the ranks' partials in rank
// order into the output rows: the same arithmetic, so the same rows, on
// every rank.  Loads go through L2 (.cg): the blocks are written by peers.
__device__ __forceinline__ void exchange_merge(const AttnArgs &A, uint32_t s_idx, size_t row0) {
    const int lane = threadIdx.x & 31;
    const uint32_t par = A.xepoch & 1u, W = A.xworld, G = A.group;
    __syncwarp();
    if ((uint32_t)lane < W) st_release_sys(xflag(A.xbuf[lane], par, A.xrank, s_idx), A.xepoch);
    uint8_t *own = A.xbuf[A.xrank];
    bool ok = true;
    if ((uint32_t)lane < W) {
        const uint32_t *f = xflag(own, par, lane, s_idx);
        const uint64_t t0 = globaltimer();
        while (ld_acquire_sys(f) != A.xepoch) {
            if (globaltimer() - t0 > A.xtimeout_ns) { ok = false; break; }
            __nanosleep(32);
        }
    }
    if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) latch(A.status, QWN_KV_STATUS_PEER_TIMEOUT);
        return;
    }
    // (m, l) of pair i = g*W + r (at most 64 pairs): lane holds i = lane, lane+32
    float mp[2], lp[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const uint32_t i = (uint32_t)lane + 32u * h;
        mp[h] = -INFINITY;
        lp[h] = 0.f;
        if (i < G * W) {
            const float *blk = xblock(own, par, i % W, A.xrows);
            const size_t row = row0 + i / W;
            mp[h] = __ldcg(blk + (size_t)A.xrows * kHeadDim + row);
            lp[h] = __ldcg(blk + (size_t)A.xrows * (kHeadDim + 1) + row);
        }
    }
    for (uint32_t g = 0; g < G; g += 2) {
        // two rows per round: all ranks' o of both rows are loaded at once
        float4 v[2][QWN_KV_MAX_RANKS];
#pragma unroll
        for (int e = 0; e < 2; e++)
#pragma unroll
            for (uint32_t r = 0; r < QWN_KV_MAX_RANKS; r++)
                v[e][r] = (r < W && g + e < G)
                              ? __ldcg(reinterpret_cast<const float4 *>(xblock(own, par, r, A.xrows) +
                                                                        (row0 + g + e) * kHeadDim) + lane)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int e = 0; e < 2; e++) {
            if (g + e >= G) break;
            float m[QWN_KV_MAX_RANKS], l[QWN_KV_MAX_RANKS];
            float M = -INFINITY;
#pragma unroll
            for (uint32_t r = 0; r < QWN_KV_MAX_RANKS; r++) {
                const uint32_t i = (g + e) * W + r;
                const float mh = __shfl_sync(0xffffffffu, i < 32 ? mp[0] : mp[1], i & 31);
                const float lh = __shfl_sync(0xffffffffu, i < 32 ? lp[0] : lp[1], i & 31);
                m[r] = r < W ? mh : -INFINITY;
                l[r] = r < W ? lh : 0.f;
                M = fmaxf(M, m[r]);
            }
            float ls = 0.f;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (uint32_t r = 0; r < QWN_KV_MAX_RANKS; r++) {
                if (r >= W) break;
                const float w = m[r] == -INFINITY ? 0.f : ex2(m[r] - M);
                ls += l[r] * w;
                acc.x += v[e][r].x * w; acc.y += v[e][r].y * w; acc.z += v[e][r].z * w; acc.w += v[e][r].w * w;
            }
            const float inv = ls > 0.f ? 1.0f / ls : 0.f;
            reinterpret_cast<float4 *>(A.output + (row0 + g + e) * kHeadDim)[lane] =
                make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        }
    }
}

// merge_small: the merge of a segment (or group) whose parts all fit in one
// warp's stage memory, so that every merger -- a lone warp or a CTA's -- does
// it in one round with the same arithmetic.  The merging warp pulls the
// nparts slots (written by other warps) into shared memory (buf, SB bytes)
// with bulk copies completed on one mbarrier and combines them there, its
// rows unrolled: GG >= G is the compile-time row count.  Output as for
// merge_chunked.  Returns false when the wait gave up.
template <int GG, bool XCHG>
__device__ __forceinline__ bool merge_small(const AttnArgs &A, uint32_t s_idx, const Parts &P, uint32_t first,
                                           uint32_t stride, uint32_t nparts, float *dst_slot, uint8_t *buf,
                                           uint32_t SB, uint64_t *bar, uint32_t &par) {
    const int lane = threadIdx.x & 31;
    const uint32_t G = A.group;
    const uint32_t PB = slot_bytes(G), rowf = G * kHeadDim;
    const uint32_t cap = SB / PB < 32u ? SB / PB : 32u;
    auto slot_of = [&](uint32_t pp) -> const float * {
        return A.partials + (size_t)(part_warp(P, first + pp * stride) + s_idx) * kPartialFloats;
    };
    // the slots were written by generic stores of other warps (ordered by the
    // acquire on the segment counter); the bulk copies read them through the
    // async proxy
    asm volatile("fence.proxy.async.global;" ::: "memory");
    float M[GG], ls[GG];
    float4 acc[GG];
#pragma unroll
    for (int g = 0; g < GG; g++) { M[g] = -INFINITY; ls[g] = 0.f; acc[g] = make_float4(0.f, 0.f, 0.f, 0.f); }
    for (uint32_t c = 0; c < nparts; c += cap) {
        const uint32_t nq = nparts - c < cap ? nparts - c : cap;
        if (lane == 0) mbar_expect_tx(bar, nq * PB);
        __syncwarp();
        if ((uint32_t)lane < nq) bulk_g2s(buf + lane * PB, slot_of(c + lane), PB, bar);
        if (!mbar_wait_bounded(bar, par)) {
            if (lane == 0) latch(A.status, QWN_KV_STATUS_WAIT_TIMEOUT);
            mbar_wait_bounded(bar, par);  // the copies into buf must land before the warp leaves
            return false;
        }
        par ^= 1u;
        float m[GG], l[GG];
#pragma unroll
        for (int g = 0; g < GG; g++) { m[g] = -INFINITY; l[g] = 0.f; }
        if ((uint32_t)lane < nq) {
            const float *ml = reinterpret_cast<const float *>(buf + lane * PB) + rowf;
#pragma unroll
            for (int g = 0; g < GG; g++)
                if ((uint32_t)g < G) { m[g] = ml[g]; l[g] = ml[G + g]; }
        }
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
        for (uint32_t q = 0; q < nq; q++) {
            const float *sl = reinterpret_cast<const float *>(buf + q * PB);
#pragma unroll
            for (int g = 0; g < GG; g++) {
                const float wg = __shfl_sync(0xffffffffu, w[g], q);
                if ((uint32_t)g < G) {
                    const float4 v = reinterpret_cast<const float4 *>(sl + g * kHeadDim)[lane];
                    acc[g].x += v.x * wg; acc[g].y += v.y * wg; acc[g].z += v.z * wg; acc[g].w += v.w * wg;
                }
            }
        }
        __syncwarp();  // all lanes are done with buf before the next chunk lands
    }
    const size_t row0 = (size_t)s_idx * G;
#pragma unroll
    for (int g = 0; g < GG; g++) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ls[g] += __shfl_xor_sync(0xffffffffu, ls[g], o);
        if ((uint32_t)g >= G) continue;
        if (dst_slot) {  // a merged group, stored as one unnormalised partial
            reinterpret_cast<float4 *>(dst_slot + g * kHeadDim)[lane] = acc[g];
            if (lane == 0) { dst_slot[rowf + g] = M[g]; dst_slot[rowf + G + g] = ls[g]; }
            continue;
        }
        const size_t row = row0 + g;
        if constexpr (XCHG) {
            for (uint32_t r = 0; r < A.xworld; r++) {
                float *blk = xblock(A.xbuf[r], A.xepoch & 1u, A.xrank, A.xrows);
                reinterpret_cast<float4 *>(blk + row * kHeadDim)[lane] = acc[g];
                if (lane == 0) {
                    blk[(size_t)A.xrows * kHeadDim + row] = M[g];
                    blk[(size_t)A.xrows * (kHeadDim + 1) + row] = ls[g];
                }
            }
        } else if (A.part_o) {
            reinterpret_cast<float4 *>(A.part_o + row * kHeadDim)[lane] = acc[g];
            if (lane == 0) { A.part_m[row] = M[g]; A.part_l[row] = ls[g]; }
        } else {
            const float inv = ls[g] > 0.f ? 1.0f / ls[g] : 0.f;
            reinterpret_cast<float4 *>(A.output + row * kHeadDim)[lane] =
                make_float4(acc[g].x * inv, acc[g].y * inv, acc[g].z * inv, acc[g].w * inv);
        }
        if (A.seg_ml && lane == 0) A.seg_ml[(size_t)s_idx * kMaxGroup + g] = make_float2(M[g], ls[g]);
    }
    if constexpr (XCHG) {
        if (!dst_slot) exchange_merge(A, s_idx, row0);
    }
    return true;
}

// one round of slot copies: parts i0 .. i0+nq-1 into cbuf, PB bytes apart,
// completed on bar; false (status latched) when the wait gave up
template <class SlotOf>
__device__ __forceinline__ bool copy_round(const AttnArgs &A, uint8_t *cbuf, uint32_t PB, uint32_t i0, uint32_t nq,
                                           const SlotOf &slot_of, uint64_t *bar, uint32_t &par) {
    const int lane = threadIdx.x & 31;
    if (lane == 0) mbar_expect_tx(bar, nq * PB);
    __syncwarp();
    if ((uint32_t)lane < nq) bulk_g2s(cbuf + lane * PB, slot_of(i0 + lane), PB, bar);
    if (!mbar_wait_bounded(bar, par)) {
        if (lane == 0) latch(A.status, QWN_KV_STATUS_WAIT_TIMEOUT);
        mbar_wait_bounded(bar, par);  // the copies into buf must land before the warp leaves
        return false;
    }
    par ^= 1u;
    return true;
}

// merge_chunked: merge nparts partial slots of segment s_idx -- part i of the map P at slot
// part_warp(P, first + i * stride) + s_idx -- into the segment's output rows
// (row0 = s_idx * G), or, given dst_slot, into one unnormalised partial
// there.  Returns false when a wait gave up.
//
// The arithmetic depends on the part order only, so every launch gives the
// same bits whichever warp merges and however much shared memory it has:
// the parts are taken in logical chunks of 32 (lane q <-> part q), each
// chunk's (m, l) read straight from L2 into a table, the chunk maximum,
// weights and sum of l per row computed from the table, the running o rows
// rescaled once per chunk, and then the o rows of the chunk's parts added in
// part order.  Those rows arrive by bulk copies into shared memory, as many
// slots per round trip as the buffer holds (a CTA's merger has four warps'
// stages, a lone warp its own).  Rows are handled in loops that are not
// unrolled: a merge runs once per segment at the end of a launch with its
// instructions fetched cold, so its code is kept short.
//
// buf layout: o[G][128] running rows, M[8], L[8], alpha[8], then per (row,
// part) the tables m, l, w (rows kTStride floats apart, so that lanes reading
// different rows hit different banks), then the copied slots.
template <bool XCHG>
__device__ __forceinline__ bool merge_chunked(const AttnArgs &A, uint32_t s_idx, const Parts &P, uint32_t first,
                                              uint32_t stride, uint32_t nparts, float *dst_slot, uint8_t *buf,
                                              uint32_t SB, uint64_t *bar, uint32_t &par) {
    const int lane = threadIdx.x & 31;
    const uint32_t G = A.group;
    const uint32_t PB = slot_bytes(G), rowf = G * kHeadDim;
    float *run = reinterpret_cast<float *>(buf);
    constexpr uint32_t kTStride = 33;
    float *Mr = run + kMaxGroup * kHeadDim, *Lr = Mr + kMaxGroup, *Ar = Lr + kMaxGroup;
    float *Tm = Ar + kMaxGroup, *Tl = Tm + kMaxGroup * kTStride, *Tw = Tl + kMaxGroup * kTStride;
    uint8_t *cbuf = buf + ((reinterpret_cast<uint8_t *>(Tw + kMaxGroup * kTStride) - buf + 15) & ~(ptrdiff_t)15);
    const uint32_t hdr = (uint32_t)(cbuf - buf);
    uint32_t cap = (SB - hdr) / PB;
    if (cap > 32u) cap = 32u;
    const size_t row0 = (size_t)s_idx * G;
    auto slot_of = [&](uint32_t i) -> const float * {
        return A.partials + (size_t)(part_warp(P, first + i * stride) + s_idx) * kPartialFloats;
    };
    // the slots were written by generic stores of other warps (ordered by the
    // acquire on the segment counter); the bulk copies read them through the
    // async proxy
    asm volatile("fence.proxy.async.global;" ::: "memory");
    for (uint32_t lc = 0; lc < nparts; lc += 32) {
        const uint32_t nl = nparts - lc < 32u ? nparts - lc : 32u;
        // a chunk that fits the buffer is copied in one round, before its
        // (m, l) are needed; otherwise the copies go round by round below
        const bool one_round = nl <= cap;
        if (one_round && !copy_round(A, cbuf, PB, lc, nl, slot_of, bar, par)) return false;
        // (m, l) of the chunk's parts: lane q takes part lc + q's rows, from
        // its copy or straight from L2
        {
            float mq[kMaxGroup], lq[kMaxGroup];
            const float *sl = (uint32_t)lane >= nl ? nullptr
                              : one_round ? reinterpret_cast<const float *>(cbuf + lane * PB) + rowf
                                          : slot_of(lc + lane) + rowf;
#pragma unroll
            for (int g = 0; g < kMaxGroup; g++) {
                mq[g] = sl && (uint32_t)g < G ? (one_round ? sl[g] : __ldcg(sl + g)) : -INFINITY;
                lq[g] = sl && (uint32_t)g < G ? (one_round ? sl[G + g] : __ldcg(sl + G + g)) : 0.f;
            }
#pragma unroll
            for (int g = 0; g < kMaxGroup; g++) {
                Tm[g * kTStride + lane] = mq[g];
                Tl[g * kTStride + lane] = lq[g];
            }
        }
        __syncwarp();
        // per row (lane g): the chunk maximum, the parts' weights and their sum of l
        if ((uint32_t)lane < G) {
            const uint32_t g = lane;
            float cm = -INFINITY;
            for (uint32_t q = 0; q < nl; q++) cm = fmaxf(cm, Tm[g * kTStride + q]);
            const float m_old = lc == 0 ? -INFINITY : Mr[g];
            const float nm = fmaxf(m_old, cm);
            float ls = 0.f;
#pragma unroll 4
            for (uint32_t q = 0; q < nl; q++) {
                const float mq = Tm[g * kTStride + q];
                const float wq = mq == -INFINITY ? 0.f : ex2(mq - nm);
                Tw[g * kTStride + q] = wq;
                ls = fmaf(Tl[g * kTStride + q], wq, ls);
            }
            const float alpha = m_old == -INFINITY ? 0.f : ex2(m_old - nm);
            Lr[g] = lc == 0 ? ls : fmaf(Lr[g], alpha, ls);
            Mr[g] = nm;
            Ar[g] = alpha;
        }
        __syncwarp();
        // the running rows, rescaled to the new maxima (zero before the first chunk)
#pragma unroll 1
        for (uint32_t g = 0; g < G; g++) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            if (lc != 0) {
                const float alpha = Ar[g];
                acc = reinterpret_cast<const float4 *>(run + g * kHeadDim)[lane];
                acc.x *= alpha; acc.y *= alpha; acc.z *= alpha; acc.w *= alpha;
            }
            reinterpret_cast<float4 *>(run + g * kHeadDim)[lane] = acc;
        }
        // the chunk's o rows, weighted, in part order
        for (uint32_t pc = 0; pc < nl; pc += cap) {
            const uint32_t nq = nl - pc < cap ? nl - pc : cap;
            __syncwarp();  // every lane is done with the previous round's slots
            if (!one_round && !copy_round(A, cbuf, PB, lc + pc, nq, slot_of, bar, par)) return false;
#pragma unroll 1
            for (uint32_t g = 0; g < G; g++) {
                float4 acc = reinterpret_cast<const float4 *>(run + g * kHeadDim)[lane];
                const uint8_t *vq = cbuf + g * (kHeadDim * 4) + lane * 16;
                const float *wg = Tw + g * kTStride + pc;
#pragma unroll 4
                for (uint32_t q = 0; q < nq; q++) {
                    const float w = wg[q];
                    const float4 v = *reinterpret_cast<const float4 *>(vq + q * PB);
                    acc.x = fmaf(v.x, w, acc.x); acc.y = fmaf(v.y, w, acc.y);
                    acc.z = fmaf(v.z, w, acc.z); acc.w = fmaf(v.w, w, acc.w);
                }
                reinterpret_cast<float4 *>(run + g * kHeadDim)[lane] = acc;
            }
        }
        __syncwarp();
    }
    // the merged rows to their destination
#pragma unroll 1
    for (uint32_t g = 0; g < G; g++) {
        const float4 acc = reinterpret_cast<const float4 *>(run + g * kHeadDim)[lane];
        const float nm = Mr[g], ls = Lr[g];
        const size_t row = row0 + g;
        if (dst_slot) {  // a merged group, stored as one unnormalised partial
            reinterpret_cast<float4 *>(dst_slot + g * kHeadDim)[lane] = acc;
            if (lane == 0) { dst_slot[rowf + g] = nm; dst_slot[rowf + G + g] = ls; }
            continue;
        }
        if constexpr (XCHG) {
            for (uint32_t r = 0; r < A.xworld; r++) {
                float *blk = xblock(A.xbuf[r], A.xepoch & 1u, A.xrank, A.xrows);
                reinterpret_cast<float4 *>(blk + row * kHeadDim)[lane] = acc;
                if (lane == 0) {
                    blk[(size_t)A.xrows * kHeadDim + row] = nm;
                    blk[(size_t)A.xrows * (kHeadDim + 1) + row] = ls;
                }
            }
        } else if (A.part_o) {
            reinterpret_cast<float4 *>(A.part_o + row * kHeadDim)[lane] = acc;
            if (lane == 0) { A.part_m[row] = nm; A.part_l[row] = ls; }
        } else {
            const float inv = ls > 0.f ? 1.0f / ls : 0.f;
            reinterpret_cast<float4 *>(A.output + row * kHeadDim)[lane] =
                make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        }
        if (A.seg_ml && lane == 0) A.seg_ml[(size_t)s_idx * kMaxGroup + g] = make_float2(nm, ls);
    }
    __syncwarp();  // buf is free again when the warp goes on
    if constexpr (XCHG) {
        if (!dst_slot) exchange_merge(A, s_idx, row0);
    }
    return true;
}


// The merge of a segment's (or group's) parts.  In the one-head-group
// kernels (G <= 4), parts that fit in one warp's stage memory (warp_sb
// bytes) are merged in one round by merge_small, whatever warp merges;
// larger merges, and every merge of the two-head-group kernels (where the
// unrolled rows cost more than they save), take merge_chunked.  The choice
// depends on the kernel and the part count only, so the result bits never
// depend on which warp merges.
template <int HG, bool XCHG>
__device__ __forceinline__ bool merge_parts(const AttnArgs &A, uint32_t s_idx, const Parts &P, uint32_t first,
                                            uint32_t stride, uint32_t nparts, float *dst_slot, uint8_t *buf,
                                            uint32_t SB, uint32_t warp_sb, uint64_t *bar, uint32_t &par) {
    if constexpr (HG == 1) {
        if (nparts * slot_bytes(A.group) <= warp_sb) {
            if (A.group <= 2)
                return merge_small<2, XCHG>(A, s_idx, P, first, stride, nparts, dst_slot, buf, SB, bar, par);
            return merge_small<4, XCHG>(A, s_idx, P, first, stride, nparts, dst_slot, buf, SB, bar, par);
        }
    }
    return merge_chunked<XCHG>(A, s_idx, P, first, stride, nparts, dst_slot, buf, SB, bar, par);
}

// End of a warp's share of segment s_idx (first unit Us, ns units).  A warp
// that saw the whole segment writes the output and returns 0.  A warp of an
// interior CTA (parts_of) writes its partial (m, l, o) into its own stage
// memory, sets in_cta and returns the number of parts; any other warp writes
// it to slot wid + s_idx and returns the number of parts.  The warp counts
// itself on the segment's counter only after its streaming loop (a release
// there waits for the slot stores to reach L2, a round trip the loop should
// not take mid-stream); the warp that draws nparts-1 merges, also after its
// loop.
template <class OPS, bool XCHG>
__device__ __forceinline__ uint32_t finish_segment(const AttnArgs &A, const typename OPS::State &st, uint32_t s_idx,
                                                   uint64_t Us, uint64_t ns, uint64_t T, uint64_t W, uint64_t wid,
                                                   uint8_t *wsm, bool &in_cta) {
    const Parts P = parts_of(Us, ns, T, W);
    const uint32_t nparts = P.n;
    const size_t row0 = (size_t)s_idx * A.group;
    in_cta = false;
    // split-KV over ranks: a whole segment is a partial too (its slot is
    // published to the ranks after the streaming loop)
    if (nparts == 1 && !XCHG) {
        float2 *sm = A.seg_ml ? A.seg_ml + (size_t)s_idx * kMaxGroup : nullptr;
        if (A.part_o)
            OPS::store_rows(A, st, A.part_o + row0 * kHeadDim, A.part_m + row0, A.part_l + row0, false, sm);
        else
            OPS::store_rows(A, st, A.output + row0 * kHeadDim, nullptr, nullptr, true, sm);
        return 0;
    }
    float *slot = A.partials + (size_t)(wid + s_idx) * kPartialFloats;
    if (interior_warp(P, wid)) {  // the CTA merges its four warps first, in shared memory
        slot = reinterpret_cast<float *>(wsm);
        in_cta = true;
    }
    OPS::store_rows(A, st, slot, slot + A.group * kHeadDim, slot + A.group * (kHeadDim + 1), false, nullptr);
    return nparts;
}

// counter a part (index idx of P.n) of segment s_idx counts on: the
// segment's when it merges in one level, else its merge group's (kept at the
// slot index of the group's first part)
__device__ __forceinline__ uint32_t *part_counter(const AttnArgs &A, uint32_t s_idx, const Parts &P, uint32_t idx) {
    if (P.n <= kMergeGroup) return &A.counters[s_idx];
    return &A.gcounters[part_warp(P, (idx / kMergeGroup) * kMergeGroup) + s_idx];
}

// The four warps of a CTA whose ranges lie inside one segment merged their
// states into their own stage memory (a slot at the start of each warp's
// stages, `stride` bytes apart); the last of them to arrive combines the four
// in warp order into the CTA's partial slot `dst` (unnormalised o, m, l).
__device__ __forceinline__ void merge_cta_slots(const AttnArgs &A, const uint8_t *base, uint32_t stride, float *dst) {
    const int lane = threadIdx.x & 31;
    const uint32_t G = A.group, rowf = G * kHeadDim;
#pragma unroll 1
    for (uint32_t g = 0; g < G; g++) {  // not unrolled: cold code, kept short
        float m[kWarpsPerCta], l[kWarpsPerCta], M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarpsPerCta; w++) {
            const float *sl = reinterpret_cast<const float *>(base + w * stride);
            m[w] = sl[rowf + g];
            l[w] = sl[rowf + G + g];
            M = fmaxf(M, m[w]);
        }
        float ls = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < kWarpsPerCta; w++) {
            const float wt = m[w] == -INFINITY ? 0.f : ex2(m[w] - M);
            const float4 v = reinterpret_cast<const float4 *>(base + w * stride)[g * (kHeadDim / 4) + lane];
            ls = fmaf(l[w], wt, ls);
            acc.x = fmaf(v.x, wt, acc.x); acc.y = fmaf(v.y, wt, acc.y);
            acc.z = fmaf(v.z, wt, acc.z); acc.w = fmaf(v.w, wt, acc.w);
        }
        reinterpret_cast<float4 *>(dst + g * kHeadDim)[lane] = acc;
        if (lane == 0) { dst[rowf + g] = M; dst[rowf + G + g] = ls; }
    }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int CODEC, int HG, bool XCHG>
__global__ void __launch_bounds__(kWarpsPerCta * 32, 3) attn_kernel(const AttnArgs A) {
    using OPS = Ops<CODEC, HG>;
    constexpr int S = OPS::kStages, B = OPS::kBytes;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t *wsm = smem + (size_t)warp * S * B;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + (size_t)kWarpsPerCta * S * B) + warp * S;
    WarpWindow *win = reinterpret_cast<WarpWindow *>(smem + (size_t)kWarpsPerCta * S * (B + 8)) + warp;
    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < S; s++) mbar_init(&bars[s], 1);
        fence_barrier_init();
    }
    __syncwarp();
    // let the stream's next kernel start its CTAs as SMs free up; wait for the
    // previous kernel's results before the first global access -- or, in the
    // early mode, before the first write that kernel could race with
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (!A.early) asm volatile("griddepcontrol.wait;" ::: "memory");
    // (returns at once once the previous kernel has finished; reading the flag
    // from the parameter bank keeps it out of the registers)
    auto dep_wait = [&]() {
        if (A.early) asm volatile("griddepcontrol.wait;" ::: "memory");
    };

    const uint32_t HK = A.kv_heads;
    uint64_t W = (uint64_t)gridDim.x * kWarpsPerCta;
    uint64_t wid = (uint64_t)blockIdx.x * kWarpsPerCta + warp;

    // The setup below depends only on the batch geometry, which is the same for
    // every layer of a decode step: it is cached per warp (per-step launch
    // plan) under a key of the pool's epoch (bumped by every change of lengths
    // or page tables) and the launch parameters.  The record is loaded while
    // the CTA reads the sequence table.
    uint32_t *plan = A.plans ? A.plans + 32 + ((size_t)blockIdx.x * kWarpsPerCta + warp) * kPlanWords : nullptr;
    uint32_t pw0 = 0, pw1 = 0, pw2 = 0, pw3 = 0, epoch = 0;
    if (plan) {
        // (in the early mode the host has checked that the previous kernel does
        // not record plans, so the records are stable while they are read)
        pw0 = plan[lane]; pw1 = plan[32 + lane]; pw2 = plan[64 + lane]; pw3 = plan[96 + lane];
        epoch = A.plans[0];
    }
    // arrivals of the CTA's warps at the shared-memory merge (interior CTAs)
    __shared__ uint32_t cta_arrivals;
    if (threadIdx.x == 0) cta_arrivals = 0u;
    fill_len_cache(A);  // (its CTA barrier also publishes cta_arrivals)
    const uint32_t key = lane == 0 ? epoch : lane == 1 ? A.num_seqs : lane == 2 ? A.attend_limit
                       : lane == 3 ? A.t_begin : lane == 4 ? A.t_end : lane == 5 ? (A.new_k ? 1u : 0u)
                       : lane == 6 ? gridDim.x : 0x504C414Eu;
    const bool hit = plan != nullptr && __all_sync(0xffffffffu, lane >= 8 || pw0 == key);

    Walk cons;
    uint32_t n = 0;
    uint64_t Tv = 0;
    int cw = 0;
    uint32_t wbase = 0;
    if (hit) {
        auto w32 = [&](int i) { return __shfl_sync(0xffffffffu, pw0, i); };
        auto w64 = [&](int i) { return (uint64_t)w32(i) | ((uint64_t)w32(i + 1) << 32); };
        n = w32(20);
        if (n == 0) {
            dep_wait();  // finishing means the previous kernel has finished too
            return;
        }
        cons.i = w32(8); cons.h = w32(9); cons.tile = w32(10);
        cons.seg_base = w64(11); cons.vbase = w64(13);
        cons.geo.seq = (int32_t)w32(15); cons.geo.tok_lo = (int32_t)w32(16); cons.geo.tok_hi = (int32_t)w32(17);
        cons.geo.tile0 = w32(18); cons.geo.ntiles = w32(19);
        Tv = w64(21); W = w64(23); wid = w64(25);
        win->pg[0][lane] = (int32_t)pw1;
        win->hv[0][lane] = pw2;
        win->off[0][lane] = (A.layer * HK * A.tpp + pw2) * A.tile_bytes;
        win->app[0][lane] = (int32_t)pw3;
        if ((int32_t)pw3 >= 0) prefetch_new_rows(A, (int32_t)pw3);
        __syncwarp();
    } else {
        // real units T of the batch and virtual units Tv (each non-empty
        // segment counts kVirtualUnits more)
        uint64_t T = 0;
        uint32_t seg_v = 0;  // virtual units of the longest segment
        for (uint32_t base = 0; base < A.num_seqs; base += 32) {
            const uint32_t i = base + lane;
            const uint32_t nt = i < A.num_seqs ? geo_of(A, i).ntiles : 0;
            const uint32_t sv = nt ? nt + kVirtualUnits + virtual_tail(A) : 0;
            uint32_t u = nt * HK, uv = sv * HK, mv = sv;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                u += __shfl_xor_sync(0xffffffffu, u, o);
                uv += __shfl_xor_sync(0xffffffffu, uv, o);
                mv = max(mv, __shfl_xor_sync(0xffffffffu, mv, o));
            }
            T += u;
            Tv += uv;
            seg_v = max(seg_v, mv);
        }
        uint64_t Wsmall = W;
        if (T != 0 && (T + kMinUnitsPerWarp - 1) / kMinUnitsPerWarp < Wsmall)
            Wsmall = (T + kMinUnitsPerWarp - 1) / kMinUnitsPerWarp;
        if (T != 0) {
            // at most kMergeGroup - 1 warp ranges start inside the longest segment
            const uint64_t W1 = (uint64_t)kOneLevelWarps * Tv / seg_v;
            if (W1 >= 1 && W1 < Wsmall && T <= W1 * kOneLevelTilesPerWarp) Wsmall = W1;
        }
        // a small batch: fewer, longer warp ranges (every split is a partial
        // to merge); the first W / 4 CTAs run (the others leave at once)
        if (Wsmall < W) W = Wsmall;
        // this warp's virtual range [v0, v1)
        const uint64_t v0 = muldiv_floor(wid, Tv, W), v1 = muldiv_floor(wid + 1, Tv, W);
        if (T != 0 && wid < W && v0 < v1) {
            // locate v0: its segment, and the warp's first real unit
            uint64_t acc = 0, accv = 0;
            for (uint32_t base = 0; base < A.num_seqs; base += 32) {
                const uint32_t i = base + lane;
                const uint32_t nt = i < A.num_seqs ? geo_of(A, i).ntiles : 0;
                const uint32_t u = nt * HK, uv = nt ? (nt + kVirtualUnits + virtual_tail(A)) * HK : 0;
                const uint32_t incl = warp_incl_scan(u), inclv = warp_incl_scan(uv);
                const uint32_t tot = __shfl_sync(0xffffffffu, incl, 31), totv = __shfl_sync(0xffffffffu, inclv, 31);
                if (v0 < accv + totv) {
                    const uint32_t ball = __ballot_sync(0xffffffffu, accv + inclv > v0);
                    const int L = __ffs(ball) - 1;
                    const uint32_t excl = __shfl_sync(0xffffffffu, incl - u, L);
                    const uint32_t exclv = __shfl_sync(0xffffffffu, inclv - uv, L);
                    cons.i = base + L;
                    cons.geo = geo_of(A, cons.i);
                    const uint32_t span = cons.geo.ntiles + kVirtualUnits + virtual_tail(A);
                    const uint32_t rem = (uint32_t)(v0 - (accv + exclv));  // < one sequence's virtual units
                    cons.h = rem / span;
                    const uint32_t off = rem - cons.h * span;
                    cons.tile = off < kVirtualUnits ? 0u : off - kVirtualUnits;
                    cons.seg_base = acc + excl + (uint64_t)cons.h * cons.geo.ntiles;
                    cons.vbase = accv + exclv + (uint64_t)cons.h * span;
                    if (cons.tile >= cons.geo.ntiles) {  // v0 is in the segment's tail: start at the next
                        cons.tile = 0;
                        walk_next_segment(A, cons);
                    }
                    break;
                }
                acc += tot;
                accv += totv;
            }
            // real units in [v0, v1): the range minus the virtual units around segments
            Walk t = cons;
            uint64_t pos = t.vbase + kVirtualUnits + t.tile;
            if (pos < v0) pos = v0;
            while (pos < v1) {
                const uint64_t seg_end = t.vbase + kVirtualUnits + t.geo.ntiles;
                n += (uint32_t)((v1 < seg_end ? v1 : seg_end) - pos);
                if (seg_end >= v1) break;
                walk_next_segment(A, t);
                if (t.i >= A.num_seqs) break;
                pos = t.vbase + kVirtualUnits;
            }
        }
        if (n) {
            fill_window(A, cons, 0, 0, n, win, 0);
            window_ready();
        }
        if (plan) {  // record the plan for the following launches of this step
            dep_wait();  // the previous kernel may still be reading this record
            if (lane == 0) {
                for (int i = 0; i < 8; i++) plan[i] = 0xFFFFFFFFu;  // key last
                plan[8] = cons.i; plan[9] = cons.h; plan[10] = cons.tile;
                plan[11] = (uint32_t)cons.seg_base; plan[12] = (uint32_t)(cons.seg_base >> 32);
                plan[13] = (uint32_t)cons.vbase; plan[14] = (uint32_t)(cons.vbase >> 32);
                plan[15] = (uint32_t)cons.geo.seq; plan[16] = (uint32_t)cons.geo.tok_lo;
                plan[17] = (uint32_t)cons.geo.tok_hi; plan[18] = cons.geo.tile0; plan[19] = cons.geo.ntiles;
                plan[20] = n;
                plan[21] = (uint32_t)Tv; plan[22] = (uint32_t)(Tv >> 32);
                plan[23] = (uint32_t)W; plan[24] = (uint32_t)(W >> 32);
                plan[25] = (uint32_t)wid; plan[26] = (uint32_t)(wid >> 32);
            }
            if (n) {
                plan[32 + lane] = (uint32_t)win->pg[0][lane];
                plan[64 + lane] = win->hv[0][lane];
                plan[96 + lane] = (uint32_t)win->app[0][lane];
            }
            __syncwarp();
            if (lane < 8) plan[lane] = key;
        }
        if (n == 0) {
            dep_wait();
            return;
        }
    }

    window_resolve(A, win, 0);
    const uint32_t npro = n < (uint32_t)S ? n : (uint32_t)S;
    for (uint32_t j = 0; j < npro; j++) {
        const int32_t seg = win->app[0][j];
        const uint8_t *src = window_src(A, win, 0, j);
        if (seg >= 0) fused_append<CODEC>(A.new_k, A.new_v, A.seq_ids, A.seq_lens, A.kv_heads, seg, src);
        if (lane == 0) {
            mbar_expect_tx(&bars[j], B);
            bulk_g2s(wsm + j * B, src, B, &bars[j]);
        }
    }

    typename OPS::Frag frag;
    typename OPS::State state;
    uint32_t st = 0, par = 0;
    // partials this warp wrote (at most two); the first is counted on its
    // segment a few tiles after it was written (its stores have landed by then,
    // so the release costs nothing), the last after the loop
    uint32_t pend_n = 0, pend_s0 = 0, pend_s1 = 0, pend_k0 = 0, tk0 = 0;
    uint32_t pend_ns0 = 0, pend_ns1 = 0;  // the pending segments' tile counts
    bool pend_cta = false;                // the (only) partial waits in shared memory for the CTA merge
    uint64_t xpend = 0;  // split-KV: segments this warp saw whole, to publish and merge after the loop
    bool counted0 = false;
    uint64_t pend_u0 = 0, pend_u1 = 0;

    for (uint32_t k = 0; k < n;) {
        if (cons.tile == 0 || k == 0) OPS::begin(frag, state, A, cons.i * HK + cons.h);
        // tiles this iteration: two consecutive tiles of one segment where the
        // codec steps pairs, else one
        const uint32_t nt = (OPS::kTilesPerStep == 2 && cons.tile + 1 < cons.geo.ntiles && k + 1 < n) ? 2u : 1u;
        if (pend_n && !counted0 && k >= pend_k0 + 4u) {
            __syncwarp();
            if (lane == 0) {
                const Parts P0 = parts_of(pend_u0, pend_ns0, Tv, W);
                tk0 = atom_add_acq_rel_gpu(part_counter(A, pend_s0, P0, part_index(P0, wid)), 1u);
            }
            counted0 = true;  // the ticket is read after the loop
        }
        if (cons.tile + 4u <= cons.geo.ntiles && cons.geo.ntiles < cons.tile + 4u + nt) {
            // the next segment's query rows (s_idx + 1 in batch order) into L1,
            // so that its begin() does not wait for them
            const size_t next = (size_t)(cons.i * HK + cons.h + 1) * A.group;
            if (next < (size_t)A.num_seqs * HK * A.group && (uint32_t)lane * 128u < A.group * kHeadDim * 4u)
                asm volatile("prefetch.global.L1 [%0];" ::"l"(A.query + next * kHeadDim + lane * 32));
        }
        uint32_t st1 = st + 1u, par1 = par;
        if (st1 == (uint32_t)S) { st1 = 0; par1 ^= 1u; }
        bool landed = mbar_wait_bounded(&bars[st], par);
        if (landed && nt == 2) landed = mbar_wait_bounded(&bars[st1], par1);
        if (!landed) {
            if (lane == 0) latch(A.status, QWN_KV_STATUS_WAIT_TIMEOUT);
            // wait (bounded) for the copies still in flight into this warp's stages
            uint32_t s2 = st, p2 = par;
            for (uint32_t d = k + 1; d < n && d < k + (uint32_t)S; ++d) {
                if (++s2 == (uint32_t)S) { s2 = 0; p2 ^= 1u; }
                mbar_wait_bounded(&bars[s2], p2);
            }
            dep_wait();
            return;
        }
        const int tile_tok0 = (int)(cons.geo.tile0 + cons.tile) * 16;
        if constexpr (OPS::kTilesPerStep == 2) {
            if (nt == 2) {
                const uint8_t *const tl[2] = {wsm + st * B, wsm + st1 * B};
                const int lo[2] = {max(cons.geo.tok_lo - tile_tok0, 0), max(cons.geo.tok_lo - tile_tok0 - 16, 0)};
                const int hi[2] = {min(cons.geo.tok_hi - tile_tok0, 16), min(cons.geo.tok_hi - tile_tok0 - 16, 16)};
                float ps[2][HG];
                OPS::template stepn<2>(tl, frag, state, lo, hi, ps);
                if (A.tile_mass) {
                    OPS::mass(A, cons.seg_base + cons.tile, state, ps[0]);
                    OPS::mass(A, cons.seg_base + cons.tile + 1, state, ps[1]);
                }
            }
        }
        if (nt == 1) {
            const int t_lo = max(cons.geo.tok_lo - tile_tok0, 0);
            const int t_hi = min(cons.geo.tok_hi - tile_tok0, 16);
            float psum[HG];
            OPS::step(wsm + st * B, frag, state, t_lo, t_hi, psum);
            if (A.tile_mass) OPS::mass(A, cons.seg_base + cons.tile, state, psum);
        }
        __syncwarp();

        // refill the consumed stages with units k + S (and k + 1 + S)
        for (uint32_t e = 0; e < nt; e++) {
            const uint32_t j = k + e + (uint32_t)S;
            if (j < n) {
                if (j - wbase == 16u && wbase + 32u < n)  // request the next window early
                    fill_window(A, cons, wbase + 32u - k, wbase + 32u, n, win, cw ^ 1);  // cons is at unit k
                if (j - wbase == 32u) {
                    wbase = j;
                    cw ^= 1;
                    window_ready();
                    window_resolve(A, win, cw);
                }
                const int32_t seg = win->app[cw][j - wbase];
                const uint8_t *src = window_src(A, win, cw, j - wbase);
                if (seg >= 0) fused_append<CODEC>(A.new_k, A.new_v, A.seq_ids, A.seq_lens, A.kv_heads, seg, src);
                // every shared-memory read of this stage fed a register that was
                // consumed before the __syncwarp above, so the copy cannot
                // overtake them
                if (lane == 0) {
                    mbar_expect_tx(&bars[st], B);
                    bulk_g2s(wsm + st * B, src, B, &bars[st]);
                }
            }
            if (++st == (uint32_t)S) { st = 0; par ^= 1u; }
        }

        // end of this warp's share of the segment?
        if (cons.tile + nt == cons.geo.ntiles || k + nt == n) {
            dep_wait();  // its slot (or output rows) may still be read by the previous kernel
            const uint32_t s_idx = cons.i * HK + cons.h;
            bool in_cta = false;
            const uint32_t np =
                finish_segment<OPS, XCHG>(A, state, s_idx, cons.vbase, cons.geo.ntiles, Tv, W, wid, wsm, in_cta);
            if (XCHG && np == 1) xpend |= 1ull << s_idx;
            else if (np) {
                const int e = pend_n++;  // at most two: the segment the range starts in and the one it ends in
                if (e == 0) {
                    pend_s0 = s_idx; pend_u0 = cons.vbase; pend_k0 = k; pend_ns0 = cons.geo.ntiles;
                    pend_cta = in_cta;  // an interior warp has this one partial only, at its last unit
                } else {
                    pend_s1 = s_idx; pend_u1 = cons.vbase; pend_ns1 = cons.geo.ntiles;
                }
            }
        }
        // next unit
        if (k + nt < n) {
            cons.tile += nt;
            if (cons.tile == cons.geo.ntiles) walk_next_segment(A, cons);
        }
        k += nt;
    }
    // the pipeline is drained: its stages hold the partials being merged,
    // completed on the next barrier in the ring
    __syncwarp();
    uint8_t *buf = wsm;  // where merges stage the slots they read
    uint32_t SB = (uint32_t)(S * B);
    // the CTA's part (all four warps inside one segment): the last of its
    // warps to get here combines the four shared-memory slots into the
    // CTA's slot and counts it; the others are done.  (No CTA barrier: a
    // warp that gave up on a wait never arrives, and the segment's result is
    // then marked invalid by the latched status.)
    uint64_t pw = wid;  // the warp whose slot holds this warp's first part
    if (pend_cta) {
        uint32_t t = 0;
        if (lane == 0) {
            __threadfence_block();
            t = atomicAdd(&cta_arrivals, 1u);
            __threadfence_block();
        }
        t = __shfl_sync(0xffffffffu, t, 0);
        if (t != kWarpsPerCta - 1) return;
        __syncwarp();
        pw = wid - wid % kWarpsPerCta;
        float *cslot = A.partials + (size_t)(pw + pend_s0) * kPartialFloats;
        const uint32_t stride = (uint32_t)(S * B);
        merge_cta_slots(A, smem, stride, cslot);
        // every warp of the CTA is done: its whole stage memory serves the merges
        buf = smem;
        SB = (uint32_t)(kWarpsPerCta * S * B);
        __syncwarp();
    }
    // count this warp's partials on their segments: the warp barrier orders
    // the lanes' slot stores before lane 0's release, the acquire orders the
    // last arriver's reads of the other slots
    const Parts P0 = parts_of(pend_u0, pend_ns0, Tv, W), P1 = parts_of(pend_u1, pend_ns1, Tv, W);
    const uint32_t idx0 = pend_n > 0 ? part_index(P0, pw) : 0u, idx1 = pend_n > 1 ? part_index(P1, wid) : 0u;
    uint32_t tk1 = 0;
    if (lane == 0) {
        if (pend_n > 0 && !counted0) tk0 = atom_add_acq_rel_gpu(part_counter(A, pend_s0, P0, idx0), 1u);
        if (pend_n > 1) tk1 = atom_add_acq_rel_gpu(part_counter(A, pend_s1, P1, idx1), 1u);
    }
    tk0 = __shfl_sync(0xffffffffu, tk0, 0);
    tk1 = __shfl_sync(0xffffffffu, tk1, 0);
    if constexpr (XCHG) {
        while (xpend) {
            const uint32_t s = (uint32_t)(__ffsll((long long)xpend) - 1);
            xpend &= xpend - 1;
            publish_slot(A, s, A.partials + (size_t)(wid + s) * kPartialFloats);
            exchange_merge(A, s, (size_t)s * A.group);
        }
    }
    for (uint32_t e = 0; e < pend_n; e++) {
        const Parts &P = e ? P1 : P0;
        const uint32_t np = P.n, s_idx = e ? pend_s1 : pend_s0, idx = e ? idx1 : idx0;
        const uint32_t tk = e ? tk1 : tk0;
        // the merge the last arrival runs: the whole segment (one level), or
        // this part's group of kMergeGroup consecutive parts, whose result
        // goes to the group's first slot and counts on the segment; the last
        // group then merges the groups (one call site keeps the code short)
        uint32_t mfirst = 0, mstride = 1, mn = np;
        float *mdst = nullptr;
        uint32_t *mctr = &A.counters[s_idx];
        if (np > kMergeGroup) {
            mfirst = (idx / kMergeGroup) * kMergeGroup;
            mn = min(kMergeGroup, np - mfirst);
            const uint64_t gw = part_warp(P, mfirst);
            mdst = A.partials + (size_t)(gw + s_idx) * kPartialFloats;
            mctr = &A.gcounters[gw + s_idx];
        }
        if (tk != mn - 1) continue;  // not the last arrival
        for (;;) {
            if (!merge_parts<HG, XCHG>(A, s_idx, P, mfirst, mstride, mn, mdst, buf, SB, (uint32_t)(S * B),
                                       &bars[st], par))
                return;
            if (lane == 0) *mctr = 0u;  // ready for the next launch
            if (!mdst) break;
            __syncwarp();
            uint32_t t2 = 0;
            if (lane == 0) t2 = atom_add_acq_rel_gpu(&A.counters[s_idx], 1u);
            t2 = __shfl_sync(0xffffffffu, t2, 0);
            const uint32_t ngroups = (np + kMergeGroup - 1) / kMergeGroup;
            if (t2 != ngroups - 1) break;
            mfirst = 0;
            mstride = kMergeGroup;
            mn = ngroups;
            mdst = nullptr;
            mctr = &A.counters[s_idx];
        }
    }
}

// merge of partial states produced on several devices (base-2 domain); part
// p's (m, l) of a row sit at p*stride_ml + row, its o row at p*stride_o +
// row*128
__global__ void merge_kernel(uint32_t parts, uint32_t rows, const float *m, const float *l, const float *o,
                             float *out, size_t stride_ml, size_t stride_o) {
    const uint32_t row = blockIdx.x;
    const uint32_t d = threadIdx.x;
    if (row >= rows || d >= kHeadDim) return;
    float ms = -INFINITY;
    for (uint32_t p = 0; p < parts; p++) ms = fmaxf(ms, m[p * stride_ml + row]);
    float ls = 0.f, acc = 0.f;
    for (uint32_t p = 0; p < parts; p++) {
        const float mp = m[p * stride_ml + row];
        const float w = mp == -INFINITY ? 0.f : ex2(mp - ms);
        ls += l[p * stride_ml + row] * w;
        acc += o[p * stride_o + (size_t)row * kHeadDim + d] * w;
    }
    out[(size_t)row * kHeadDim + d] = ls > 0.f ? acc / ls : 0.f;
}

template <int CODEC, int HG>
constexpr size_t codec_smem() {
    using O = Ops<CODEC, HG>;
    return (size_t)kWarpsPerCta * O::kStages * (O::kBytes + 8) + (size_t)kWarpsPerCta * sizeof(WarpWindow);
}

// kernel variants: one or two head groups of four query heads
template <int CODEC>
cudaError_t configure_codec() {
    cudaError_t e = cudaFuncSetAttribute(attn_kernel<CODEC, 1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)codec_smem<CODEC, 1>());
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_kernel<CODEC, 2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)codec_smem<CODEC, 2>());
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_kernel<CODEC, 1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)codec_smem<CODEC, 1>());
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_kernel<CODEC, 2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)codec_smem<CODEC, 2>());
    return e;
}
// ctas[hg-1]: the resident grid of each variant.  Launched as a
// programmatic dependent: its CTAs may start on SMs the previous kernel of
// the stream has left while that kernel finishes, and wait (griddepcontrol)
// for it to complete before touching global memory.
template <int CODEC>
cudaError_t launch_variant(const uint32_t (&ctas)[2], const AttnArgs &A, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.blockDim = dim3(kWarpsPerCta * 32);
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // split-KV over ranks (the exchange) is its own instantiation, so the
    // decode kernels carry none of its code
    const bool x = A.xworld != 0;
    if (A.group > 4) {
        cfg.gridDim = dim3(ctas[1]);
        cfg.dynamicSmemBytes = codec_smem<CODEC, 2>();
        return x ? cudaLaunchKernelEx(&cfg, attn_kernel<CODEC, 2, true>, A)
                 : cudaLaunchKernelEx(&cfg, attn_kernel<CODEC, 2, false>, A);
    }
    cfg.gridDim = dim3(ctas[0]);
    cfg.dynamicSmemBytes = codec_smem<CODEC, 1>();
    return x ? cudaLaunchKernelEx(&cfg, attn_kernel<CODEC, 1, true>, A)
             : cudaLaunchKernelEx(&cfg, attn_kernel<CODEC, 1, false>, A);
}

template <int CODEC>
cudaError_t launch_codec(Pool *p, const AttnArgs &A, cudaStream_t s) {
    static bool configured[64] = {false};
    if (!configured[p->device & 63]) {
        const cudaError_t e = configure_codec<CODEC>();
        if (e != cudaSuccess) return e;
        configured[p->device & 63] = true;
    }
    const uint32_t ctas[2] = {p->attn_ctas, p->attn_ctas2};
    const cudaError_t e = launch_variant<CODEC>(ctas, A, s);
    count_launch();
    return e;
}

}  // namespace

size_t attention_smem_bytes(uint32_t codec, int hg) {
    switch (codec) {
        case QWN_KV_CODEC_Q8_HEAD_F16:
            return hg == 1 ? codec_smem<QWN_KV_CODEC_Q8_HEAD_F16, 1>() : codec_smem<QWN_KV_CODEC_Q8_HEAD_F16, 2>();
        case QWN_KV_CODEC_Q8_B64_F32:
            return hg == 1 ? codec_smem<QWN_KV_CODEC_Q8_B64_F32, 1>() : codec_smem<QWN_KV_CODEC_Q8_B64_F32, 2>();
        case QWN_KV_CODEC_Q4_G32:
            return hg == 1 ? codec_smem<QWN_KV_CODEC_Q4_G32, 1>() : codec_smem<QWN_KV_CODEC_Q4_G32, 2>();
        case QWN_KV_CODEC_F16:
            return hg == 1 ? codec_smem<QWN_KV_CODEC_F16, 1>() : codec_smem<QWN_KV_CODEC_F16, 2>();
        case QWN_KV_CODEC_TQ35_G64:
            return hg == 1 ? codec_smem<QWN_KV_CODEC_TQ35_G64, 1>() : codec_smem<QWN_KV_CODEC_TQ35_G64, 2>();
        default: return 0;
    }
}

const void *attention_kernel_ptr(uint32_t codec, int hg) {
    switch (codec) {
        case QWN_KV_CODEC_Q8_HEAD_F16:
            return hg == 1 ? (const void *)attn_kernel<QWN_KV_CODEC_Q8_HEAD_F16, 1, false>
                           : (const void *)attn_kernel<QWN_KV_CODEC_Q8_HEAD_F16, 2, false>;
        case QWN_KV_CODEC_Q8_B64_F32:
            return hg == 1 ? (const void *)attn_kernel<QWN_KV_CODEC_Q8_B64_F32, 1, false>
                           : (const void *)attn_kernel<QWN_KV_CODEC_Q8_B64_F32, 2, false>;
        case QWN_KV_CODEC_Q4_G32:
            return hg == 1 ? (const void *)attn_kernel<QWN_KV_CODEC_Q4_G32, 1, false>
                           : (const void *)attn_kernel<QWN_KV_CODEC_Q4_G32, 2, false>;
        case QWN_KV_CODEC_F16:
            return hg == 1 ? (const void *)attn_kernel<QWN_KV_CODEC_F16, 1, false>
                           : (const void *)attn_kernel<QWN_KV_CODEC_F16, 2, false>;
        case QWN_KV_CODEC_TQ35_G64:
            return hg == 1 ? (const void *)attn_kernel<QWN_KV_CODEC_TQ35_G64, 1, false>
                           : (const void *)attn_kernel<QWN_KV_CODEC_TQ35_G64, 2, false>;
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
    A.gcounters = p->counters + p->max_segments;
    // plans are keyed by the pool's epoch, not by the contents of a caller's
    // sequence-id array: cache them only for the identity batch
    A.plans = a.seq_ids ? nullptr : p->plans;
    A.tile_mass = a.page_mass ? p->tile_mass : nullptr;
    A.seg_ml = a.page_mass ? p->seg_ml : nullptr;
    A.part_m = a.part_m;
    A.part_l = a.part_l;
    A.part_o = a.part_o;
    A.new_k = a.new_k;
    A.new_v = a.new_v;
    A.status = p->status;
    // Early start.  Every other kernel of this library is an ordinary launch
    // (the next launch waits for it to finish) -- except seq_append_kernel,
    // which lets the next launch start at once and therefore clears
    // last_attn, so that the launch after it is never early -- so this
    // attention kernel can overlap only an attention kernel of the stream that
    // precedes it directly.  That kernel writes its layer's newest-token tiles, its output
    // rows, the pool's partial slots, counters and plans.  When the previous
    // attention launch of this pool on this stream was of another layer,
    // recorded no plans (the records this launch reads early), exported no
    // page mass or partials, and its output rows do not overlap
    // this launch's query, new K/V or output, this launch reads nothing it
    // writes before the kernel's dependency wait, which then sits before the
    // first write of slots, counters, plans or outputs.  (An operation queued
    // in between only delays the start, so the check stays sound.)
    {
        const size_t qbytes = (size_t)a.num_seqs * a.query_heads * kHeadDim * sizeof(float);
        const size_t kvbytes = (size_t)a.num_seqs * p->kv_heads * kHeadDim * sizeof(float);
        const uintptr_t q0 = (uintptr_t)a.query, o0 = (uintptr_t)a.output;
        const uintptr_t k0 = (uintptr_t)a.new_k, v0 = (uintptr_t)a.new_v;
        const bool eligible = !a.part_o && !a.peers && !a.page_mass && a.output;
        std::lock_guard<std::mutex> lk(p->last_mu);
        // does this launch record plans?  The kernel records on a key miss; the
        // host mirrors the key (the epoch part through plan_valid, which every
        // kernel that changes lengths or tables clears)
        const uint32_t pkey[6] = {a.num_seqs, a.attend_limit, a.t_begin, a.t_end, a.new_k ? 1u : 0u,
                                  A.group > 4 ? 2u : 1u};
        bool records = false;
        if (A.plans) {
            records = !p->plan_valid || std::memcmp(pkey, p->plan_key, sizeof(pkey)) != 0;
            p->plan_valid = true;
            std::memcpy(p->plan_key, pkey, sizeof(pkey));
        }
        const Pool::LastAttention &L = p->last_attn;
        auto clear = [&](uintptr_t lo, size_t n) { return lo + n <= L.out_lo || lo >= L.out_hi; };
        A.early = eligible && L.valid && !L.recorded && L.stream == s && L.layer != a.layer && clear(q0, qbytes) &&
                  clear(o0, qbytes) && (!a.new_k || (clear(k0, kvbytes) && clear(v0, kvbytes)));
        p->last_attn.valid = eligible;
        p->last_attn.recorded = records;
        p->last_attn.stream = s;
        p->last_attn.layer = a.layer;
        p->last_attn.out_lo = o0;
        p->last_attn.out_hi = o0 + qbytes;
    }
    if (a.peers) {
        for (uint32_t r = 0; r < a.peers->world; r++) A.xbuf[r] = static_cast<uint8_t *>(a.peers->buffers[r]);
        A.xrank = a.peers->rank;
        A.xworld = a.peers->world;
        A.xrows = a.peers->max_rows;
        A.xepoch = a.epoch;
        A.xtimeout_ns = a.peers->timeout_ns ? a.peers->timeout_ns : 2000000000ull;
    }
    switch (p->codec) {
        case QWN_KV_CODEC_Q8_HEAD_F16: return launch_codec<QWN_KV_CODEC_Q8_HEAD_F16>(p, A, s);
        case QWN_KV_CODEC_Q8_B64_F32: return launch_codec<QWN_KV_CODEC_Q8_B64_F32>(p, A, s);
        case QWN_KV_CODEC_Q4_G32: return launch_codec<QWN_KV_CODEC_Q4_G32>(p, A, s);
        case QWN_KV_CODEC_F16: return launch_codec<QWN_KV_CODEC_F16>(p, A, s);
        case QWN_KV_CODEC_TQ35_G64: return launch_codec<QWN_KV_CODEC_TQ35_G64>(p, A, s);
        default: return cudaErrorNotSupported;
    }
}

cudaError_t launch_merge(uint32_t parts, uint32_t rows, const float *m, const float *l,
                         const float *o, float *out, size_t stride_ml, size_t stride_o, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    merge_kernel<<<rows, kHeadDim, 0, s>>>(parts, rows, m, l, o, out, stride_ml, stride_o);
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
constexpr size_t kStaticFloats = (size_t)kStaticSlots * kPartialFloats + kStaticSegments + kStaticSlots;
static __device__ __align__(256) float g_static_scratch[kStaticFloats];
constexpr int kStaticMaxDevices = 64;
std::mutex g_static_mu;
float *g_static_addr[kStaticMaxDevices] = {};
uint32_t g_static_ctas[kStaticMaxDevices][6][2] = {};

template <int CODEC>
cudaError_t static_setup(int dev) {
    cudaError_t e = configure_codec<CODEC>();
    if (e != cudaSuccess) return e;
    int sms = 0;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    for (int hg = 1; hg <= 2; hg++) {
        int per_sm = 0;
        if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attention_kernel_ptr(CODEC, hg),
                                                               kWarpsPerCta * 32, attention_smem_bytes(CODEC, hg))) !=
            cudaSuccess)
            return e;
        g_static_ctas[dev][CODEC][hg - 1] = (uint32_t)(sms * (per_sm > 0 ? per_sm : 1));
    }
    return cudaSuccess;
}
}  // namespace
}  // namespace qkv

extern "C" QWN_CUDA_ABI_API int qwn_kv_attention_static(const QwnKvStaticAttentionRequest *r) {
    using namespace qkv;
    if (!r || !header_ok(r->header, sizeof(*r))) return QWN_CUDA_STATUS_ABI_MISMATCH;
    const size_t tb = tile_bytes_of(r->codec);
    if (!tb || r->head_dim != (uint32_t)kHeadDim || r->kv_heads == 0 ||
        r->page_tokens == 0 || r->page_tokens % 16 || r->layer >= r->layers || r->query_heads == 0 ||
        r->query_heads % r->kv_heads || r->query_heads / r->kv_heads > (uint32_t)kMaxGroup || !r->pages_dev ||
        !r->page_table_dev || !r->seq_lens_dev || !r->query_dev || !r->output_dev || r->total_pages == 0 ||
        r->max_seqs == 0 || r->max_pages_per_seq == 0 || r->num_seqs > r->max_seqs) {
        set_error("qwn_kv_attention_static: invalid request");
        return QWN_CUDA_STATUS_INVALID_ARGUMENT;
    }
    // the tiles arrive by 1-D bulk copies (16-byte source and size), the query
    // rows by 16-byte loads and the output by 16-byte stores; the int32
    // arrays are read 4 bytes at a time
    auto misaligned = [](const void *ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) != 0; };
    if (misaligned(r->pages_dev, 16) || misaligned(r->query_dev, 16) || misaligned(r->output_dev, 16) ||
        misaligned(r->page_table_dev, 4) || misaligned(r->seq_lens_dev, 4) || misaligned(r->seq_ids_dev, 4) ||
        misaligned(r->status_dev, 4) || tb % 16) {
        set_error("qwn_kv_attention_static: pages, query and output must be 16-byte aligned, the int32 arrays 4-byte");
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
                (e = static_setup<QWN_KV_CODEC_Q4_G32>(dev)) != cudaSuccess ||
                (e = static_setup<QWN_KV_CODEC_TQ35_G64>(dev)) != cudaSuccess ||
                (e = static_setup<QWN_KV_CODEC_F16>(dev)) != cudaSuccess) {
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
    // the merge counters (per segment, then per merge group) must start at
    // zero; the slots are written before they are read
    e = cudaMemsetAsync(counters, 0, sizeof(uint32_t) * (kStaticSegments + kStaticSlots), s);
    if (e != cudaSuccess) { set_cuda_error("qwn_kv_attention_static: clear", e); return QWN_CUDA_STATUS_RUNTIME_ERROR; }
    const uint32_t segs = r->num_seqs * r->kv_heads;
    const uint32_t max_ctas = (kStaticSlots - segs) / kWarpsPerCta;  // warps + segments <= slots
    uint32_t ctas[2] = {g_static_ctas[dev][r->codec][0], g_static_ctas[dev][r->codec][1]};
    for (uint32_t &c : ctas)
        if (c > max_ctas) c = max_ctas;
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
    A.gcounters = counters + kStaticSegments;
    A.status = r->status_dev;
    switch (r->codec) {
        case QWN_KV_CODEC_Q8_HEAD_F16: e = launch_variant<QWN_KV_CODEC_Q8_HEAD_F16>(ctas, A, s); break;
        case QWN_KV_CODEC_Q8_B64_F32: e = launch_variant<QWN_KV_CODEC_Q8_B64_F32>(ctas, A, s); break;
        case QWN_KV_CODEC_Q4_G32: e = launch_variant<QWN_KV_CODEC_Q4_G32>(ctas, A, s); break;
        case QWN_KV_CODEC_F16: e = launch_variant<QWN_KV_CODEC_F16>(ctas, A, s); break;
        case QWN_KV_CODEC_TQ35_G64: e = launch_variant<QWN_KV_CODEC_TQ35_G64>(ctas, A, s); break;
        default:
            set_error("qwn_kv_attention_static: unsupported codec");
            return QWN_CUDA_STATUS_UNSUPPORTED;
    }
    count_launch();
    if (e != cudaSuccess) {
        set_cuda_error("qwn_kv_attention_static: launch", e);
        return QWN_CUDA_STATUS_RUNTIME_ERROR;
    }
    return QWN_CUDA_STATUS_OK;
}
