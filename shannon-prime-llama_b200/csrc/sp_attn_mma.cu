// sp_attn_mma.cu — tensor-core fused decode attention for the ship layout
// (head_dim 128, K bands 32/32/32/32 at 5/5/4/3 bits, V one 3-bit band,
// up to 4 query heads per KV head).
//
// The attention is taken in the VHT2 coefficient domain, as in the generic
// kernel (sp_attn.cu): score_t = sum_i q'[i] * c_t[i] with q' the
// transformed, Möbius-permuted query, and the V sum accumulated on the
// dequantised coefficients, transformed once per head at the end.
//
// Why tensor cores here: at 70% of HBM bandwidth a B200 SM receives one
// 126-byte K+V row every ~7 clocks, i.e. ~28 warp-instruction issue slots
// per row across its four schedulers.  A SIMT unpack + FMA loop needs
// ~110 warp instructions per row (4 GQA FMAs per K element, 4 per V
// element), so the decode would be issue-bound at ~25% of HBM.  Both
// contractions are instead done with mma.sync.m16n8k16 (fp16 in, fp32
// accumulate) straight from registers:
//
//   K side:  S[16 tokens][8] = codes_K[16 tokens][16 slots] x Bq[16][8]
//            per band (two k-steps of 16 slots per 32-code band);
//   V side:  O[16 coeffs][8] += codes_V[16 coeffs][16 tokens] x P[16][8]
//
// with the 8 columns = 4 query heads x {hi, lo} fp16 halves of an fp32
// operand (q' for K, p*scale_v for V), so both operands carry ~22 bits.
//
// Unpacking without conversion instructions: a packed code u masked into
// bits d..d+b-1 of a 16-bit half is the fp16 subnormal u * 2^(d-24),
// exact, and the tensor cores take fp16 subnormals exactly.  So an
// A-fragment register (two fp16) is one shift/funnel-shift plus one AND of
// the packed row, with the 2^d of each slot folded into the B operand
// (K side) or into the per-coefficient epilogue (V side).  Code pairs in
// one register are chosen so both land in mantissa bits:
//   K band of b bits, lane c owns codes 8c..8c+7, registers pair code j
//   with code j+4 (same token); V registers pair one coefficient of two
//   consecutive tokens (16-bit windows of both rows interleaved with prmt).
//
// Tiles of 16 tokens (K 1216 B, V 800 B, both multiples of 16 B and
// 16-B aligned) are staged per warp by cp.async.bulk (the TMA engine)
// into a 4-deep ring completed on mbarriers; every wait is bounded.
//
// Work split: the flattened (layer, KV head, tile) space is cut into equal
// contiguous ranges, one per CTA (a single wave on the 148 SMs), so load
// balance is exact to a tile; a CTA writes one partial per (layer, KV head)
// segment it touches, and a combine kernel merges the segments.
#include "sp_attn.cuh"
#include "sp_bulk.cuh"

#include <atomic>
#include <math.h>
#include <stdlib.h>
#include <string.h>


namespace {

constexpr int kKTile = 16 * 76;       // 1216: one 16-position MMA tile of K rows
constexpr int kVTile = 16 * 50;       // 800
// MMA tiles per ring stage (16 x this many positions per bulk-copied
// stage): 3 for up to 4 query heads per KV head, 4 for 5..8 (measured best
// for each; the stage work is paid once per stage).
__host__ __device__ constexpr int stage_sub(int gt) { return gt == 8 ? 4 : 3; }
constexpr int kN = 128;
constexpr float kEmptyMax = -1.0e30f; // running max before the first valid token
constexpr int kFlushTiles = 16;       // tiles between V-accumulator recentrings

// Fixed ship layout (checked on the host against the cache's band config).
// Bit position of band b's first code within a K row.
__host__ __device__ constexpr int kKBit(int b) { return b == 0 ? 16 : b == 1 ? 192 : b == 2 ? 368 : 512; }
__host__ __device__ constexpr int kKBits(int b) { return b < 2 ? 5 : (b == 2 ? 4 : 3); }
// fp16 scale of band b: 32-bit word of the row holding it (low half for
// bands 0 and 2, high half for bands 1 and 3).
__host__ __device__ constexpr int kKScaleWord(int b) { return b == 0 ? 0 : b == 1 ? 5 : b == 2 ? 11 : 15; }

// Pre-shift d (the code's value is u * 2^(d-24)) of the low / high code of
// pair p of band b, as produced by the unpack sequence of k_attn_ship_mma.
__host__ __device__ constexpr int pair_dlo(int b, int p)
{
    return b < 2 ? 0 : (b == 2 ? ((p & 1) ? 4 : 0) : ((p & 1) ? 7 : 4));
}
__host__ __device__ constexpr int pair_dhi(int b, int p)
{
    return b < 2 ? 4 : (b == 2 ? ((p & 1) ? 4 : 0) : ((p & 1) ? 3 : 0));
}
// Pre-shift of V code j of a lane's 16-code chunk (windows of 5 codes at
// bits 0,3,6,9,12: the first two taken after a left shift by 4 (d 4, 7), the
// third in place (d 6), the last two after a right shift by 5 (d 4, 7);
// code 15 at d 4).  The tensor cores' products lose precision on the
// smallest subnormals (codes below bit 4 of a half: up to 2e-6 of an MMA's
// magnitude at d = 0, a systematic error), so no code sits there.
__host__ __device__ constexpr int vcode_d(int j)
{
    return j == 15 ? 4 : ((j % 5) == 2 ? 6 : ((j % 5) == 0 || (j % 5) == 3) ? 4 : 7);
}

using Sched = SpSched;

__host__ __device__ inline long long tile_begin(long long i, const Sched &s) { return sp_tile_begin(i, s); }
__host__ __device__ inline int cta_of_tile(long long g, const Sched &s) { return sp_cta_of_tile(g, s); }

// ------------------------------------------------------------------ PTX --

using spb::smem_u32;
using spb::mbar_init;
using spb::mbar_expect_tx;
using spb::bulk_g2s;
using spb::evict_first_policy;
using spb::wait_stage;

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1)
{
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The same with the accumulator input taken from separate registers (the
// first MMA of a band starts from its constant offset without copies).
__device__ __forceinline__ void mma16816_c(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1, float c0, float c1, float c2, float c3)
{
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c0), "f"(c1), "f"(c2), "f"(c3));
}

// 2^x on the XU pipe (one MUFU op; rel. error ~2^-22, flushes subnormal
// results, which are far below the softmax's resolution).
__device__ __forceinline__ float fast_exp2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t shf(uint32_t lo, uint32_t hi, uint32_t s)
{
    return __funnelshift_r(lo, hi, s);
}

// fp16 bits of x (round to nearest even) and of the residual x - fp16(x):
// the hi/lo split of an fp32 operand.
__device__ __forceinline__ uint32_t split_hi_lo(float x)
{
    __half h = __float2half_rn(x);
    __half l = __float2half_rn(x - __half2float(h));
    return (uint32_t)__half_as_ushort(h) | ((uint32_t)__half_as_ushort(l) << 16);
}

// x * 2^e by one multiply (e inside the normal exponent range, where that is
// exactly ldexpf), else ldexpf.
__device__ __forceinline__ float scale2(float x, int e)
{
    return (e >= -126 && e <= 127) ? x * __int_as_float((e + 127) << 23) : ldexpf(x, e);
}
// ilogbf of a normal, positive float.
__device__ __forceinline__ int ilogb_normal(float x) { return ((__float_as_int(x) >> 23) & 0xff) - 127; }

// Zero the non-finite halves of a half2 (the reference zeroes a band whose
// stored scale is not finite, shannon_prime_cuda.cu:236-245).
__device__ __forceinline__ __half2 finite_or_zero(__half2 h)
{
    const unsigned m = __hle2_mask(__habs2(h), __float2half2_rn(65504.0f));
    const unsigned v = *reinterpret_cast<unsigned *>(&h) & m;
    return *reinterpret_cast<const __half2 *>(&v);
}

template <int kWarps, int kStages, int GT>
struct Smem {
    static constexpr int kSub = stage_sub(GT);
    static constexpr int kStageBytes = kSub * (kKTile + kVTile);
    unsigned char ring[kWarps][kStages][kStageBytes];
    unsigned char pad[16];
    unsigned long long bar[kWarps][kStages];
    float q[GT][kN];         // transformed, permuted, scaled queries
    float qt[GT][kN];        // scratch for the permutation
    float qsum[GT][4];       // per query, per band: sum of q'
    float qmax[GT];
    float merge[kWarps][GT][4 + kN];
    float scl[kWarps][kStages][16 * kSub][8];   // per stage position: K band scales 0..3, V scale (fp32)
};

// kWarps warps per CTA, a kStages-deep copy ring per warp, kMinBlocks CTAs
// per SM requested from the register allocator.
// GT query heads per KV head (4 or 8): NT = GT / 4 column tiles of the MMAs,
// each 4 queries x {hi, lo}.
// Segment merge of one (layer, q head) row.
__device__ __forceinline__ void combine_row(const SpAttnArgs &a, const Sched &sc, int li, int qh, int lane)
{
    const long long u = (long long)li * a.n_kv_heads + qh / a.group;
    const int i0 = cta_of_tile(u * sc.tiles_per_unit, sc);
    const int i1 = cta_of_tile((u + 1) * sc.tiles_per_unit - 1, sc);
    const int nseg = i1 - i0 + 1;
    // Lane s owns segments s, s + 32, s + 64, s + 96 (at most kAttnMaxSplits
    // = 128): their maxima and sums arrive in one round of loads, the
    // weights stay in the owning lanes, and the accumulator rows are loaded
    // 16 segments at a time, all in flight together, so a row costs about
    // 1 + nseg / 16 L2 round trips.
    static_assert(kAttnMaxSplits <= 128, "four segments per lane");
    float mv[4], lv[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int sg = lane + 32 * j;
        mv[j] = kEmptyMax;
        lv[j] = 0.0f;
        if (sg < nseg) {
            const float2 ml = __ldcg(reinterpret_cast<const float2 *>(sp_attn_partial(a, li, qh, sg)));
            mv[j] = ml.x;
            lv[j] = ml.y;
        }
    }
    float M = fmaxf(fmaxf(mv[0], mv[1]), fmaxf(mv[2], mv[3]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float wv[4], L = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        wv[j] = lane + 32 * j < nseg ? exp2f(mv[j] - M) : 0.0f;
        L += wv[j] * lv[j];
    }
    float x[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int c0 = 0; c0 < nseg; c0 += 16) {
        const int jw = c0 >> 5;                         // weights of this chunk live in wv[jw]
        const float wsrc = jw == 0 ? wv[0] : jw == 1 ? wv[1] : jw == 2 ? wv[2] : wv[3];
        float4 v[16];
#pragma unroll
        for (int t = 0; t < 16; t++)
            v[t] = c0 + t < nseg
                       ? __ldcg(reinterpret_cast<const float4 *>(sp_attn_partial(a, li, qh, c0 + t) + 4 + lane * 4))
                       : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int t = 0; t < 16; t++) {
            const float wt = __shfl_sync(0xffffffffu, wsrc, (c0 + t) & 31);
            x[0] += wt * v[t].x; x[1] += wt * v[t].y; x[2] += wt * v[t].z; x[3] += wt * v[t].w;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
    sp_warp_wht<4>(x, lane);
    __half h[4];
#pragma unroll
    for (int e = 0; e < 4; e++) h[e] = __float2half_rn(x[e] * a.inv_sqrt_n * inv);
    sp_attn_store_row<4>(a, li, qh, lane, h);
}

// NBK: K bands read (4, or fewer for a partial-band read, which then skips
// the unpack and the MMAs of the bands it leaves out).
template <int kWarps, int kStages, int kMinBlocks, int GT, int NBK>
__global__ void __launch_bounds__(kWarps * 32, kMinBlocks)
k_attn_ship_mma(SpAttnArgs a, Sched sc)
{
    static_assert(GT == 4 || GT == 8, "4 or 8 query heads per KV head");
    constexpr int kSub = stage_sub(GT);
    constexpr int kKStage = kSub * kKTile;
    constexpr int kStageBytes = kSub * (kKTile + kVTile);
    // Launched as a programmatic dependent of the stream's previous kernel.
    // The only kernel of this library that lets its dependents start early
    // is the previous decode call's combine, which writes no cache byte; so
    // the ring's first copies of the (unchanged) compressed cache and the
    // Möbius order are fetched before the wait, and the queries, the
    // partials and everything else only after it.  The combine of this call
    // may then launch and wait on this grid.
    sp_pdl_trigger();
    constexpr int NT = GT / 4;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    Smem<kWarps, kStages, GT> &sm = *reinterpret_cast<Smem<kWarps, kStages, GT> *>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = lane >> 2, c = lane & 3;
    const int cta = blockIdx.x;
    const long long g_begin = tile_begin(cta, sc), g_end = tile_begin(cta + 1, sc);
    const int n_t = sc.tiles_per_unit;
    const int G = a.group;
    const int H = a.n_kv_heads;

    // ---- per-warp ring --------------------------------------------------
    const long long my_first = g_begin + warp;
    const int n_my = my_first < g_end ? (int)((g_end - my_first + kWarps - 1) / kWarps) : 0;
    const uint32_t bar0 = smem_u32(&sm.bar[warp][0]);
    const uint32_t ring0 = smem_u32(&sm.ring[warp][0][0]);
    uint64_t policy = 0;
    if (lane == 0) {
        for (int s = 0; s < kStages; s++) mbar_init(bar0 + 8 * s, 1);
        spb::mbar_init_fence();
        policy = evict_first_policy();
    }
    __syncwarp();

    // Issue cursor (lane 0): (layer index, KV head, tile) of the next of my
    // tiles to fetch and its K / V source addresses, advanced by kWarps
    // tiles per issue.
    int ic_tile = 0, ic_h = 0, ic_li = 0;
    const uint8_t *ic_k = nullptr, *ic_v = nullptr;
    auto ic_point = [&]() {
        const long long slot = (long long)(a.layer0 + ic_li) * H + ic_h;
        ic_k = a.k_cache + slot * a.k_slot_stride + (long long)ic_tile * kKStage;
        ic_v = a.v_cache + slot * a.v_slot_stride + (long long)ic_tile * (kSub * kVTile);
    };
    if (lane == 0 && n_my > 0) {
        const long long u0 = my_first / n_t;
        ic_tile = (int)(my_first - u0 * n_t);
        ic_h = (int)(u0 % H);
        ic_li = (int)(u0 / H);
        ic_point();
    }
    auto issue = [&](int k) {
        const int st = k % kStages;
        const uint32_t bar = bar0 + 8 * st;
        const uint32_t dst = ring0 + st * kStageBytes;
        // the stage's 16-position tiles that start before kv_len (whole
        // 16-row tiles lie inside the slot; the rows past kv_len are masked)
        const int rem = a.kv_len - ic_tile * 16 * kSub;
        const int nsub = rem >= 16 * kSub ? kSub : (rem + 15) / 16;
        spb::fence_proxy_async();
        mbar_expect_tx(bar, (uint32_t)nsub * (kKTile + kVTile));
        bulk_g2s(dst, ic_k, (uint32_t)nsub * kKTile, bar, policy);
        bulk_g2s(dst + kKStage, ic_v, (uint32_t)nsub * kVTile, bar, policy);
        ic_tile += kWarps;
        if (ic_tile < n_t) {
            ic_k += kWarps * kKStage;
            ic_v += kWarps * (kSub * kVTile);
        } else {
            while (ic_tile >= n_t) {
                ic_tile -= n_t;
                if (++ic_h == H) { ic_h = 0; ++ic_li; }
            }
            ic_point();
        }
    };
    if (lane == 0)
        for (int k = 0; k < kStages && k < n_my; k++) issue(k);
    int ord[4];                         // Möbius order entries of this lane's four coefficients
#pragma unroll
    for (int e = 0; e < 4; e++) ord[e] = a.order ? __ldg(a.order + lane * 4 + e) : lane * 4 + e;
    sp_pdl_wait();

    // ---- lane constants ---------------------------------------------------
    // K: window word and shift of lane c's chunk in each band.
    int kw[4], ks[4];
#pragma unroll
    for (int b = 0; b < 4; b++) {
        const int bit = kKBit(b) + 8 * c * kKBits(b);
        kw[b] = bit >> 5;
        ks[b] = bit & 31;
    }
    // V: lane r's 16-code chunk (bits 16+48r .. ) in row A (4-byte aligned
    // pair base) and in row B (starting 400 bits later).
    const int vbitA = 16 + 48 * r, vbitB = 416 + 48 * r;
    const int vwA = vbitA >> 5, vsA = vbitA & 31, vwB = vbitB >> 5, vsB = vbitB & 31;
    const uint32_t psel = (r & 1) ? 0x7632u : 0x5410u;
    const int src0 = (2 * c) * 4 + (r >> 1), src1 = (2 * c + 1) * 4 + (r >> 1);

    int k_next = 0;                     // next of my tiles to consume
    long long seg_start = g_begin;
    bool failed = false;
    while (seg_start < g_end) {
        const long long u = seg_start / n_t;
        const long long seg_end = min(g_end, (u + 1) * (long long)n_t);
        const int li = (int)(u / H), h = (int)(u % H);

        // ---- queries of this (layer, KV head): q' = perm(H q) * scale ----
        __syncthreads();
        for (int g = warp; g < GT; g += kWarps) {
            if (g < G) {
                const __half *qg = a.q + ((long long)li * a.n_q_heads + h * G + g) * kN;
                float x[4];
#pragma unroll
                for (int e = 0; e < 4; e++) x[e] = __half2float(qg[lane * 4 + e]);
                sp_warp_wht<4>(x, lane);
                const float sc_all = a.logit_scale * 1.4426950408889634f * a.inv_sqrt_n;
#pragma unroll
                for (int e = 0; e < 4; e++) sm.qt[g][lane * 4 + e] = x[e] * sc_all;
                __syncwarp();
                float mx = 0.0f;
                float bs = 0.0f;
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int i = lane * 4 + e;
                    const float v = sm.qt[g][ord[e]];
                    sm.q[g][i] = v;
                    mx = fmaxf(mx, fabsf(v));
                    bs += v;
                }
                // lanes 8b..8b+7 hold band b
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) bs += __shfl_xor_sync(0xffffffffu, bs, o);
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                if ((lane & 7) == 0) sm.qsum[g][lane >> 3] = bs;
                if (lane == 0) sm.qmax[g] = mx;
            } else {
                for (int i = lane; i < kN; i += 32) sm.q[g][i] = 0.0f;
                if (lane < 4) sm.qsum[g][lane] = 0.0f;
                if (lane == 0) sm.qmax[g] = 0.0f;
            }
        }
        __syncthreads();

        // B fragments of the K side: lane (r, c) supplies column r = query
        // r/2, fp16 part r%2, for the slots of lane group c.
        uint32_t bq[NT][8][2];
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const int g = 4 * nt + (r >> 1);
            const float qm = sm.qmax[g];
            const int F = qm > 1e-30f ? 6 - ilogb_normal(qm) : 0;
#pragma unroll
            for (int b = 0; b < 4; b++) {
#pragma unroll
                for (int p = 0; p < 4; p++) {
                    const int lo = 32 * b + 8 * c + p, hi = lo + 4;
                    float vlo = scale2(sm.q[g][lo], F - pair_dlo(b, p));
                    float vhi = scale2(sm.q[g][hi], F - pair_dhi(b, p));
                    if (b >= a.nb_k) vlo = vhi = 0.0f;
                    const uint32_t slo = split_hi_lo(vlo), shi = split_hi_lo(vhi);
                    const uint32_t w = (r & 1) ? ((slo >> 16) | (shi & 0xffff0000u))
                                               : ((slo & 0xffffu) | (shi << 16));
                    bq[nt][2 * b + (p >> 1)][p & 1] = w;
                }
            }
        }
        // Score constants for query 4nt + c: s = kc * sum_b s_b (acc_b + cinit_b),
        // cinit_b = -m_b * sum_{i in b} q'_i / kc.
        float kc[NT], cinit[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const int g = 4 * nt + c;
            const float qm = sm.qmax[g];
            const int F = qm > 1e-30f ? 6 - ilogb_normal(qm) : 0;
            kc[nt] = scale2(1.0f, 24 - F);
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const float m_b = (float)((1 << (kKBits(b) - 1)) - 1);
                cinit[nt][b] = b < a.nb_k ? -scale2(m_b * sm.qsum[g][b], F - 24) : 0.0f;
            }
        }

        float oacc[NT][8][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 8; i++) oacc[nt][i][0] = oacc[nt][i][1] = oacc[nt][i][2] = oacc[nt][i][3] = 0.0f;
        // Running max of the scores in units of 1/kc (kc > 0, so it orders
        // like the base-2 logits); nkm = -kc * m_run.
        float m_run[NT], nkm[NT], l_sum[NT], p_sum[NT];
#pragma unroll
        for (int nt = 0; nt < NT; nt++) { m_run[nt] = kEmptyMax; nkm[nt] = 0.0f; l_sum[nt] = 0.0f; p_sum[nt] = 0.0f; }
        // The MMAs accumulate p * vscale * u over the raw codes u (0..6); the
        // offset 3 * sum(p * vscale) comes off afterwards.  Over a long, flat
        // softmax the raw sum is ~3 sqrt(T) times the centered one, and the
        // tensor cores' accumulation (not IEEE-rounded per add) drifts in
        // proportion to the accumulator's size: 1e-3 of the output after a
        // few hundred tiles.  Every kFlushTiles tiles the window's offset is
        // taken off the accumulators with fp32 fmas, so they stay centered.
        int n_since_flush = 0;
        auto recenter = [&]() {
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                float ps = p_sum[nt];                   // window sum over the warp's positions
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
                const float off = -3.0f * ps;           // V offset 2^(3-1)-1
#pragma unroll
                for (int mt = 0; mt < 8; mt++) {
#pragma unroll
                    for (int rr = 0; rr < 2; rr++)      // hi column, in units of 2^(d-24)
                        oacc[nt][mt][2 * rr] = fmaf(off, 1.0f / (float)(1 << (24 - vcode_d(2 * mt + rr))),
                                                    oacc[nt][mt][2 * rr]);
                }
                p_sum[nt] = 0.0f;
            }
            n_since_flush = 0;
        };

        // ---- my tiles of this segment ------------------------------------
        // One ring stage per iteration: the scores of its two 16-position
        // tiles, one running-max update, then the weights and V products of
        // both tiles.  The two tiles are independent chains, which is the
        // overlap the schedule needs (a cross-stage software pipeline that
        // took the next stage's scores beside this stage's V products held
        // more registers and ran 4% slower).
        //
        // Band scales of ring stage st to fp32 (scl[st]): lane t converts
        // the four K bands and the V scale of the stage's positions t,
        // t + 32, ...
        auto stage_scales = [&](int st) {
            const unsigned char *kt = sm.ring[warp][st];
#pragma unroll
            for (int p = lane; p < 16 * kSub; p += 32) {
                const int sub = p >> 4, t = p & 15;
                const uint32_t *row = reinterpret_cast<const uint32_t *>(kt + sub * kKTile) + 19 * t;
                const uint32_t w0 = row[kKScaleWord(0)], w1 = row[kKScaleWord(1)];
                const uint32_t w2 = row[kKScaleWord(2)], w3 = row[kKScaleWord(3)];
                const uint32_t h01 = __byte_perm(w0, w1, 0x7610), h23 = __byte_perm(w2, w3, 0x7610);
                const float2 f01 = __half22float2(finite_or_zero(*reinterpret_cast<const __half2 *>(&h01)));
                const float2 f23 = __half22float2(finite_or_zero(*reinterpret_cast<const __half2 *>(&h23)));
                *reinterpret_cast<float4 *>(&sm.scl[warp][st][p][0]) = make_float4(f01.x, f01.y, f23.x, f23.y);
                const unsigned short vb =
                    *reinterpret_cast<const unsigned short *>(kt + kKStage + sub * kVTile + 50 * t);
                sm.scl[warp][st][p][4] = __low2float(finite_or_zero(__half2half2(__ushort_as_half(vb))));
            }
        };
        // K side of MMA tile `sub` of ring stage st (positions
        // tok0..tok0+15): code unpack, band MMAs, and the scores of
        // positions r, r+8 for query 4nt+c in units of 1/kc.
        auto k_scores = [&](int st, int sub, int tok0, float (&su)[NT][2]) {
            const unsigned char *kt = sm.ring[warp][st] + sub * kKTile;
            const uint32_t *K32 = reinterpret_cast<const uint32_t *>(kt);
            // Band dot products; the accumulator starts at -m_b * sum(q') in
            // its hi column, so acc_hi + acc_lo = sum_i (u_i - m_b) q'_i / kc.
            // Each MMA's A quad is unpacked right before it, so the four
            // registers can be allocated as the operand tuple directly.
            float acc[NT][4][4];
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int b = NBK; b < 4; b++) {
                    acc[nt][b][0] = cinit[nt][b]; acc[nt][b][1] = 0.0f; acc[nt][b][2] = cinit[nt][b]; acc[nt][b][3] = 0.0f;
                }
#pragma unroll
            for (int b = 0; b < 4; b++) {
                // Bands a partial read leaves out keep their zero start and
                // contribute nothing.
                if (b >= NBK) continue;
                // band window of rows r and r+8: x (low), y (high / shifted)
                uint32_t wx[2], wy[2];
#pragma unroll
                for (int hh = 0; hh < 2; hh++) {
                    const uint32_t *row = K32 + 19 * (r + 8 * hh);
                    if (b < 2) {
                        const uint32_t w0 = row[kw[b]], w1 = row[kw[b] + 1];
                        wx[hh] = shf(w0, w1, ks[b]);
                        wy[hh] = w1 >> ks[b];
                    } else if (b == 2) {
                        wx[hh] = shf(row[kw[2]], row[kw[2] + 1], 16);
                        wy[hh] = wx[hh] >> 8;
                    } else {
                        const uint32_t x = shf(row[kw[3]], row[kw[3] + 1], ks[3]);
                        wx[hh] = x << 4;
                        wy[hh] = x >> 2;
                    }
                }
                auto code = [&](int hh, int i) -> uint32_t {
                    if (b < 2) {
                        const uint32_t v = i == 0 ? wx[hh] : shf(wx[hh], wy[hh], 5 * i);
                        return v & 0x01F0001Fu;
                    } else if (b == 2) {
                        return (i < 2 ? wx[hh] : wy[hh]) & ((i & 1) ? 0x00F000F0u : 0x000F000Fu);
                    } else {
                        return (i < 2 ? wx[hh] : wy[hh]) & ((i & 1) ? 0x00380380u : 0x00070070u);
                    }
                };
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const uint32_t a0 = code(0, 2 * j), a1 = code(1, 2 * j), a2 = code(0, 2 * j + 1),
                                   a3 = code(1, 2 * j + 1);
#pragma unroll
                    for (int nt = 0; nt < NT; nt++)
                        if (j == 0)
                            mma16816_c(acc[nt][b], a0, a1, a2, a3, bq[nt][2 * b][0], bq[nt][2 * b][1], cinit[nt][b],
                                       0.0f, cinit[nt][b], 0.0f);
                        else
                            mma16816(acc[nt][b], a0, a1, a2, a3, bq[nt][2 * b + j][0], bq[nt][2 * b + j][1]);
                }
            }
            __syncwarp();
            float4 fs[2];
#pragma unroll
            for (int hh = 0; hh < 2; hh++)
                fs[hh] = *reinterpret_cast<const float4 *>(&sm.scl[warp][st][16 * sub + r + 8 * hh][0]);
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
#pragma unroll
                for (int hh = 0; hh < 2; hh++) {
                    const float4 f = fs[hh];
                    float v = f.x * (acc[nt][0][2 * hh] + acc[nt][0][2 * hh + 1]);
                    v = fmaf(f.y, acc[nt][1][2 * hh] + acc[nt][1][2 * hh + 1], v);
                    v = fmaf(f.z, acc[nt][2][2 * hh] + acc[nt][2][2 * hh + 1], v);
                    v = fmaf(f.w, acc[nt][3][2 * hh] + acc[nt][3][2 * hh + 1], v);
                    su[nt][hh] = tok0 + r + 8 * hh < a.kv_len ? v : -INFINITY;
                }
            }
        };
        // Online softmax max update (rescale only when the running max grows).
        auto update_max = [&](const float (&su)[kSub][NT][2]) {
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                float mx = fmaxf(su[0][nt][0], su[0][nt][1]);
#pragma unroll
                for (int sb = 1; sb < kSub; sb++) mx = fmaxf(mx, fmaxf(su[sb][nt][0], su[sb][nt][1]));
                if (__any_sync(0xffffffffu, mx > m_run[nt])) {
                    float mt = mx;
                    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
                    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
                    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
                    const float m_new = fmaxf(m_run[nt], mt);
                    const float alpha = fast_exp2(kc[nt] * (m_run[nt] - m_new));
                    m_run[nt] = m_new;
                    nkm[nt] = -kc[nt] * m_new;
                    l_sum[nt] *= alpha;
                    p_sum[nt] *= alpha;
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        oacc[nt][i][0] *= alpha; oacc[nt][i][1] *= alpha;
                        oacc[nt][i][2] *= alpha; oacc[nt][i][3] *= alpha;
                    }
                }
            }
        };
        // Softmax weights of the tile in stage st and its V product: lane r
        // unpacks its 16-coefficient chunk of position pairs (2c, 2c+1) and
        // (2c+8, 2c+9).
        auto v_step = [&](int st, int sub, const float (&su)[NT][2]) {
            const unsigned char *kt = sm.ring[warp][st];
            const uint32_t *V32 = reinterpret_cast<const uint32_t *>(kt + kKStage + sub * kVTile);
            // 16-bit windows of the two position rows, interleaved per half:
            // W[hh][wi] holds 5 codes of each row (the last one code).
            uint32_t W[2][4];
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                const uint32_t *pr = V32 + 25 * (c + 4 * hh);
                const uint32_t a0 = pr[vwA], a1 = pr[vwA + 1], b0 = pr[vwB], b1 = pr[vwB + 1];
                const uint32_t xal = shf(a0, a1, vsA), xah = a1 >> vsA;
                const uint32_t xbl = shf(b0, b1, vsB), xbh = b1 >> vsB;
                W[hh][0] = __byte_perm(xal, xbl, 0x5410);
                W[hh][1] = __byte_perm(shf(xal, xah, 15), shf(xbl, xbh, 15), 0x5410);
                W[hh][2] = __byte_perm(shf(xal, xah, 30), shf(xbl, xbh, 30), 0x5410);
                W[hh][3] = __byte_perm(xah, xbh, 0x5410) >> 9;
            }
            // Register j of the chunk: every code lands at bit 4 or above of
            // its half (the tensor cores lose precision on the smallest
            // subnormals, d < 4).
            auto vreg = [&](int hh, int j) -> uint32_t {
                if (j == 15) return W[hh][3] & 0x00700070u;
                const uint32_t w = W[hh][j / 5];
                switch (j % 5) {
                case 0: return (w << 4) & 0x00700070u;
                case 1: return (w << 4) & 0x03800380u;
                case 2: return w & 0x01C001C0u;
                case 3: return (w >> 5) & 0x00700070u;
                default: return (w >> 5) & 0x03800380u;
                }
            };
            float vscale[2];
#pragma unroll
            for (int hh = 0; hh < 2; hh++) vscale[hh] = sm.scl[warp][st][16 * sub + r + 8 * hh][4];
            uint32_t pb[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                float pv[2];
#pragma unroll
                for (int hh = 0; hh < 2; hh++) {
                    const float p = fast_exp2(fmaf(kc[nt], su[nt][hh], nkm[nt]));
                    l_sum[nt] += p;
                    pv[hh] = p * vscale[hh];
                    p_sum[nt] += pv[hh];
                }
                // P' (hi/lo) into the B layout of the V product.
                uint32_t pk0, pk1;
                {
                    const __half2 hi2 = __floats2half2_rn(pv[0], pv[1]);
                    const float2 back = __half22float2(hi2);
                    const __half2 lo2 = __floats2half2_rn(pv[0] - back.x, pv[1] - back.y);
                    const uint32_t hb = *reinterpret_cast<const uint32_t *>(&hi2);
                    const uint32_t lb = *reinterpret_cast<const uint32_t *>(&lo2);
                    pk0 = __byte_perm(hb, lb, 0x5410);
                    pk1 = __byte_perm(hb, lb, 0x7632);
                }
                const uint32_t x0 = __shfl_sync(0xffffffffu, pk0, src0);
                const uint32_t x1 = __shfl_sync(0xffffffffu, pk0, src1);
                const uint32_t x2 = __shfl_sync(0xffffffffu, pk1, src0);
                const uint32_t x3 = __shfl_sync(0xffffffffu, pk1, src1);
                pb[nt][0] = __byte_perm(x0, x1, psel);
                pb[nt][1] = __byte_perm(x2, x3, psel);
            }
#pragma unroll
            for (int mt = 0; mt < 8; mt++) {
                const uint32_t a0 = vreg(0, 2 * mt), a1 = vreg(0, 2 * mt + 1), a2 = vreg(1, 2 * mt),
                               a3 = vreg(1, 2 * mt + 1);
#pragma unroll
                for (int nt = 0; nt < NT; nt++) mma16816(oacc[nt][mt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
            }
        };

        int ctile = (int)(my_first + (long long)k_next * kWarps - u * n_t);
        while (k_next < n_my && ctile < n_t) {
            if (!wait_stage(bar0 + 8 * (k_next % kStages), (k_next / kStages) & 1, a.status)) {
                failed = true;
                break;
            }
            float su[kSub][NT][2];
            stage_scales(k_next % kStages);
            __syncwarp();
#pragma unroll
            for (int sb = 0; sb < kSub; sb++) k_scores(k_next % kStages, sb, ctile * 16 * kSub + 16 * sb, su[sb]);
            update_max(su);
#pragma unroll
            for (int sb = 0; sb < kSub; sb++) v_step(k_next % kStages, sb, su[sb]);
            n_since_flush += kSub;
            if (n_since_flush >= kFlushTiles) recenter();
            __syncwarp();
            if (lane == 0 && k_next + kStages < n_my) issue(k_next + kStages);
            k_next++;
            ctile += kWarps;
        }

        // ---- warp partial -> shared memory ---------------------------------
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                l_sum[nt] += __shfl_xor_sync(0xffffffffu, l_sum[nt], o);
                p_sum[nt] += __shfl_xor_sync(0xffffffffu, p_sum[nt], o);
            }
            const float mv = 3.0f;   // V offset 2^(3-1)-1
            float *mrow = sm.merge[warp][4 * nt + c];
#pragma unroll
            for (int mt = 0; mt < 8; mt++) {
#pragma unroll
                for (int rr = 0; rr < 2; rr++) {
                    const int j = 2 * mt + rr;
                    const float v = (oacc[nt][mt][2 * rr] + oacc[nt][mt][2 * rr + 1]) * (float)(1 << (24 - vcode_d(j)));
                    mrow[4 + 16 * r + j] = v - mv * p_sum[nt];
                }
            }
            if (r == 0) {
                mrow[0] = fmaxf(kc[nt] * m_run[nt], kEmptyMax);   // base-2 logit units
                mrow[1] = l_sum[nt];
            }
        }
        __syncthreads();
        // ---- CTA merge -> global partial of segment j of unit u ----------
        {
            const int seg = cta - cta_of_tile(u * (long long)n_t, sc);
            for (int idx = threadIdx.x; idx < G * (kN + 1); idx += blockDim.x) {
                const int g = idx / (kN + 1), i = idx % (kN + 1);
                float M = kEmptyMax;
#pragma unroll
                for (int w = 0; w < kWarps; w++) M = fmaxf(M, sm.merge[w][g][0]);
                float v = 0.0f;
#pragma unroll
                for (int w = 0; w < kWarps; w++) {
                    const float wt = exp2f(sm.merge[w][g][0] - M);
                    v += wt * (i < kN ? sm.merge[w][g][4 + i] : sm.merge[w][g][1]);
                }
                float *part = sp_attn_partial(a, li, h * G + g, seg);
                if (i < kN) {
                    part[4 + i] = v;
                } else {
                    part[0] = M;
                    part[1] = v;
                }
            }
        }
        if (failed) break;
        seg_start = seg_end;
    }
    // On a timed-out wait, wait (bounded) for this warp's copies in flight
    // before the CTA's shared memory is released.
    if (failed) {
        for (int k = k_next; k < n_my && k < k_next + kStages; k++)
            wait_stage(bar0 + 8 * (k % kStages), (k / kStages) & 1, nullptr);
    }
}

// Merge the segment partials of one (layer, q head), transform, write fp16
// (locally, or into every rank's gather buffer).
__global__ void k_attn_combine_seg(SpAttnArgs a, Sched sc)
{
    sp_pdl_wait();                      // launched early: the main grid's partials first
    sp_pdl_trigger();                   // the next call's main kernel may launch and wait on this grid
    const int lane = threadIdx.x & 31;
    const int qh = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int li = blockIdx.y;
    if (qh < a.n_q_heads) combine_row(a, sc, li, qh, lane);
    sp_attn_gather_signal(a);
}


}  // namespace

int sp_attn_mma_supported(const SpAttnArgs &a)
{
    if (a.kl.n != 128 || a.vl.n != 128) return SP_ERR_UNSUPPORTED;
    if (a.kl.n_bands != 4 || a.vl.n_bands != 1) return SP_ERR_UNSUPPORTED;
    for (int b = 0; b < 4; b++)
        if (a.kl.size[b] != 32 || a.kl.bits[b] != kKBits(b) || a.kl.byte_off[b] * 8 + 16 != kKBit(b))
            return SP_ERR_UNSUPPORTED;
    if (a.kl.total_bytes != 76 || a.vl.total_bytes != 50 || a.vl.bits[0] != 3) return SP_ERR_UNSUPPORTED;
    if (a.group < 1 || a.group > 8) return SP_ERR_UNSUPPORTED;
    // Whole 16-position tiles must lie inside each slot.
    const long long tiles = (a.kv_len + 15) / 16;
    if (tiles * kKTile > a.k_slot_stride || tiles * kVTile > a.v_slot_stride) return SP_ERR_UNSUPPORTED;
    if (a.nb_k < 1 || a.nb_v < 1) return SP_ERR_UNSUPPORTED;
    // 16-byte aligned tile starts for the bulk copies.
    if (((uintptr_t)a.k_cache & 15) || ((uintptr_t)a.v_cache & 15) || (a.k_slot_stride & 15) ||
        (a.v_slot_stride & 15))
        return SP_ERR_UNSUPPORTED;
    return SP_OK;
}

// Launch configuration: 4 warps per CTA, a ring of 2 stages per warp (48
// positions per stage, 64 with 5..8 query heads per KV head), and 3 CTAs
// per SM (12 warps, up to 168 registers per thread); 2 CTAs per SM with
// 5..8 query heads (two column tiles, more registers).  Measured against
// 16 x 4, 32 x 3, 32 x 2, 48 x 2 and 64 x 2 position stages for both query
// group sizes; configurations that force fewer registers spill and run
// slower.
constexpr int kCtaWarps = 4, kRingStages = 2, kCtasPerSm = 3, kCtasPerSm8 = 2;

int sp_attn_mma_launch(const SpAttnArgs &a_in, cudaStream_t s, cudaEvent_t ev_begin, cudaEvent_t ev_end)
{
    SpAttnArgs a = a_in;
    const bool wide = a.group > 4;
    using Kern = void (*)(SpAttnArgs, Sched);
    static const Kern narrow_k[4] = {k_attn_ship_mma<kCtaWarps, kRingStages, kCtasPerSm, 4, 1>,
                                     k_attn_ship_mma<kCtaWarps, kRingStages, kCtasPerSm, 4, 2>,
                                     k_attn_ship_mma<kCtaWarps, kRingStages, kCtasPerSm, 4, 3>,
                                     k_attn_ship_mma<kCtaWarps, kRingStages, kCtasPerSm, 4, 4>};
    static const Kern wide_k[4] = {k_attn_ship_mma<kCtaWarps, kRingStages, kCtasPerSm8, 8, 1>,
                                   k_attn_ship_mma<kCtaWarps, kRingStages, kCtasPerSm8, 8, 2>,
                                   k_attn_ship_mma<kCtaWarps, kRingStages, kCtasPerSm8, 8, 3>,
                                   k_attn_ship_mma<kCtaWarps, kRingStages, kCtasPerSm8, 8, 4>};
    const int nbk = a.nb_k < 1 ? 1 : (a.nb_k > 4 ? 4 : a.nb_k);
    Kern kernel = wide ? wide_k[nbk - 1] : narrow_k[nbk - 1];
    const size_t smem = wide ? sizeof(Smem<kCtaWarps, kRingStages, 8>) : sizeof(Smem<kCtaWarps, kRingStages, 4>);
    const int threads = kCtaWarps * 32;
    // Per device and per kernel: the shared-memory attribute is set and the
    // occupancy looked up once.  The table is written with atomics, so
    // host threads driving different devices (or the same one) may race on
    // it harmlessly: both compute the same values.
    constexpr int kMaxDev = 64;
    static std::atomic<int> occ_tab[kMaxDev][2][4];
    static std::atomic<int> sms_tab[kMaxDev];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDev) return sp_set_error(SP_ERR_CUDA, "tensor-core attention: device %d", dev);
    int occ_now = occ_tab[dev][wide][nbk - 1].load(std::memory_order_acquire);
    if (occ_now == 0) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return sp_check_cuda(cudaGetLastError(), "attention smem attribute");
        int occ = 0, sms = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, threads, smem);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        sms_tab[dev].store(sms > 0 ? sms : 148, std::memory_order_relaxed);
        occ_now = occ > 0 ? occ : 1;
        occ_tab[dev][wide][nbk - 1].store(occ_now, std::memory_order_release);
    }
    const int sms_cached = sms_tab[dev].load(std::memory_order_relaxed);
    const int units = a.n_layers * a.n_kv_heads;
    Sched sc;
    const int stage_pos = 16 * stage_sub(wide ? 8 : 4);
    sc.tiles_per_unit = (a.kv_len + stage_pos - 1) / stage_pos;
    sc.total_tiles = (long long)units * sc.tiles_per_unit;
    long long n = (long long)sms_cached * occ_now;
    if (n > sc.total_tiles) n = sc.total_tiles;
    // At most kAttnMaxSplits segments per (layer, KV head): N/units + 2.
    if (n > (long long)units * (kAttnMaxSplits - 2)) n = (long long)units * (kAttnMaxSplits - 2);
    sc.n_ctas = (int)n;
    a.n_splits = 0;
    if (ev_begin) cudaEventRecord(ev_begin, s);
    // A programmatic dependent of the stream's previous kernel (the previous
    // call's combine, in a decode loop): its blocks are placed while that
    // kernel finishes and start at its completion.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sc.n_ctas);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int rc = sp_check_cuda(cudaLaunchKernelEx(&cfg, kernel, a, sc), "tensor-core attention launch");
    if (ev_end) cudaEventRecord(ev_end, s);
    if (rc) return rc;
    return sp_attn_seg_combine_launch(a, sc, s);
}

// The combine is launched as a programmatic dependent of the main kernel:
// it may start as soon as every main block has begun (sp_pdl_trigger) and
// waits in sp_pdl_wait for the main grid's completion, which takes the
// kernel-to-kernel launch gap off the step.
int sp_attn_seg_combine_launch(const SpAttnArgs &a, const SpSched &sc, cudaStream_t s)
{
    const int per_block = 4;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.n_q_heads + per_block - 1) / per_block, a.n_layers);
    cfg.blockDim = dim3(per_block * 32);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return sp_check_cuda(cudaLaunchKernelEx(&cfg, k_attn_combine_seg, a, sc), "tensor-core attention combine launch");
}
