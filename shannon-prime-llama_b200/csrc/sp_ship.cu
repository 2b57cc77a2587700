// sp_ship.cu — ship-path codec kernels for sm_100a: the write path
// (VHT2 -> Möbius reorder -> band quantise -> pack) and the read path
// (unpack -> dequantise -> Möbius unreorder -> VHT2), plus the
// reference-named C-ABI launchers of shannon_prime_cuda.h.
//
// Design: one warp per vector.  The vector lives in registers (E = n/32
// floats per lane); the Hartley butterfly runs in registers and warp
// shuffles (sp_warp_wht) instead of one __syncthreads per stage in shared
// memory (reference kernel_vht2_p2, shannon_prime_cuda.cu:37-75).  The
// reorder is one shared-memory gather, the band absmax one redux.sync per
// band, and packing is output-byte-stationary: each lane assembles whole
// output bytes from the codes that overlap them, so no serial bit loop
// (reference kernel_band_quantize_simple packs 128 codes in one thread,
// shannon_prime_cuda.cu:131-204) and no atomics.  A CTA handles 8
// consecutive positions of one head, so its packed rows are one contiguous
// range written by the whole CTA.
//
// Bit-exactness: every float step is the single IEEE operation the CPU
// restatement performs (__fadd_rn/__fsub_rn/__fmul_rn/__fdiv_rn, no
// contraction), __float2half_rn for the scale, round-half-even for codes.
#include "sp_internal.cuh"

#include <atomic>

#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <type_traits>

namespace {

constexpr int kWarps = 8;   // vectors (positions) per CTA

struct EncodeArgs {
    const void *in;            // [n_tokens][nh][n] elements
    uint8_t *out_base;         // slab base
    long long slot0;           // slot of head 0
    long long slot_stride;     // bytes per slot
    int n_tokens;
    int nh;
    int start_pos;
    const int *order;          // Möbius order or nullptr
    float inv_sqrt_n;
    SpBandLayout bl;
};

struct DecodeArgs {
    const uint8_t *in_base;
    long long slot;
    long long slot_stride;
    int start_pos;
    int n_pos;
    float *out;                // [n_pos][n]
    const int *order;          // Möbius order or nullptr (unreorder)
    float inv_sqrt_n;
    int max_bands;
    SpBandLayout bl;
};

__device__ __forceinline__ int band_of(const SpBandLayout &bl, int i)
{
    int b = 0;
#pragma unroll 1
    for (int k = 1; k < bl.n_bands; k++)
        if (i >= bl.off[k]) b = k;
    return b;
}

// Assemble packed byte j of a row from the codes in shared memory.
__device__ __forceinline__ uint8_t pack_byte(const SpBandLayout &bl, const uint8_t *codes,
                                             const uint16_t *scale_bits, int j)
{
    int b = 0;
#pragma unroll 1
    for (int k = 1; k < bl.n_bands; k++)
        if (j >= bl.byte_off[k]) b = k;
    int r = j - bl.byte_off[b];
    if (r == 0) return (uint8_t)(scale_bits[b] & 0xff);
    if (r == 1) return (uint8_t)(scale_bits[b] >> 8);
    const int d = r - 2, bits = bl.bits[b], sz = bl.size[b];
    const uint8_t *c = codes + bl.off[b];
    int k0 = (8 * d) / bits;
    int k1 = (8 * d + 7) / bits;
    if (k1 > sz - 1) k1 = sz - 1;
    uint32_t v = 0;
    for (int k = k0; k <= k1; k++) {
        int sh = k * bits - 8 * d;
        v |= sh >= 0 ? ((uint32_t)c[k] << sh) : ((uint32_t)c[k] >> (-sh));
    }
    return (uint8_t)(v & 0xff);
}

// Write path.  Grid: x = head-major tiles of kWarps positions, one warp per
// vector.  Dynamic smem: order[n] ints, per-warp float buf[n] + codes[n],
// per-warp scale info, and the CTA's packed rows.
template <int E, typename Tin, bool WHT>
__global__ void __launch_bounds__(kWarps * 32)
k_encode(EncodeArgs a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int n = 32 * E;
    const SpBandLayout &bl = a.bl;
    int *s_order = reinterpret_cast<int *>(smem);
    float *s_buf = reinterpret_cast<float *>(s_order + n);             // [kWarps][n]
    float *s_inv = s_buf + kWarps * n;                                  // [kWarps][16]
    uint16_t *s_sbits = reinterpret_cast<uint16_t *>(s_inv + kWarps * SP_MAX_BANDS);
    uint8_t *s_codes = reinterpret_cast<uint8_t *>(s_sbits + kWarps * SP_MAX_BANDS);
    uint8_t *s_rows = s_codes + kWarps * n;                             // [kWarps][total]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tiles = (a.n_tokens + kWarps - 1) / kWarps;
    const int h = blockIdx.x % a.nh;
    const int tile = blockIdx.x / a.nh;
    if (tile >= n_tiles) return;
    const int t0 = tile * kWarps;
    const int t = t0 + warp;
    const bool active = t < a.n_tokens;

    if (a.order)
        for (int i = threadIdx.x; i < n; i += blockDim.x) s_order[i] = a.order[i];
    __syncthreads();

    float *buf = s_buf + warp * n;
    uint8_t *codes = s_codes + warp * n;
    float x[E];
    if (active) {
        const Tin *src = reinterpret_cast<const Tin *>(a.in) +
                         ((long long)t * a.nh + h) * n + lane * E;
        if constexpr (sizeof(Tin) == 4 && E % 4 == 0) {
#pragma unroll
            for (int e = 0; e < E; e += 4) {
                float4 v = __ldg(reinterpret_cast<const float4 *>(src + e));
                x[e] = v.x; x[e + 1] = v.y; x[e + 2] = v.z; x[e + 3] = v.w;
            }
        } else {
#pragma unroll
            for (int e = 0; e < E; e++) x[e] = sp_load_as_float(src, e);
        }
        if constexpr (WHT) {
            sp_warp_wht<E>(x, lane);
#pragma unroll
            for (int e = 0; e < E; e++) x[e] = __fmul_rn(x[e], a.inv_sqrt_n);
        }
        if (a.order) {
#pragma unroll
            for (int e = 0; e < E; e++) buf[lane * E + e] = x[e];
            __syncwarp();
#pragma unroll
            for (int e = 0; e < E; e++) x[e] = buf[s_order[lane * E + e]];
        }
        // Per-band absmax: |x| of a non-NaN float orders like its bit pattern.
        for (int b = 0; b < bl.n_bands; b++) {
            unsigned m = 0;
#pragma unroll
            for (int e = 0; e < E; e++) {
                int i = lane * E + e;
                if (i >= bl.off[b] && i < bl.off[b] + bl.size[b]) {
                    float av = fabsf(x[e]);
                    unsigned u = __float_as_uint(av);
                    if (!(av != av) && u > m) m = u;
                }
            }
            m = __reduce_max_sync(0xffffffffu, m);
            if (lane == b) {
                float amax = __uint_as_float(m);
                int max_val = (1 << (bl.bits[b] - 1)) - 1;
                float scale = amax > 0.0f ? __fdiv_rn(amax, (float)max_val) : 0.0f;
                __half hs = __float2half_rn(scale);
                float stored = __half2float(hs);
                s_sbits[warp * SP_MAX_BANDS + b] = __half_as_ushort(hs);
                s_inv[warp * SP_MAX_BANDS + b] = stored > 0.0f ? __fdiv_rn(1.0f, stored) : 0.0f;
            }
        }
        __syncwarp();
#pragma unroll
        for (int e = 0; e < E; e++) {
            int i = lane * E + e;
            int b = band_of(bl, i);
            int max_val = (1 << (bl.bits[b] - 1)) - 1;
            float p = __fmul_rn(x[e], s_inv[warp * SP_MAX_BANDS + b]);
            int q = __float2int_rn(p);            // NaN -> 0, saturating
            q = q > max_val ? max_val : (q < -max_val ? -max_val : q);
            codes[i] = (uint8_t)(q + max_val);
        }
        __syncwarp();
        uint8_t *row = s_rows + warp * bl.total_bytes;
        for (int j = lane; j < bl.total_bytes; j += 32)
            row[j] = pack_byte(bl, codes, s_sbits + warp * SP_MAX_BANDS, j);
    }
    __syncthreads();
    // The CTA's rows are contiguous in the slot: copy them out together.
    const int n_rows = min(kWarps, a.n_tokens - t0);
    const long long nbytes = (long long)n_rows * bl.total_bytes;
    uint8_t *dst = a.out_base + (a.slot0 + h) * a.slot_stride +
                   (long long)(a.start_pos + t0) * bl.total_bytes;
    if ((((uintptr_t)dst) & 3) == 0 && (nbytes & 3) == 0) {
        const uint32_t *s32 = reinterpret_cast<const uint32_t *>(s_rows);
        uint32_t *d32 = reinterpret_cast<uint32_t *>(dst);
        for (int j = threadIdx.x; j < nbytes / 4; j += blockDim.x) d32[j] = s32[j];
    } else {
        for (int j = threadIdx.x; j < nbytes; j += blockDim.x) dst[j] = s_rows[j];
    }
}

// Read path.  One warp per position of one slot; the CTA's packed rows are
// first copied (coalesced) into shared memory, then each lane unpacks the
// codes of its E reordered coefficients.
template <int E, bool WHT>
__global__ void __launch_bounds__(kWarps * 32)
k_decode(DecodeArgs a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int n = 32 * E;
    const SpBandLayout &bl = a.bl;
    int *s_order = reinterpret_cast<int *>(smem);
    float *s_buf = reinterpret_cast<float *>(s_order + n);   // [kWarps][n]
    uint8_t *s_rows = reinterpret_cast<uint8_t *>(s_buf + kWarps * n);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * kWarps;
    const int n_rows = min(kWarps, a.n_pos - t0);
    if (n_rows <= 0) return;
    if (a.order)
        for (int i = threadIdx.x; i < n; i += blockDim.x) s_order[i] = a.order[i];
    const uint8_t *src = a.in_base + a.slot * a.slot_stride +
                         (long long)(a.start_pos + t0) * bl.total_bytes;
    const int nbytes = n_rows * bl.total_bytes;
    for (int j = threadIdx.x; j < nbytes; j += blockDim.x) s_rows[j] = __ldg(src + j);
    __syncthreads();

    const int t = t0 + warp;
    if (t >= a.n_pos) return;
    const int nb_use = (a.max_bands < 0 || a.max_bands >= bl.n_bands) ? bl.n_bands : a.max_bands;
    const uint8_t *row = s_rows + warp * bl.total_bytes;
    float x[E];
#pragma unroll
    for (int e = 0; e < E; e++) {
        const int i = lane * E + e;
        const int b = band_of(bl, i);
        float v = 0.0f;
        if (b < nb_use) {
            const int bits = bl.bits[b];
            const int max_val = (1 << (bits - 1)) - 1;
            const uint8_t *p = row + bl.byte_off[b];
            float scale = __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
            if (!isfinite(scale)) scale = 0.0f;
            const int bp = (i - bl.off[b]) * bits;
            const int byte = 2 + (bp >> 3);
            uint32_t w = p[byte];
            if ((bp & 7) + bits > 8) w |= (uint32_t)p[byte + 1] << 8;
            const int u = (int)((w >> (bp & 7)) & ((1u << bits) - 1u));
            v = __fmul_rn((float)(u - max_val), scale);
        }
        x[e] = v;
    }
    if (a.order) {
        float *buf = s_buf + warp * n;
#pragma unroll
        for (int e = 0; e < E; e++) buf[s_order[lane * E + e]] = x[e];
        __syncwarp();
#pragma unroll
        for (int e = 0; e < E; e++) x[e] = buf[lane * E + e];
    }
    if constexpr (WHT) {
        sp_warp_wht<E>(x, lane);
#pragma unroll
        for (int e = 0; e < E; e++) x[e] = __fmul_rn(x[e], a.inv_sqrt_n);
    }
    float *dst = a.out + (long long)t * n + lane * E;
    if constexpr (E % 4 == 0) {
#pragma unroll
        for (int e = 0; e < E; e += 4)
            *reinterpret_cast<float4 *>(dst + e) = make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]);
    } else {
#pragma unroll
        for (int e = 0; e < E; e++) dst[e] = x[e];
    }
}

// In-place Möbius (un)reorder of n_vecs vectors of length n (one warp each).
template <bool INVERSE>
__global__ void k_permute(float *data, const int *order, int n, int n_vecs)
{
    extern __shared__ float pbuf[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long v = (long long)blockIdx.x * kWarps + warp;
    if (v >= n_vecs) return;
    float *buf = pbuf + warp * n;
    float *x = data + v * n;
    for (int i = lane; i < n; i += 32) buf[i] = x[i];
    __syncwarp();
    for (int i = lane; i < n; i += 32) {
        if (INVERSE) x[order[i]] = buf[i];
        else x[i] = buf[order[i]];
    }
}

// ---------------------------------------------------------------------------
// Fast write path for band layouts that map onto whole lane groups.  A
// vector of n coefficients is spread over LPV = n/8 lanes, 8 consecutive
// coefficients per lane (two vectors per warp at head_dim 128), and every
// band must start and end on a lane boundary and span a power-of-two,
// aligned group of lanes.  The ship layouts (K 4 x 32, V 1 x 128 at
// head_dim 128) qualify.  Then:
//   - the lane's 8 reordered coefficients belong to one band, so the band
//     absmax is an xor-reduction over the band's lane group;
//   - the lane's 8 codes are consecutive in the band's bit stream: one bit
//     field ORed into the packed row with two or three shared-memory
//     atomics;
//   - the Hartley butterfly runs 3 stages in registers and log2(LPV)
//     stages as one shuffle plus one FMA with +-1 per element
//     (fma(-1, v, u) rounds exactly like u - v);
//   - the lane's Möbius gather indices are loaded once per CTA.
// CTAs are persistent (grid-stride over vectors, token-major), and each
// vector's lanes store its row themselves, so no CTA-wide barrier is taken.
constexpr int kFastWarps = 8;
constexpr int kFastRowWords = 80;      // per-vector packed-row buffer (320 B)

struct FastBand {
    int group_log2[32];    // per lane of a vector: log2 of its band's lane-group size
    int bits[32];          // bits of its band
    int bitpos[32];        // row bit of its first code
    int scale_word[32];    // row word of its band's fp16 scale
    int scale_shift[32];   // 0 or 16; -1 if the lane does not write the scale
};

struct FastArgs {
    EncodeArgs e;
    FastBand fb;
    int store_width;       // 4, 2 or 1: widest aligned store for every row
};

template <int LPV, int E, typename Tin, bool WHT>
__global__ void __launch_bounds__(kFastWarps * 32)
k_encode_fast(FastArgs fa)
{
    static_assert(E == 8 || E == 16, "codes are packed in groups of 8");
    constexpr int VPW = 32 / LPV;             // vectors per warp
    constexpr int n = LPV * E;
    constexpr int kStages = LPV == 32 ? 5 : LPV == 16 ? 4 : LPV == 8 ? 3 : LPV == 4 ? 2 : 1;
    __shared__ uint32_t s_row[kFastWarps][VPW][kFastRowWords];
    __shared__ __align__(16) float s_buf[kFastWarps][VPW][n];
    const EncodeArgs &a = fa.e;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = lane / LPV, ln = lane % LPV;        // vector within the warp, lane within it
    const int words = (a.bl.total_bytes + 3) >> 2;

    // Lane constants.
    int ord[E];
#pragma unroll
    for (int e = 0; e < E; e++) ord[e] = a.order ? a.order[ln * E + e] : ln * E + e;
    const int glog = fa.fb.group_log2[ln];
    const int bits = fa.fb.bits[ln];
    const int max_val = (1 << (bits - 1)) - 1;
    const unsigned mult = 1u << bits;
    const unsigned off4 = (unsigned)max_val * (1u + mult + mult * mult + mult * mult * mult);
    const int bitpos = fa.fb.bitpos[ln];
    const int sword = fa.fb.scale_word[ln];
    const int sshift = fa.fb.scale_shift[ln];
    float sgn[5];                           // butterfly sign of this lane per stage
#pragma unroll
    for (int k = 0; k < 5; k++) sgn[k] = (ln >> k) & 1 ? -1.0f : 1.0f;

    const long long n_vec = (long long)a.n_tokens * a.nh;
    const int stride = gridDim.x * kFastWarps * VPW;
    // (token, head) of vector v = t * nh + h, stepped without division.
    const int dt = stride / a.nh, dh = stride - dt * a.nh;
    long long v = ((long long)blockIdx.x * kFastWarps + warp) * VPW + sub;
    int t = (int)(v / a.nh), h = (int)(v - (long long)t * a.nh);
    uint32_t *row = s_row[warp][sub];
    float *buf = s_buf[warp][sub];
    // Every lane of the warp runs the same number of iterations (shuffles
    // span the warp); vectors past the end are computed but not stored.
    const long long v_first = ((long long)blockIdx.x * kFastWarps + warp) * VPW;
    for (long long vw = v_first; vw < n_vec; vw += stride, v += stride, t += dt, h += dh) {
        if (h >= a.nh) { h -= a.nh; t++; }
        const bool live = v < n_vec;
        // ---- load ----
        float x[E];
        const Tin *src = reinterpret_cast<const Tin *>(a.in) + (live ? v : vw) * n + ln * E;
        if constexpr (sizeof(Tin) == 4) {
#pragma unroll
            for (int e = 0; e < E; e += 4) {
                const float4 q = __ldcs(reinterpret_cast<const float4 *>(src + e));
                x[e] = q.x; x[e + 1] = q.y; x[e + 2] = q.z; x[e + 3] = q.w;
            }
        } else {
#pragma unroll
            for (int e = 0; e < E; e += 8) {
                const uint4 q = __ldcs(reinterpret_cast<const uint4 *>(src + e));
                const Tin *hv = reinterpret_cast<const Tin *>(&q);
#pragma unroll
                for (int i = 0; i < 8; i++) x[e + i] = sp_load_as_float(hv, i);
            }
        }
        for (int j = ln; j < words; j += LPV) row[j] = 0u;
        // ---- VHT2 (ascending butterfly lengths, as the CPU path) ----
        if constexpr (WHT) {
#pragma unroll
            for (int len = 1; len < E; len <<= 1) {
#pragma unroll
                for (int i = 0; i < E; i += len << 1) {
#pragma unroll
                    for (int j = 0; j < len; j++) {
                        const float u = x[i + j], w = x[i + j + len];
                        x[i + j] = __fadd_rn(u, w);
                        x[i + j + len] = __fsub_rn(u, w);
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < kStages; k++) {
#pragma unroll
                for (int e = 0; e < E; e++) {
                    const float o = __shfl_xor_sync(0xffffffffu, x[e], 1 << k);
                    x[e] = __fmaf_rn(sgn[k], x[e], o);
                }
            }
#pragma unroll
            for (int e = 0; e < E; e++) x[e] = __fmul_rn(x[e], a.inv_sqrt_n);
        }
        // ---- Möbius reorder through shared memory ----
        if (a.order) {
#pragma unroll
            for (int e = 0; e < E; e += 4)
                *reinterpret_cast<float4 *>(&buf[ln * E + e]) = make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]);
            __syncwarp();
#pragma unroll
            for (int e = 0; e < E; e++) x[e] = buf[ord[e]];
        }
        // ---- band absmax over the lane group (fmaxf skips NaN, as the CPU
        //      path's "a > amax" does) ----
        float amax = 0.0f;
#pragma unroll
        for (int e = 0; e < E; e++) amax = fmaxf(amax, fabsf(x[e]));
#pragma unroll
        for (int k = 0; k < kStages; k++) {
            const float o = __shfl_xor_sync(0xffffffffu, amax, 1 << k);
            if (k < glog) amax = fmaxf(amax, o);
        }
        const float scale = amax > 0.0f ? __fdiv_rn(amax, (float)max_val) : 0.0f;
        const __half hs = __float2half_rn(scale);
        const float stored = __half2float(hs);
        const float inv = stored > 0.0f ? __frcp_rn(stored) : 0.0f;     // = 1.0f / stored
        // ---- quantise and pack the lane's codes into one field: codes
        //      0..3 and 4..7 are accumulated Horner-style (q3*m + q2)*m ...
        //      with m = 2^bits, one integer multiply-add per code ----
        int qv[E];
#pragma unroll
        for (int e = 0; e < E; e++) {
            const int q = __float2int_rn(__fmul_rn(x[e], inv));   // NaN -> 0, saturating
            qv[e] = min(max(q, -max_val), max_val);
        }
        __syncwarp();                       // row zeroed, buf reads done
#pragma unroll
        for (int g = 0; g < E / 8; g++) {
            // codes 8g..8g+7 as one field of 8 * bits <= 64 bits, over the
            // signed codes; the offset max_val of all four codes of a half
            // is added once (exact modulo 2^32: the field fits in 32 bits)
            unsigned f_lo = (unsigned)qv[8 * g + 3], f_hi = (unsigned)qv[8 * g + 7];
#pragma unroll
            for (int e = 2; e >= 0; e--) {
                f_lo = f_lo * mult + (unsigned)qv[8 * g + e];
                f_hi = f_hi * mult + (unsigned)qv[8 * g + 4 + e];
            }
            f_lo += off4;
            f_hi += off4;
            const unsigned long long field = ((unsigned long long)f_hi << (4 * bits)) | f_lo;
            const int pos = bitpos + 8 * g * bits;
            const int w0 = pos >> 5, sh = pos & 31;
            const unsigned long long lo = field << sh;
            atomicOr(&row[w0], (unsigned)lo);
            if (8 * bits + sh > 32) atomicOr(&row[w0 + 1], (unsigned)(lo >> 32));
            if (sh && 8 * bits + sh > 64) atomicOr(&row[w0 + 2], (unsigned)(field >> (64 - sh)));
        }
        if (sshift >= 0) atomicOr(&row[sword], (unsigned)__half_as_ushort(hs) << sshift);
        __syncwarp();
        // ---- store the packed row ----
        if (live) {
            uint8_t *dst = a.out_base + (a.slot0 + h) * a.slot_stride +
                           (long long)(a.start_pos + t) * a.bl.total_bytes;
            const int tb = a.bl.total_bytes;
            if (fa.store_width == 4) {
                for (int j = ln; j < (tb >> 2); j += LPV) reinterpret_cast<uint32_t *>(dst)[j] = row[j];
            } else if (fa.store_width == 2) {
                const uint16_t *r16 = reinterpret_cast<const uint16_t *>(row);
                for (int j = ln; j < (tb >> 1); j += LPV) reinterpret_cast<uint16_t *>(dst)[j] = r16[j];
            } else {
                const uint8_t *r8 = reinterpret_cast<const uint8_t *>(row);
                for (int j = ln; j < tb; j += LPV) dst[j] = r8[j];
            }
        }
        __syncwarp();                       // row fully read before the next zeroing
    }
}

// Lane tables for the fast path at E coefficients per lane, or false if the
// layout does not qualify.
bool fast_bands(const SpBandLayout &bl, int E, FastBand &fb)
{
    if (bl.n % E || bl.n / E > 32 || bl.n / E < 1) return false;
    if ((bl.total_bytes + 3) / 4 + 3 > kFastRowWords) return false;
    for (int b = 0; b < bl.n_bands; b++) {
        if (bl.off[b] % E || bl.size[b] % E || bl.bits[b] < 1 || bl.bits[b] > 8) return false;
        const int g = bl.size[b] / E;
        if (g < 1 || (g & (g - 1)) || (bl.off[b] / E) % g) return false;
        int glog = 0;
        while ((1 << glog) < g) glog++;
        for (int l = bl.off[b] / E; l < (bl.off[b] + bl.size[b]) / E; l++) {
            fb.group_log2[l] = glog;
            fb.bits[l] = bl.bits[b];
            fb.bitpos[l] = 8 * (bl.byte_off[b] + 2) + (l * E - bl.off[b]) * bl.bits[b];
            fb.scale_word[l] = bl.byte_off[b] >> 2;
            fb.scale_shift[l] = (l * E == bl.off[b]) ? 8 * (bl.byte_off[b] & 3) : -1;
        }
    }
    return true;
}

template <int LPV, int E, typename Tin>
int launch_encode_fast(const FastArgs &fa, bool wht, cudaStream_t s)
{
    // occupancy and SM count looked up once per kernel (atomics: host
    // threads race harmlessly; every device here is the same B200 part)
    static std::atomic<int> blocks_per_sm[2], sms_cached{0};
    auto k = wht ? k_encode_fast<LPV, E, Tin, true> : k_encode_fast<LPV, E, Tin, false>;
    int bps = blocks_per_sm[wht ? 1 : 0].load(std::memory_order_acquire);
    if (!bps) {
        int dev = 0, sm = 0, o = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, k, kFastWarps * 32, 0);
        sms_cached.store(sm > 0 ? sm : 148, std::memory_order_relaxed);
        bps = o > 0 ? o : 1;
        blocks_per_sm[wht ? 1 : 0].store(bps, std::memory_order_release);
    }
    const int sms = sms_cached.load(std::memory_order_relaxed);
    const long long per_cta = (long long)kFastWarps * (32 / LPV);
    const long long n_vec = (long long)fa.e.n_tokens * fa.e.nh;
    long long blocks = (n_vec + per_cta - 1) / per_cta;
    if (blocks > (long long)sms * bps) blocks = (long long)sms * bps;
    k<<<(unsigned)blocks, kFastWarps * 32, 0, s>>>(fa);
    return sp_check_cuda(cudaGetLastError(), "encode launch");
}

size_t encode_smem(int n, int total_bytes)
{
    return (size_t)n * 4 + (size_t)kWarps * n * 4 + (size_t)kWarps * SP_MAX_BANDS * 6 +
           (size_t)kWarps * n + (size_t)kWarps * total_bytes + 16;
}

size_t decode_smem(int n, int total_bytes)
{
    return (size_t)n * 4 + (size_t)kWarps * n * 4 + (size_t)kWarps * total_bytes + 16;
}

template <int E, typename Tin>
int launch_encode_t(const EncodeArgs &a, bool wht, cudaStream_t s)
{
    const int n_tiles = (a.n_tokens + kWarps - 1) / kWarps;
    const long long blocks = (long long)n_tiles * a.nh;
    if (blocks > 0x7fffffffLL) return sp_set_error(SP_ERR_ARG, "encode: too many vectors");
    const size_t sm = encode_smem(32 * E, a.bl.total_bytes);
    if (wht) {
        auto k = k_encode<E, Tin, true>;
        if (sm > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        k<<<(unsigned)blocks, kWarps * 32, sm, s>>>(a);
    } else {
        auto k = k_encode<E, Tin, false>;
        if (sm > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        k<<<(unsigned)blocks, kWarps * 32, sm, s>>>(a);
    }
    return sp_check_cuda(cudaGetLastError(), "encode launch");
}

template <typename Tin>
int launch_encode_dt(const EncodeArgs &a, bool wht, cudaStream_t s)
{
    FastArgs fa;
    fa.e = a;
    const uintptr_t base = (uintptr_t)(a.out_base + a.slot0 * a.slot_stride + (long long)a.start_pos * a.bl.total_bytes);
    const int tb = a.bl.total_bytes;
    fa.store_width = ((tb | base | (uintptr_t)a.slot_stride) & 3) == 0 ? 4
                   : ((tb | base | (uintptr_t)a.slot_stride) & 1) == 0 ? 2 : 1;
    // The inputs must allow 16-byte loads of each lane's 8 elements.
    const bool in_aligned = ((uintptr_t)a.in % 16) == 0;
    // 8 coefficients per lane (two head_dim-128 vectors per warp); 16 per lane
    // (four vectors per warp) measured 5% slower on config 1 at the same
    // occupancy, so only 8 is dispatched.
    if (in_aligned && fast_bands(a.bl, 8, fa.fb)) {
        switch (a.bl.n / 8) {
        case 4:  return launch_encode_fast<4, 8, Tin>(fa, wht, s);
        case 8:  return launch_encode_fast<8, 8, Tin>(fa, wht, s);
        case 16: return launch_encode_fast<16, 8, Tin>(fa, wht, s);
        case 32: return launch_encode_fast<32, 8, Tin>(fa, wht, s);
        }
    }
    switch (a.bl.n) {
    case 32:  return launch_encode_t<1, Tin>(a, wht, s);
    case 64:  return launch_encode_t<2, Tin>(a, wht, s);
    case 128: return launch_encode_t<4, Tin>(a, wht, s);
    case 256: return launch_encode_t<8, Tin>(a, wht, s);
    case 512: return launch_encode_t<16, Tin>(a, wht, s);
    default:
        return sp_set_error(SP_ERR_UNSUPPORTED, "ship path: head_dim %d is not a power of two in [32,512]", a.bl.n);
    }
}

template <int E>
int launch_decode_t(const DecodeArgs &a, bool wht, cudaStream_t s)
{
    const int blocks = (a.n_pos + kWarps - 1) / kWarps;
    const size_t sm = decode_smem(32 * E, a.bl.total_bytes);
    if (wht) {
        auto k = k_decode<E, true>;
        if (sm > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        k<<<blocks, kWarps * 32, sm, s>>>(a);
    } else {
        auto k = k_decode<E, false>;
        if (sm > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        k<<<blocks, kWarps * 32, sm, s>>>(a);
    }
    return sp_check_cuda(cudaGetLastError(), "decode launch");
}

}  // namespace

// ------------------------------------------------------------ launchers --

int sp_launch_encode(const void *d_in, int dtype, int n_tokens, int nh,
                     uint8_t *d_out_base, long long slot0, long long slot_stride_bytes,
                     int start_pos, const int *d_order, bool do_wht,
                     const SpBandLayout &bl, cudaStream_t s, bool std_order,
                     unsigned int *d_status)
{
    if (n_tokens == 0) return SP_OK;
    if (!d_in || !d_out_base || n_tokens < 0 || nh <= 0)
        return sp_set_error(SP_ERR_ARG, "encode: bad arguments");
    int rc = SP_OK;
    if (sp_encode_lane_try(d_in, dtype, n_tokens, nh, d_out_base, slot0, slot_stride_bytes, start_pos,
                           std_order, d_order, do_wht, bl, d_status, s, &rc))
        return rc;
    EncodeArgs a;
    a.in = d_in; a.out_base = d_out_base; a.slot0 = slot0; a.slot_stride = slot_stride_bytes;
    a.n_tokens = n_tokens; a.nh = nh; a.start_pos = start_pos; a.order = d_order;
    a.inv_sqrt_n = sp_inv_sqrt_n(bl.n); a.bl = bl;
    switch (dtype) {
    case SP_DTYPE_F32:  return launch_encode_dt<float>(a, do_wht, s);
    case SP_DTYPE_F16:  return launch_encode_dt<__half>(a, do_wht, s);
    case SP_DTYPE_BF16: return launch_encode_dt<__nv_bfloat16>(a, do_wht, s);
    default: return sp_set_error(SP_ERR_ARG, "encode: unknown dtype %d", dtype);
    }
}

int sp_launch_decode(const uint8_t *d_in_base, long long slot, long long slot_stride_bytes,
                     int start_pos, int n_pos, float *d_out, const int *d_order,
                     bool do_wht, int max_bands, const SpBandLayout &bl, cudaStream_t s,
                     bool std_order, unsigned int *d_status)
{
    if (n_pos == 0) return SP_OK;
    if (!d_in_base || !d_out || n_pos < 0)
        return sp_set_error(SP_ERR_ARG, "decode: bad arguments");
    {
        int rc = SP_OK;
        const uint8_t *rows = d_in_base + slot * slot_stride_bytes + (long long)start_pos * bl.total_bytes;
        if (sp_decode_lane_try(rows, n_pos, d_out, d_order, std_order, do_wht, max_bands, bl, d_status, s, &rc))
            return rc;
    }
    DecodeArgs a;
    a.in_base = d_in_base; a.slot = slot; a.slot_stride = slot_stride_bytes;
    a.start_pos = start_pos; a.n_pos = n_pos; a.out = d_out; a.order = d_order;
    a.inv_sqrt_n = sp_inv_sqrt_n(bl.n); a.max_bands = max_bands; a.bl = bl;
    switch (bl.n) {
    case 32:  return launch_decode_t<1>(a, do_wht, s);
    case 64:  return launch_decode_t<2>(a, do_wht, s);
    case 128: return launch_decode_t<4>(a, do_wht, s);
    case 256: return launch_decode_t<8>(a, do_wht, s);
    case 512: return launch_decode_t<16>(a, do_wht, s);
    default:
        return sp_set_error(SP_ERR_UNSUPPORTED, "ship path: head_dim %d is not a power of two in [32,512]", bl.n);
    }
}

// In-place VHT2 of [n_vecs][n]: the encode kernel without quantisation is
// not reusable here, so run a small dedicated warp-per-vector kernel.
namespace {
template <int E>
__global__ void k_vht2_inplace(float *data, int n_vecs, float s)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long v = (long long)blockIdx.x * kWarps + warp;
    if (v >= n_vecs) return;
    float *p = data + v * (32 * E) + lane * E;
    float x[E];
#pragma unroll
    for (int e = 0; e < E; e++) x[e] = p[e];
    sp_warp_wht<E>(x, lane);
#pragma unroll
    for (int e = 0; e < E; e++) p[e] = __fmul_rn(x[e], s);
}
}  // namespace

extern "C" {

void sp_cuda_vht2_forward(float *d_data, int n, int n_vecs, void *stream)
{
    sp_clear_error();
    if (!d_data || n_vecs < 0) { sp_set_error(SP_ERR_ARG, "vht2: bad arguments"); return; }
    if (n_vecs == 0) return;
    cudaStream_t s = (cudaStream_t)stream;
    const int blocks = (n_vecs + kWarps - 1) / kWarps;
    const float sc = sp_inv_sqrt_n(n);
    switch (n) {
    case 32:  k_vht2_inplace<1><<<blocks, kWarps * 32, 0, s>>>(d_data, n_vecs, sc); break;
    case 64:  k_vht2_inplace<2><<<blocks, kWarps * 32, 0, s>>>(d_data, n_vecs, sc); break;
    case 128: k_vht2_inplace<4><<<blocks, kWarps * 32, 0, s>>>(d_data, n_vecs, sc); break;
    case 256: k_vht2_inplace<8><<<blocks, kWarps * 32, 0, s>>>(d_data, n_vecs, sc); break;
    case 512: k_vht2_inplace<16><<<blocks, kWarps * 32, 0, s>>>(d_data, n_vecs, sc); break;
    default:
        sp_set_error(SP_ERR_UNSUPPORTED, "vht2: n=%d is not a power of two in [32,512]", n);
        return;
    }
    sp_check_cuda(cudaGetLastError(), "vht2 launch");
}

static void permute(float *d_data, const int *d_order, int n, int n_vecs, void *stream, bool inverse)
{
    sp_clear_error();
    if (!d_data || !d_order || n <= 0 || n > SP_MAX_HEAD_DIM || n_vecs < 0) {
        sp_set_error(SP_ERR_ARG, "mobius: bad arguments");
        return;
    }
    if (n_vecs == 0) return;
    const int blocks = (n_vecs + kWarps - 1) / kWarps;
    const size_t sm = (size_t)kWarps * n * 4;
    if (inverse) k_permute<true><<<blocks, kWarps * 32, sm, (cudaStream_t)stream>>>(d_data, d_order, n, n_vecs);
    else k_permute<false><<<blocks, kWarps * 32, sm, (cudaStream_t)stream>>>(d_data, d_order, n, n_vecs);
    sp_check_cuda(cudaGetLastError(), "mobius launch");
}

void sp_cuda_mobius_reorder(float *d_data, const int *d_order, int n, int n_vecs, void *stream)
{
    permute(d_data, d_order, n, n_vecs, stream, false);
}

void sp_cuda_mobius_unreorder(float *d_data, const int *d_order, int n, int n_vecs, void *stream)
{
    permute(d_data, d_order, n, n_vecs, stream, true);
}

void sp_cuda_band_quantize(const float *d_input, void *d_output, const sp_band_config_t *bc,
                           int n_vecs, void *stream)
{
    sp_clear_error();
    if (!bc) { sp_set_error(SP_ERR_ARG, "band_quantize: bc is NULL"); return; }
    SpBandLayout bl = sp_layout_from(*bc);
    sp_launch_encode(d_input, SP_DTYPE_F32, n_vecs, 1, (uint8_t *)d_output, 0, 0, 0,
                     nullptr, false, bl, (cudaStream_t)stream);
}

void sp_cuda_band_dequantize(const void *d_input, float *d_output, const sp_band_config_t *bc,
                             int n_vecs, void *stream)
{
    sp_clear_error();
    if (!bc) { sp_set_error(SP_ERR_ARG, "band_dequantize: bc is NULL"); return; }
    SpBandLayout bl = sp_layout_from(*bc);
    sp_launch_decode((const uint8_t *)d_input, 0, 0, 0, n_vecs, d_output, nullptr, false, -1,
                     bl, (cudaStream_t)stream);
}

}  // extern "C"
