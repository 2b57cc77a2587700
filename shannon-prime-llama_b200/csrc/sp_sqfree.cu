// sp_sqfree.cu — sqfree+spinor and hierarchical-Vilenkin caches on sm_100a:
// compress, decompress and (sqfree) fused decode attention, plus the
// reference-named C-ABI of shannon_prime_cuda.h.
//
// Both paths share one pipeline (reference shannon_prime_sqfree.cu:750-1069,
// shannon_prime_hier.cu:399-571), here fused into single kernels instead of
// the reference's ~10 launches per vector:
//   write: pad head_dim -> pad_dim with the mean; staged Vilenkin (prime
//          Hartley) transform; skeleton coefficients band-quantised; the
//          other coefficients predicted from the skeleton (sqfree: Möbius CSR
//          sum with the spinor sheet bit; hier: W . skeleton with fp16 W);
//          deviation magnitude; residual levels packed LSB-first.
//   read:  the inverse, predictions taken from the dequantised skeleton.
// One warp per vector; the padded vector lives in shared memory for the
// transform (stages of p = 2, 3, 5, 7, 11 at growing strides), every other
// intermediate in registers or a per-warp shared buffer; the packed slot is
// assembled in shared memory with bitwise ORs and stored by the warp.
//
// Exactness: every float step is the single operation the CPU restatement
// performs (the transform's cas table is built on the host in double and
// rounded once; each output is an fma chain over j ascending, then one
// multiply by 1/sqrt(p); sums over lanes use the fixed "lane tree": lane l
// sums elements l, l+32, ... in order, then an xor butterfly), so packed
// skeleton codes, magnitudes, residual levels and sheet bits are
// bit-identical to the CPU path.
#include "sp_internal.cuh"
#include "sp_bulk.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <algorithm>
#include <atomic>
#include <vector>
#include <type_traits>
#include <utility>

namespace {

constexpr int kSqMaxPd = 512;
constexpr int kSqWarps = 8;
constexpr int kSqRowWords = 160;     // per-warp slot buffer (640 B)
constexpr int kSqMaxStages = 8;

// Transform and layout description passed by value to every kernel.
struct SpSqDev {
    int hd, pd, nf;
    int p[kSqMaxStages];
    int cas_off[kSqMaxStages];
    float isp[kSqMaxStages];
    float cas[224];                   // concatenated p x p tables (2,3,5,7,11: 208)
    int n_skel, n_res, n_terms;
    int res_bits, use_spinor, hier;
    int mag_off, res_off, sheet_off, bytes_per_pos;
    SpBandLayout bl;                  // skeleton bands (bl.n = n_skel)
    const int *tables;                // skel_idx[n_skel], res_idx[n_res], csr_off[n_res+1], csr_term[n_terms]
};

__host__ __device__ inline int tab_skel(const SpSqDev &) { return 0; }
__host__ __device__ inline int tab_res(const SpSqDev &t) { return t.n_skel; }
__host__ __device__ inline int tab_csr_off(const SpSqDev &t) { return t.n_skel + t.n_res; }
__host__ __device__ inline int tab_csr_term(const SpSqDev &t) { return 2 * t.n_res + t.n_skel + 1; }
__host__ __device__ inline int tab_len(const SpSqDev &t) { return 2 * t.n_res + t.n_skel + 1 + t.n_terms; }

// ------------------------------------------------------------- device --

// Sum over the warp in the lane-tree order (all lanes get the result).
__device__ __forceinline__ float lane_tree_reduce(float s)
{
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s = s + __shfl_xor_sync(0xffffffffu, s, off);
    return s;
}

// One Vilenkin stage of prime P at the given stride: every group of P
// elements (stride apart) becomes its P x P Hartley transform.
template <int P>
__device__ __forceinline__ void vilenkin_stage(float *buf, int pd, int stride, const float *cas, float isp,
                                               int lane)
{
    const int bs = stride * P;
    const int groups = pd / P;
    for (int g = lane; g < groups; g += 32) {
        const int blk = g / stride, o = g - blk * stride;
        const int base = blk * bs + o;
        float x[P], y[P];
#pragma unroll
        for (int j = 0; j < P; j++) x[j] = buf[base + j * stride];
#pragma unroll
        for (int k = 0; k < P; k++) {
            float acc = 0.0f;
#pragma unroll
            for (int j = 0; j < P; j++) acc = __fmaf_rn(cas[k * P + j], x[j], acc);
            y[k] = __fmul_rn(acc, isp);
        }
#pragma unroll
        for (int k = 0; k < P; k++) buf[base + k * stride] = y[k];
    }
}

// In-place staged Vilenkin transform of buf[0..pd) by one warp: primes in
// ascending order, strides growing (reference shannon_prime_sqfree.cu:66-106).
__device__ void vilenkin_warp(float *buf, const SpSqDev &t, const float *cas_s, int lane)
{
    int stride = 1;
    for (int st = 0; st < t.nf; st++) {
        const float *cas = cas_s + t.cas_off[st];
        switch (t.p[st]) {
        case 2:  vilenkin_stage<2>(buf, t.pd, stride, cas, t.isp[st], lane); break;
        case 3:  vilenkin_stage<3>(buf, t.pd, stride, cas, t.isp[st], lane); break;
        case 5:  vilenkin_stage<5>(buf, t.pd, stride, cas, t.isp[st], lane); break;
        case 7:  vilenkin_stage<7>(buf, t.pd, stride, cas, t.isp[st], lane); break;
        default: vilenkin_stage<11>(buf, t.pd, stride, cas, t.isp[st], lane); break;
        }
        __syncwarp();
        stride *= t.p[st];
    }
}

// Hartley (cas) tables of the five primes, concatenated in the order
// 2, 3, 5, 7, 11 (offsets 0, 4, 13, 38, 87), and 1/sqrt(p) in the same
// order, as fp32 values computed on the host in double.  In constant memory
// every lane reads the same entry, so each fma takes its coefficient
// straight from the constant bank.
__constant__ float c_sq_cas[208];
__constant__ float c_sq_isp[5];

template <int P>
__host__ __device__ constexpr int prime_slot()
{
    return P == 2 ? 0 : P == 3 ? 1 : P == 5 ? 2 : P == 7 ? 3 : 4;
}
template <int P>
__host__ __device__ constexpr int cas_base()
{
    return P == 2 ? 0 : P == 3 ? 4 : P == 5 ? 13 : P == 7 ? 38 : 87;
}

// One stage of the compile-time transform: the same arithmetic as
// vilenkin_stage (an fma chain over j, then one multiply by 1/sqrt(p)), with
// the group layout fixed at compile time.
template <int PD, int P, int STRIDE>
__device__ __forceinline__ void vstage_c(float *buf, int lane)
{
    constexpr int groups = PD / P;
    const float isp = c_sq_isp[prime_slot<P>()];
#pragma unroll
    for (int g0 = 0; g0 < groups; g0 += 32) {
        const int g = g0 + lane;
        if (g < groups) {
            const int blk = g / STRIDE;
            const int base = blk * (STRIDE * P) + (g - blk * STRIDE);
            float x[P];
#pragma unroll
            for (int j = 0; j < P; j++) x[j] = buf[base + j * STRIDE];
#pragma unroll
            for (int k = 0; k < P; k++) {
                float acc = 0.0f;
#pragma unroll
                for (int j = 0; j < P; j++) acc = __fmaf_rn(c_sq_cas[cas_base<P>() + k * P + j], x[j], acc);
                buf[base + k * STRIDE] = __fmul_rn(acc, isp);
            }
        }
    }
}

// Compile-time staged transform of buf[0..PD) for the pad sizes of head_dim
// 32, 64, 128 and 256 (33 = 3.11, 66 = 2.3.11, 154 = 2.7.11,
// 330 = 2.3.5.11): primes ascending, strides growing.
template <int PD>
__device__ __forceinline__ void vilenkin_pd(float *buf, int lane)
{
    if constexpr (PD == 33) {
        vstage_c<33, 3, 1>(buf, lane); __syncwarp();
        vstage_c<33, 11, 3>(buf, lane); __syncwarp();
    } else if constexpr (PD == 66) {
        vstage_c<66, 2, 1>(buf, lane); __syncwarp();
        vstage_c<66, 3, 2>(buf, lane); __syncwarp();
        vstage_c<66, 11, 6>(buf, lane); __syncwarp();
    } else if constexpr (PD == 154) {
        vstage_c<154, 2, 1>(buf, lane); __syncwarp();
        vstage_c<154, 7, 2>(buf, lane); __syncwarp();
        vstage_c<154, 11, 14>(buf, lane); __syncwarp();
    } else {
        static_assert(PD == 330, "pad size without a compile-time plan");
        vstage_c<330, 2, 1>(buf, lane); __syncwarp();
        vstage_c<330, 3, 2>(buf, lane); __syncwarp();
        vstage_c<330, 5, 6>(buf, lane); __syncwarp();
        vstage_c<330, 11, 30>(buf, lane); __syncwarp();
    }
}

__host__ __device__ constexpr bool sq_fast_pd(int pd) { return pd == 33 || pd == 66 || pd == 154 || pd == 330; }

// Transform by the compile-time plan when PD names one, else by the
// table-driven stages.
template <int PD>
__device__ __forceinline__ void vilenkin_sel(float *buf, const SpSqDev &t, const float *cas_s, int lane)
{
    if constexpr (PD != 0) vilenkin_pd<PD>(buf, lane);
    else vilenkin_warp(buf, t, cas_s, lane);
}

// Row stride (floats) of the fp32 copy of W in shared memory: a multiple of
// 4 with an odd quotient, so the 16-byte loads of 8 consecutive rows hit
// distinct banks.
__host__ __device__ inline int hier_w_stride(int n_skel)
{
    int ws = (n_skel + 3) & ~3;
    if (((ws >> 2) & 1) == 0) ws += 4;
    return ws;
}

// W . skeleton for residual r with the skeleton held in registers (the fma
// chain in s order of hier_predict).
template <int NSK>
__device__ __forceinline__ float hier_predict_reg(const float *W, int ws, const float (&sk)[NSK], int r)
{
    const float *w = W + (size_t)r * ws;
    float acc = 0.0f;
#pragma unroll
    for (int s0 = 0; s0 < NSK; s0 += 4) {
        const float4 w4 = *reinterpret_cast<const float4 *>(w + s0);
        acc = __fmaf_rn(w4.x, sk[s0], acc);
        if (s0 + 1 < NSK) acc = __fmaf_rn(w4.y, sk[s0 + 1], acc);
        if (s0 + 2 < NSK) acc = __fmaf_rn(w4.z, sk[s0 + 2], acc);
        if (s0 + 3 < NSK) acc = __fmaf_rn(w4.w, sk[s0 + 3], acc);
    }
    return acc;
}

template <int NSK>
__device__ __forceinline__ void load_skel_regs(const float *skel, float (&sk)[NSK])
{
#pragma unroll
    for (int s = 0; s < NSK; s++) sk[s] = skel[s];
}

// OR the low `bits` bits of v into the packed row at bit position pos.
__device__ __forceinline__ void row_or(uint32_t *row, int pos, uint32_t v, int bits)
{
    const int w = pos >> 5, sh = pos & 31;
    if (v == 0) return;
    atomicOr(&row[w], v << sh);
    if (sh + bits > 32) atomicOr(&row[w + 1], v >> (32 - sh));
}

__device__ __forceinline__ uint32_t row_bits(const uint32_t *row, int pos, int bits)
{
    const int w = pos >> 5, sh = pos & 31;
    uint32_t v = row[w] >> sh;
    if (sh + bits > 32) v |= row[w + 1] << (32 - sh);
    return v & ((1u << bits) - 1u);
}

__device__ __forceinline__ float row_f16(const uint32_t *row, int byte)
{
    const unsigned short h = (unsigned short)row_bits(row, 8 * byte, 16);
    float f = __half2float(__ushort_as_half(h));
    return isfinite(f) ? f : 0.0f;
}

// Band of skeleton value s.
__device__ __forceinline__ int band_of_s(const SpBandLayout &bl, int s)
{
    int b = 0;
#pragma unroll 1
    for (int k = 1; k < bl.n_bands; k++)
        if (s >= bl.off[k]) b = k;
    return b;
}

// Band-quantise skel[0..n_skel) (shared) into the row (the ship quantiser:
// amax / max_val -> fp16 scale, codes rint(x / stored scale) + max_val).
__device__ void quantize_skeleton(const float *skel, uint32_t *row, const SpBandLayout &bl, int lane)
{
    for (int b = 0; b < bl.n_bands; b++) {
        const int off = bl.off[b], sz = bl.size[b], bits = bl.bits[b];
        float amax = 0.0f;
        for (int i = lane; i < sz; i += 32) amax = fmaxf(amax, fabsf(skel[off + i]));
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const int max_val = (1 << (bits - 1)) - 1;
        const float scale = amax > 0.0f ? __fdiv_rn(amax, (float)max_val) : 0.0f;
        const __half hs = __float2half_rn(scale);
        const float stored = __half2float(hs);
        const float inv = stored > 0.0f ? __frcp_rn(stored) : 0.0f;
        const int base = 8 * (bl.byte_off[b] + 2);
        for (int i = lane; i < sz; i += 32) {
            int q = __float2int_rn(__fmul_rn(skel[off + i], inv));
            q = q > max_val ? max_val : (q < -max_val ? -max_val : q);
            row_or(row, base + i * bits, (uint32_t)(q + max_val), bits);
        }
        if (lane == 0) row_or(row, 8 * bl.byte_off[b], (uint32_t)__half_as_ushort(hs), 16);
    }
}

// Dequantised skeleton value s from the row (partial bands never apply).
__device__ __forceinline__ float dequant_skel(const uint32_t *row, const SpBandLayout &bl, int s)
{
    const int b = band_of_s(bl, s);
    const int bits = bl.bits[b];
    const int max_val = (1 << (bits - 1)) - 1;
    const float scale = row_f16(row, bl.byte_off[b]);
    const uint32_t u = row_bits(row, 8 * (bl.byte_off[b] + 2) + (s - bl.off[b]) * bits, bits);
    return __fmul_rn((float)((int)u - max_val), scale);
}

// Sqfree Möbius prediction of residual r from skeleton values (shared).
__device__ __forceinline__ float csr_predict(const int *csr_off, const int *csr_term, const float *skel, int r)
{
    float p = 0.0f;
    for (int k = csr_off[r]; k < csr_off[r + 1]; k++) {
        const int term = csr_term[k];
        const float v = skel[term >> 1];
        p = (term & 1) ? __fsub_rn(p, v) : __fadd_rn(p, v);
    }
    return p;
}

__device__ __forceinline__ float hier_predict(const float *W, const float *skel, int n_skel, int r)
{
    const float *w = W + (size_t)r * hier_w_stride(n_skel);
    float acc = 0.0f;
    for (int s = 0; s < n_skel; s++) acc = __fmaf_rn(w[s], skel[s], acc);
    return acc;
}

struct SqIo {
    const void *in;              // write: [n_layers][n_tokens][nh][hd]
    float *out;                  // read:  [n_layers][n_pos][nh][hd] or [n_pos][hd] (one slot)
    uint8_t *cache;              // slab base
    long long slot_stride;       // bytes per slot
    int layer0, n_layers, nh, start_pos, n_tok;
    int tokens_per_cta;
    int store_width;             // 4, 2 or 1
    const __half *W;             // hier: [n_slots][n_res][n_skel]
    int single_slot;             // read of one (layer, head): output [n_pos][hd]
};

size_t sq_smem_bytes(const SpSqDev &t)
{
    size_t s = (size_t)tab_len(t) * 4 + 224 * 4;
    s += (size_t)kSqWarps * (t.pd + t.n_skel + t.n_res + 4) * 4;   // buf, skel, dev
    s += (size_t)kSqWarps * kSqRowWords * 4;
    if (t.hier) s += (size_t)t.n_res * hier_w_stride(t.n_skel) * 4;
    return s + 64;
}

struct SqSmem {
    int *tab;
    float *cas;
    float *buf, *skel, *dev;
    uint32_t *row;
    float *W;
};

__device__ SqSmem sq_carve(unsigned char *smem, const SpSqDev &t, int warp)
{
    SqSmem s;
    s.tab = reinterpret_cast<int *>(smem);
    s.cas = reinterpret_cast<float *>(s.tab + tab_len(t));
    float *f = s.cas + 224;
    const int per = t.pd + t.n_skel + t.n_res + 4;
    float *mine = f + (size_t)warp * per;
    s.buf = mine;
    s.skel = mine + t.pd;
    s.dev = s.skel + t.n_skel;
    s.row = reinterpret_cast<uint32_t *>(f + (size_t)kSqWarps * per) + warp * kSqRowWords;
    const uintptr_t w0 = reinterpret_cast<uintptr_t>(reinterpret_cast<uint32_t *>(f + (size_t)kSqWarps * per) +
                                                     kSqWarps * kSqRowWords);
    s.W = reinterpret_cast<float *>((w0 + 15) & ~uintptr_t(15));    // 16-byte rows for float4 loads
    return s;
}

__device__ void sq_load_common(unsigned char *smem, const SpSqDev &t, const SqIo &io, int slot)
{
    SqSmem s0 = sq_carve(smem, t, 0);
    for (int i = threadIdx.x; i < tab_len(t); i += blockDim.x) s0.tab[i] = t.tables[i];
    for (int i = threadIdx.x; i < 224; i += blockDim.x) s0.cas[i] = t.cas[i];
    if (t.hier) {
        const __half *w = io.W + (size_t)slot * t.n_res * t.n_skel;
        const int ws = hier_w_stride(t.n_skel);
        for (int i = threadIdx.x; i < t.n_res * t.n_skel; i += blockDim.x) {
            const int r = i / t.n_skel, c = i - r * t.n_skel;
            s0.W[r * ws + c] = __half2float(w[i]);
        }
    }
    __syncthreads();
}

// Compress.  Grid: x = token chunks, y = slot within the call (layer-major).
template <typename Tin, int PD>
__global__ void __launch_bounds__(kSqWarps * 32)
k_sq_encode(SpSqDev t, SqIo io)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int li = blockIdx.y / io.nh, h = blockIdx.y % io.nh;
    const int slot = (io.layer0 + li) * io.nh + h;
    sq_load_common(smem, t, io, slot);
    SqSmem S = sq_carve(smem, t, warp);
    const int *skel_idx = S.tab + tab_skel(t), *res_idx = S.tab + tab_res(t);
    const int *csr_off = S.tab + tab_csr_off(t), *csr_term = S.tab + tab_csr_term(t);
    const int words = (t.bytes_per_pos + 3) >> 2;
    const int tb = blockIdx.x * io.tokens_per_cta;
    const int te = min(io.n_tok, tb + io.tokens_per_cta);
    // The next vector's inputs (up to 8 per lane, head_dim <= 256) are
    // loaded into registers while the current one is processed.
    constexpr int KP = 8;
    auto src_of = [&](int tk) {
        return reinterpret_cast<const Tin *>(io.in) + (((long long)li * io.n_tok + tk) * io.nh + h) * t.hd;
    };
    const bool pre_ok = t.hd <= 32 * KP;
    float pre[KP];
    if (pre_ok && tb + warp < te) {
        const Tin *s0 = src_of(tb + warp);
#pragma unroll
        for (int k = 0; k < KP; k++) pre[k] = lane + 32 * k < t.hd ? sp_load_as_float(s0, lane + 32 * k) : 0.0f;
    }
    for (int tok = tb + warp; tok < te; tok += kSqWarps) {
        const Tin *src = src_of(tok);
        // pad with the lane-tree mean
        float sum = 0.0f;
        if (pre_ok) {
#pragma unroll
            for (int k = 0; k < KP; k++) {
                const int i = lane + 32 * k;
                if (i < t.hd) {
                    S.buf[i] = pre[k];
                    sum = __fadd_rn(sum, pre[k]);
                }
            }
            if (tok + kSqWarps < te) {
                const Tin *sn = src_of(tok + kSqWarps);
#pragma unroll
                for (int k = 0; k < KP; k++)
                    if (lane + 32 * k < t.hd) pre[k] = sp_load_as_float(sn, lane + 32 * k);
            }
        } else {
            for (int i = lane; i < t.hd; i += 32) {
                const float x = sp_load_as_float(src, i);
                S.buf[i] = x;
                sum = __fadd_rn(sum, x);
            }
        }
        const float mean = __fdiv_rn(lane_tree_reduce(sum), (float)t.hd);
        for (int i = t.hd + lane; i < t.pd; i += 32) S.buf[i] = mean;
        for (int j = lane; j < words; j += 32) S.row[j] = 0u;
        __syncwarp();
        vilenkin_sel<PD>(S.buf, t, S.cas, lane);
        for (int s = lane; s < t.n_skel; s += 32) S.skel[s] = S.buf[skel_idx[s]];
        __syncwarp();
        quantize_skeleton(S.skel, S.row, t.bl, lane);
        if (t.n_res > 0) {
            constexpr int NSK = PD > 0 ? PD / 11 : 1;    // hier skeleton size of the compile-time plans
            float asum = 0.0f;
            bool done = false;
            if constexpr (PD > 0) {
                if (t.hier) {
                    // the lane's W . skeleton predictions as independent fma
                    // chains (same per-lane order of the |d| sum)
                    constexpr int KR = (PD + 31) / 32;
                    float skr[NSK];
                    load_skel_regs(S.skel, skr);
#pragma unroll
                    for (int k = 0; k < KR; k++) {
                        const int r = lane + 32 * k;
                        if (r < t.n_res) {
                            const float p = hier_predict_reg<NSK>(S.W, hier_w_stride(NSK), skr, r);
                            const float d = __fsub_rn(S.buf[res_idx[r]], p);
                            S.dev[r] = d;
                            asum = __fadd_rn(asum, fabsf(d));
                        }
                    }
                    done = true;
                }
            }
            for (int r = lane; r < t.n_res && !done; r += 32) {
                const float a = S.buf[res_idx[r]];
                float d;
                if (t.hier) {
                    d = __fsub_rn(a, hier_predict(S.W, S.skel, t.n_skel, r));
                } else {
                    const float p = csr_predict(csr_off, csr_term, S.skel, r);
                    if (t.use_spinor) {
                        const float vp = __fsub_rn(a, p), vm = __fadd_rn(a, p);
                        const bool use_minus = fabsf(vm) < fabsf(vp);
                        d = use_minus ? vm : vp;
                        if (use_minus) row_or(S.row, 8 * t.sheet_off + r, 1u, 1);
                    } else {
                        d = __fsub_rn(a, p);
                    }
                }
                S.dev[r] = d;
                asum = __fadd_rn(asum, fabsf(d));
            }
            float mag = __fdiv_rn(lane_tree_reduce(asum), (float)t.n_res);
            if (mag < 1e-12f) mag = 1e-12f;
            const int L = 1 << t.res_bits;
            float inv, center;
            if (t.hier) {
                const float step = __fdiv_rn(__fmul_rn(2.0f, mag), (float)(L - 1));
                center = __fdiv_rn((float)(L - 1), 2.0f);
                inv = step > 0.0f ? __frcp_rn(step) : 0.0f;
            } else {
                center = __fmul_rn(0.5f, (float)(L - 1));
                const float sat = __fmul_rn(mag, (float)t.res_bits);
                const float step = __fdiv_rn(__fmul_rn(2.0f, sat), (float)(L - 1));
                inv = __frcp_rn(step);
            }
            __syncwarp();
            for (int r = lane; r < t.n_res; r += 32) {
                const float q = __fmaf_rn(S.dev[r], inv, center);
                int level = t.hier ? __float2int_rn(q) : (int)__fadd_rn(q, 0.5f);
                level = level < 0 ? 0 : (level >= L ? L - 1 : level);
                row_or(S.row, 8 * t.res_off + r * t.res_bits, (uint32_t)level, t.res_bits);
            }
            if (lane == 0) row_or(S.row, 8 * t.mag_off, __float_as_uint(mag) & 0xffffu, 16),
                           row_or(S.row, 8 * t.mag_off + 16, __float_as_uint(mag) >> 16, 16);
        }
        __syncwarp();
        uint8_t *dst = io.cache + (long long)slot * io.slot_stride +
                       (long long)(io.start_pos + tok) * t.bytes_per_pos;
        if (io.store_width == 4) {
            for (int j = lane; j < (t.bytes_per_pos >> 2); j += 32) reinterpret_cast<uint32_t *>(dst)[j] = S.row[j];
        } else if (io.store_width == 2) {
            const uint16_t *r16 = reinterpret_cast<const uint16_t *>(S.row);
            for (int j = lane; j < (t.bytes_per_pos >> 1); j += 32) reinterpret_cast<uint16_t *>(dst)[j] = r16[j];
        } else {
            const uint8_t *r8 = reinterpret_cast<const uint8_t *>(S.row);
            for (int j = lane; j < t.bytes_per_pos; j += 32) dst[j] = r8[j];
        }
        __syncwarp();
    }
}

// Load a packed slot into the warp's row buffer.
__device__ __forceinline__ void load_row(uint32_t *row, const uint8_t *src, int bytes, int width, int lane)
{
    if (width == 4) {
        for (int j = lane; j < (bytes >> 2); j += 32) row[j] = reinterpret_cast<const uint32_t *>(src)[j];
        if ((bytes & 3) && lane == 0) {
            uint32_t w = 0;
            for (int k = bytes & ~3; k < bytes; k++) w |= (uint32_t)src[k] << (8 * (k & 3));
            row[bytes >> 2] = w;
        }
    } else {
        uint8_t *r8 = reinterpret_cast<uint8_t *>(row);
        for (int j = lane; j < bytes; j += 32) r8[j] = src[j];
    }
    if (lane == 0) row[(bytes + 3) >> 2] = 0u;
}

// Coefficient vector of one packed slot into buf[0..pd) (before the inverse
// transform).  skel/dev are per-warp shared scratch.
template <int PD>
__device__ void sq_coeffs(const SpSqDev &t, const SqSmem &S, const float *W, int lane)
{
    const int *skel_idx = S.tab + tab_skel(t), *res_idx = S.tab + tab_res(t);
    const int *csr_off = S.tab + tab_csr_off(t), *csr_term = S.tab + tab_csr_term(t);
    for (int i = lane; i < t.pd; i += 32) S.buf[i] = 0.0f;
    for (int s = lane; s < t.n_skel; s += 32) S.skel[s] = dequant_skel(S.row, t.bl, s);
    __syncwarp();
    for (int s = lane; s < t.n_skel; s += 32) S.buf[skel_idx[s]] = S.skel[s];
    if (t.n_res > 0) {
        const float mag = __uint_as_float(row_bits(S.row, 8 * t.mag_off, 16) |
                                          (row_bits(S.row, 8 * t.mag_off + 16, 16) << 16));
        const int L = 1 << t.res_bits;
        float step, center;
        if (t.hier) {
            step = __fdiv_rn(__fmul_rn(2.0f, mag), (float)(L - 1));
            center = __fdiv_rn((float)(L - 1), 2.0f);
        } else {
            center = __fmul_rn(0.5f, (float)(L - 1));
            const float sat = __fmul_rn(mag, (float)t.res_bits);
            step = L > 1 ? __fdiv_rn(__fmul_rn(2.0f, sat), (float)(L - 1)) : 0.0f;
        }
        constexpr int NSK = PD > 0 ? PD / 11 : 1;
        if constexpr (PD > 0) {
            if (t.hier) {
                // lane's residuals as independent W . skeleton fma chains
                constexpr int KR = (PD + 31) / 32;
                float skr[NSK];
                __syncwarp();
                load_skel_regs(S.skel, skr);
#pragma unroll
                for (int k = 0; k < KR; k++) {
                    const int r = lane + 32 * k;
                    if (r < t.n_res) {
                        const uint32_t lv = row_bits(S.row, 8 * t.res_off + r * t.res_bits, t.res_bits);
                        const float dev = __fmul_rn(__fsub_rn((float)lv, center), step);
                        const float p = hier_predict_reg<NSK>(W, hier_w_stride(NSK), skr, r);
                        S.buf[res_idx[r]] = __fadd_rn(p, dev);
                    }
                }
                __syncwarp();
                return;
            }
        }
        for (int r = lane; r < t.n_res; r += 32) {
            const uint32_t lv = row_bits(S.row, 8 * t.res_off + r * t.res_bits, t.res_bits);
            const float dev = __fmul_rn(__fsub_rn((float)lv, center), step);
            float p;
            if (t.hier) {
                p = hier_predict(W, S.skel, t.n_skel, r);
            } else {
                p = csr_predict(csr_off, csr_term, S.skel, r);
                if (t.use_spinor && row_bits(S.row, 8 * t.sheet_off + r, 1)) p = -p;
            }
            S.buf[res_idx[r]] = __fadd_rn(p, dev);
        }
    }
    __syncwarp();
}

// Decompress.  Grid: x = position chunks, y = slot within the call.
template <int PD>
__global__ void __launch_bounds__(kSqWarps * 32)
k_sq_decode(SpSqDev t, SqIo io)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int li = blockIdx.y / io.nh, h = blockIdx.y % io.nh;
    const int slot = (io.layer0 + li) * io.nh + h;
    sq_load_common(smem, t, io, slot);
    SqSmem S = sq_carve(smem, t, warp);
    const int tb = blockIdx.x * io.tokens_per_cta;
    const int te = min(io.n_tok, tb + io.tokens_per_cta);
    for (int tok = tb + warp; tok < te; tok += kSqWarps) {
        const uint8_t *src = io.cache + (long long)slot * io.slot_stride +
                             (long long)(io.start_pos + tok) * t.bytes_per_pos;
        load_row(S.row, src, t.bytes_per_pos, io.store_width, lane);
        __syncwarp();
        sq_coeffs<PD>(t, S, S.W, lane);
        vilenkin_sel<PD>(S.buf, t, S.cas, lane);
        float *dst = io.single_slot ? io.out + (long long)tok * t.hd
                                    : io.out + (((long long)li * io.n_tok + tok) * io.nh + h) * t.hd;
        for (int i = lane; i < t.hd; i += 32) dst[i] = S.buf[i];
        __syncwarp();
    }
}

// ---------------------------------------------------- fused decode (sqfree) --

struct SqAttn {
    const uint8_t *k_cache, *v_cache;
    long long k_slot_stride, v_slot_stride;
    const __half *q;
    __half *out;
    float *ws;                    // partials [n_layers][n_q][kSqMaxSplits][pd + 4]
    int layer0, n_layers, n_kv_heads, n_q_heads, group, kv_len, chunk, n_splits;
    float logit_scale;
    int store_width_k, store_width_v;
    unsigned int *status;         // bit 0: a bounded copy wait ran out
    float *qws;                   // lane decode: transformed queries [n_layers][n_q][kSaQWords]
};

constexpr int kSqMaxSplits = 64;
constexpr int kSaQWords = 164;
constexpr int kSqAttnWarps = 4;

__device__ __forceinline__ float *sq_partial(const SqAttn &a, int pd, int li, int qh, int split)
{
    return a.ws + (((long long)li * a.n_q_heads + qh) * kSqMaxSplits + split) * (pd + 4);
}

size_t sq_attn_smem(const SpSqDev &t, int G)
{
    return (size_t)tab_len(t) * 4 + 224 * 4 + (size_t)G * t.pd * 4 +
           (size_t)kSqAttnWarps * ((t.pd + t.n_skel + t.n_res + 4) * 4 + kSqRowWords * 4) +
           (size_t)kSqAttnWarps * 8 * (t.pd + 4) * 4 + 64;
}

// Scores and the V sum in the Vilenkin coefficient domain: the transform is
// symmetric and self-inverse, so q . unpad(V(c)) = (V q_pad) . c with q_pad
// the query zero-extended to pad_dim, and sum_t p_t unpad(V(c_t)) =
// unpad(V(sum_t p_t c_t)).  One warp reconstructs one position's K
// coefficients (skeleton slots, then the CSR-predicted residuals) and V
// coefficients cooperatively.
__global__ void __launch_bounds__(kSqAttnWarps * 32)
k_sq_attn(SpSqDev tk, SpSqDev tv, SqAttn a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x, h = blockIdx.y, li = blockIdx.z;
    const int layer = a.layer0 + li;
    const int G = a.group, pd = tk.pd;
    // shared layout: tables(K) | cas | q'[G][pd] | per-warp (buf, skel, dev, row) | acc
    int *tab = reinterpret_cast<int *>(smem);
    float *cas = reinterpret_cast<float *>(tab + tab_len(tk));
    float *qp = cas + 224;
    float *wbase = qp + G * pd;
    const int per = pd + tk.n_skel + tk.n_res + 4;
    SqSmem S;
    S.tab = tab; S.cas = cas;
    S.buf = wbase + warp * per;
    S.skel = S.buf + pd;
    S.dev = S.skel + tk.n_skel;
    S.row = reinterpret_cast<uint32_t *>(wbase + kSqAttnWarps * per) + warp * kSqRowWords;
    S.W = nullptr;
    float *accs = reinterpret_cast<float *>(reinterpret_cast<uint32_t *>(wbase + kSqAttnWarps * per) +
                                            kSqAttnWarps * kSqRowWords);   // [warps][G][pd + 4]
    for (int i = threadIdx.x; i < tab_len(tk); i += blockDim.x) tab[i] = tk.tables[i];
    for (int i = threadIdx.x; i < 224; i += blockDim.x) cas[i] = tk.cas[i];
    __syncthreads();
    // Transformed queries (zero-padded), base-2 logit scale folded in.
    for (int g = warp; g < G; g += kSqAttnWarps) {
        const __half *qg = a.q + ((long long)li * a.n_q_heads + h * G + g) * tk.hd;
        float *b = qp + g * pd;
        for (int i = lane; i < pd; i += 32) b[i] = i < tk.hd ? __half2float(qg[i]) : 0.0f;
        __syncwarp();
        vilenkin_warp(b, tk, cas, lane);
        for (int i = lane; i < pd; i += 32) b[i] *= a.logit_scale * 1.4426950408889634f;
    }
    float *acc = accs + (size_t)warp * G * (pd + 4);
    for (int i = lane; i < G * (pd + 4); i += 32) acc[i] = 0.0f;
    __syncthreads();

    float m[8], l[8];
#pragma unroll
    for (int g = 0; g < 8; g++) { m[g] = -INFINITY; l[g] = 0.0f; }
    const long long slot = (long long)layer * a.n_kv_heads + h;
    const int t_begin = split * a.chunk, t_end = min(a.kv_len, t_begin + a.chunk);
    for (int tok = t_begin + warp; tok < t_end; tok += kSqAttnWarps) {
        // K coefficients -> scores
        load_row(S.row, a.k_cache + slot * a.k_slot_stride + (long long)tok * tk.bytes_per_pos,
                 tk.bytes_per_pos, a.store_width_k, lane);
        __syncwarp();
        sq_coeffs<0>(tk, S, nullptr, lane);
        float s[8];
#pragma unroll
        for (int g = 0; g < 8; g++) {
            float d = 0.0f;
            if (g < G)
                for (int i = lane; i < pd; i += 32) d = __fmaf_rn(qp[g * pd + i], S.buf[i], d);
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
            s[g] = d;
        }
        __syncwarp();
        // V coefficients, accumulated with online-softmax weights
        load_row(S.row, a.v_cache + slot * a.v_slot_stride + (long long)tok * tv.bytes_per_pos,
                 tv.bytes_per_pos, a.store_width_v, lane);
        __syncwarp();
        sq_coeffs<0>(tv, S, nullptr, lane);
#pragma unroll
        for (int g = 0; g < 8; g++) {
            if (g >= G) break;
            const float mn = fmaxf(m[g], s[g]);
            const float alpha = exp2f(m[g] - mn), p = exp2f(s[g] - mn);
            l[g] = l[g] * alpha + p;
            m[g] = mn;
            float *ag = acc + g * (pd + 4);
            for (int i = lane; i < pd; i += 32) ag[4 + i] = ag[4 + i] * alpha + p * S.buf[i];
        }
        __syncwarp();
    }
    if (lane == 0)
        for (int g = 0; g < G; g++) { acc[g * (pd + 4)] = m[g]; acc[g * (pd + 4) + 1] = l[g]; }
    __syncthreads();
    for (int g = 0; g < G; g++) {
        float M = -INFINITY;
        for (int w = 0; w < kSqAttnWarps; w++) M = fmaxf(M, accs[((size_t)w * G + g) * (pd + 4)]);
        float *part = sq_partial(a, pd, li, h * G + g, split);
        for (int i = threadIdx.x; i < pd + 1; i += blockDim.x) {
            float v = 0.0f;
            for (int w = 0; w < kSqAttnWarps; w++) {
                const float *aw = accs + ((size_t)w * G + g) * (pd + 4);
                const float wt = aw[0] == -INFINITY ? 0.0f : exp2f(aw[0] - M);
                v += wt * (i < pd ? aw[4 + i] : aw[1]);
            }
            if (i < pd) part[4 + i] = v;
            else { part[0] = M; part[1] = v; }
        }
    }
}

// Sum N per-lane values over the warp; every lane gets all N sums.  For N = 4
// the values are reduced in a transposed butterfly (2 + 1 + 3 shuffles and 4
// broadcasts instead of 20 shuffles).
template <int N>
__device__ __forceinline__ void warp_sum_multi(float (&v)[N], int lane)
{
    if constexpr (N == 4) {
        const bool b4 = lane & 16, b3 = lane & 8;
        float k0 = b4 ? v[2] : v[0], k1 = b4 ? v[3] : v[1];
        const float g0 = b4 ? v[0] : v[2], g1 = b4 ? v[1] : v[3];
        k0 += __shfl_xor_sync(0xffffffffu, g0, 16);
        k1 += __shfl_xor_sync(0xffffffffu, g1, 16);
        float kk = b3 ? k1 : k0;
        const float gg = b3 ? k0 : k1;
        kk += __shfl_xor_sync(0xffffffffu, gg, 8);
        kk += __shfl_xor_sync(0xffffffffu, kk, 4);
        kk += __shfl_xor_sync(0xffffffffu, kk, 2);
        kk += __shfl_xor_sync(0xffffffffu, kk, 1);
#pragma unroll
        for (int j = 0; j < 4; j++) v[j] = __shfl_sync(0xffffffffu, kk, 8 * j);
    } else {
#pragma unroll
        for (int j = 0; j < N; j++)
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
    }
}

constexpr int kSqRing = 4;          // positions prefetched ahead per warp

__host__ __device__ inline int sq_ring_row_words(const SpSqDev &tk, const SpSqDev &tv)
{
    const int w = (tk.bytes_per_pos > tv.bytes_per_pos ? tk.bytes_per_pos : tv.bytes_per_pos);
    return ((w + 3) >> 2) + 2;       // + guard words read past the row end
}

__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}

// Per-lane field descriptor: word << 16 | shift << 8 | (bits - 1) << 4 | band
// (bits 1..16), so a field is funnelshift(row[word], row[word + 1], shift)
// & mask(bits).
__device__ __forceinline__ int field_desc(int bitpos, int bits, int band)
{
    return ((bitpos >> 5) << 16) | ((bitpos & 31) << 8) | ((bits - 1) << 4) | band;
}

__device__ __forceinline__ uint32_t field_get(const uint32_t *row, int d)
{
    const int w = d >> 16, sh = (d >> 8) & 31, bm1 = (d >> 4) & 15;
    return __funnelshift_r(row[w], row[w + 1], sh) & ((2u << bm1) - 1u);
}

// Per-lane slot descriptor of skeleton value s.
__device__ __forceinline__ int slot_desc(const SpBandLayout &bl, int s)
{
    const int b = band_of_s(bl, s);
    return field_desc(8 * (bl.byte_off[b] + 2) + (s - bl.off[b]) * bl.bits[b], bl.bits[b], b);
}

// Skeleton values of the lane's KS slots from the row in smem (band scales
// converted once per row by lanes 0..n_bands-1 and fetched by shuffle).
template <int KS>
__device__ __forceinline__ void skel_values(const uint32_t *row, int scdesc, const int (&desc)[KS],
                                            const float (&offs)[KS], int n_skel, int lane, float (&val)[KS],
                                            float *skbuf)
{
    // lane b < n_bands converts band b's fp16 scale (0 if not finite)
    float bsc = __half2float(__ushort_as_half((unsigned short)field_get(row, scdesc)));
    bsc = fabsf(bsc) <= 65504.0f ? bsc : 0.0f;
#pragma unroll
    for (int k = 0; k < KS; k++) {
        const int d = desc[k];
        const float sc = __shfl_sync(0xffffffffu, bsc, d & 15);
        const float u = (float)field_get(row, d);
        const int s = lane + 32 * k;
        val[k] = s < n_skel ? (u - offs[k]) * sc : 0.0f;
        if (s < n_skel) skbuf[s] = val[k];
    }
}

constexpr int kSqMaxTerms = 8;       // Möbius terms per residual held in registers

// Residual coefficients of the lane's KR slots (after skel_values + syncwarp).
// terms[k][j]: the lane's CSR terms (skeleton slot << 1 | negative), nt[k]
// their count; step_mul = 2 * bits / (L - 1), so step = mag * step_mul.
template <int KR>
__device__ __forceinline__ void res_values(const uint32_t *row, int magw, const int (&lvdesc)[KR],
                                           const int (&shdesc)[KR], const int (&terms)[KR][kSqMaxTerms],
                                           const int (&nt)[KR], float center, float step_mul, const float *skbuf,
                                           float (&val)[KR])
{
    const float mag = __uint_as_float(__funnelshift_r(row[magw >> 8], row[(magw >> 8) + 1], magw & 31));
    const float step = mag * step_mul;
#pragma unroll
    for (int k = 0; k < KR; k++) {
        float p = 0.0f;
#pragma unroll
        for (int j = 0; j < kSqMaxTerms; j++) {
            if (j < nt[k]) {
                const float v = skbuf[terms[k][j] >> 1];
                p = (terms[k][j] & 1) ? p - v : p + v;
            }
        }
        const float lv = (float)field_get(row, lvdesc[k]);
        if (shdesc[k] >= 0 && field_get(row, shdesc[k])) p = -p;
        val[k] = nt[k] >= 0 ? p + (lv - center) * step : 0.0f;
    }
}

// Register-resident fused decode: lane l owns skeleton slots l, l+32, ...
// (KS of them) and residual slots l, l+32, ... (KR), holds its slots' q'
// entries and V accumulators in registers, and only the skeleton values go
// through shared memory (the Möbius prediction reads other lanes' slots).
__device__ __forceinline__ float ex2_fast(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int GT, int KS, int KR>
__global__ void __launch_bounds__(kSqAttnWarps * 32, 3)
k_sq_attn_reg(SpSqDev tk, SpSqDev tv, SqAttn a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x, h = blockIdx.y, li = blockIdx.z;
    const int layer = a.layer0 + li;
    const int G = a.group, pd = tk.pd;
    int *tab = reinterpret_cast<int *>(smem);
    float *cas = reinterpret_cast<float *>(tab + tab_len(tk));
    float *qp = cas + 224;                                       // [GT][pd]
    float *skb = qp + GT * pd + warp * (tk.n_skel + 4);          // per warp
    // per warp: a ring of kSqRing stages, each the K row then the V row
    const int rw = sq_ring_row_words(tk, tv);
    uint32_t *ring = reinterpret_cast<uint32_t *>(qp + GT * pd + kSqAttnWarps * (tk.n_skel + 4)) +
                     warp * kSqRing * 2 * rw;
    float *merge = reinterpret_cast<float *>(reinterpret_cast<uint32_t *>(qp + GT * pd + kSqAttnWarps * (tk.n_skel + 4)) +
                                             kSqAttnWarps * kSqRing * 2 * rw);    // [warps][GT][pd + 4]
    for (int i = threadIdx.x; i < tab_len(tk); i += blockDim.x) tab[i] = tk.tables[i];
    for (int i = threadIdx.x; i < 224; i += blockDim.x) cas[i] = tk.cas[i];
    __syncthreads();
    for (int g = warp; g < GT; g += kSqAttnWarps) {
        float *b = qp + g * pd;
        const __half *qg = a.q + ((long long)li * a.n_q_heads + h * G + g) * tk.hd;
        for (int i = lane; i < pd; i += 32) b[i] = (g < G && i < tk.hd) ? __half2float(qg[i]) : 0.0f;
        __syncwarp();
        vilenkin_warp(b, tk, cas, lane);
        for (int i = lane; i < pd; i += 32) b[i] *= a.logit_scale * 1.4426950408889634f;
    }
    __syncthreads();
    const int *skel_idx = tab + tab_skel(tk), *res_idx = tab + tab_res(tk);
    const int *csr_off = tab + tab_csr_off(tk), *csr_term = tab + tab_csr_term(tk);
    int terms[KR][kSqMaxTerms], nt[KR];
#pragma unroll
    for (int k = 0; k < KR; k++) {
        const int r = lane + 32 * k;
        nt[k] = r < tk.n_res ? csr_off[r + 1] - csr_off[r] : 0;
#pragma unroll
        for (int j = 0; j < kSqMaxTerms; j++) terms[k][j] = j < nt[k] ? csr_term[csr_off[r] + j] : 0;
    }
    const int Lr = 1 << tk.res_bits;
    const float center = 0.5f * (float)(Lr - 1);
    const float kmul = Lr > 1 ? 2.0f * (float)tk.res_bits / (float)(Lr - 1) : 0.0f;
    const float vmul = Lr > 1 ? 2.0f * (float)tv.res_bits / (float)(Lr - 1) : 0.0f;
    int kdesc[KS], vdesc[KS], lvk[KR], lvv[KR], shk[KR], shv[KR];
    float koffs[KS], voffs[KS];
    float qs[GT][KS], qr[GT][KR];
    const int ksc = field_desc(8 * tk.bl.byte_off[lane < tk.bl.n_bands ? lane : 0], 16, 0);
    const int vsc = field_desc(8 * tv.bl.byte_off[lane < tv.bl.n_bands ? lane : 0], 16, 0);
    const int kmag = ((8 * tk.mag_off) >> 5 << 8) | ((8 * tk.mag_off) & 31);
    const int vmag = ((8 * tv.mag_off) >> 5 << 8) | ((8 * tv.mag_off) & 31);
#pragma unroll
    for (int k = 0; k < KR; k++) {
        const int r = lane + 32 * k, rc = r < tk.n_res ? r : 0;
        lvk[k] = field_desc(8 * tk.res_off + rc * tk.res_bits, tk.res_bits, 0);
        lvv[k] = field_desc(8 * tv.res_off + rc * tv.res_bits, tv.res_bits, 0);
        shk[k] = tk.use_spinor ? field_desc(8 * tk.sheet_off + rc, 1, 0) : -1;
        shv[k] = tv.use_spinor ? field_desc(8 * tv.sheet_off + rc, 1, 0) : -1;
        if (r >= tk.n_res) nt[k] = -1;          // not a residual slot: value 0
    }
#pragma unroll
    for (int k = 0; k < KS; k++) {
        const int s = lane + 32 * k;
        const int sc = s < tk.n_skel ? s : 0;
        kdesc[k] = slot_desc(tk.bl, sc);
        vdesc[k] = slot_desc(tv.bl, sc);
        koffs[k] = (float)((1 << (tk.bl.bits[band_of_s(tk.bl, sc)] - 1)) - 1);
        voffs[k] = (float)((1 << (tv.bl.bits[band_of_s(tv.bl, sc)] - 1)) - 1);
#pragma unroll
        for (int g = 0; g < GT; g++) qs[g][k] = s < tk.n_skel ? qp[g * pd + skel_idx[s]] : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < KR; k++) {
        const int r = lane + 32 * k;
#pragma unroll
        for (int g = 0; g < GT; g++) qr[g][k] = r < tk.n_res ? qp[g * pd + res_idx[r]] : 0.0f;
    }
    float as[GT][KS], ar[GT][KR], m[GT], l[GT];
#pragma unroll
    for (int g = 0; g < GT; g++) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int k = 0; k < KS; k++) as[g][k] = 0.0f;
#pragma unroll
        for (int k = 0; k < KR; k++) ar[g][k] = 0.0f;
    }
    const long long slot = (long long)layer * a.n_kv_heads + h;
    const int t_begin = split * a.chunk, t_end = min(a.kv_len, t_begin + a.chunk);
    const uint8_t *kbase = a.k_cache + slot * a.k_slot_stride;
    const uint8_t *vbase = a.v_cache + slot * a.v_slot_stride;
    const int kw = tk.bytes_per_pos >> 2, vw = tv.bytes_per_pos >> 2;   // 4-byte rows (checked on the host)
    // Prefetch rows kSqRing positions ahead with 4-byte cp.async per lane.
    auto issue = [&](int tok, int st) {
        uint32_t *dk = ring + st * 2 * rw, *dv = dk + rw;
        if (tok < t_end) {
            const uint32_t *sk = reinterpret_cast<const uint32_t *>(kbase + (long long)tok * tk.bytes_per_pos);
            const uint32_t *svp = reinterpret_cast<const uint32_t *>(vbase + (long long)tok * tv.bytes_per_pos);
            for (int j = lane; j < kw; j += 32)
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dk + j)), "l"(sk + j) : "memory");
            for (int j = lane; j < vw; j += 32)
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dv + j)), "l"(svp + j) : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    if (lane == 0)
        for (int st = 0; st < kSqRing; st++) { ring[st * 2 * rw + kw] = 0u; ring[st * 2 * rw + rw + vw] = 0u; }
    __syncwarp();
    for (int st = 0; st < kSqRing; st++) issue(t_begin + warp + st * kSqAttnWarps, st);
    int it = 0;
    for (int tok = t_begin + warp; tok < t_end; tok += kSqAttnWarps, it++) {
        const int st = it % kSqRing;
        asm volatile("cp.async.wait_group %0;" ::"n"(kSqRing - 1) : "memory");
        __syncwarp();
        const uint32_t *row = ring + st * 2 * rw;
        // ---- K: scores ----
        float sv[KS], rv[KR];
        skel_values<KS>(row, ksc, kdesc, koffs, tk.n_skel, lane, sv, skb);
        __syncwarp();
        res_values<KR>(row, kmag, lvk, shk, terms, nt, center, kmul, skb, rv);
        float sc[GT];
#pragma unroll
        for (int g = 0; g < GT; g++) {
            float d = 0.0f;
#pragma unroll
            for (int k = 0; k < KS; k++) d = __fmaf_rn(qs[g][k], sv[k], d);
#pragma unroll
            for (int k = 0; k < KR; k++) d = __fmaf_rn(qr[g][k], rv[k], d);
            sc[g] = d;
        }
        warp_sum_multi<GT>(sc, lane);
        float p[GT];
#pragma unroll
        for (int g = 0; g < GT; g++) {
            if (sc[g] > m[g]) {                 // uniform across the warp
                const float alpha = ex2_fast(m[g] - sc[g]);
                m[g] = sc[g];
                l[g] *= alpha;
#pragma unroll
                for (int k = 0; k < KS; k++) as[g][k] *= alpha;
#pragma unroll
                for (int k = 0; k < KR; k++) ar[g][k] *= alpha;
            }
            p[g] = ex2_fast(sc[g] - m[g]);
            l[g] += p[g];
        }
        __syncwarp();
        // ---- V: accumulate ----
        row += rw;
        skel_values<KS>(row, vsc, vdesc, voffs, tv.n_skel, lane, sv, skb);
        __syncwarp();
        res_values<KR>(row, vmag, lvv, shv, terms, nt, center, vmul, skb, rv);
#pragma unroll
        for (int g = 0; g < GT; g++) {
#pragma unroll
            for (int k = 0; k < KS; k++) as[g][k] = __fmaf_rn(p[g], sv[k], as[g][k]);
#pragma unroll
            for (int k = 0; k < KR; k++) ar[g][k] = __fmaf_rn(p[g], rv[k], ar[g][k]);
        }
        __syncwarp();
        issue(tok + kSqRing * kSqAttnWarps, st);
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    // ---- merge the warps, write the CTA's partial ----
    float *mw = merge + (size_t)warp * GT * (pd + 4);
#pragma unroll
    for (int g = 0; g < GT; g++) {
#pragma unroll
        for (int k = 0; k < KS; k++) {
            const int s = lane + 32 * k;
            if (s < tk.n_skel) mw[g * (pd + 4) + 4 + skel_idx[s]] = as[g][k];
        }
#pragma unroll
        for (int k = 0; k < KR; k++) {
            const int r = lane + 32 * k;
            if (r < tk.n_res) mw[g * (pd + 4) + 4 + res_idx[r]] = ar[g][k];
        }
        if (lane == 0) { mw[g * (pd + 4)] = m[g]; mw[g * (pd + 4) + 1] = l[g]; }
    }
    __syncthreads();
    for (int g = 0; g < G; g++) {
        float M = -INFINITY;
        for (int w = 0; w < kSqAttnWarps; w++) M = fmaxf(M, merge[((size_t)w * GT + g) * (pd + 4)]);
        float *part = sq_partial(a, pd, li, h * G + g, split);
        for (int i = threadIdx.x; i < pd + 1; i += blockDim.x) {
            float v = 0.0f;
            for (int w = 0; w < kSqAttnWarps; w++) {
                const float *aw = merge + ((size_t)w * GT + g) * (pd + 4);
                const float wt = aw[0] == -INFINITY ? 0.0f : exp2f(aw[0] - M);
                v += wt * (i < pd ? aw[4 + i] : aw[1]);
            }
            if (i < pd) part[4 + i] = v;
            else { part[0] = M; part[1] = v; }
        }
    }
}

// ------------------------------------------- fused decode (sqfree), blocked --
// Register-resident decode over 4-position blocks staged by bulk copies.
// Per lane: KS consecutive skeleton slots (one 64-bit window per field,
// dequantised as ((u | 2^23 bits) - (2^23 + m_b)) * scale, which equals
// (u - m_b) * scale exactly), up to KR residual slots assigned on the host
// so that the Möbius terms are spread evenly (at most KT terms per lane,
// each an fma with a +-1 or 0 coefficient into one of the lane's residual
// sums, which adds or subtracts exactly as the CSR sum does).  Two positions
// are processed per step: their skeleton values share one 8-byte
// shared-memory word per slot, their 8 scores one transposed butterfly,
// and one softmax update covers both.
constexpr int kSq3Warps = 4;
constexpr int kSq3Stages = 4;
constexpr int kSq3Block = 4;           // positions per bulk copy
constexpr int kSq3LaneRes = 2;         // residual slots per lane in the assignment table

__host__ __device__ inline int sq3_tab_len(const SpSqDev &t) { return tab_len(t) + 32 * kSq3LaneRes; }

size_t sq_attn3_smem(const SpSqDev &tk, const SpSqDev &tv)
{
    size_t s = (size_t)sq3_tab_len(tk) * 4 + 224 * 4 + (size_t)4 * tk.pd * 4;
    s = (s + 7) & ~size_t(7);
    s += (size_t)kSq3Warps * 2 * (tk.n_skel + 2) * 4;
    s = (s + 15) & ~size_t(15);
    s += (size_t)kSq3Warps * kSq3Stages * kSq3Block * (tk.bytes_per_pos + tv.bytes_per_pos);
    s += (size_t)kSq3Warps * kSq3Stages * 8;
    s += (size_t)kSq3Warps * 4 * (tk.pd + 4) * 4;
    return s + 64;
}

// Sum of 8 values over the warp (all lanes get all 8 sums).
__device__ __forceinline__ void warp_sum8(float (&v)[8], int lane)
{
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
    float k[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float keep = b4 ? v[4 + i] : v[i], give = b4 ? v[i] : v[4 + i];
        k[i] = keep + __shfl_xor_sync(0xffffffffu, give, 16);
    }
    float m[2];
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const float keep = b3 ? k[2 + i] : k[i], give = b3 ? k[i] : k[2 + i];
        m[i] = keep + __shfl_xor_sync(0xffffffffu, give, 8);
    }
    float x = b2 ? m[1] : m[0];
    const float gx = b2 ? m[0] : m[1];
    x += __shfl_xor_sync(0xffffffffu, gx, 4);
    x += __shfl_xor_sync(0xffffffffu, x, 2);
    x += __shfl_xor_sync(0xffffffffu, x, 1);
    // lane with bits (b4, b3, b2) holds sum index 4*b4 + 2*b3 + b2
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = __shfl_sync(0xffffffffu, x, 4 * j);
}

// Per-lane field descriptors of one cache half (K or V).
template <int KS, int KR>
struct Sq3Fields {
    int wo[KS], sh[KS], bd[KS];        // byte offset of the field's word, shift, band
    uint32_t mk[KS];                   // code mask (0 for an absent slot)
    float mo[KS];                      // 2^23 + m_b (2^23 for an absent slot)
    int sc_wo, sc_sh;                  // lane b < n_bands: its band scale
    int mag_wo, mag_sh;
    int lwo[KR], lsh[KR], swo[KR], ssh[KR];
    uint32_t lmask;
    int spinor;
    float step_mul, center;
};

template <int KS, int KR>
__device__ __forceinline__ void sq3_fields(const SpSqDev &t, int lane, const int (&rr)[KR], Sq3Fields<KS, KR> &f)
{
#pragma unroll
    for (int k = 0; k < KS; k++) {
        const int s = KS * lane + k;
        const bool ok = s < t.n_skel;
        const int sc = ok ? s : 0;
        const int b = band_of_s(t.bl, sc);
        const int bits = t.bl.bits[b];
        const int pos = 8 * (t.bl.byte_off[b] + 2) + (sc - t.bl.off[b]) * bits;
        f.wo[k] = (pos >> 5) * 4;
        f.sh[k] = pos & 31;
        f.bd[k] = b;
        f.mk[k] = ok ? (1u << bits) - 1u : 0u;
        f.mo[k] = ok ? 8388608.0f + (float)((1 << (bits - 1)) - 1) : 8388608.0f;
    }
    const int bl = lane < t.bl.n_bands ? lane : 0;
    f.sc_wo = t.bl.byte_off[bl] / 4 * 4;
    f.sc_sh = 8 * (t.bl.byte_off[bl] & 3);
    f.mag_wo = t.mag_off / 4 * 4;
    f.mag_sh = 8 * (t.mag_off & 3);
#pragma unroll
    for (int j = 0; j < KR; j++) {
        const int r = rr[j] >= 0 ? rr[j] : 0;
        const int lp = 8 * t.res_off + r * t.res_bits, sp = 8 * t.sheet_off + r;
        f.lwo[j] = (lp >> 5) * 4;
        f.lsh[j] = lp & 31;
        f.swo[j] = (sp >> 5) * 4;
        f.ssh[j] = sp & 31;
    }
    f.lmask = (1u << t.res_bits) - 1u;
    f.spinor = t.use_spinor;
    const int L = 1 << t.res_bits;
    f.step_mul = L > 1 ? 2.0f * (float)t.res_bits / (float)(L - 1) : 0.0f;
    f.center = 0.5f * (float)(L - 1);
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr)
{
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ float2 lds_f2(uint32_t addr)
{
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
    return v;
}

__device__ __forceinline__ void sts_f2(uint32_t addr, float x, float y)
{
    asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(x), "f"(y) : "memory");
}

// 32 bits of a staged row starting at bit sh of the word at byte offset wo
// (row: shared-memory address).
__device__ __forceinline__ uint32_t sq3_word2(uint32_t row, int wo, int sh)
{
    return __funnelshift_r(lds32(row + wo), lds32(row + wo + 4), sh);
}

// Coefficient values of positions A (row rA) and B (row rA + bpp): the
// lane's skeleton slots (also stored to skb as (A, B) pairs) and residuals.
template <int KS, int KR, int KT>
__device__ __forceinline__ void sq3_values(uint32_t rA, int bpp, const Sq3Fields<KS, KR> &f,
                                           int n_bands, int n_skel, float *skb, uint32_t skb_s, int lane,
                                           const int (&toff)[KT], const float (&tcf)[KT], int n0,
                                           float (&vA)[KS], float (&vB)[KS], float (&cA)[KR], float (&cB)[KR])
{
    const uint32_t rB = rA + bpp;
    float scA = 0.0f, scB = 0.0f;
    if (lane < n_bands) {
        scA = __half2float(__ushort_as_half((unsigned short)(sq3_word2(rA, f.sc_wo, f.sc_sh) & 0xffffu)));
        scB = __half2float(__ushort_as_half((unsigned short)(sq3_word2(rB, f.sc_wo, f.sc_sh) & 0xffffu)));
        scA = fabsf(scA) <= 65504.0f ? scA : 0.0f;
        scB = fabsf(scB) <= 65504.0f ? scB : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < KS; k++) {
        const float sa = __shfl_sync(0xffffffffu, scA, f.bd[k]);
        const float sb = __shfl_sync(0xffffffffu, scB, f.bd[k]);
        const uint32_t xa = (sq3_word2(rA, f.wo[k], f.sh[k]) & f.mk[k]) | 0x4B000000u;
        const uint32_t xb = (sq3_word2(rB, f.wo[k], f.sh[k]) & f.mk[k]) | 0x4B000000u;
        vA[k] = __fmul_rn(__fsub_rn(__uint_as_float(xa), f.mo[k]), sa);
        vB[k] = __fmul_rn(__fsub_rn(__uint_as_float(xb), f.mo[k]), sb);
        const int s = KS * lane + k;
        if (s < n_skel) sts_f2(skb_s + 8 * s, vA[k], vB[k]);
    }
    __syncwarp();
    const float stepA = __uint_as_float(sq3_word2(rA, f.mag_wo, f.mag_sh)) * f.step_mul;
    const float stepB = __uint_as_float(sq3_word2(rB, f.mag_wo, f.mag_sh)) * f.step_mul;
    float pA[KR], pB[KR];
#pragma unroll
    for (int j = 0; j < KR; j++) { pA[j] = 0.0f; pB[j] = 0.0f; }
    static_assert(KR == 2, "two residual sums per lane");
#pragma unroll
    for (int t = 0; t < KT; t++) {
        const float2 v = lds_f2(skb_s + toff[t]);
        // terms t < n0 belong to the lane's first residual, the rest to the second
        const float c0 = t < n0 ? tcf[t] : 0.0f, c1 = t < n0 ? 0.0f : tcf[t];
        pA[0] = __fmaf_rn(c0, v.x, pA[0]);
        pB[0] = __fmaf_rn(c0, v.y, pB[0]);
        pA[1] = __fmaf_rn(c1, v.x, pA[1]);
        pB[1] = __fmaf_rn(c1, v.y, pB[1]);
    }
#pragma unroll
    for (int j = 0; j < KR; j++) {
        const uint32_t la = (sq3_word2(rA, f.lwo[j], f.lsh[j]) & f.lmask) | 0x4B000000u;
        const uint32_t lb = (sq3_word2(rB, f.lwo[j], f.lsh[j]) & f.lmask) | 0x4B000000u;
        const float da = __fmul_rn(__fsub_rn(__fsub_rn(__uint_as_float(la), 8388608.0f), f.center), stepA);
        const float db = __fmul_rn(__fsub_rn(__fsub_rn(__uint_as_float(lb), 8388608.0f), f.center), stepB);
        float a = pA[j], b = pB[j];
        if (f.spinor) {
            const uint32_t sa = sq3_word2(rA, f.swo[j], f.ssh[j]) << 31;   // sheet bit -> sign
            const uint32_t sb = sq3_word2(rB, f.swo[j], f.ssh[j]) << 31;
            a = __uint_as_float(__float_as_uint(a) ^ sa);
            b = __uint_as_float(__float_as_uint(b) ^ sb);
        }
        cA[j] = __fadd_rn(a, da);
        cB[j] = __fadd_rn(b, db);
    }
}

template <int KS, int KR, int KT>
__global__ void __launch_bounds__(kSq3Warps * 32, 3)
k_sq_attn3(SpSqDev tk, SpSqDev tv, SqAttn a)
{
    constexpr int GT = 4;
    extern __shared__ __align__(16) unsigned char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x, h = blockIdx.y, li = blockIdx.z;
    const int layer = a.layer0 + li;
    const int G = a.group, pd = tk.pd;
    const int ntab = sq3_tab_len(tk);
    int *tab = reinterpret_cast<int *>(smem);
    float *cas = reinterpret_cast<float *>(tab + ntab);
    float *qp = cas + 224;
    float *skb_all = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(qp + GT * pd) + 7) & ~uintptr_t(7));
    float *skb = skb_all + warp * 2 * (tk.n_skel + 2);
    const uint32_t skb_s = spb::smem_u32(skb);
    unsigned char *ring_all = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(skb_all + kSq3Warps * 2 * (tk.n_skel + 2)) + 15) & ~uintptr_t(15));
    const int kblk = kSq3Block * tk.bytes_per_pos, vblk = kSq3Block * tv.bytes_per_pos;
    const int stage_bytes = kblk + vblk;
    unsigned char *ring = ring_all + warp * kSq3Stages * stage_bytes;
    unsigned long long *bars = reinterpret_cast<unsigned long long *>(ring_all + kSq3Warps * kSq3Stages * stage_bytes);
    float *merge = reinterpret_cast<float *>(bars + kSq3Warps * kSq3Stages);

    // ---- copy ring: blocks of 4 positions, warp w takes blocks w, w+4, ...
    const int t_begin = split * a.chunk, t_end = min(a.kv_len, t_begin + a.chunk);
    const int n_blk = (t_end - t_begin + kSq3Block - 1) / kSq3Block;
    const int n_my = warp < n_blk ? (n_blk - warp + kSq3Warps - 1) / kSq3Warps : 0;
    const long long slot = (long long)layer * a.n_kv_heads + h;
    const uint8_t *kbase = a.k_cache + slot * a.k_slot_stride;
    const uint8_t *vbase = a.v_cache + slot * a.v_slot_stride;
    const uint32_t bar0 = spb::smem_u32(bars + warp * kSq3Stages);
    const uint32_t ring0 = spb::smem_u32(ring);
    uint64_t policy = 0;
    if (lane == 0) {
        for (int st = 0; st < kSq3Stages; st++) spb::mbar_init(bar0 + 8 * st, 1);
        spb::mbar_init_fence();
        policy = spb::evict_first_policy();
    }
    __syncwarp();
    // Block k of this warp: first position, and whether all 4 positions exist
    // (only those are bulk-copied; a ragged last block is loaded by lanes).
    auto blk_pos = [&](int k) { return t_begin + (warp + k * kSq3Warps) * kSq3Block; };
    auto issue = [&](int k) {
        const int p0 = blk_pos(k);
        if (p0 + kSq3Block > t_end) return;
        const int st = k % kSq3Stages;
        const uint32_t bar = bar0 + 8 * st, dst = ring0 + st * stage_bytes;
        spb::fence_proxy_async();
        spb::mbar_expect_tx(bar, stage_bytes);
        spb::bulk_g2s(dst, kbase + (long long)p0 * tk.bytes_per_pos, kblk, bar, policy);
        spb::bulk_g2s(dst + kblk, vbase + (long long)p0 * tv.bytes_per_pos, vblk, bar, policy);
    };
    if (lane == 0)
        for (int k = 0; k < kSq3Stages && k < n_my; k++) issue(k);

    // ---- tables, queries --------------------------------------------------
    for (int i = threadIdx.x; i < ntab; i += blockDim.x) tab[i] = tk.tables[i];
    for (int i = threadIdx.x; i < 224; i += blockDim.x) cas[i] = tk.cas[i];
    __syncthreads();
    for (int g = warp; g < GT; g += kSq3Warps) {
        float *b = qp + g * pd;
        const __half *qg = a.q + ((long long)li * a.n_q_heads + h * G + (g < G ? g : 0)) * tk.hd;
        for (int i = lane; i < pd; i += 32) b[i] = (g < G && i < tk.hd) ? __half2float(qg[i]) : 0.0f;
        __syncwarp();
        vilenkin_warp(b, tk, cas, lane);
        for (int i = lane; i < pd; i += 32) b[i] *= a.logit_scale * 1.4426950408889634f;
    }
    __syncthreads();
    const int *skel_idx = tab + tab_skel(tk), *res_idx = tab + tab_res(tk);
    const int *csr_off = tab + tab_csr_off(tk), *csr_term = tab + tab_csr_term(tk);
    const int *lane_res = tab + tab_len(tk);

    // ---- lane constants ---------------------------------------------------
    int rr[KR];
#pragma unroll
    for (int j = 0; j < KR; j++) rr[j] = lane_res[kSq3LaneRes * lane + j];
    // flattened Möbius terms: byte offset of the (A, B) skeleton pair and
    // the coefficient into each of the lane's residual sums
    int toff[KT], n0;
    float tcf[KT];
    {
        int n[KR], o[KR];
#pragma unroll
        for (int j = 0; j < KR; j++) {
            n[j] = rr[j] >= 0 ? csr_off[rr[j] + 1] - csr_off[rr[j]] : 0;
            o[j] = rr[j] >= 0 ? csr_off[rr[j]] : 0;
        }
#pragma unroll
        for (int t = 0; t < KT; t++) {
            int idx = t, which = -1;
#pragma unroll
            for (int j = 0; j < KR; j++) {
                if (which < 0 && idx < n[j]) which = j;
                else if (which < 0) idx -= n[j];
            }
            int term = 0;
#pragma unroll
            for (int j = 0; j < KR; j++)
                if (which == j) term = csr_term[o[j] + idx];
            toff[t] = which >= 0 ? 8 * (term >> 1) : 0;
            tcf[t] = which >= 0 ? ((term & 1) ? -1.0f : 1.0f) : 0.0f;
        }
        n0 = n[0];
    }
    // K and V rows share one layout (checked on the host)
    Sq3Fields<KS, KR> fk;
    sq3_fields<KS, KR>(tk, lane, rr, fk);
    float qs[GT][KS], qr[GT][KR];
#pragma unroll
    for (int g = 0; g < GT; g++) {
#pragma unroll
        for (int k = 0; k < KS; k++) {
            const int s = KS * lane + k;
            qs[g][k] = s < tk.n_skel ? qp[g * pd + skel_idx[s]] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < KR; j++) qr[g][j] = rr[j] >= 0 ? qp[g * pd + res_idx[rr[j]]] : 0.0f;
    }
    float as[GT][KS], ar[GT][KR], m[GT], l[GT];
#pragma unroll
    for (int g = 0; g < GT; g++) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int k = 0; k < KS; k++) as[g][k] = 0.0f;
#pragma unroll
        for (int j = 0; j < KR; j++) ar[g][j] = 0.0f;
    }

    // ---- blocks -----------------------------------------------------------
    bool failed = false;
    int k_fail = 0;
    for (int k = 0; k < n_my; k++) {
        const int st = k % kSq3Stages;
        const int p0 = blk_pos(k);
        const int nvalid = min(kSq3Block, t_end - p0);
        unsigned char *sk_row = ring + st * stage_bytes;
        unsigned char *sv_row = sk_row + kblk;
        const uint32_t sk_s = ring0 + st * stage_bytes, sv_s = sk_s + kblk;
        if (nvalid == kSq3Block) {
            if (!spb::wait_stage(bar0 + 8 * st, (k / kSq3Stages) & 1, a.status)) {
                failed = true;
                k_fail = k;
                break;
            }
        } else {
            // ragged last block: lanes copy the valid rows, zero the rest
            const int kw = tk.bytes_per_pos / 4, vw = tv.bytes_per_pos / 4;
            for (int i = lane; i < kSq3Block * kw; i += 32)
                reinterpret_cast<uint32_t *>(sk_row)[i] =
                    i < nvalid * kw ? reinterpret_cast<const uint32_t *>(kbase + (long long)p0 * tk.bytes_per_pos)[i] : 0u;
            for (int i = lane; i < kSq3Block * vw; i += 32)
                reinterpret_cast<uint32_t *>(sv_row)[i] =
                    i < nvalid * vw ? reinterpret_cast<const uint32_t *>(vbase + (long long)p0 * tv.bytes_per_pos)[i] : 0u;
            __syncwarp();
        }
#pragma unroll 1
        for (int pp = 0; pp < kSq3Block; pp += 2) {
            if (pp >= nvalid) break;
            const bool okB = pp + 1 < nvalid;
            float vA[KS], vB[KS], cA[KR], cB[KR];
            sq3_values<KS, KR, KT>(sk_s + pp * tk.bytes_per_pos, tk.bytes_per_pos, fk, tk.bl.n_bands, tk.n_skel,
                                   skb, skb_s, lane, toff, tcf, n0, vA, vB, cA, cB);
            float sc[8];
#pragma unroll
            for (int g = 0; g < GT; g++) {
                float dA = 0.0f, dB = 0.0f;
#pragma unroll
                for (int kk = 0; kk < KS; kk++) {
                    dA = __fmaf_rn(qs[g][kk], vA[kk], dA);
                    dB = __fmaf_rn(qs[g][kk], vB[kk], dB);
                }
#pragma unroll
                for (int j = 0; j < KR; j++) {
                    dA = __fmaf_rn(qr[g][j], cA[j], dA);
                    dB = __fmaf_rn(qr[g][j], cB[j], dB);
                }
                sc[g] = dA;
                sc[4 + g] = dB;
            }
            warp_sum8(sc, lane);
            __syncwarp();
            sq3_values<KS, KR, KT>(sv_s + pp * tv.bytes_per_pos, tv.bytes_per_pos, fk, tv.bl.n_bands, tv.n_skel,
                                   skb, skb_s, lane, toff, tcf, n0, vA, vB, cA, cB);
#pragma unroll
            for (int g = 0; g < GT; g++) {
                const float sA = sc[g], sB = okB ? sc[4 + g] : -INFINITY;
                const float mx = fmaxf(sA, sB);
                if (mx > m[g]) {                 // uniform across the warp
                    const float alpha = ex2_fast(m[g] - mx);
                    m[g] = mx;
                    l[g] *= alpha;
#pragma unroll
                    for (int kk = 0; kk < KS; kk++) as[g][kk] *= alpha;
#pragma unroll
                    for (int j = 0; j < KR; j++) ar[g][j] *= alpha;
                }
                const float pa = ex2_fast(sA - m[g]), pb = ex2_fast(sB - m[g]);
                l[g] += pa + pb;
#pragma unroll
                for (int kk = 0; kk < KS; kk++) as[g][kk] = __fmaf_rn(pb, vB[kk], __fmaf_rn(pa, vA[kk], as[g][kk]));
#pragma unroll
                for (int j = 0; j < KR; j++) ar[g][j] = __fmaf_rn(pb, cB[j], __fmaf_rn(pa, cA[j], ar[g][j]));
            }
            __syncwarp();
        }
        __syncwarp();
        if (lane == 0 && k + kSq3Stages < n_my) issue(k + kSq3Stages);
    }
    if (failed) {
        // bounded wait for this warp's bulk copies still in flight (blocks
        // k_fail .. k_fail + stages - 1 were issued) before the CTA exits
        for (int k = k_fail; k < n_my && k < k_fail + kSq3Stages; k++)
            if (blk_pos(k) + kSq3Block <= t_end)
                spb::wait_stage(bar0 + 8 * (k % kSq3Stages), (k / kSq3Stages) & 1, nullptr);
    }
    // ---- merge the warps, write the CTA's partial ---------------------------
    float *mw = merge + (size_t)warp * GT * (pd + 4);
#pragma unroll
    for (int g = 0; g < GT; g++) {
#pragma unroll
        for (int kk = 0; kk < KS; kk++) {
            const int s = KS * lane + kk;
            if (s < tk.n_skel) mw[g * (pd + 4) + 4 + skel_idx[s]] = as[g][kk];
        }
#pragma unroll
        for (int j = 0; j < KR; j++)
            if (rr[j] >= 0) mw[g * (pd + 4) + 4 + res_idx[rr[j]]] = ar[g][j];
        if (lane == 0) { mw[g * (pd + 4)] = m[g]; mw[g * (pd + 4) + 1] = l[g]; }
    }
    __syncthreads();
    for (int g = 0; g < G; g++) {
        float M = -INFINITY;
        for (int w = 0; w < kSq3Warps; w++) M = fmaxf(M, merge[((size_t)w * GT + g) * (pd + 4)]);
        float *part = sq_partial(a, pd, li, h * G + g, split);
        for (int i = threadIdx.x; i < pd + 1; i += blockDim.x) {
            float v = 0.0f;
            for (int w = 0; w < kSq3Warps; w++) {
                const float *aw = merge + ((size_t)w * GT + g) * (pd + 4);
                const float wt = aw[0] == -INFINITY ? 0.0f : exp2f(aw[0] - M);
                v += wt * (i < pd ? aw[4 + i] : aw[1]);
            }
            if (i < pd) part[4 + i] = v;
            else { part[0] = M; part[1] = v; }
        }
    }
}

size_t sq_attn_reg_smem(const SpSqDev &t, const SpSqDev &tv, int GT)
{
    return (size_t)tab_len(t) * 4 + 224 * 4 + (size_t)GT * t.pd * 4 + (size_t)kSqAttnWarps * (t.n_skel + 4) * 4 +
           (size_t)kSqAttnWarps * kSqRing * 2 * sq_ring_row_words(t, tv) * 4 +
           (size_t)kSqAttnWarps * GT * (t.pd + 4) * 4 + 64;
}

using SqAttnKernel = void (*)(SpSqDev, SpSqDev, SqAttn);

// Register-resident instantiations: (query group bound, skeleton slots per
// lane, residual slots per lane) for the sqfree shapes of head_dim 64, 128
// and 256 at skeleton fractions 0.5 and 0.75.
SqAttnKernel sq_attn_reg_kernel(int G, int KS, int KR, int *GT)
{
#define SQ_CASE(ks, kr)                                                                 \
    if (KS == ks && KR == kr) {                                                         \
        if (G <= 4) { *GT = 4; return k_sq_attn_reg<4, ks, kr>; }                       \
        *GT = 8; return k_sq_attn_reg<8, ks, kr>;                                       \
    }
    SQ_CASE(4, 2) SQ_CASE(3, 3) SQ_CASE(2, 1) SQ_CASE(2, 2) SQ_CASE(8, 3) SQ_CASE(6, 6)
#undef SQ_CASE
    return nullptr;
}

// Split merge of one (layer, query head): 128 threads.  The splits' maxima
// and sums are read in parallel, the weights go to shared memory, and every
// coefficient's sum over the splits keeps several independent loads in
// flight; one warp then applies the transform.
constexpr int kSqCombineThreads = 128;

__global__ void __launch_bounds__(kSqCombineThreads)
k_sq_attn_combine(SpSqDev t, SqAttn a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    float *cas = reinterpret_cast<float *>(smem);
    float *buf = cas + 224;
    float *wts = buf + ((t.pd + 3) & ~3);
    float *red = wts + kSqMaxSplits;                 // [4 warps][2]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int qh = blockIdx.x, li = blockIdx.y;
    for (int i = tid; i < 224; i += blockDim.x) cas[i] = t.cas[i];
    const int ns = a.n_splits;
    float m = -INFINITY, l = 0.0f;
    for (int s = tid; s < ns; s += blockDim.x) m = fmaxf(m, __ldcg(sq_partial(a, t.pd, li, qh, s)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[2 * warp] = m;
    __syncthreads();
    float M = red[0];
    for (int w = 1; w < kSqCombineThreads / 32; w++) M = fmaxf(M, red[2 * w]);
    for (int s = tid; s < kSqMaxSplits; s += blockDim.x) {
        float w = 0.0f;
        if (s < ns) {
            const float *p = sq_partial(a, t.pd, li, qh, s);
            const float ms = __ldcg(p);
            if (ms != -INFINITY) {
                w = exp2f(ms - M);
                l += w * __ldcg(p + 1);
            }
        }
        wts[s] = w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) red[2 * warp + 1] = l;
    __syncthreads();
    float L = 0.0f;
    for (int w = 0; w < kSqCombineThreads / 32; w++) L += red[2 * w + 1];
    for (int i = tid; i < t.pd; i += blockDim.x) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        int s = 0;
        for (; s + 4 <= ns; s += 4) {
#pragma unroll
            for (int u = 0; u < 4; u++) acc[u] += wts[s + u] * __ldcg(sq_partial(a, t.pd, li, qh, s + u) + 4 + i);
        }
        for (; s < ns; s++) acc[0] += wts[s] * __ldcg(sq_partial(a, t.pd, li, qh, s) + 4 + i);
        buf[i] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
    }
    __syncthreads();
    if (warp == 0) vilenkin_warp(buf, t, cas, lane);
    __syncthreads();
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
    __half *o = a.out + ((long long)li * a.n_q_heads + qh) * t.hd;
    for (int i = tid; i < t.hd; i += blockDim.x) o[i] = __float2half_rn(buf[i] * inv);
}

size_t sq_combine_smem(const SpSqDev &t)
{
    return (224 + ((t.pd + 3) & ~3) + kSqMaxSplits + 2 * (kSqCombineThreads / 32)) * sizeof(float);
}

// ------------------------------------------------ lane-per-vector sqfree --
// Compress for the sqfree+spinor layout at head_dim 128 (pad 154 = 2.7.11,
// skeleton of SK = 115 values (sk_frac 0.75), bands 5,4,4,4,5,
// 3-bit residuals, sheet bits).  One thread owns one whole vector, as in the
// ship lane encoder: the warp's 32 input rows arrive by tiled TMA copies
// (128-byte swizzle) from one elected lane, the pad mean, the 154-point
// staged transform, the skeleton quantiser, the Möbius CSR prediction, the
// spinor choice and the residual quantiser all run in the thread's registers
// with compile-time tables, and the 32 packed slots leave by one bulk store.
// Every float operation is the one k_sq_encode performs, in the same order
// (the lane-tree sums of the mean and of |dev| are replayed as the same
// tree), so slots are bit-identical.
constexpr int kSlPD = 154, kSlHD = 128, kSlNR = 3;   // pad, head_dim, residual bits
constexpr int kSlWarps = 4;
__host__ __device__ constexpr int sl_bits(int b) { return b == 0 || b == 4 ? 5 : 4; }

template <int SK>
struct SlTab {
    int skel[SK];
    int res[kSlPD - SK];
    int off[kSlPD - SK + 1];
    int term[384];                // (slot << 1) | negative
    int term_res[384];            // residual of each term
    int band_off[5], band_size[5], band_byte[5];
    int mag_off, res_off, sheet_off, bytes;
};

__host__ __device__ constexpr bool sl_sqfree(int m)
{
    for (int p = 2; p * p <= m; p++)
        if (m % (p * p) == 0) return false;
    return true;
}
__host__ __device__ constexpr int sl_mu(int m)
{
    int k = 0;
    for (int p = 2; p * p <= m; p++) {
        if (m % p == 0) {
            m /= p;
            if (m % p == 0) return 0;
            k++;
        }
    }
    if (m > 1) k++;
    return (k & 1) ? -1 : 1;
}

// The tables sp_cuda_sqfree_cache_init_ex builds (squarefree-first Knight
// ranking, residual CSR over proper divisors with Möbius signs, skeleton
// bands as sp_band_config_init) and the slot byte layout of sq_build_desc.
template <int SK>
__host__ __device__ constexpr SlTab<SK> sl_tab()
{
    SlTab<SK> t{};
    int rank[kSlPD] = {};
    int k = 0;
    for (int i = 0; i < kSlPD; i++) if (sl_sqfree(i + 1)) rank[k++] = i;
    for (int i = 0; i < kSlPD; i++) if (!sl_sqfree(i + 1)) rank[k++] = i;
    int slot_of[kSlPD] = {};
    for (int i = 0; i < kSlPD; i++) slot_of[i] = -1;
    for (int s = 0; s < SK; s++) { t.skel[s] = rank[s]; slot_of[rank[s]] = s; }
    int nr = 0;
    for (int i = 0; i < kSlPD; i++) if (slot_of[i] < 0) t.res[nr++] = i;
    int nt = 0;
    for (int r = 0; r < kSlPD - SK; r++) {
        t.off[r] = nt;
        const int n = t.res[r] + 1;
        for (int d = 1; d < n; d++) {
            if (n % d) continue;
            const int mu = sl_mu(n / d);
            if (!mu || slot_of[d - 1] < 0) continue;
            t.term_res[nt] = r;
            t.term[nt++] = (slot_of[d - 1] << 1) | (mu < 0 ? 1 : 0);
        }
    }
    t.off[kSlPD - SK] = nt;
    int byte = 0;
    for (int b = 0; b < 5; b++) {
        t.band_off[b] = b * (SK / 5);
        t.band_size[b] = b == 4 ? SK - 4 * (SK / 5) : SK / 5;
        t.band_byte[b] = byte;
        byte += 2 + (t.band_size[b] * sl_bits(b) + 7) / 8;
    }
    t.mag_off = byte;
    t.res_off = byte + 4;
    t.sheet_off = t.res_off + ((kSlPD - SK) * kSlNR + 7) / 8;
    t.bytes = t.sheet_off + (kSlPD - SK + 7) / 8;
    return t;
}

// The tables of the one compiled skeleton size, evaluated at compile time;
// device code reads them only inside constant expressions, so every table
// lookup becomes a register name.
constexpr int kSlSK = 115;
constexpr int kSlNRes = kSlPD - kSlSK;
constexpr SlTab<kSlSK> kSlTab = sl_tab<kSlSK>();
constexpr int kSlNT = kSlTab.off[kSlNRes];
constexpr int kSlBytes = kSlTab.bytes, kSlMagOff = kSlTab.mag_off, kSlResOff = kSlTab.res_off,
              kSlSheetOff = kSlTab.sheet_off;
// Byte offset of skeleton band b (bands of kSlSK / 5 values).
__host__ __device__ constexpr int sl_band_byte(int b)
{
    int byte = 0;
    for (int k = 0; k < b; k++) byte += 2 + ((kSlSK / 5) * sl_bits(k) + 7) / 8;
    return byte;
}

template <int I>
__device__ __forceinline__ float sl_skel_of(const float (&x)[kSlPD])
{
    constexpr int i = kSlTab.skel[I];
    return x[i];
}
template <int I>
__device__ __forceinline__ float sl_res_of(const float (&x)[kSlPD])
{
    constexpr int i = kSlTab.res[I];
    return x[i];
}
template <size_t... I>
__device__ __forceinline__ void sl_gather(const float (&x)[kSlPD], float (&sk)[kSlSK], float (&rs)[kSlNRes],
                                          std::index_sequence<I...>)
{
    ((sk[I] = sl_skel_of<I>(x)), ...);
}
template <size_t... I>
__device__ __forceinline__ void sl_gather_res(const float (&x)[kSlPD], float (&rs)[kSlNRes], std::index_sequence<I...>)
{
    ((rs[I] = sl_res_of<I>(x)), ...);
}
// CSR term K: pr[r] +/-= skeleton value (csr_predict's chain, term by term).
template <int K>
__device__ __forceinline__ void sl_term(float (&pr)[kSlNRes], const float (&sk)[kSlSK])
{
    constexpr int term = kSlTab.term[K], r = kSlTab.term_res[K], si = term >> 1;
    pr[r] = (term & 1) ? __fsub_rn(pr[r], sk[si]) : __fadd_rn(pr[r], sk[si]);
}
template <size_t... K>
__device__ __forceinline__ void sl_terms(float (&pr)[kSlNRes], const float (&sk)[kSlSK], std::index_sequence<K...>)
{
    (sl_term<K>(pr, sk), ...);
}

// One launch writes the K half (0) and/or the V half (1) of the same tokens.
// Skeleton and residual values back to coefficient positions (the inverse
// of sl_gather / sl_gather_res).
template <int I>
__device__ __forceinline__ void sl_put_skel(float (&x)[kSlPD], const float (&sk)[kSlSK])
{
    constexpr int i = kSlTab.skel[I];
    x[i] = sk[I];
}
template <int I>
__device__ __forceinline__ void sl_put_res(float (&x)[kSlPD], const float (&rs)[kSlNRes])
{
    constexpr int i = kSlTab.res[I];
    x[i] = rs[I];
}
template <size_t... I, size_t... R>
__device__ __forceinline__ void sl_scatter(float (&x)[kSlPD], const float (&sk)[kSlSK], const float (&rs)[kSlNRes],
                                           std::index_sequence<I...>, std::index_sequence<R...>)
{
    (sl_put_skel<I>(x, sk), ...);
    (sl_put_res<R>(x, rs), ...);
}

template <int SK>
struct SlArgs {
    uint8_t *cache[2];           // slab bases (head 0 of the slot numbering)
    long long slot_stride[2];
    int first, n_halves;         // first half present, 1 or 2 halves
    int layer0, n_layers, nh, start_pos, n_tok;
    int nb;                      // batches per half: n_layers * nh * ceil(n_tok / 32)
    unsigned int *status;
};

struct alignas(64) SlMap { CUtensorMap m[2]; };

template <typename Tin>
__device__ __forceinline__ void lane_unpack16_sq(const uint4 &w, float *x)
{
    if constexpr (sizeof(Tin) == 4) {
        x[0] = __uint_as_float(w.x); x[1] = __uint_as_float(w.y);
        x[2] = __uint_as_float(w.z); x[3] = __uint_as_float(w.w);
    } else {
        const Tin *hv = reinterpret_cast<const Tin *>(&w);
#pragma unroll
        for (int i = 0; i < 8; i++) x[i] = sp_load_as_float(hv, i);
    }
}
__device__ __forceinline__ void sl_bulk_s2g(void *dst, uint32_t src, uint32_t bytes)
{
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src), "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void sl_bulk_wait_read()
{
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

template <typename Tin>
struct SlSmem {
    static constexpr int RB = kSlHD * (int)sizeof(Tin);
    alignas(1024) unsigned char in[kSlWarps][32][RB];
    unsigned char out[kSlWarps][32 * 100];
    unsigned long long bar[kSlWarps];
};

// One stage of prime P at stride STRIDE of the compile-time plan, in the
// thread's registers (vstage_c's arithmetic).
template <int P, int STRIDE>
__device__ __forceinline__ void sl_stage(float (&x)[kSlPD])
{
    const float isp = c_sq_isp[prime_slot<P>()];
#pragma unroll
    for (int g = 0; g < kSlPD / P; g++) {
        const int blk = g / STRIDE, base = blk * (STRIDE * P) + (g - blk * STRIDE);
        float y[P];
#pragma unroll
        for (int kk = 0; kk < P; kk++) {
            float acc = 0.0f;
#pragma unroll
            for (int j = 0; j < P; j++) acc = __fmaf_rn(c_sq_cas[cas_base<P>() + kk * P + j], x[base + j * STRIDE], acc);
            y[kk] = __fmul_rn(acc, isp);
        }
#pragma unroll
        for (int kk = 0; kk < P; kk++) x[base + kk * STRIDE] = y[kk];
    }
}

// Sum of v[0..32) in the order lane_tree_reduce adds them across a warp.
__device__ __forceinline__ float sl_tree32(float (&v)[32])
{
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
        for (int j = 0; j < off; j++) v[j] = __fadd_rn(v[j], v[j + off]);
    return v[0];
}

template <typename Tin, int SK>
__global__ void __launch_bounds__(kSlWarps * 32, 2)
k_sq_encode_lane(SlArgs<SK> a, const __grid_constant__ SlMap map)
{
    static_assert(SK == kSlSK, "one compiled skeleton size");
    constexpr int NR = kSlPD - SK;
    constexpr int TB = kSlBytes;
    constexpr int W = (TB + 3) / 4;
    static_assert(TB % 4 == 0 && TB <= 100, "slot rows of whole words, at most 100 bytes");
    using S = SlSmem<Tin>;
    constexpr int RB = S::RB, C = RB / 16, NQ = RB / 128, EPC = 16 / (int)sizeof(Tin);
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    S &sm = *reinterpret_cast<S *>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t bar = spb::smem_u32(&sm.bar[warp]);
    const uint32_t in0 = spb::smem_u32(&sm.in[warp][0][0]);
    const int gw = blockIdx.x * kSlWarps + warp, n_w = gridDim.x * kSlWarps;
    const int nbt = (a.n_tok + 31) >> 5;
    const int n_total = a.nb * a.n_halves;
    if (in0 & 1023) {
        if (threadIdx.x == 0 && a.status) atomicOr(a.status, 4u);
        return;
    }
    if (lane == 0) {
        spb::mbar_init(bar, 1);
        spb::mbar_init_fence();
    }
    const uint64_t policy = spb::evict_first_policy();
    __syncwarp();
    // batch g: half first + g / nb; within it slot gl / nbt (layer-major,
    // then head), tokens 32 * (gl % nbt) ...
    auto issue = [&](int g) {
        if (lane == 0) {
            const int hx = a.first + g / a.nb, gl = g % a.nb;
            const int sl = gl / nbt, li = sl / a.nh, h = sl - li * a.nh, t0 = (gl - sl * nbt) * 32;
            const CUtensorMap *tm = hx ? &map.m[1] : &map.m[0];
            spb::mbar_expect_tx(bar, (uint32_t)(32 * RB));
#pragma unroll
            for (int q = 0; q < NQ; q++)
                asm volatile(
                    "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                    ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(in0 + q * 4096),
                    "l"(tm), "r"(q * (128 / (int)sizeof(Tin))), "r"(h), "r"(li * a.n_tok + t0), "r"(bar),
                    "l"(policy)
                    : "memory");
        }
    };
    uint32_t parity = 0;
    if (gw < n_total) issue(gw);
    for (int g = gw; g < n_total; g += n_w) {
        const int hx = a.first + g / a.nb, gl = g % a.nb;
        const int sl = gl / nbt, li = sl / a.nh, h = sl - li * a.nh, t0 = (gl - sl * nbt) * 32;
        const int live = min(32, a.n_tok - t0);
        if (!spb::wait_stage(bar, parity, a.status)) {
            spb::wait_stage(bar, parity, nullptr);
            break;
        }
        parity ^= 1u;
        float x[kSlPD];
#pragma unroll
        for (int j = 0; j < C; j++) {
            const int off = (j >> 3) * 4096 + lane * 128 + (((j & 7) ^ (lane & 7)) << 4);
            const uint4 w = *reinterpret_cast<const uint4 *>(&sm.in[warp][0][0] + off);
            lane_unpack16_sq<Tin>(w, &x[j * EPC]);
        }
        __syncwarp();
        spb::fence_proxy_async();
        if (g + n_w < n_total) issue(g + n_w);

        // ---- pad with the lane-tree mean ----
        {
            float part[32];
#pragma unroll
            for (int l = 0; l < 32; l++) {
                float s = 0.0f;
#pragma unroll
                for (int i = l; i < kSlHD; i += 32) s = __fadd_rn(s, x[i]);
                part[l] = s;
            }
            const float mean = __fdiv_rn(sl_tree32(part), (float)kSlHD);
#pragma unroll
            for (int i = kSlHD; i < kSlPD; i++) x[i] = mean;
        }
        // ---- staged transform 2.7.11 ----
        sl_stage<2, 1>(x);
        sl_stage<7, 2>(x);
        sl_stage<11, 14>(x);

        uint32_t row[W];
#pragma unroll
        for (int k = 0; k < W; k++) row[k] = 0u;
        auto put = [&](int p, uint32_t v, int bits) {
            row[p >> 5] |= v << (p & 31);
            if ((p & 31) + bits > 32) row[(p >> 5) + 1] |= v >> (32 - (p & 31));
        };
        // ---- skeleton / residual coefficients in table order ----
        float sk[kSlSK], rs[kSlNRes];
        sl_gather(x, sk, rs, std::make_index_sequence<kSlSK>{});
        sl_gather_res(x, rs, std::make_index_sequence<kSlNRes>{});
        // ---- skeleton bands (the ship quantiser) ----
        constexpr int BS = SK / 5;           // every band holds SK / 5 values
        static_assert(SK % 5 == 0, "equal skeleton bands");
#pragma unroll
        for (int b = 0; b < 5; b++) {
            const int bits = sl_bits(b), mv = (1 << (bits - 1)) - 1;
            float am[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int i = 0; i < BS; i++) am[i & 3] = fmaxf(am[i & 3], fabsf(sk[b * BS + i]));
            const float amax = fmaxf(fmaxf(am[0], am[1]), fmaxf(am[2], am[3]));
            const float scale = amax > 0.0f ? __fdiv_rn(amax, (float)mv) : 0.0f;
            const __half hs = __float2half_rn(scale);
            const float stored = __half2float(hs);
            const float inv = stored > 0.0f ? __frcp_rn(stored) : 0.0f;
            put(8 * sl_band_byte(b), (uint32_t)__half_as_ushort(hs), 16);
#pragma unroll
            for (int i = 0; i < BS; i++) {
                int q = __float2int_rn(__fmul_rn(sk[b * BS + i], inv));
                q = q > mv ? mv : (q < -mv ? -mv : q);
                put(8 * (sl_band_byte(b) + 2) + i * bits, (uint32_t)(q + mv), bits);
            }
        }
        // ---- residuals: Möbius prediction from the skeleton, spinor sheet ----
        float pr[NR];
#pragma unroll
        for (int r = 0; r < NR; r++) pr[r] = 0.0f;
        sl_terms(pr, sk, std::make_index_sequence<kSlNT>{});
        float dev[NR];
#pragma unroll
        for (int r = 0; r < NR; r++) {
            const float av = rs[r], p = pr[r];
            const float vp = __fsub_rn(av, p), vm = __fadd_rn(av, p);
            const bool use_minus = fabsf(vm) < fabsf(vp);
            const float d = use_minus ? vm : vp;
            put(8 * kSlSheetOff + r, use_minus ? 1u : 0u, 1);
            dev[r] = d;
        }
        // lane l of k_sq_encode sums |dev| of r = l, l + 32, ... in order
        float part[32];
#pragma unroll
        for (int l = 0; l < 32; l++) {
            float sacc = 0.0f;
#pragma unroll
            for (int r = l; r < NR; r += 32) sacc = __fadd_rn(sacc, fabsf(dev[r]));
            part[l] = sacc;
        }
        float mag = __fdiv_rn(sl_tree32(part), (float)NR);
        if (mag < 1e-12f) mag = 1e-12f;
        {
            constexpr int L = 1 << kSlNR;
            const float center = __fmul_rn(0.5f, (float)(L - 1));
            const float sat = __fmul_rn(mag, (float)kSlNR);
            const float step = __fdiv_rn(__fmul_rn(2.0f, sat), (float)(L - 1));
            const float inv = __frcp_rn(step);
#pragma unroll
            for (int r = 0; r < NR; r++) {
                const float q = __fmaf_rn(dev[r], inv, center);
                int level = (int)__fadd_rn(q, 0.5f);
                level = level < 0 ? 0 : (level >= L ? L - 1 : level);
                put(8 * kSlResOff + r * kSlNR, (uint32_t)level, kSlNR);
            }
            put(8 * kSlMagOff, __float_as_uint(mag), 32);
        }

        // ---- stage the 32 slots, write them back ----
        if (lane == 0) sl_bulk_wait_read();
        __syncwarp();
        unsigned char *stage = sm.out[warp];
        {
            uint32_t *r32 = reinterpret_cast<uint32_t *>(stage + lane * TB);
#pragma unroll
            for (int k = 0; k < TB / 4; k++) r32[k] = row[k];
        }
        spb::fence_proxy_async();
        __syncwarp();
        const int slot = (a.layer0 + li) * a.nh + h;
        uint8_t *dst = (hx ? a.cache[1] : a.cache[0]) + (long long)slot * (hx ? a.slot_stride[1] : a.slot_stride[0]) +
                       (long long)(a.start_pos + t0) * TB;
        const uint32_t bytes = (uint32_t)(live * TB);
        if ((((uintptr_t)dst | bytes) & 15) == 0) {
            if (lane == 0) sl_bulk_s2g(dst, spb::smem_u32(stage), bytes);
        } else {
            const uint32_t *s32 = reinterpret_cast<const uint32_t *>(stage);
            for (uint32_t i = lane; i < bytes / 4; i += 32) reinterpret_cast<uint32_t *>(dst)[i] = s32[i];
        }
        __syncwarp();
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Lane-per-vector read of the same layout: one thread per position
// rebuilds the 154 coefficients in registers (skeleton dequantised with the
// ship rule, residuals as the signed Möbius prediction plus the dequantised
// deviation, the order of sq_coeffs), runs the self-inverse transform and
// writes the first 128 values through a 128-byte-swizzled tile and tiled
// TMA stores.  Bit-identical with k_sq_decode.
struct alignas(64) SlOutMap { CUtensorMap m; };

struct SlReadSmem {
    alignas(1024) unsigned char out[kSlWarps][4][4096];
    alignas(16) uint32_t rows[kSlWarps][32 * 25];   // 32 slots of 100 bytes
    unsigned long long bar[kSlWarps];
};

// Slots a lane read covers: n_layers x n_heads slots, slot (l, h) at
// slab + (slot0 + l * n_heads + h) * slot_stride + pos0 * bytes_per_pos; its
// rows go to the output tensor at coordinates (h * hd, t, l).
struct SlGrid {
    long long slot_stride, slot0;
    int n_heads, n_layers, pos0;
};

__global__ void __launch_bounds__(kSlWarps * 32, 2)
k_sq_decode_lane(const uint8_t *slab, SlGrid g, int n_pos, unsigned int *status, const __grid_constant__ SlOutMap map)
{
    constexpr int NR = kSlNRes, TW = kSlBytes / 4;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    SlReadSmem &sm = *reinterpret_cast<SlReadSmem *>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t out0 = spb::smem_u32(&sm.out[warp][0][0]);
    if (out0 & 1023) {
        if (threadIdx.x == 0 && status) atomicOr(status, 4u);
        return;
    }
    const int n_bs = (n_pos + 31) >> 5;                 // batches per slot
    const long long n_b = (long long)n_bs * g.n_heads * g.n_layers;
    const long long b_step = (long long)gridDim.x * kSlWarps;
    // A full batch's 32 slots (3200 contiguous bytes) arrive by one bulk
    // copy when their start is 16-byte aligned, issued as soon as the
    // previous batch's fields are in registers; the lanes load ragged or
    // unaligned batches.
    const uint32_t bar0 = spb::smem_u32(&sm.bar[warp]);
    const uint32_t rows0 = spb::smem_u32(&sm.rows[warp][0]);
    uint64_t policy = 0;
    if (lane == 0) {
        spb::mbar_init(bar0, 1);
        spb::mbar_init_fence();
        policy = spb::evict_first_policy();
    }
    __syncwarp();
    auto batch_src = [&](long long bt, int &sl, int &t0, int &live) {
        sl = (int)(bt / n_bs);
        t0 = (int)(bt - (long long)sl * n_bs) * 32;
        live = min(32, n_pos - t0);
        return slab + (g.slot0 + sl) * g.slot_stride + (long long)(g.pos0 + t0) * kSlBytes;
    };
    auto next_src = [&](long long bt) -> const uint8_t * {
        if (bt >= n_b) return nullptr;
        int sl, t0, live;
        const uint8_t *src = batch_src(bt, sl, t0, live);
        return live == 32 && ((uintptr_t)src & 15) == 0 ? src : nullptr;
    };
    uint32_t par = 0u;
    bool pending = false, failed = false;
    auto issue = [&](const uint8_t *src) {
        if (!src) return;
        pending = true;
        if (lane == 0) {
            spb::fence_proxy_async();
            spb::mbar_expect_tx(bar0, 32 * kSlBytes);
            spb::bulk_g2s(rows0, src, 32 * kSlBytes, bar0, policy);
        }
    };
    long long bt = (long long)blockIdx.x * kSlWarps + warp;
    issue(next_src(bt));
    for (; bt < n_b; bt += b_step) {
        const uint8_t *nsrc = next_src(bt + b_step);
        int sl, t0, live;
        const uint8_t *srcb = batch_src(bt, sl, t0, live);
        const int l = sl / g.n_heads, hh = sl - l * g.n_heads;
        uint32_t *rows = sm.rows[warp];
        if (pending) {
            if (!spb::wait_stage(bar0, par, status)) {
                failed = true;                  // the copy may still land: waited for below
                break;
            }
            pending = false;
            par ^= 1u;
        } else {
            const uint32_t *src = reinterpret_cast<const uint32_t *>(srcb);
            for (int i = lane; i < live * TW; i += 32) rows[i] = src[i];
            __syncwarp();
        }
        const uint32_t *rw = rows + lane * TW;
        auto bits_at = [&](int p, int nb) -> uint32_t {
            const int w = p >> 5, sh = p & 31;
            uint32_t v = rw[w] >> sh;
            if (sh + nb > 32) v |= rw[w + 1] << (32 - sh);
            return nb == 32 ? v : (v & ((1u << nb) - 1u));
        };
        // skeleton values in slot order
        constexpr int BS = kSlSK / 5;
        float sk[kSlSK];
#pragma unroll
        for (int b = 0; b < 5; b++) {
            const int bits = sl_bits(b), mv = (1 << (bits - 1)) - 1;
            float scale = __half2float(__ushort_as_half((unsigned short)bits_at(8 * sl_band_byte(b), 16)));
            if (!isfinite(scale)) scale = 0.0f;
#pragma unroll
            for (int i = 0; i < BS; i++)
                sk[b * BS + i] =
                    __fmul_rn((float)((int)bits_at(8 * (sl_band_byte(b) + 2) + i * bits, bits) - mv), scale);
        }
        const float mag = __uint_as_float(bits_at(8 * kSlMagOff, 32));
        constexpr int L = 1 << kSlNR;
        const float center = __fmul_rn(0.5f, (float)(L - 1));
        const float sat = __fmul_rn(mag, (float)kSlNR);
        const float step = __fdiv_rn(__fmul_rn(2.0f, sat), (float)(L - 1));
        float pr[NR];
#pragma unroll
        for (int r = 0; r < NR; r++) pr[r] = 0.0f;
        sl_terms(pr, sk, std::make_index_sequence<kSlNT>{});
        float rs[NR];
#pragma unroll
        for (int r = 0; r < NR; r++) {
            const float lv = (float)bits_at(8 * kSlResOff + r * kSlNR, kSlNR);
            const float dev = __fmul_rn(__fsub_rn(lv, center), step);
            const float p = bits_at(8 * kSlSheetOff + r, 1) ? -pr[r] : pr[r];
            rs[r] = __fadd_rn(p, dev);
        }
        __syncwarp();                           // every lane's fields are in registers
        issue(nsrc);
        float x[kSlPD];
        sl_scatter(x, sk, rs, std::make_index_sequence<kSlSK>{}, std::make_index_sequence<NR>{});
        sl_stage<2, 1>(x);
        sl_stage<7, 2>(x);
        sl_stage<11, 14>(x);
        if (lane == 0) sl_bulk_wait_read();
        __syncwarp();
#pragma unroll
        for (int c = 0; c < kSlHD / 4; c++) {
            const int off = (c >> 3) * 4096 + lane * 128 + (((c & 7) ^ (lane & 7)) << 4);
            *reinterpret_cast<float4 *>(&sm.out[warp][0][0] + off) =
                make_float4(x[4 * c], x[4 * c + 1], x[4 * c + 2], x[4 * c + 3]);
        }
        spb::fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
#pragma unroll
            for (int q = 0; q < 4; q++)
                asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
                                 &map.m),
                             "r"(hh * kSlHD + q * 32), "r"(t0), "r"(l), "r"(out0 + q * 4096)
                             : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
    }
    if (failed && pending) spb::wait_stage(bar0, par, nullptr);
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// -------------------------------------------- fused decode, lane per slot --
// Fused decode attention for the same layout (k_sq_attn_lane): one thread
// rebuilds the 154 coefficients of one position's K (then V) slot in its
// registers from compile-time field offsets, as the lane read does, and the
// two contractions run on the tensor cores (mma.sync m16n8k16, fp16 in,
// fp32 accumulate) over a warp's 32 positions:
//   scores  S[32 pos][8]   = C_K[32 pos][160] x Q[160][8]
//   values  O[160][8]     += C_V^T[160][32 pos] x W[32 pos][8]
// with the 8 columns = 4 query heads x {hi, lo} fp16 halves of an fp32
// operand (the transformed query for K, the softmax weight for V).  The
// coefficient rows go through a per-warp shared-memory tile as fp16 (times
// 2^-4, which keeps any coefficient of a finite slot inside the fp16 range)
// and come back as MMA fragments by ldmatrix (transposed for the V side).
// Coefficients are in slot order: skeleton slots 0..114, residuals 0..38,
// six zero columns; the query is transformed once per CTA and gathered into
// the same order, so the score is the coefficient-domain dot product
// q'.c = q.unpad(V c) of the other decode kernels.
//
// Residual predictions are accumulated slot by slot (each skeleton value is
// added into the residuals whose Möbius terms name it, in slot order) so a
// thread keeps 39 running sums instead of all 115 skeleton values.
constexpr int kSaWarps = 4;
constexpr int kSaRowHalves = 168;                 // 160 + 8: conflict-free ldmatrix rows
constexpr int kSaTile = 32 * kSlBytes;            // 3200 bytes of K (or V) rows per tile

struct SaTerms {
    int slot[kSlNT], res[kSlNT], neg[kSlNT];
    int grp[16];                                  // first term of skeleton group k (slots 8k..8k+7)
};
__host__ __device__ constexpr SaTerms sa_terms()
{
    SaTerms t{};
    int n = 0;
    for (int s = 0; s < kSlSK; s++) {
        if ((s & 7) == 0) t.grp[s >> 3] = n;
        for (int k = 0; k < kSlNT; k++)
            if ((kSlTab.term[k] >> 1) == s) {
                t.slot[n] = s;
                t.res[n] = kSlTab.term_res[k];
                t.neg[n] = kSlTab.term[k] & 1;
                n++;
            }
    }
    for (int g = (kSlSK + 7) / 8; g < 16; g++) t.grp[g] = n;
    return t;
}
constexpr SaTerms kSaTerms = sa_terms();

// Row order of the lane decode's coefficient tile.  Skeleton slots that no
// Möbius term names are dequantised two per instruction in fp16x2
// arithmetic from a masked window of the row words (the fp32 path's value
// rounded to fp16, exactly); they take the first row positions, in pairs of
// one band whose codes fit the two halves of one 32-bit window.  The slots
// the predictions need follow in slot order on the fp32 path, then the
// residuals, then zero columns up to 160.
constexpr int kSaMaxPairs = 64;
struct SaPlan {
    int n_pairs, n_f32;
    int lo[kSaMaxPairs], hi[kSaMaxPairs];     // skeleton slot in the low / high half
    int win[kSaMaxPairs];                     // row bit where the pair's window starts
    int dlo[kSaMaxPairs], dhi[kSaMaxPairs];   // bit of each code inside its half
    int f32[kSlSK];                           // skeleton slots on the fp32 path, ascending
    int row[kSlPD];                           // row position of slot s (< kSlSK) or residual s - kSlSK
    int pd[160];                              // pad index at a row position, -1 for zero columns
};
__host__ __device__ constexpr SaPlan sa_plan()
{
    SaPlan p{};
    bool named[kSlSK] = {}, used[kSlSK] = {};
    for (int k = 0; k < kSlNT; k++) named[kSlTab.term[k] >> 1] = true;
    constexpr int BS = kSlSK / 5;
    for (int b = 0; b < 5; b++) {
        const int bits = sl_bits(b), n_b = b == 4 ? kSlSK - 4 * BS : BS;
        for (int i = 0; i < n_b; i++) {
            const int s = b * BS + i;
            if (named[s] || used[s]) continue;
            for (int dl = 3; dl <= 5; dl++) {
                const int t = s + dl, D = dl * bits;
                if (i + dl >= n_b || named[t] || used[t]) continue;
                const int d1 = D < 16 ? 16 - D : 0, d2 = d1 + D - 16;
                if (d1 + bits > 10 || d2 + bits > 10) continue;
                const int k = p.n_pairs++;
                p.lo[k] = s;
                p.hi[k] = t;
                p.win[k] = 8 * (sl_band_byte(b) + 2) + i * bits - d1;
                p.dlo[k] = d1;
                p.dhi[k] = d2;
                used[s] = used[t] = true;
                break;
            }
        }
    }
    for (int s = 0; s < kSlSK; s++)
        if (!used[s]) p.f32[p.n_f32++] = s;
    for (int k = 0; k < p.n_pairs; k++) { p.row[p.lo[k]] = 2 * k; p.row[p.hi[k]] = 2 * k + 1; }
    for (int k = 0; k < p.n_f32; k++) p.row[p.f32[k]] = 2 * p.n_pairs + k;
    for (int r = 0; r < kSlNRes; r++) p.row[kSlSK + r] = 2 * p.n_pairs + p.n_f32 + r;
    for (int j = 0; j < 160; j++) p.pd[j] = -1;
    for (int s = 0; s < kSlPD; s++) p.pd[p.row[s]] = s < kSlSK ? kSlTab.skel[s] : kSlTab.res[s - kSlSK];
    return p;
}
constexpr SaPlan kSaPlan = sa_plan();
static_assert(kSaPlan.n_pairs <= kSaMaxPairs && 2 * kSaPlan.n_pairs + kSaPlan.n_f32 == kSlSK, "row plan");

// Row position of pad index i.
struct SaPdIdx { int v[kSlPD]; };
__host__ __device__ constexpr SaPdIdx sa_pd_idx()
{
    SaPdIdx x{};
    for (int j = 0; j < 160; j++)
        if (kSaPlan.pd[j] >= 0) x.v[kSaPlan.pd[j]] = j;
    return x;
}
__constant__ SaPdIdx c_sa_j_of = sa_pd_idx();

template <int P, int NB>
__device__ __forceinline__ uint32_t sa_bits(const uint32_t (&w)[26])
{
    constexpr int i = P >> 5, s = P & 31;
    constexpr uint32_t m = NB == 32 ? 0xffffffffu : (1u << NB) - 1u;
    if constexpr (s + NB > 32) return __funnelshift_r(w[i], w[i + 1], s) & m;
    else return (w[i] >> s) & m;
}

// Skeleton value of slot S (times 2^-4): (u - m_b) * scale_b, exact.
template <int S>
__device__ __forceinline__ float sa_skel(const uint32_t (&w)[26], const float (&scl)[5])
{
    constexpr int BS = kSlSK / 5, b = S / BS, bits = sl_bits(b), mv = (1 << (bits - 1)) - 1;
    constexpr int pos = 8 * (sl_band_byte(b) + 2) + (S - b * BS) * bits;
    const uint32_t u = sa_bits<pos, bits>(w) | 0x4B000000u;
    return __fmul_rn(__fsub_rn(__uint_as_float(u), 8388608.0f + (float)mv), scl[b]);
}

template <int K>
__device__ __forceinline__ void sa_term(float (&pr)[kSlNRes], float v)
{
    constexpr int r = kSaTerms.res[K];
    constexpr bool neg = kSaTerms.neg[K] != 0;
    pr[r] = neg ? __fsub_rn(pr[r], v) : __fadd_rn(pr[r], v);
}
// Terms [B, E) of the slot-sorted list whose slot is S.
template <int S, int B, int E>
__device__ __forceinline__ void sa_terms_of(float (&pr)[kSlNRes], float v)
{
    if constexpr (B < E) {
        if constexpr (kSaTerms.slot[B] == S) sa_term<B>(pr, v);
        sa_terms_of<S, B + 1, E>(pr, v);
    }
}

__device__ __forceinline__ void sa_st4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d)
{
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}
__device__ __forceinline__ uint32_t sa_h2(float lo, float hi)
{
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

template <int B>
__device__ __forceinline__ float sa_scale(const uint32_t (&w)[26])
{
    const float s = __half2float(__ushort_as_half((unsigned short)sa_bits<8 * sl_band_byte(B), 16>(w)));
    return fabsf(s) <= 65504.0f ? __fmul_rn(s, 0.0625f) : 0.0f;
}
template <size_t... B>
__device__ __forceinline__ void sa_scales(const uint32_t (&w)[26], float (&scl)[5], std::index_sequence<B...>)
{
    ((scl[B] = sa_scale<(int)B>(w)), ...);
}
// Residual R (times 2^-4): the signed Möbius prediction plus the deviation.
template <int R>
__device__ __forceinline__ float sa_res(const uint32_t (&w)[26], const float (&pr)[kSlNRes], float step, float nc)
{
    const uint32_t lv = sa_bits<8 * kSlResOff + R * kSlNR, kSlNR>(w) | 0x4B000000u;
    const float dev = __fmaf_rn(__fsub_rn(__uint_as_float(lv), 8388608.0f), step, nc);
    const uint32_t sgn = sa_bits<8 * kSlSheetOff + R, 1>(w) << 31;
    return __fadd_rn(__uint_as_float(__float_as_uint(pr[R]) ^ sgn), dev);
}

// fp16 bits of a value fp16 holds exactly in its normal range (the
// constants of the paired dequantisation).
__host__ __device__ constexpr uint32_t sa_f16_bits(double x)
{
    const uint32_t sign = x < 0 ? 0x8000u : 0u;
    double a = x < 0 ? -x : x;
    int e = 0;
    while (a >= 2.0) { a /= 2.0; e++; }
    while (a < 1.0) { a *= 2.0; e--; }
    return sign | ((uint32_t)(e + 15) << 10) | (uint32_t)((a - 1.0) * 1024.0);
}
__host__ __device__ constexpr double sa_pow2(int e)
{
    double x = 1.0;
    for (; e > 0; e--) x *= 2.0;
    for (; e < 0; e++) x *= 0.5;
    return x;
}
// Band scale B as fp16x2 (both halves), zero if not finite.
template <int B>
__device__ __forceinline__ uint32_t sa_scale_h2(const uint32_t (&w)[26])
{
    const uint32_t h = sa_bits<8 * sl_band_byte(B), 16>(w);
    const uint32_t f = (h & 0x7C00u) == 0x7C00u ? 0u : h;
    return f | (f << 16);
}
// Pair K as one fp16x2 word: the window's two codes masked into halves
// 1024 + u * 2^d, one fma to (u - m) * 2^-4 (exact), one multiply by the
// band scale (the single rounding of the exact product, as the fp32 path's
// conversion).
template <int K>
__device__ __forceinline__ uint32_t sa_pair(const uint32_t (&w)[26], const uint32_t (&sb)[5])
{
    constexpr int b = kSaPlan.lo[K] / (kSlSK / 5), bits = sl_bits(b), mv = (1 << (bits - 1)) - 1;
    constexpr int W = kSaPlan.win[K], i = W >> 5, s = W & 31, d1 = kSaPlan.dlo[K], d2 = kSaPlan.dhi[K];
    constexpr uint32_t m = (1u << bits) - 1u;
    constexpr uint32_t mask = (m << d1) | (m << (16 + d2));
    constexpr uint32_t kk = sa_f16_bits(sa_pow2(-4 - d1)) | (sa_f16_bits(sa_pow2(-4 - d2)) << 16);
    constexpr uint32_t cc = sa_f16_bits(-(1024.0 + mv * sa_pow2(d1)) * sa_pow2(-4 - d1)) |
                            (sa_f16_bits(-(1024.0 + mv * sa_pow2(d2)) * sa_pow2(-4 - d2)) << 16);
    uint32_t win;
    if constexpr (s == 0) win = w[i];
    else win = __funnelshift_r(w[i], w[i + 1], s);
    const uint32_t x = (win & mask) | 0x64006400u;
    const __half2 v = __hfma2(*reinterpret_cast<const __half2 *>(&x), *reinterpret_cast<const __half2 *>(&kk),
                              *reinterpret_cast<const __half2 *>(&cc));
    const __half2 r = __hmul2_rn(v, *reinterpret_cast<const __half2 *>(&sb[b]));
    return *reinterpret_cast<const uint32_t *>(&r);
}

// What row position J holds: 0 pair, 1 fp32 skeleton slot, 2 residual, 3 zero.
__host__ __device__ constexpr int sa_kind(int j)
{
    return j < 2 * kSaPlan.n_pairs ? 0 : j < kSlSK ? 1 : j < kSlPD ? 2 : 3;
}
// Phase after which group G (row positions 8G..8G+7) is complete: 0 after
// the pairs, 1 + k after fp32 slot k, 1 + n_f32 after the residuals.
__host__ __device__ constexpr int sa_group_stage(int g)
{
    int st = 0;
    for (int j = 8 * g; j < 8 * g + 8; j++) {
        const int k = sa_kind(j);
        const int sj = k == 1 ? 1 + (j - 2 * kSaPlan.n_pairs) : k == 2 ? 1 + kSaPlan.n_f32 : 0;
        st = sj > st ? sj : st;
    }
    return st;
}
struct SaRowVals {
    float fv[kSlSK];      // fp32 skeleton values, by fp32-path index
    float rv[kSlNRes];    // residual coefficients
};
template <int J>
__device__ __forceinline__ float sa_val(const SaRowVals &v)
{
    constexpr int k = sa_kind(J);
    if constexpr (k == 1) return v.fv[J - 2 * kSaPlan.n_pairs];
    else if constexpr (k == 2) return v.rv[J - kSlSK];
    else return 0.0f;
}
template <int Wd>
__device__ __forceinline__ uint32_t sa_word(const uint32_t (&w)[26], const uint32_t (&sb)[5], const SaRowVals &v)
{
    if constexpr (2 * Wd + 1 < 2 * kSaPlan.n_pairs) return sa_pair<Wd>(w, sb);
    else return sa_h2(sa_val<2 * Wd>(v), sa_val<2 * Wd + 1>(v));
}
template <int ST, size_t... G>
__device__ __forceinline__ void sa_store_stage(const uint32_t (&w)[26], const uint32_t (&sb)[5], const SaRowVals &v,
                                               uint32_t row, std::index_sequence<G...>)
{
    ((sa_group_stage((int)G) == ST
          ? sa_st4(row + 16 * (int)G, sa_word<4 * (int)G>(w, sb, v), sa_word<4 * (int)G + 1>(w, sb, v),
                   sa_word<4 * (int)G + 2>(w, sb, v), sa_word<4 * (int)G + 3>(w, sb, v))
          : (void)0),
     ...);
}
template <int K>
__device__ __forceinline__ void sa_f32_slot(const uint32_t (&w)[26], const float (&scl)[5], const uint32_t (&sb)[5],
                                            float (&pr)[kSlNRes], SaRowVals &v, uint32_t row)
{
    constexpr int S = kSaPlan.f32[K];
    v.fv[K] = sa_skel<S>(w, scl);
    sa_terms_of<S, kSaTerms.grp[S >> 3], kSaTerms.grp[(S >> 3) + 1]>(pr, v.fv[K]);
    sa_store_stage<1 + K>(w, sb, v, row, std::make_index_sequence<20>{});
}
template <size_t... K>
__device__ __forceinline__ void sa_f32_slots(const uint32_t (&w)[26], const float (&scl)[5], const uint32_t (&sb)[5],
                                             float (&pr)[kSlNRes], SaRowVals &v, uint32_t row, std::index_sequence<K...>)
{
    (sa_f32_slot<(int)K>(w, scl, sb, pr, v, row), ...);
}

// Residual levels in pairs (r, r + 3..7) whose 3-bit codes fit the two
// halves of one 32-bit window: one fma turns both into lv - center exactly
// (fp16x2), and each residual is then one fp32 fma with the step onto its
// signed prediction.  An odd one left over takes sa_res.
struct SaResPlan {
    int n_pairs, n_left;
    int lo[kSlNRes], hi[kSlNRes], win[kSlNRes], dlo[kSlNRes], dhi[kSlNRes];
    int left[kSlNRes];
};
__host__ __device__ constexpr SaResPlan sa_res_plan()
{
    SaResPlan p{};
    bool used[kSlNRes] = {};
    for (int r = 0; r < kSlNRes; r++) {
        if (used[r]) continue;
        for (int dl = 5; dl <= 7; dl++) {
            const int t = r + dl, D = dl * kSlNR;
            if (t >= kSlNRes || used[t]) continue;
            // d >= 1 keeps 1024 + center * 2^d an fp16 integer
            const int d1 = D < 17 ? 17 - D : 1, d2 = d1 + D - 16;
            if (d1 + kSlNR > 10 || d2 + kSlNR > 10) continue;
            const int k = p.n_pairs++;
            p.lo[k] = r;
            p.hi[k] = t;
            p.win[k] = 8 * kSlResOff + r * kSlNR - d1;
            p.dlo[k] = d1;
            p.dhi[k] = d2;
            used[r] = used[t] = true;
            break;
        }
    }
    for (int r = 0; r < kSlNRes; r++)
        if (!used[r]) p.left[p.n_left++] = r;
    return p;
}
constexpr SaResPlan kSaResPlan = sa_res_plan();
__host__ __device__ constexpr int sa_left_res(int k) { return kSaResPlan.left[k]; }

// Every fp16x2 constant of both pair plans is exact in fp16 (checked at
// compile time: the paired dequantisation relies on it).
__host__ __device__ constexpr bool sa_f16_exact(double x)
{
    double a = x < 0 ? -x : x;
    int e = 0;
    while (a >= 2.0) { a /= 2.0; e++; }
    while (a < 1.0) { a *= 2.0; e--; }
    const double m = (a - 1.0) * 1024.0;
    return e >= -14 && e <= 15 && m == (double)(long long)m;
}
__host__ __device__ constexpr bool sa_plans_exact()
{
    for (int k = 0; k < kSaPlan.n_pairs; k++) {
        const int mv = (1 << (sl_bits(kSaPlan.lo[k] / (kSlSK / 5)) - 1)) - 1;
        for (int d : {kSaPlan.dlo[k], kSaPlan.dhi[k]})
            if (!sa_f16_exact(sa_pow2(-4 - d)) || !sa_f16_exact((1024.0 + mv * sa_pow2(d)) * sa_pow2(-4 - d)))
                return false;
    }
    for (int k = 0; k < kSaResPlan.n_pairs; k++)
        for (int d : {kSaResPlan.dlo[k], kSaResPlan.dhi[k]})
            if (!sa_f16_exact(sa_pow2(-d)) || !sa_f16_exact((1024.0 + 0.5 * ((1 << kSlNR) - 1) * sa_pow2(d)) * sa_pow2(-d)))
                return false;
    return true;
}
static_assert(sa_plans_exact(), "fp16x2 pair constants must be exact");

// Signed prediction of residual R: the sheet bit flips its sign.
template <int R>
__device__ __forceinline__ float sa_signed_pred(const uint32_t (&w)[26], const float (&pr)[kSlNRes])
{
    const uint32_t sgn = sa_bits<8 * kSlSheetOff + R, 1>(w) << 31;
    return __uint_as_float(__float_as_uint(pr[R]) ^ sgn);
}
template <int K>
__device__ __forceinline__ void sa_res_pair(const uint32_t (&w)[26], const float (&pr)[kSlNRes], float step,
                                            float *c)
{
    constexpr int W = kSaResPlan.win[K], i = W >> 5, s = W & 31, d1 = kSaResPlan.dlo[K], d2 = kSaResPlan.dhi[K];
    constexpr uint32_t m = (1u << kSlNR) - 1u, mask = (m << d1) | (m << (16 + d2));
    constexpr double ctr = 0.5 * ((1 << kSlNR) - 1);
    constexpr uint32_t kk = sa_f16_bits(sa_pow2(-d1)) | (sa_f16_bits(sa_pow2(-d2)) << 16);
    constexpr uint32_t cc = sa_f16_bits(-(1024.0 + ctr * sa_pow2(d1)) * sa_pow2(-d1)) |
                            (sa_f16_bits(-(1024.0 + ctr * sa_pow2(d2)) * sa_pow2(-d2)) << 16);
    uint32_t win;
    if constexpr (s == 0) win = w[i];
    else win = __funnelshift_r(w[i], w[i + 1], s);
    const uint32_t x = (win & mask) | 0x64006400u;
    const __half2 v = __hfma2(*reinterpret_cast<const __half2 *>(&x), *reinterpret_cast<const __half2 *>(&kk),
                              *reinterpret_cast<const __half2 *>(&cc));        // lv - center, both halves
    constexpr int rl = kSaResPlan.lo[K], rh = kSaResPlan.hi[K];
    c[rl] = __fmaf_rn(__low2float(v), step, sa_signed_pred<rl>(w, pr));
    c[rh] = __fmaf_rn(__high2float(v), step, sa_signed_pred<rh>(w, pr));
}
template <size_t... K>
__device__ __forceinline__ void sa_res_pairs(const uint32_t (&w)[26], const float (&pr)[kSlNRes], float step,
                                             float *c, std::index_sequence<K...>)
{
    (sa_res_pair<(int)K>(w, pr, step, c), ...);
}
template <size_t... K>
__device__ __forceinline__ void sa_res_left(const uint32_t (&w)[26], const float (&pr)[kSlNRes], float step,
                                            float nc, float *c, std::index_sequence<K...>)
{
    ((c[sa_left_res((int)K)] = sa_res<sa_left_res((int)K)>(w, pr, step, nc)), ...);
}

// One slot (row words in w, w[25] zero) to its fp16 staging row (shared-
// memory address row): 160 halves, coefficients times 2^-4 in row order
// (kSaPlan).  Predictions accumulate term by term in slot order, as the
// other decoders do.
__device__ __forceinline__ void sa_slot_row(const uint32_t (&w)[26], uint32_t row)
{
    uint32_t sb[5] = {sa_scale_h2<0>(w), sa_scale_h2<1>(w), sa_scale_h2<2>(w), sa_scale_h2<3>(w),
                      sa_scale_h2<4>(w)};
    SaRowVals v;
    sa_store_stage<0>(w, sb, v, row, std::make_index_sequence<20>{});
    float scl[5];
    sa_scales(w, scl, std::make_index_sequence<5>{});
    float pr[kSlNRes];
#pragma unroll
    for (int r = 0; r < kSlNRes; r++) pr[r] = 0.0f;
    sa_f32_slots(w, scl, sb, pr, v, row, std::make_index_sequence<kSaPlan.n_f32>{});
    constexpr int L = 1 << kSlNR;
    const float mag = __uint_as_float(sa_bits<8 * kSlMagOff, 32>(w));
    // step = 2 mag bits / (L - 1), times 2^-4 (one multiply; the decode
    // needs no bit-exact step)
    const float step = __fmul_rn(mag, (float)(2.0 * kSlNR / (L - 1) * 0.0625));
    const float nc = -0.5f * (float)(L - 1) * step;
    sa_res_pairs(w, pr, step, v.rv, std::make_index_sequence<kSaResPlan.n_pairs>{});
    sa_res_left(w, pr, step, nc, v.rv, std::make_index_sequence<kSaResPlan.n_left>{});
    sa_store_stage<1 + kSaPlan.n_f32>(w, sb, v, row, std::make_index_sequence<20>{});
}

__device__ __forceinline__ void sa_ldsm4(uint32_t addr, uint32_t (&r)[4])
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}
__device__ __forceinline__ void sa_ldsm4t(uint32_t addr, uint32_t (&r)[4])
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}
__device__ __forceinline__ void sa_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// fp16 of x (hi) or of x - fp16(x) (lo).
__device__ __forceinline__ __half sa_part(float x, int lo)
{
    const __half h = __float2half_rn(x);
    return lo ? __float2half_rn(x - __half2float(h)) : h;
}

struct SaSmem {
    uint32_t kring[kSaWarps][kSaTile / 4];          // one tile of K rows per warp
    uint32_t vring[kSaWarps][kSaTile / 4];          // and of V rows
    uint32_t ct[kSaWarps][32 * kSaRowHalves / 2];
    uint32_t wt[kSaWarps][8 * 20];                  // weights [column][position], 40-half rows
    unsigned long long bar[kSaWarps][2];            // K, V copy completion
    float q[4][160];                                // transformed queries, slot order, 2^F scaled
    int qf[4];
};

// The transformed queries of the lane decode, one warp per (layer, query
// head): q' = V q_pad * logit_scale * log2(e) in slot order (160 words, six
// zeros at the end), times 2^F with F chosen so max|q'| lands in [64, 128),
// and F itself in word 160.
struct SaPdOf { int v[160]; };
__host__ __device__ constexpr SaPdOf sa_pd_of_tab()
{
    SaPdOf x{};
    for (int j = 0; j < 160; j++) x.v[j] = kSaPlan.pd[j];
    return x;
}
__constant__ SaPdOf c_sa_pd_of = sa_pd_of_tab();

__global__ void __launch_bounds__(128)
k_sa_query(SqAttn a)
{
    __shared__ float qbuf[4][kSlPD + 2];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i = blockIdx.x * 4 + warp;
    if (i >= a.n_layers * a.n_q_heads) return;
    float *b = qbuf[warp];
    const __half *qg = a.q + (long long)i * kSlHD;
    for (int j = lane; j < kSlPD; j += 32) b[j] = j < kSlHD ? __half2float(qg[j]) : 0.0f;
    __syncwarp();
    vilenkin_pd<kSlPD>(b, lane);
    const float s = a.logit_scale * 1.4426950408889634f;
    float mx = 0.0f;
    for (int j = lane; j < kSlPD; j += 32) mx = fmaxf(mx, fabsf(b[j] * s));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int F = mx > 1e-30f ? 6 - ilogbf(mx) : 0;
    const float sf = ldexpf(s, F);
    float *o = a.qws + (long long)i * kSaQWords;
    for (int j = lane; j < 160; j += 32) {
        const int pi = c_sa_pd_of.v[j];
        o[j] = pi >= 0 ? b[pi] * sf : 0.0f;
    }
    if (lane == 0) o[160] = (float)F;
}

__global__ void __launch_bounds__(kSaWarps * 32, 3)
k_sq_attn_lane(SqAttn a)
{
    extern __shared__ __align__(128) unsigned char smem_raw[];
    SaSmem &sm = *reinterpret_cast<SaSmem *>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = lane >> 2, c = lane & 3;
    const int split = blockIdx.x, h = blockIdx.y, li = blockIdx.z;
    const int G = a.group;

    // ---- copies: tiles of 32 positions, warp w takes tiles w, w+4, ...;
    // one K and one V buffer per warp, each refilled as soon as its rows are
    // in registers, so a copy has the rest of the tile's work to land.
    const int t_begin = split * a.chunk, t_end = min(a.kv_len, t_begin + a.chunk);
    const int n_blk = (t_end - t_begin + 31) / 32;
    const int n_my = warp < n_blk ? (n_blk - warp + kSaWarps - 1) / kSaWarps : 0;
    const long long slot = (long long)(a.layer0 + li) * a.n_kv_heads + h;
    const uint8_t *kbase = a.k_cache + slot * a.k_slot_stride;
    const uint8_t *vbase = a.v_cache + slot * a.v_slot_stride;
    const uint32_t bar0 = spb::smem_u32(&sm.bar[warp][0]);
    const uint32_t kring0 = spb::smem_u32(&sm.kring[warp][0]), vring0 = spb::smem_u32(&sm.vring[warp][0]);
    uint64_t policy = 0;
    if (lane == 0) {
        spb::mbar_init(bar0, 1);
        spb::mbar_init(bar0 + 8, 1);
        spb::mbar_init_fence();
        policy = spb::evict_first_policy();
    }
    __syncwarp();
    auto blk_pos = [&](int k) { return t_begin + (warp + k * kSaWarps) * 32; };
    int issued_k = 0, issued_v = 0, waited_k = 0, waited_v = 0;   // copies issued / completions consumed
    auto issue = [&](int k, int half) {
        const int p0 = blk_pos(k);
        if (p0 + 32 > t_end) return;
        const uint32_t bar = bar0 + 8 * half;
        spb::fence_proxy_async();
        spb::mbar_expect_tx(bar, kSaTile);
        spb::bulk_g2s(half ? vring0 : kring0, (half ? vbase : kbase) + (long long)p0 * kSlBytes, kSaTile, bar,
                      policy);
        if (half) issued_v++; else issued_k++;
    };
    if (lane == 0 && n_my > 0) { issue(0, 0); issue(0, 1); }

    // ---- queries (k_sa_query's output for this layer and KV head) -------
    for (int i = threadIdx.x; i < 4 * 160; i += blockDim.x) {
        const int g = i / 160, j = i - g * 160;
        sm.q[g][j] = g < G ? a.qws[((long long)li * a.n_q_heads + h * G + g) * kSaQWords + j] : 0.0f;
    }
    if (threadIdx.x < 4) {
        const int g = threadIdx.x;
        sm.qf[g] = g < G ? (int)a.qws[((long long)li * a.n_q_heads + h * G + g) * kSaQWords + 160] : 0;
    }
    __syncthreads();
    // B fragments of the score MMAs: column r = query r/2, half r%2.
    uint32_t bq[10][2];
    {
        const int g = r >> 1, lo = r & 1;
#pragma unroll
        for (int ks = 0; ks < 10; ks++)
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                const int k0 = 16 * ks + 8 * hh + 2 * c;
                const __half2 v = __halves2half2(sa_part(sm.q[g][k0], lo), sa_part(sm.q[g][k0 + 1], lo));
                bq[ks][hh] = *reinterpret_cast<const uint32_t *>(&v);
            }
    }
    // score of query c = kc * (acc_hi + acc_lo): 2^-F for the query, 2^4 for
    // the coefficients
    const float kc = ldexpf(1.0f, 4 - sm.qf[c]);

    const uint32_t ct0 = spb::smem_u32(&sm.ct[warp][0]);
    const uint32_t my_row = ct0 + lane * (2 * kSaRowHalves);
    __half *wt = reinterpret_cast<__half *>(&sm.wt[warp][0]);
    const uint32_t wt0 = spb::smem_u32(wt);
    // ldmatrix row addresses: K side (rows = positions), V side (transposed)
    const int lq = lane >> 3, l8 = lane & 7;
    const uint32_t ka = ct0 + ((lq & 1) * 8 + l8) * (2 * kSaRowHalves) + (lq >> 1) * 16;
    const uint32_t va = ct0 + ((lq >> 1) * 8 + l8) * (2 * kSaRowHalves) + (lq & 1) * 16;

    float o[10][4];
#pragma unroll
    for (int mt = 0; mt < 10; mt++) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.0f;
    float m_run = -INFINITY, l_sum = 0.0f;

    bool failed = false;
    for (int k = 0; k < n_my; k++) {
        const int p0 = blk_pos(k);
        const int nvalid = min(32, t_end - p0);
        const uint32_t *krow = sm.kring[warp];
        const uint32_t *vrow = sm.vring[warp];
        if (nvalid < 32) {
            // ragged last tile (no copy was issued for it): lanes copy the
            // valid rows and zero the rest
            constexpr int TW = kSlBytes / 4;
            const uint32_t *ks = reinterpret_cast<const uint32_t *>(kbase + (long long)p0 * kSlBytes);
            const uint32_t *vs = reinterpret_cast<const uint32_t *>(vbase + (long long)p0 * kSlBytes);
            for (int i = lane; i < 32 * TW; i += 32) {
                sm.kring[warp][i] = i < nvalid * TW ? ks[i] : 0u;
                sm.vring[warp][i] = i < nvalid * TW ? vs[i] : 0u;
            }
            __syncwarp();
        }
        // K half, then V half; one copy of the (long, straight-line) slot
        // rebuild serves both.
#pragma unroll 1
        for (int half = 0; half < 2; half++) {
            if (nvalid == 32) {
                if (!spb::wait_stage(bar0 + 8 * half, (half ? waited_v : waited_k) & 1, a.status)) {
                    failed = true;
                    break;
                }
                if (half) waited_v++; else waited_k++;
            }
            {
                const uint32_t *rows = half ? vrow : krow;
                uint32_t w[26];
#pragma unroll
                for (int i = 0; i < 25; i++) w[i] = rows[lane * 25 + i];
                w[25] = 0u;
                __syncwarp();
                if (lane == 0 && k + 1 < n_my) issue(k + 1, half);
                sa_slot_row(w, my_row);
            }
            __syncwarp();
            if (half == 0) {
                // ---- scores, then the online softmax of query c over
                // positions r, r+8, 16+r, 24+r
                float s[2][4];
#pragma unroll
                for (int mt = 0; mt < 2; mt++) {
                    s[mt][0] = s[mt][1] = s[mt][2] = s[mt][3] = 0.0f;
#pragma unroll
                    for (int ks = 0; ks < 10; ks++) {
                        uint32_t af[4];
                        sa_ldsm4(ka + mt * 16 * (2 * kSaRowHalves) + ks * 32, af);
                        sa_mma(s[mt], af, bq[ks][0], bq[ks][1]);
                    }
                }
                float sc[4];
#pragma unroll
                for (int mt = 0; mt < 2; mt++)
#pragma unroll
                    for (int hh = 0; hh < 2; hh++) {
                        const int t = 16 * mt + 8 * hh + r;
                        sc[2 * mt + hh] = t < nvalid ? kc * (s[mt][2 * hh] + s[mt][2 * hh + 1]) : -INFINITY;
                    }
                float mx = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                if (mx > m_run) {
                    const float alpha = ex2_fast(m_run - mx);
                    m_run = mx;
                    l_sum *= alpha;
#pragma unroll
                    for (int mt = 0; mt < 10; mt++) {
                        o[mt][0] *= alpha; o[mt][1] *= alpha; o[mt][2] *= alpha; o[mt][3] *= alpha;
                    }
                }
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float p = ex2_fast(sc[i] - m_run);
                    l_sum += p;
                    const int t = 16 * (i >> 1) + 8 * (i & 1) + r;
                    const __half ph = __float2half_rn(p);
                    wt[(2 * c) * 40 + t] = ph;
                    wt[(2 * c + 1) * 40 + t] = __float2half_rn(p - __half2float(ph));
                }
            } else {
                // ---- values
                uint32_t bw[2][2];
#pragma unroll
                for (int kt = 0; kt < 2; kt++)
#pragma unroll
                    for (int hh = 0; hh < 2; hh++)
                        bw[kt][hh] = lds32(wt0 + 2 * (r * 40 + 16 * kt + 8 * hh + 2 * c));
#pragma unroll
                for (int mt = 0; mt < 10; mt++)
#pragma unroll
                    for (int kt = 0; kt < 2; kt++) {
                        uint32_t af[4];
                        sa_ldsm4t(va + kt * 16 * (2 * kSaRowHalves) + mt * 32, af);
                        sa_mma(o[mt], af, bw[kt][0], bw[kt][1]);
                    }
            }
            __syncwarp();
        }
        if (failed) break;
    }
    if (failed && lane == 0) {
        // bounded waits for this warp's copies still in flight before exit
        for (; waited_k < issued_k; waited_k++) spb::wait_stage(bar0, waited_k & 1, nullptr);
        for (; waited_v < issued_v; waited_v++) spb::wait_stage(bar0 + 8, waited_v & 1, nullptr);
    }
    __syncwarp();
    // ---- merge the warps, write the CTA's partial ---------------------------
#pragma unroll
    for (int o2 = 4; o2 < 32; o2 <<= 1) l_sum += __shfl_xor_sync(0xffffffffu, l_sum, o2);
    __syncwarp();
    float *mw = reinterpret_cast<float *>(&sm.ct[warp][0]);       // [4 queries][4 + 160]
#pragma unroll
    for (int mt = 0; mt < 10; mt++)
#pragma unroll
        for (int hh = 0; hh < 2; hh++)
            mw[c * 164 + 4 + 16 * mt + 8 * hh + r] = 16.0f * (o[mt][2 * hh] + o[mt][2 * hh + 1]);
    if (r == 0) { mw[c * 164] = m_run; mw[c * 164 + 1] = l_sum; }
    __syncthreads();
    for (int g = 0; g < G; g++) {
        float M = -INFINITY;
        for (int w = 0; w < kSaWarps; w++) M = fmaxf(M, reinterpret_cast<const float *>(&sm.ct[w][0])[g * 164]);
        float *part = sq_partial(a, kSlPD, li, h * G + g, split);
        for (int i = threadIdx.x; i < kSlPD + 1; i += blockDim.x) {
            const int j = i < kSlPD ? c_sa_j_of.v[i] : 0;
            float v = 0.0f;
            for (int w = 0; w < kSaWarps; w++) {
                const float *aw = reinterpret_cast<const float *>(&sm.ct[w][0]) + g * 164;
                const float wgt = aw[0] == -INFINITY ? 0.0f : exp2f(aw[0] - M);
                v += wgt * (i < kSlPD ? aw[4 + j] : aw[1]);
            }
            if (i < kSlPD) part[4 + i] = v;
            else { part[0] = M; part[1] = v; }
        }
    }
}

// --------------------------------------------------------------- host --

bool sq_squarefree(int m)
{
    for (int p = 2; p * p <= m; p++)
        if (m % (p * p) == 0) return false;
    return true;
}

int sq_mu(int m)
{
    int k = 0;
    for (int p = 2; p * p <= m; p++) {
        if (m % p == 0) {
            m /= p;
            if (m % p == 0) return 0;
            k++;
        }
    }
    if (m > 1) k++;
    return (k & 1) ? -1 : 1;
}

// Smallest squarefree {2,3,5,7,11}-smooth number >= hd.
int sq_pad_dim(int hd)
{
    for (int m = hd > 1 ? hd : 2; m <= 4 * kSqMaxPd; m++) {
        if (!sq_squarefree(m)) continue;
        int r = m;
        for (int p : {2, 3, 5, 7, 11})
            if (r % p == 0) r /= p;
        if (r == 1) return m;
    }
    return -1;
}

// Fill the transform part of t for pad_dim pd.
int sq_fill_transform(SpSqDev &t, int pd)
{
    t.pd = pd;
    t.nf = 0;
    int r = pd, off = 0;
    for (int p : {2, 3, 5, 7, 11}) {
        while (r % p == 0) {
            if (t.nf >= kSqMaxStages) return -1;
            t.p[t.nf] = p;
            t.cas_off[t.nf] = off;
            t.isp[t.nf] = (float)(1.0 / sqrt((double)p));
            bool seen = false;
            for (int k = 0; k < t.nf; k++)
                if (t.p[k] == p) { t.cas_off[t.nf] = t.cas_off[k]; seen = true; }
            if (!seen) {
                if (off + p * p > 224) return -1;
                for (int k = 0; k < p; k++)
                    for (int j = 0; j < p; j++) {
                        const double ang = 2.0 * 3.14159265358979323846 * (double)((k * j) % p) / (double)p;
                        t.cas[off + k * p + j] = (float)(cos(ang) + sin(ang));
                    }
                off += p * p;
            }
            t.nf++;
            r /= p;
        }
    }
    return r == 1 ? 0 : -1;
}

int store_width_for(int bytes, long long stride, const void *base)
{
    const uintptr_t x = (uintptr_t)bytes | (uintptr_t)stride | (uintptr_t)base;
    return (x & 3) == 0 ? 4 : ((x & 1) == 0 ? 2 : 1);
}

// Pad size of the compile-time plan for t (0: table-driven kernels).  The
// hier plans assume the skeleton of pad_dim / 11 values.
int sq_plan_pd(const SpSqDev &t)
{
    if (!sq_fast_pd(t.pd)) return 0;
    if (t.hier && t.n_skel != t.pd / 11) return 0;
    return t.pd;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point.
PFN_cuTensorMapEncodeTiled_v12000 sq_encode_fn()
{
    // looked up once, thread-safely (function-local static)
    static const PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        return nullptr;
    }();
    return fn;
}

// Whether t is the layout of the lane-per-vector sqfree encoder
// (sqfree+spinor, head_dim 128, pad 154, skeleton 115, bands 5,4,4,4,5,
// 3-bit residuals) and io's buffers suit it.
bool sq_lane_fits(const SpSqDev &t, const SqIo &io)
{
    constexpr const SlTab<kSlSK> &T = kSlTab;
    if (t.hier || !t.use_spinor || t.hd != kSlHD || t.pd != kSlPD || t.n_skel != kSlSK || t.n_res != kSlNRes ||
        t.res_bits != kSlNR || t.bl.n_bands != 5 || t.mag_off != T.mag_off || t.res_off != T.res_off ||
        t.sheet_off != T.sheet_off || t.bytes_per_pos != T.bytes || t.n_terms != T.off[kSlNRes])
        return false;
    for (int b = 0; b < 5; b++)
        if (t.bl.bits[b] != sl_bits(b) || t.bl.off[b] != T.band_off[b] || t.bl.size[b] != T.band_size[b] ||
            t.bl.byte_off[b] != T.band_byte[b])
            return false;
    return !(((uintptr_t)io.in & 15) || ((uintptr_t)io.cache & 3) || (io.slot_stride & 3));
}

// The fused lane decode's layout: the compiled config-2 slot.
bool sa_fits(const SpSqDev &t)
{
    constexpr const SlTab<kSlSK> &T = kSlTab;
    if (t.hier || !t.use_spinor || t.hd != kSlHD || t.pd != kSlPD || t.n_skel != kSlSK || t.n_res != kSlNRes ||
        t.res_bits != kSlNR || t.bl.n_bands != 5 || t.mag_off != T.mag_off || t.res_off != T.res_off ||
        t.sheet_off != T.sheet_off || t.bytes_per_pos != T.bytes || t.n_terms != T.off[kSlNRes])
        return false;
    for (int b = 0; b < 5; b++)
        if (t.bl.bits[b] != sl_bits(b) || t.bl.off[b] != T.band_off[b] || t.bl.size[b] != T.band_size[b] ||
            t.bl.byte_off[b] != T.band_byte[b])
            return false;
    return true;
}

bool sq_lane_map(CUtensorMap *m, const SqIo &io, int dtype)
{
    auto fn = sq_encode_fn();
    if (!fn) return false;
    const int es = dtype == SP_DTYPE_F32 ? 4 : 2;
    const CUtensorMapDataType dt = dtype == SP_DTYPE_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == SP_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                         : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const cuuint64_t dims[3] = {(cuuint64_t)kSlHD, (cuuint64_t)io.nh, (cuuint64_t)io.n_layers * io.n_tok};
    const cuuint64_t strides[2] = {(cuuint64_t)kSlHD * es, (cuuint64_t)kSlHD * es * io.nh};
    const cuuint32_t box[3] = {(cuuint32_t)(128 / es), 1, 32};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, dt, 3, const_cast<void *>(io.in), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// K (io[0]) and/or V (io[1], null = skipped) of the same tokens through the
// lane-per-vector encoder: 1 and *rc set if it took the call.
template <typename Tin>
int sq_lane_launch(const SpSqDev *t[2], const SqIo *io[2], int dtype, unsigned int *status, cudaStream_t s,
                   int *rc)
{
    if (getenv("SHANNON_PRIME_SQFREE_ENCODE_WARP")) return 0;
    const SqIo *i0 = io[0] ? io[0] : io[1];
    if (!i0) return 0;
    for (int hx = 0; hx < 2; hx++)
        if (io[hx] && (!sq_lane_fits(*t[hx], *io[hx]) || io[hx]->n_tok != i0->n_tok || io[hx]->nh != i0->nh ||
                       io[hx]->n_layers != i0->n_layers || io[hx]->layer0 != i0->layer0 ||
                       io[hx]->start_pos != i0->start_pos))
            return 0;
    const long long nb = (long long)i0->n_layers * i0->nh * ((i0->n_tok + 31) / 32);
    if (2 * nb > 0x7fffffffLL || (long long)i0->n_layers * i0->n_tok > 0xffffffffLL) return 0;
    SlMap map;
    memset(&map, 0, sizeof(map));
    SlArgs<kSlSK> a;
    memset(&a, 0, sizeof(a));
    for (int hx = 0; hx < 2; hx++) {
        if (!io[hx]) continue;
        if (!sq_lane_map(&map.m[hx], *io[hx], dtype)) return 0;
        a.cache[hx] = io[hx]->cache;
        a.slot_stride[hx] = io[hx]->slot_stride;
    }
    a.first = io[0] ? 0 : 1;
    a.n_halves = (io[0] && io[1]) ? 2 : 1;
    a.layer0 = i0->layer0; a.n_layers = i0->n_layers; a.nh = i0->nh; a.start_pos = i0->start_pos;
    a.n_tok = i0->n_tok;
    a.nb = (int)nb;
    a.status = status;
    auto k = k_sq_encode_lane<Tin, kSlSK>;
    const size_t smem = sizeof(SlSmem<Tin>);
    // per device and input type: attribute set and occupancy looked up once
    // (atomics, so host threads driving any devices race harmlessly)
    constexpr int kMaxDev = 64;
    static std::atomic<int> occ_tab[kMaxDev][3], sms_tab[kMaxDev];
    const int ti = sizeof(Tin) == 4 ? 0 : (std::is_same<Tin, __half>::value ? 1 : 2);
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDev) return 0;
    int occ = occ_tab[dev][ti].load(std::memory_order_acquire);
    if (occ == 0) {
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
            *rc = sp_check_cuda(cudaGetLastError(), "sqfree lane encoder smem attribute");
            return 1;
        }
        int o = 0, sm = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, k, kSlWarps * 32, smem);
        cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev);
        sms_tab[dev].store(sm > 0 ? sm : 148, std::memory_order_relaxed);
        occ = o > 0 ? o : 1;
        occ_tab[dev][ti].store(occ, std::memory_order_release);
    }
    const int sms = sms_tab[dev].load(std::memory_order_relaxed);
    long long blocks = (nb * a.n_halves + kSlWarps - 1) / kSlWarps;
    if (blocks > (long long)sms * occ) blocks = (long long)sms * occ;
    k<<<(unsigned)blocks, kSlWarps * 32, smem, s>>>(a, map);
    *rc = sp_check_cuda(cudaGetLastError(), "sqfree lane encoder launch");
    return 1;
}

int sq_lane_try(const SpSqDev *t[2], const SqIo *io[2], int dtype, unsigned int *status, cudaStream_t s, int *rc)
{
    return dtype == SP_DTYPE_F32 ? sq_lane_launch<float>(t, io, dtype, status, s, rc)
         : dtype == SP_DTYPE_F16 ? sq_lane_launch<__half>(t, io, dtype, status, s, rc)
         : dtype == SP_DTYPE_BF16 ? sq_lane_launch<__nv_bfloat16>(t, io, dtype, status, s, rc) : 0;
}

// ----------------------------------------------- lane-per-vector hier write --
// Compress for the hier layout of head_dim 256 (pad 330 = 2.3.5.11, skeleton
// of 30 values in two 15-value bands of 5 bits, 300 targets at 2 bits).  One
// thread owns one whole vector, so none of the warp encoder's cross-lane
// bookkeeping (group loops, shuffles, shared-memory atomics on the slot
// image) is left; every float operation is the one k_sq_encode performs, in
// the same order (the lane-tree sums of the inputs and of |dev| are replayed
// as the same tree), so slots are bit-identical.
//   pass 0  the input sum (lane-tree order) -> pad mean;
//   pass A  the transform stages 2, 3, 5 act inside blocks of 30 consecutive
//           coefficients (30 = 2.3.5): each block is loaded from the input
//           (or the mean) into registers, transformed there and stored into
//           the thread's 330-float row in shared memory;
//   pass B  the stride-30 stage 11: 30 groups of 11 values, all 330 outputs
//           written back; the skeleton then goes to registers;
//   pass C  prediction W . skeleton (fp32 fma chain in skeleton order, W rows
//           read as broadcasts) and the deviation, in place;
//   pass D  magnitude (lane-tree order), levels, packing into the row words,
//           which the warp then writes out byte-contiguously.
constexpr int kHlPD = 330, kHlHD = 256, kHlSK = 30, kHlNR = 300;
constexpr int kHlRow = 357;              // floats per thread: 330 + 26 row words + 1 (odd: conflict-free)
constexpr int kHlWs = 32;                // W row stride in floats (16-byte loads)
constexpr int kHlBandBits = 5, kHlBand = 15;
constexpr int kHlMagOff = 24, kHlResOff = 28, kHlBytes = 103;
__host__ __device__ constexpr int hl_band_byte(int b) { return b == 0 ? 0 : 12; }

struct HlArgs {
    const void *in;              // [n_layers][n_tok][nh][256]
    uint8_t *cache;
    long long slot_stride;
    int layer0, nh, start_pos, n_tok, tokens_per_cta;
    const __half *W;             // [n_slots][300][30]
    const int *tables;           // skel_idx[30], res_idx[300]
};

size_t hl_smem_bytes()
{
    return (size_t)kHlNR * kHlWs * 4 + (size_t)128 * kHlRow * 4 + (size_t)(kHlSK + kHlNR) * 4 + 16;
}

// Stage of prime P at stride STRIDE inside one 30-block held in registers
// (vstage_c's arithmetic and group layout restricted to the block).
template <int P, int STRIDE>
__device__ __forceinline__ void hl_stage(float (&x)[30])
{
    const float isp = c_sq_isp[prime_slot<P>()];
#pragma unroll
    for (int g = 0; g < 30 / P; g++) {
        const int blk = g / STRIDE, base = blk * (STRIDE * P) + (g - blk * STRIDE);
        float y[P];
#pragma unroll
        for (int k = 0; k < P; k++) {
            float acc = 0.0f;
#pragma unroll
            for (int j = 0; j < P; j++) acc = __fmaf_rn(c_sq_cas[cas_base<P>() + k * P + j], x[base + j * STRIDE], acc);
            y[k] = __fmul_rn(acc, isp);
        }
#pragma unroll
        for (int k = 0; k < P; k++) x[base + k * STRIDE] = y[k];
    }
}

// R lanes share one vector (32 / R vectors per warp, 128 per CTA); role
// rho = lane / (32 / R) takes the rho-th share of each split pass.
template <typename Tin, int R>
__global__ void __launch_bounds__(R * 128, 1)
k_hier_encode_lane(HlArgs a)
{
    constexpr int VPW = 32 / R, NW = 4 * R;          // vectors per warp, warps per CTA
    constexpr int U = R == 4 ? 5 : 6;                // residuals per prediction step
    static_assert((kHlNR / R) % U == 0, "prediction steps tile a role's residuals");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float *Ws = reinterpret_cast<float *>(smem_raw);                      // [300][32]
    float *rows = Ws + kHlNR * kHlWs;                                      // [128][357]
    int *tab = reinterpret_cast<int *>(rows + 128 * kHlRow);               // skel_idx, res_idx
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int v = lane % VPW, role = lane / VPW;
    const int li = blockIdx.y / a.nh, h = blockIdx.y % a.nh;
    const int slot = (a.layer0 + li) * a.nh + h;
    {
        const __half *w = a.W + (size_t)slot * kHlNR * kHlSK;
        for (int i = threadIdx.x; i < kHlNR * kHlWs; i += blockDim.x) {
            const int r = i / kHlWs, s = i - r * kHlWs;
            Ws[i] = s < kHlSK ? __half2float(w[r * kHlSK + s]) : 0.0f;
        }
        for (int i = threadIdx.x; i < kHlSK + kHlNR; i += blockDim.x) tab[i] = a.tables[i];
    }
    __syncthreads();
    float *y = rows + (size_t)(warp * VPW + v) * kHlRow;
    uint32_t *rw = reinterpret_cast<uint32_t *>(y + kHlPD);               // 26 row words
    // this role's shares: transform blocks, stage-11 groups, residuals, level words
    const int b0 = (kHlPD / 30) * role / R, b1 = (kHlPD / 30) * (role + 1) / R;
    const int g0 = 30 * role / R, g1 = 30 * (role + 1) / R;
    const int r0 = kHlNR / R * role;
    constexpr int NWORD = (2 * kHlNR + 31) / 32;
    const int w0 = NWORD * role / R, w1 = NWORD * (role + 1) / R;
    const int lo = 30 * b0, hi = 30 * b1;                                  // y range of the blocks
    const int tb = blockIdx.x * a.tokens_per_cta;
    const int te = min(a.n_tok, tb + a.tokens_per_cta);
    for (int t0 = tb + warp * VPW; t0 < te; t0 += NW * VPW) {
        const int tok = t0 + v;
        const bool live = tok < te;
        const Tin *src = reinterpret_cast<const Tin *>(a.in) +
                         (((long long)li * a.n_tok + (live ? tok : t0)) * a.nh + h) * kHlHD;
        // ---- pass 0: lane-tree sum of the inputs (every role); each role
        // stores the inputs of its own blocks and their mean pad
        float part[32];
#pragma unroll
        for (int l = 0; l < 32; l++) part[l] = 0.0f;
        constexpr int EPV = 16 / (int)sizeof(Tin);          // elements per 16-byte load
#pragma unroll 2
        for (int k = 0; k < kHlHD / 32; k++) {
            float x[32];
#pragma unroll
            for (int c = 0; c < 32; c += EPV) {
                const uint4 q = *reinterpret_cast<const uint4 *>(src + 32 * k + c);
                lane_unpack16_sq<Tin>(q, &x[c]);
            }
#pragma unroll
            for (int l = 0; l < 32; l++) {
                part[l] = __fadd_rn(part[l], x[l]);
                const int i = 32 * k + l;
                if (i >= lo && i < hi) y[i] = x[l];
            }
        }
        const float mean = __fdiv_rn(sl_tree32(part), (float)kHlHD);
        for (int i = max(lo, kHlHD); i < hi; i++) y[i] = mean;
        // ---- pass A: stages 2, 3, 5 on this role's blocks of 30 ------------
#pragma unroll 1
        for (int b = b0; b < b1; b++) {
            float x[30];
#pragma unroll
            for (int i = 0; i < 30; i++) x[i] = y[30 * b + i];
            hl_stage<2, 1>(x);
            hl_stage<3, 2>(x);
            hl_stage<5, 6>(x);
#pragma unroll
            for (int i = 0; i < 30; i++) y[30 * b + i] = x[i];
        }
        __syncwarp();
        // ---- pass B: stage 11 at stride 30 on this role's groups (a
        // group's outputs replace its own inputs) -----------------------------
        {
            const float isp = c_sq_isp[prime_slot<11>()];
#pragma unroll 1
            for (int g = g0; g < g1; g++) {
                float x[11];
#pragma unroll
                for (int j = 0; j < 11; j++) x[j] = y[g + 30 * j];
#pragma unroll
                for (int k = 0; k < 11; k++) {
                    float acc = 0.0f;
#pragma unroll
                    for (int j = 0; j < 11; j++) acc = __fmaf_rn(c_sq_cas[cas_base<11>() + k * 11 + j], x[j], acc);
                    y[g + 30 * k] = __fmul_rn(acc, isp);
                }
            }
        }
        __syncwarp();
        float sk[kHlSK];
#pragma unroll
        for (int s = 0; s < kHlSK; s++) sk[s] = y[tab[s]];
        // ---- skeleton bands (role 0) -----------------------------------------
        if (role == 0) {
            uint32_t row[6];
#pragma unroll
            for (int w = 0; w < 6; w++) row[w] = 0u;
#pragma unroll
            for (int b = 0; b < 2; b++) {
                float amax = 0.0f;
#pragma unroll
                for (int i = 0; i < kHlBand; i++) amax = fmaxf(amax, fabsf(sk[kHlBand * b + i]));
                constexpr int mv = (1 << (kHlBandBits - 1)) - 1;
                const float scale = amax > 0.0f ? __fdiv_rn(amax, (float)mv) : 0.0f;
                const __half hs = __float2half_rn(scale);
                const float stored = __half2float(hs);
                const float inv = stored > 0.0f ? __frcp_rn(stored) : 0.0f;
                const int sb = 8 * hl_band_byte(b);
                row[sb >> 5] |= (uint32_t)__half_as_ushort(hs) << (sb & 31);
#pragma unroll
                for (int i = 0; i < kHlBand; i++) {
                    int q = __float2int_rn(__fmul_rn(sk[kHlBand * b + i], inv));
                    q = q > mv ? mv : (q < -mv ? -mv : q);
                    const uint32_t u = (uint32_t)(q + mv);
                    const int pos = 8 * (hl_band_byte(b) + 2) + i * kHlBandBits;
                    row[pos >> 5] |= u << (pos & 31);
                    if ((pos & 31) + kHlBandBits > 32) row[(pos >> 5) + 1] |= u >> (32 - (pos & 31));
                }
            }
            static_assert(kHlMagOff == 24, "skeleton bands fill words 0-5");
#pragma unroll
            for (int w = 0; w < 6; w++) rw[w] = row[w];
        }
        // ---- pass C: prediction and deviation, in place, on this role's
        // residuals, U at a time so their fma chains interleave
#pragma unroll 1
        for (int rr = r0; rr < r0 + kHlNR / R; rr += U) {
            float acc[U];
#pragma unroll
            for (int u = 0; u < U; u++) acc[u] = 0.0f;
#pragma unroll
            for (int s0 = 0; s0 < kHlSK; s0 += 4) {
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const float4 w4 = reinterpret_cast<const float4 *>(Ws + (rr + u) * kHlWs)[s0 >> 2];
                    acc[u] = __fmaf_rn(w4.x, sk[s0], acc[u]);
                    acc[u] = __fmaf_rn(w4.y, sk[s0 + 1], acc[u]);
                    if (s0 + 2 < kHlSK) acc[u] = __fmaf_rn(w4.z, sk[s0 + 2], acc[u]);
                    if (s0 + 3 < kHlSK) acc[u] = __fmaf_rn(w4.w, sk[s0 + 3], acc[u]);
                }
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int i = tab[kHlSK + rr + u];
                y[i] = __fsub_rn(y[i], acc[u]);
            }
        }
        __syncwarp();
        // ---- pass D: magnitude (every role), this role's level words -------
#pragma unroll
        for (int l = 0; l < 32; l++) {
            float s = 0.0f;
#pragma unroll
            for (int r = l; r < kHlNR; r += 32) s = __fadd_rn(s, fabsf(y[tab[kHlSK + r]]));
            part[l] = s;
        }
        float mag = __fdiv_rn(sl_tree32(part), (float)kHlNR);
        if (mag < 1e-12f) mag = 1e-12f;
        const float step = __fdiv_rn(__fmul_rn(2.0f, mag), 3.0f);
        const float center = __fdiv_rn(3.0f, 2.0f);
        const float inv = step > 0.0f ? __frcp_rn(step) : 0.0f;
        static_assert(kHlMagOff % 4 == 0 && kHlResOff == kHlMagOff + 4, "word-aligned fields");
        if (role == 0) rw[kHlMagOff / 4] = __float_as_uint(mag);
#pragma unroll 1
        for (int w = w0; w < w1; w++) {
            uint32_t word = 0u;
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int r = 16 * w + j;
                if (r < kHlNR) {
                    int level = __float2int_rn(__fmaf_rn(y[tab[kHlSK + r]], inv, center));
                    level = level < 0 ? 0 : (level > 3 ? 3 : level);
                    word |= (uint32_t)level << (2 * j);
                }
            }
            rw[kHlResOff / 4 + w] = word;
        }
        __syncwarp();
        // ---- the warp's rows, byte-contiguous in the slot -------------------
        const int n_live = min(VPW, te - t0);
        uint8_t *dst = a.cache + (long long)slot * a.slot_stride + (long long)(a.start_pos + t0) * kHlBytes;
        const float *wbase = rows + (size_t)(warp * VPW) * kHlRow;
        for (int i = lane; i < n_live * kHlBytes; i += 32) {
            const int t = i / kHlBytes, bb = i - t * kHlBytes;
            dst[i] = reinterpret_cast<const uint8_t *>(wbase + (size_t)t * kHlRow + kHlPD)[bb];
        }
        __syncwarp();
    }
}

// The lane writer's layout: hd 256, pad 330, skeleton 30 in two 15-value
// 5-bit bands, 300 targets at 2 bits (103-byte slots).
bool hl_fits(const SpSqDev &t)
{
    return t.hier && t.hd == kHlHD && t.pd == kHlPD && t.n_skel == kHlSK && t.n_res == kHlNR && t.res_bits == 2 &&
           t.bl.n_bands == 2 && t.bl.bits[0] == kHlBandBits && t.bl.bits[1] == kHlBandBits &&
           t.bl.size[0] == kHlBand && t.bl.size[1] == kHlBand && t.bl.off[1] == kHlBand &&
           t.bl.byte_off[0] == hl_band_byte(0) && t.bl.byte_off[1] == hl_band_byte(1) && t.mag_off == kHlMagOff &&
           t.res_off == kHlResOff && t.bytes_per_pos == kHlBytes;
}

int hl_launch(const SpSqDev &t, const SqIo &io, int dtype, cudaStream_t s, bool *done)
{
    *done = false;
    if (!hl_fits(t) || !io.W || getenv("SHANNON_PRIME_HIER_ENCODE_WARP")) return SP_OK;
    if (dtype != SP_DTYPE_F32 && dtype != SP_DTYPE_F16 && dtype != SP_DTYPE_BF16) return SP_OK;
    if (((uintptr_t)io.in & 15)) return SP_OK;        // 16-byte row loads (rows are 256 elements)
    // two lanes per vector, 8 warps per CTA (four lanes, 16 warps at 128
    // registers, measured slower: 45.0 against 31.0 ms for config 4)
    constexpr int R = 2;
    void (*k)(HlArgs) = dtype == SP_DTYPE_F32 ? k_hier_encode_lane<float, R>
                      : dtype == SP_DTYPE_F16 ? k_hier_encode_lane<__half, R> : k_hier_encode_lane<__nv_bfloat16, R>;
    const size_t sm = hl_smem_bytes();
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
        return sp_check_cuda(cudaGetLastError(), "hier lane write smem attribute");
    HlArgs a;
    a.in = io.in;
    a.cache = io.cache;
    a.slot_stride = io.slot_stride;
    a.layer0 = io.layer0;
    a.nh = io.nh;
    a.start_pos = io.start_pos;
    a.n_tok = io.n_tok;
    a.W = io.W;
    a.tables = t.tables;
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms < 1) sms = 148;
    const int slots = io.n_layers * io.nh;
    // chunks of whole warp tiles; the count that fills the last wave best
    const int max_chunks = std::max(1, (io.n_tok + 127) / 128);
    const int c0 = std::min(max_chunks, std::max(1, (4 * sms + slots - 1) / slots));
    int chunks = c0;
    double best = -1.0;
    for (int c = c0; c <= std::min(max_chunks, 4 * c0); c++) {
        const long long ctas = (long long)slots * c;
        const double eff = (double)ctas / (double)(((ctas + sms - 1) / sms) * sms);
        if (eff > best + 1e-3) { best = eff; chunks = c; }
    }
    a.tokens_per_cta = ((io.n_tok + chunks - 1) / chunks + 7) / 8 * 8;
    chunks = (io.n_tok + a.tokens_per_cta - 1) / a.tokens_per_cta;
    k<<<dim3(chunks, slots), R * 128, sm, s>>>(a);
    *done = true;
    return sp_check_cuda(cudaGetLastError(), "hier lane write launch");
}

int sq_launch_encode(const SpSqDev &t, SqIo io, int dtype, cudaStream_t s, unsigned int *status = nullptr)
{
    if (io.n_tok <= 0 || io.n_layers <= 0) return SP_OK;
    {
        int rc = SP_OK;
        const SpSqDev *tt[2] = {&t, nullptr};
        const SqIo *ii[2] = {&io, nullptr};
        if (sq_lane_try(tt, ii, dtype, status, s, &rc)) return rc;
        bool done = false;
        if ((rc = hl_launch(t, io, dtype, s, &done)) || done) return rc;
    }
    const size_t sm = sq_smem_bytes(t);
    io.store_width = store_width_for(t.bytes_per_pos, io.slot_stride, io.cache);
    const int slots = io.n_layers * io.nh;
    const int pd = sq_plan_pd(t);
    void (*k)(SpSqDev, SqIo) = nullptr;
#define SQ_ENC(T)                                                                          \
    k = pd == 33 ? k_sq_encode<T, 33> : pd == 66 ? k_sq_encode<T, 66> :                    \
        pd == 154 ? k_sq_encode<T, 154> : pd == 330 ? k_sq_encode<T, 330> : k_sq_encode<T, 0>
    switch (dtype) {
    case SP_DTYPE_F32: SQ_ENC(float); break;
    case SP_DTYPE_F16: SQ_ENC(__half); break;
    case SP_DTYPE_BF16: SQ_ENC(__nv_bfloat16); break;
    default: return sp_set_error(SP_ERR_ARG, "sqfree/hier write: unknown dtype %d", dtype);
    }
#undef SQ_ENC
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    // Token chunks per slot: the count (from enough for ~4 waves up to 4x
    // that, at least one warp-round of tokens each) whose CTAs fill the last
    // wave best, so a long call does not end on a partly empty wave.
    int occ = 0, dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, kSqWarps * 32, sm);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long resident = (long long)std::max(occ, 1) * std::max(sms, 1);
    const int max_chunks = std::max(1, (io.n_tok + kSqWarps - 1) / kSqWarps);
    const int c0 = std::min(max_chunks, std::max(1, (int)((4 * resident + slots - 1) / slots)));
    int chunks = c0;
    double best = -1.0;
    for (int c = c0; c <= std::min(max_chunks, 4 * c0); c++) {
        const long long ctas = (long long)slots * c;
        const double eff = (double)ctas / (double)(((ctas + resident - 1) / resident) * resident);
        if (eff > best + 1e-3) { best = eff; chunks = c; }
    }
    io.tokens_per_cta = (io.n_tok + chunks - 1) / chunks;
    chunks = (io.n_tok + io.tokens_per_cta - 1) / io.tokens_per_cta;
    dim3 grid(chunks, slots);
    k<<<grid, kSqWarps * 32, sm, s>>>(t, io);
    return sp_check_cuda(cudaGetLastError(), "sqfree/hier encode launch");
}

int sq_launch_decode(const SpSqDev &t, SqIo io, cudaStream_t s)
{
    if (io.n_tok <= 0 || io.n_layers <= 0) return SP_OK;
    const size_t sm = sq_smem_bytes(t);
    io.store_width = store_width_for(t.bytes_per_pos, io.slot_stride, io.cache);
    const int slots = io.n_layers * io.nh;
    int chunks = (148 * 4 + slots - 1) / slots;
    const int max_chunks = (io.n_tok + kSqWarps - 1) / kSqWarps;
    if (chunks > max_chunks) chunks = max_chunks;
    if (chunks < 1) chunks = 1;
    io.tokens_per_cta = (io.n_tok + chunks - 1) / chunks;
    const int pd = sq_plan_pd(t);
    void (*k)(SpSqDev, SqIo) = pd == 33 ? k_sq_decode<33> : pd == 66 ? k_sq_decode<66>
                             : pd == 154 ? k_sq_decode<154> : pd == 330 ? k_sq_decode<330> : k_sq_decode<0>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    k<<<dim3(chunks, slots), kSqWarps * 32, sm, s>>>(t, io);
    return sp_check_cuda(cudaGetLastError(), "sqfree/hier decode launch");
}

// Host copy of the kernel description of a cache half (K or V).
struct SqHost {
    SpSqDev t;
};

// Upload the constant-memory cas tables to the current device (once per
// device; called from the cache constructors, outside any stream capture).
int sq_upload_constants()
{
    static std::atomic<bool> done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && done[dev].load(std::memory_order_acquire)) return SP_OK;
    float cas[208], isp[5];
    int off = 0, i = 0;
    for (int p : {2, 3, 5, 7, 11}) {
        for (int k = 0; k < p; k++)
            for (int j = 0; j < p; j++) {
                const double ang = 2.0 * 3.14159265358979323846 * (double)((k * j) % p) / (double)p;
                cas[off + k * p + j] = (float)(cos(ang) + sin(ang));
            }
        off += p * p;
        isp[i++] = (float)(1.0 / sqrt((double)p));
    }
    int rc = sp_check_cuda(cudaMemcpyToSymbol(c_sq_cas, cas, sizeof(cas)), "sqfree cas tables");
    if (!rc) rc = sp_check_cuda(cudaMemcpyToSymbol(c_sq_isp, isp, sizeof(isp)), "sqfree cas tables");
    if (!rc && dev >= 0 && dev < 64) done[dev] = true;
    return rc;
}

int sq_build_desc(SpSqDev &t, int hd, int pd, int n_skel, int n_res, int n_terms,
                  const sp_band_config_t &bands, int res_bits, int use_spinor, int hier,
                  const int *d_tables)
{
    memset(&t, 0, sizeof(t));
    t.hd = hd;
    if (sq_fill_transform(t, pd)) return -1;
    t.n_skel = n_skel;
    t.n_res = n_res;
    t.n_terms = n_terms;
    t.res_bits = res_bits;
    t.use_spinor = use_spinor;
    t.hier = hier;
    t.bl = sp_layout_from(bands);
    t.mag_off = t.bl.total_bytes;
    t.res_off = t.mag_off + 4;
    t.sheet_off = t.res_off + (n_res * res_bits + 7) / 8;
    t.bytes_per_pos = t.sheet_off + (use_spinor ? (n_res + 7) / 8 : 0);
    t.tables = d_tables;
    return (t.bytes_per_pos + 3) / 4 + 2 <= kSqRowWords ? 0 : -1;
}

SpSqDev sq_desc(const sp_cuda_sqfree_cache_t *cc, int which)
{
    SpSqDev t;
    sq_build_desc(t, cc->config.head_dim, cc->pad_dim, cc->sk_k, cc->n_res, cc->n_terms,
                  which ? cc->v_bands : cc->k_bands, cc->residual_bits, cc->use_spinor, 0,
                  (const int *)cc->d_tables);
    return t;
}

// ------------------------------------------ hier decompress on tensor cores --
// Decompression is linear in the dequantised slot: with c = [sk ; W sk + dev]
// placed at the skeleton / residual coefficient indices, the output is
//     out = V[:hd, :] c = (V_s + V_r W) sk + V_r dev
// (V the orthonormal staged transform, V_s / V_r its columns at the skeleton
// / residual indices).  Per slot the build kernel forms
//     B = [ V_s + V_r W  |  V_r ]        (hd rows, K = 16 * n_bands + pad16(n_res))
// in fp16, one 16-wide K block per skeleton band and the residuals after;
// a decode tile of 16 positions is then one [16 x K] x [K x hd] product on
// mma.sync, with A = the dequantised values (fp16) built in registers and B
// staged in shared memory and fetched with ldmatrix.  The result is within
// 1e-3 relative L2 of the exact reconstruction (fp16 A and B: ~3e-4), which
// is the bound for reconstructed K/V; the per-vector read APIs keep the exact
// SIMT kernel.
constexpr int kHrWarps = 8;
constexpr int kHrPrefetchWords = 16;    // staged words per lane: rows of up to 127 bytes

__host__ __device__ inline int hr_kp(int n_bands, int n_res) { return 16 * n_bands + (n_res + 15) / 16 * 16; }
// Row stride of B in halves: K + 8, so 8 consecutive rows of 16 bytes land on
// distinct bank groups for ldmatrix.
__host__ __device__ inline int hr_stride(int n_bands, int n_res) { return hr_kp(n_bands, n_res) + 8; }

// Transform matrix rows 0..hd-1 (fp32, [hd][pd]) of the staged Vilenkin
// transform, from the transform of unit vectors in double (same stages and
// tables as the codec).
std::vector<float> hr_transform_rows(int pd, int hd)
{
    std::vector<double> x(pd), y(pd);
    std::vector<float> v((size_t)hd * pd);
    int f[kSqMaxStages], nf = 0, r = pd;
    for (int p : {2, 3, 5, 7, 11}) while (r % p == 0) { f[nf++] = p; r /= p; }
    for (int i = 0; i < pd; i++) {
        for (int j = 0; j < pd; j++) x[j] = j == i ? 1.0 : 0.0;
        int stride = 1;
        for (int st = 0; st < nf; st++) {
            const int p = f[st], bs = stride * p;
            const double isp = 1.0 / sqrt((double)p);
            for (int blk = 0; blk < pd / bs; blk++)
                for (int o = 0; o < stride; o++) {
                    const int base = blk * bs + o;
                    double g[11];
                    for (int j = 0; j < p; j++) g[j] = x[base + j * stride];
                    for (int k = 0; k < p; k++) {
                        double acc = 0.0;
                        for (int j = 0; j < p; j++) {
                            const double ang = 2.0 * 3.14159265358979323846 * (double)((k * j) % p) / (double)p;
                            acc += (cos(ang) + sin(ang)) * g[j];
                        }
                        y[base + k * stride] = acc * isp;
                    }
                }
            for (int j = 0; j < pd; j++) x[j] = y[j];
            stride *= p;
        }
        for (int j = 0; j < hd; j++) v[(size_t)j * pd + i] = (float)x[j];   // column i = T e_i
    }
    return v;
}

// B of every slot: grid x = slot, one thread per output row j.
__global__ void k_hier_build_recon(const float *vrows, const __half *W, const int *skel_idx, const int *res_idx,
                                   SpBandLayout bl, int hd, int pd, int n_skel, int n_res, __half *recon)
{
    const int slot = blockIdx.x, stride = hr_stride(bl.n_bands, n_res);
    const __half *w = W + (size_t)slot * n_res * n_skel;
    for (int j = threadIdx.x; j < hd; j += blockDim.x) {
        const float *vj = vrows + (size_t)j * pd;
        __half *bj = recon + ((size_t)slot * hd + j) * stride;
        for (int k = 0; k < stride; k++) bj[k] = __float2half_rn(0.0f);
        for (int s = 0; s < n_skel; s++) {
            int b = 0;
            for (int q = 1; q < bl.n_bands; q++) if (s >= bl.off[q]) b = q;
            float m = vj[skel_idx[s]];
            for (int r = 0; r < n_res; r++) m = fmaf(vj[res_idx[r]], __half2float(w[(size_t)r * n_skel + s]), m);
            bj[16 * b + (s - bl.off[b])] = __float2half_rn(m);
        }
        for (int r = 0; r < n_res; r++) bj[16 * bl.n_bands + r] = __float2half_rn(vj[res_idx[r]]);
    }
}

struct HrArgs {
    const uint8_t *cache;         // slab base
    const uint8_t *cache_end;     // one past the slab's last byte
    long long slot_stride;
    const __half *recon;          // [n_slots][hd][stride]
    float *out;                   // [n_layers][n_tok][nh][hd]
    int layer0, n_layers, nh, start_pos, n_tok, tokens_per_cta;
};

__device__ __forceinline__ uint32_t hr_bits(const uint32_t *w, int pos)
{
    return __funnelshift_r(w[pos >> 5], w[(pos >> 5) + 1], pos & 31);
}

__device__ __forceinline__ void hr_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi)
{
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// NB skeleton bands (each <= 16 values), KSR residual K blocks, 2-bit residual
// levels, hd a multiple of 64 (HD).
template <int NB, int KSR, int HD>
__global__ void __launch_bounds__(kHrWarps * 32, 1)
k_hier_recon(SpSqDev t, HrArgs h)
{
    constexpr int KS = NB + KSR, KP = 16 * KS, STRIDE = KP + 8;
    extern __shared__ __align__(16) unsigned char smem[];
    __half *Bs = reinterpret_cast<__half *>(smem);
    const int bpp = t.bytes_per_pos;
    const int stage_words = (16 * bpp + 8) / 4 + 2;
    uint32_t *stage_all = reinterpret_cast<uint32_t *>(smem + (size_t)HD * STRIDE * 2);
    uint16_t *lut = reinterpret_cast<uint16_t *>(stage_all + kHrWarps * stage_words);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int li = blockIdx.y / h.nh, hh = blockIdx.y % h.nh;
    const int slot = (h.layer0 + li) * h.nh + hh;

    // B of this slot -> shared memory (16-byte copies)
    {
        const uint4 *src = reinterpret_cast<const uint4 *>(h.recon + (size_t)slot * HD * STRIDE);
        uint4 *dst = reinterpret_cast<uint4 *>(Bs);
        for (int i = threadIdx.x; i < HD * STRIDE / 8; i += blockDim.x) dst[i] = src[i];
    }
    if (threadIdx.x < 16) {       // PRMT selectors: nibble (l0 | l1 << 2) -> halves T[l0], T[l1]
        const int l0 = threadIdx.x & 3, l1 = threadIdx.x >> 2;
        lut[threadIdx.x] = (uint16_t)((2 * l0) | ((2 * l0 + 1) << 4) | ((2 * l1) << 8) | ((2 * l1 + 1) << 12));
    }
    __syncthreads();

    uint32_t *stw = stage_all + warp * stage_words;
    const uint8_t *slot_base = h.cache + (long long)slot * h.slot_stride;
    const int L = 1 << t.res_bits;
    const float center = __fdiv_rn((float)(L - 1), 2.0f);
    const int tb = blockIdx.x * h.tokens_per_cta, te = min(h.n_tok, tb + h.tokens_per_cta);
    // ldmatrix row address of this lane: matrix lane>>3, row lane&7
    const int lm = lane >> 3, lr = lane & 7;
    const uint32_t b_lane = spb::smem_u32(Bs) + (uint32_t)(((8 * (lm >> 1) + lr) * STRIDE + 8 * (lm & 1)) * 2);

    // The packed rows of a tile (word-aligned cover, zero past the tile) are
    // loaded into registers one tile ahead: lane holds words lane + 32 i.
    constexpr int NPW = kHrPrefetchWords;
    uint32_t pf[NPW];
    auto fetch = [&](int p0) {
        const int nrows = min(16, te - p0);
        const uint8_t *gs = slot_base + (long long)(h.start_pos + p0) * bpp;
        const uint8_t *ga = reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(gs) & ~uintptr_t(3));
        const int nwords = (nrows * bpp + (int)(gs - ga) + 3) / 4;
#pragma unroll
        for (int i = 0; i < NPW; i++) {
            const int wi = lane + 32 * i;
            uint32_t v = 0;
            if (wi < nwords) {
                const uint8_t *p = ga + 4 * wi;
                if (p + 4 <= h.cache_end) {
                    v = __ldcs(reinterpret_cast<const unsigned int *>(p));
                } else {
                    for (int b = 0; b < 4; b++)
                        if (p + b < h.cache_end) v |= (uint32_t)p[b] << (8 * b);
                }
            }
            pf[i] = v;
        }
    };
    if (tb + 16 * warp < te) fetch(tb + 16 * warp);
    for (int p0 = tb + 16 * warp; p0 < te; p0 += 16 * kHrWarps) {
        const int nrows = min(16, te - p0);
        const uint8_t *gs = slot_base + (long long)(h.start_pos + p0) * bpp;
        const int soff = (int)(reinterpret_cast<uintptr_t>(gs) & 3);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < NPW; i++)
            if (lane + 32 * i < stage_words) stw[lane + 32 * i] = pf[i];
        __syncwarp();
        if (p0 + 16 * kHrWarps < te) fetch(p0 + 16 * kHrWarps);
        // ---- A fragments: rows g and g+8 of the tile ----
        uint32_t A[KS][4];
#pragma unroll
        for (int hv = 0; hv < 2; hv++) {
            const int v = g + 8 * hv;
            const int rb = 8 * (soff + v * bpp);
            // residual value table T[lv] = (lv - center) * step, fp16
            const float mag = __uint_as_float(hr_bits(stw, rb + 8 * t.mag_off));
            const float step = __fdiv_rn(__fmul_rn(2.0f, mag), (float)(L - 1));
            const uint32_t tlo = pack_h2(__fmul_rn(__fsub_rn(0.0f, center), step), __fmul_rn(__fsub_rn(1.0f, center), step));
            const uint32_t thi = pack_h2(__fmul_rn(__fsub_rn(2.0f, center), step), __fmul_rn(__fsub_rn(3.0f, center), step));
#pragma unroll
            for (int b = 0; b < NB; b++) {
                float sc = __half2float(__ushort_as_half((unsigned short)(hr_bits(stw, rb + 8 * t.bl.byte_off[b]) & 0xffffu)));
                sc = fabsf(sc) <= 65504.0f ? sc : 0.0f;
                const int bits = t.bl.bits[b];
                const uint32_t mask = (1u << bits) - 1u;
                const float m = (float)((1 << (bits - 1)) - 1);
                const int cb = rb + 8 * (t.bl.byte_off[b] + 2);
                float q[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int i = 2 * c + (e & 1) + 8 * (e >> 1);
                    const uint32_t u = i < t.bl.size[b] ? (hr_bits(stw, cb + i * bits) & mask) : 0u;
                    q[e] = i < t.bl.size[b] ? __fmul_rn(__fsub_rn((float)u, m), sc) : 0.0f;
                }
                A[b][hv] = pack_h2(q[0], q[1]);
                A[b][2 + hv] = pack_h2(q[2], q[3]);
            }
            const int resb = rb + 8 * t.res_off;
#pragma unroll
            for (int j = 0; j < KSR; j++) {
                const uint32_t w = hr_bits(stw, resb + 32 * j);
                A[NB + j][hv] = __byte_perm(tlo, thi, lut[(w >> (4 * c)) & 15u]);
                A[NB + j][2 + hv] = __byte_perm(tlo, thi, lut[(w >> (4 * c + 16)) & 15u]);
            }
        }
        // ---- products: 64 output columns at a time ----
        float *orow0 = h.out + (((long long)li * h.n_tok + p0 + g) * h.nh + hh) * HD;
        const long long rstep8 = 8LL * h.nh * HD;
#pragma unroll 1
        for (int n0 = 0; n0 < HD; n0 += 64) {
            float acc[8][4];
#pragma unroll
            for (int nt = 0; nt < 8; nt++) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;
#pragma unroll
            for (int ks = 0; ks < KS; ks++) {
#pragma unroll
                for (int np = 0; np < 4; np++) {
                    uint32_t b0, b1, b2, b3;
                    const uint32_t addr = b_lane + (uint32_t)(((n0 + 16 * np) * STRIDE + 16 * ks) * 2);
                    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                                 : "=r"(b0), "=r"(b1), "=r"(b2), "=r"(b3) : "r"(addr));
                    hr_mma(acc[2 * np], A[ks], b0, b1);
                    hr_mma(acc[2 * np + 1], A[ks], b2, b3);
                }
            }
#pragma unroll
            for (int nt = 0; nt < 8; nt++) {
                const int col = n0 + 8 * nt + 2 * c;
                if (g < nrows) *reinterpret_cast<float2 *>(orow0 + col) = make_float2(acc[nt][0], acc[nt][1]);
                if (g + 8 < nrows) *reinterpret_cast<float2 *>(orow0 + rstep8 + col) = make_float2(acc[nt][2], acc[nt][3]);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// The same reconstruction on the 5th-generation tensor cores (tcgen05):
// one persistent CTA per SM, 128 positions per tile, D = A x B with
//   A [128 positions x 336] fp16  (dequantised skeleton bands, 16 each, then
//                                   the residual deviations): built by the
//                                   thread that owns the position and written
//                                   to tensor memory (tcgen05.st), one row per
//                                   TMEM lane;
//   B [336 x 256] fp16            (the slot's reconstruction matrix, resident
//                                   in shared memory in the K-major core-
//                                   matrix layout, reloaded when the slot
//                                   changes);
//   D [128 x 256] fp32            (tensor memory; drained by tcgen05.ld, one
//                                   output row per thread).
// One elected thread issues the 21 K=16 MMAs (kind::f16, A from tensor
// memory, B by shared-memory descriptor) and commits them to an mbarrier;
// every wait is bounded and sets status bit 0 on timeout.

namespace tc {

constexpr int kM = 128;            // positions per tile (= TMEM lanes = threads)
constexpr int kN = 256;            // output columns (head_dim)
constexpr int kKSteps = 21;        // 2 skeleton bands + 19 residual blocks of 16
constexpr int kKGroups = 2 * kKSteps;          // 8-element core-matrix columns
constexpr int kBBytes = kN * kKGroups * 16;    // 172032
constexpr int kThreads = 2 * kM;  // two warps per TMEM lane quarter
constexpr int kResSplit = 9;       // residual K blocks of the first warp of a quarter (it also has 2 skeleton blocks)
constexpr int kPfWords = 13;       // prefetched words per thread
constexpr int kXStride = 36;       // floats per row of the output staging block (32 + 4: no bank conflicts)
constexpr int kStageWords = kThreads * kPfWords;   // 3328 >= (128 * 103 + 6) / 4 + 2 words of packed rows
constexpr uint32_t kColD = 0;      // TMEM columns 0..255: D
constexpr uint32_t kColA = 256;    // TMEM columns 256..423: A (168 x 32 bit)
constexpr int kTmemCols = 512;

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};"
                 ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]),
                 "r"(v[7]) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
                 "%12, %13, %14, %15}, [%16];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                   "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
                   "=r"(v[14]), "=r"(v[15])
                 : "r"(taddr));
}

// Shared-memory matrix descriptor, K-major, no swizzle: core matrices of 8
// rows x 16 bytes stored contiguously; lbo = bytes between the two K halves
// of one MMA, sbo = bytes between consecutive groups of 8 rows.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo)
{
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFFu) >> 4);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;                      // descriptor version for sm_100
    return d;                                    // base offset 0, legacy LBO mode, no swizzle
}

// Instruction descriptor of kind::f16: f16 A and B, f32 D, both K-major,
// M = 128, N = 256.
constexpr uint32_t kIdesc = (1u << 4)            // D format f32
                          | (0u << 7) | (0u << 10) // A, B f16
                          | ((uint32_t)(kN >> 3) << 17)
                          | ((uint32_t)(kM >> 4) << 24);

__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %3, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %4, {%5, %5, %5, %5}, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(accumulate), "r"(kIdesc), "r"(0u) : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

}  // namespace tc

struct HrTcArgs {
    HrArgs h;
    unsigned int *status;
    long long total_tiles;        // n_layers * nh * tiles_per_slot
    int tiles_per_slot;
};

__global__ void __launch_bounds__(tc::kThreads, 1)
k_hier_recon_tc(SpSqDev t, HrTcArgs ta)
{
    using namespace tc;
    const HrArgs &h = ta.h;
    extern __shared__ __align__(16) unsigned char smem[];
    unsigned char *Bs = smem;                                          // kBBytes
    uint32_t *stage = reinterpret_cast<uint32_t *>(smem + kBBytes);    // kStageWords
    uint16_t *lut = reinterpret_cast<uint16_t *>(stage + kStageWords);  // 16
    unsigned long long *bar = reinterpret_cast<unsigned long long *>(lut + 16);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar + 1);
    int *ok_flag = reinterpret_cast<int *>(tmem_slot + 1);
    float *xbuf = reinterpret_cast<float *>(smem + kBBytes + kStageWords * 4 + 128);   // [8 warps][32][kXStride]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // Warps w and w + 4 share TMEM lanes 32 (w % 4) .. +31 (a warp reaches
    // only its quarter of the lanes): both serve the same 32 positions,
    // warp w the first 11 K blocks of their A rows and the first 128 output
    // columns, warp w + 4 the other 10 K blocks and columns.
    const int quarter = warp & 3, half = warp >> 2;
    const int row = 32 * quarter + lane;
    const uint32_t bar_a = spb::smem_u32(bar);

    const long long g0 = blockIdx.x * ta.total_tiles / gridDim.x;
    const long long g1 = (blockIdx.x + 1) * ta.total_tiles / gridDim.x;

    if (tid < 16) {       // PRMT selectors: nibble (l0 | l1 << 2) -> halves T[l0], T[l1]
        const int l0 = tid & 3, l1 = tid >> 2;
        lut[tid] = (uint16_t)((2 * l0) | ((2 * l0 + 1) << 4) | ((2 * l1) << 8) | ((2 * l1 + 1) << 12));
    }
    if (tid == 0) {
        spb::mbar_init(bar_a, 1);
        spb::mbar_init_fence();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(spb::smem_u32(tmem_slot)), "r"((uint32_t)kTmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;

    const int L = 1 << t.res_bits;
    const float center = __fdiv_rn((float)(L - 1), 2.0f);
    const int bpp = t.bytes_per_pos;
    int cur_slot = -1;
    uint32_t phase = 0;
    bool failed = false;

    // Packed rows of tile gg: the word-aligned cover of its rows, word
    // tid + kThreads i in pf[i] (zero past the rows), loaded one tile ahead.
    uint32_t pf[kPfWords];
    int pf_soff = 0;
    auto prefetch = [&](long long gg) {
        const int sl = (int)(gg / ta.tiles_per_slot);
        const int q0 = (int)(gg - (long long)sl * ta.tiles_per_slot) * kM;
        const int li = sl / h.nh, hh = sl - li * h.nh;
        const int slot = (h.layer0 + li) * h.nh + hh;
        const int nr = min(kM, h.n_tok - q0);
        const uint8_t *gs = h.cache + (long long)slot * h.slot_stride + (long long)(h.start_pos + q0) * bpp;
        const uint8_t *ga = reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(gs) & ~uintptr_t(3));
        pf_soff = (int)(gs - ga);
        const int nwords = (nr * bpp + pf_soff + 3) / 4;
#pragma unroll
        for (int i = 0; i < kPfWords; i++) {
            const int w = tid + kThreads * i;
            const uint8_t *p = ga + 4 * w;
            uint32_t v = 0;
            if (w < nwords) {
                if (p + 4 <= h.cache_end) {
                    v = __ldcs(reinterpret_cast<const unsigned int *>(p));
                } else {
                    for (int b = 0; b < 4; b++)
                        if (p + b < h.cache_end) v |= (uint32_t)p[b] << (8 * b);
                }
            }
            pf[i] = v;
        }
    };
    if (g0 < g1) prefetch(g0);

    for (long long g = g0; g < g1 && !failed; g++) {
        const int sl = (int)(g / ta.tiles_per_slot);               // slot within the call
        const int p0 = (int)(g - (long long)sl * ta.tiles_per_slot) * kM;
        const int li = sl / h.nh, hh = sl - li * h.nh;
        const int slot = (h.layer0 + li) * h.nh + hh;
        const int nrows = min(kM, h.n_tok - p0);
        // ---- B of the slot -> shared memory, core-matrix layout ----------
        if (slot != cur_slot) {
            const uint4 *src = reinterpret_cast<const uint4 *>(h.recon + (size_t)slot * kN * (16 * kKSteps + 8));
            // thread = one row n of B; its 42 chunks are loaded 14 at a time
            // before they are stored
            const int n = tid;
            unsigned char *dst = Bs + (n >> 3) * kKGroups * 128 + (n & 7) * 16;
#pragma unroll 1
            for (int kg0 = 0; kg0 < kKGroups; kg0 += 14) {
                uint4 v[14];
#pragma unroll
                for (int j = 0; j < 14; j++) v[j] = __ldg(src + (size_t)n * (kKGroups + 1) + kg0 + j);
#pragma unroll
                for (int j = 0; j < 14; j++) *reinterpret_cast<uint4 *>(dst + (kg0 + j) * 128) = v[j];
            }
            cur_slot = slot;
            spb::fence_proxy_async();      // generic writes of B before the tensor core reads them
        }
        // ---- packed rows of the tile -> shared memory, from the registers
        // prefetched during the previous tile
        const int soff = pf_soff;
#pragma unroll
        for (int i = 0; i < kPfWords; i++) stage[tid + kThreads * i] = pf[i];
        __syncthreads();
        if (g + 1 < g1) prefetch(g + 1);

        // ---- A row blocks of this thread -> tensor memory ------------------
        {
            const bool live = row < nrows;
            const int rb = 8 * (soff + row * bpp);
            const float mag = live ? __uint_as_float(hr_bits(stage, rb + 8 * t.mag_off)) : 0.0f;
            const float step = __fdiv_rn(__fmul_rn(2.0f, mag), (float)(L - 1));
            const uint32_t tlo = pack_h2(__fmul_rn(__fsub_rn(0.0f, center), step), __fmul_rn(__fsub_rn(1.0f, center), step));
            const uint32_t thi = pack_h2(__fmul_rn(__fsub_rn(2.0f, center), step), __fmul_rn(__fsub_rn(3.0f, center), step));
            if (half == 0) {
#pragma unroll
                for (int b = 0; b < 2; b++) {
                    float sc = live ? __half2float(__ushort_as_half(
                                          (unsigned short)(hr_bits(stage, rb + 8 * t.bl.byte_off[b]) & 0xffffu)))
                                    : 0.0f;
                    sc = fabsf(sc) <= 65504.0f ? sc : 0.0f;
                    const int bits = t.bl.bits[b];
                    const uint32_t mask = (1u << bits) - 1u;
                    const float m = (float)((1 << (bits - 1)) - 1);
                    const int cb = rb + 8 * (t.bl.byte_off[b] + 2);
                    uint32_t v[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        float q[2];
#pragma unroll
                        for (int k = 0; k < 2; k++) {
                            const int i = 2 * e + k;
                            const bool ok = live && i < t.bl.size[b];
                            const uint32_t u = ok ? (hr_bits(stage, cb + i * bits) & mask) : 0u;
                            q[k] = ok ? __fmul_rn(__fsub_rn((float)u, m), sc) : 0.0f;
                        }
                        v[e] = pack_h2(q[0], q[1]);
                    }
                    tmem_st8(tmem + lane_base + kColA + 8 * b, v);
                }
            }
            const int resb = rb + 8 * t.res_off;
            const int j0 = half == 0 ? 0 : kResSplit;
            const int nj = half == 0 ? kResSplit : kKSteps - 2 - kResSplit;
            // all of this thread's residual words first (independent loads),
            // then the blocks
            uint32_t rw[kKSteps - 2 - kResSplit];
#pragma unroll
            for (int j = 0; j < kKSteps - 2 - kResSplit; j++)
                rw[j] = (live && j < nj) ? hr_bits(stage, resb + 32 * (j0 + j)) : 0u;
#pragma unroll
            for (int j = 0; j < kKSteps - 2 - kResSplit; j++) {
                if (j < nj) {
                    const int r0 = 16 * (j0 + j);
                    // residuals past n_res meet zero rows of B; write them as 0
                    uint32_t v[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        const uint32_t sel = lut[(rw[j] >> (4 * e)) & 15u];
                        v[e] = (live && r0 + 2 * e < t.n_res) ? __byte_perm(tlo, thi, sel) : 0u;
                    }
                    tmem_st8(tmem + lane_base + kColA + 8 * (2 + j0 + j), v);
                }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        fence_before();
        __syncthreads();
        // ---- MMAs (one thread) -------------------------------------------
        if (tid == 0) {
            fence_after();
            const uint32_t bsm = spb::smem_u32(Bs);
#pragma unroll 1
            for (int s = 0; s < kKSteps; s++) {
                const uint64_t bd = smem_desc(bsm + (uint32_t)(2 * s) * 128u, 128u, (uint32_t)kKGroups * 128u);
                mma_f16_ts(tmem + kColD, tmem + kColA + 8 * s, bd, s > 0 ? 1u : 0u);
            }
            mma_commit(bar_a);
        }
        // ---- wait for the products (bounded; thread 0 decides for the CTA)
        if (tid == 0) *ok_flag = spb::wait_stage(bar_a, phase, ta.status) ? 1 : 0;
        __syncthreads();
        if (!*ok_flag) {
            failed = true;
            break;
        }
        phase ^= 1u;
        fence_after();
        // ---- D -> global: each warp moves its 32 rows x 128 columns in
        // blocks of 32 columns through shared memory, so that every store
        // instruction writes four whole 128-byte row segments
        {
            float *xb = xbuf + warp * 32 * kXStride;
            const int r4 = lane >> 3, c4 = (lane & 7) * 4;
#pragma unroll 1
            for (int c0 = 0; c0 < 128; c0 += 32) {
                uint32_t v[2][16];
                tmem_ld16(tmem + lane_base + kColD + 128 * half + c0, v[0]);
                tmem_ld16(tmem + lane_base + kColD + 128 * half + c0 + 16, v[1]);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int j = 0; j < 2; j++)
#pragma unroll
                    for (int e = 0; e < 16; e += 4)
                        *reinterpret_cast<float4 *>(xb + lane * kXStride + 16 * j + e) =
                            make_float4(__uint_as_float(v[j][e]), __uint_as_float(v[j][e + 1]),
                                        __uint_as_float(v[j][e + 2]), __uint_as_float(v[j][e + 3]));
                __syncwarp();
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int rr = 4 * i + r4;                 // row within the warp's 32
                    const int prow = 32 * quarter + rr;
                    if (prow < nrows) {
                        float *o = h.out + (((long long)li * h.n_tok + p0 + prow) * h.nh + hh) * kN + 128 * half + c0 + c4;
                        __stcs(reinterpret_cast<float4 *>(o), *reinterpret_cast<const float4 *>(xb + rr * kXStride + c4));
                    }
                }
                __syncwarp();
            }
        }
        fence_before();
        __syncthreads();       // D drained and the stage read before the next tile reuses them
    }
    if (failed) {
        // The commit may still arrive: wait once more (bounded) before the
        // tensor memory is released.
        if (tid == 0) spb::wait_stage(bar_a, phase, nullptr);
        __syncthreads();
    }
    fence_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)kTmemCols)
                     : "memory");
}

size_t hr_tc_smem_bytes()
{
    return (size_t)tc::kBBytes + tc::kStageWords * 4 + 128 + (size_t)8 * 32 * tc::kXStride * 4;
}

// The tcgen05 read serves the shape its matrices are laid out for: two
// skeleton bands of at most 16 values, 19 residual blocks (n_res <= 304),
// 2-bit residuals, head_dim 256, rows of at most 103 bytes.
bool hr_tc_supported(const SpSqDev &t)
{
    if (!t.hier || t.res_bits != 2 || t.hd != 256 || t.bl.n_bands != 2) return false;
    if (t.bl.size[0] > 16 || t.bl.size[1] > 16 || (t.n_res + 15) / 16 != 19) return false;
    return (tc::kM * t.bytes_per_pos + 3 + 3) / 4 + 2 <= tc::kStageWords;
}

size_t hr_smem_bytes(const SpSqDev &t, int hd)
{
    const int stride = hr_stride(t.bl.n_bands, t.n_res);
    const int stage_words = (16 * t.bytes_per_pos + 8) / 4 + 2;
    return (size_t)hd * stride * 2 + (size_t)kHrWarps * stage_words * 4 + 64;
}

// The tensor-core kernel for the slot shape, or nullptr (then the SIMT kernel
// serves the read).
using HrKernel = void (*)(SpSqDev, HrArgs);
HrKernel hr_kernel(const SpSqDev &t)
{
    if (!t.hier || t.res_bits != 2 || t.hd != 256) return nullptr;
    for (int b = 0; b < t.bl.n_bands; b++) if (t.bl.size[b] > 16) return nullptr;
    if (hr_smem_bytes(t, t.hd) > 220 * 1024) return nullptr;
    if ((16 * t.bytes_per_pos + 8) / 4 + 2 > 32 * kHrPrefetchWords) return nullptr;
    const int ksr = (t.n_res + 15) / 16;
    if (t.bl.n_bands == 2 && ksr == 19) return k_hier_recon<2, 19, 256>;
    return nullptr;
}

SpSqDev hier_desc(const sp_cuda_hier_cache_t *hc)
{
    SpSqDev t;
    sq_build_desc(t, hc->config.head_dim, hc->pad_dim, hc->n_skeleton, hc->n_target, 0, hc->skel_bands,
                  hc->target_res_bits, 0, 1, (const int *)hc->d_tables);
    return t;
}

// (Re)build the per-slot reconstruction matrices from the current W.
int hr_build(const sp_cuda_hier_cache_t *hc)
{
    if (!hc->d_recon) return SP_OK;
    const SpSqDev t = hier_desc(hc);
    k_hier_build_recon<<<hc->n_slots, 256, 0, (cudaStream_t)hc->stream>>>(
        hc->d_vrows, (const __half *)hc->d_W, hc->d_skeleton_idx, hc->d_target_idx, t.bl, hc->config.head_dim,
        hc->pad_dim, hc->n_skeleton, hc->n_target, (__half *)hc->d_recon);
    return sp_check_cuda(cudaGetLastError(), "hier reconstruction build");
}

}  // namespace

// ===================================================================== C-ABI

extern "C" {

// Bytes of the lane decode's query area, after the partials and the status
// word of the attention workspace.
static size_t sq_qws_bytes(const sp_config_t *cfg)
{
    return (size_t)cfg->n_layers * 8 * cfg->n_heads_kv * kSaQWords * sizeof(float);
}

int sp_cuda_sqfree_cache_init_ex(sp_cuda_sqfree_cache_t *cc, const sp_config_t *cfg, int max_seq_len,
                                 int residual_bits, int use_spinor, float sk_frac, void *stream)
{
    sp_clear_error();
    if (!cc || !cfg) return sp_set_error(SP_ERR_ARG, "sqfree_cache_init: NULL argument");
    memset(cc, 0, sizeof(*cc));
    if (cfg->n_layers <= 0 || cfg->n_heads_kv <= 0 || max_seq_len <= 0 || cfg->head_dim < 1)
        return sp_set_error(SP_ERR_ARG, "sqfree_cache_init: bad dims");
    if (residual_bits < 1 || residual_bits > 8)
        return sp_set_error(SP_ERR_ARG, "sqfree_cache_init: residual_bits %d outside 1..8", residual_bits);
    const int pd = sq_pad_dim(cfg->head_dim);
    if (pd < 0 || pd > kSqMaxPd)
        return sp_set_error(SP_ERR_UNSUPPORTED, "sqfree_cache_init: head_dim %d has no pad_dim <= %d",
                            cfg->head_dim, kSqMaxPd);
    int sk_k = sk_frac > 0.0f ? (int)floor((double)sk_frac * pd) : pd / 2;
    if (sk_k < 1) sk_k = 1;
    if (sk_k > pd) sk_k = pd;
    cc->config = *cfg;
    cc->pad_dim = pd;
    cc->sk_k = sk_k;
    cc->n_res = pd - sk_k;
    cc->residual_bits = residual_bits;
    cc->use_spinor = use_spinor ? 1 : 0;
    cc->max_seq_len = max_seq_len;
    cc->n_slots = cfg->n_layers * cfg->n_heads_kv;
    cc->stream = stream;
    cudaGetDevice(&cc->device);
    // skeleton bands over sk_k; default 5,4,4,4,5 (shannon_prime_sqfree.cu:614-623)
    const int defb[5] = {5, 4, 4, 4, 5};
    int kb[SP_MAX_BANDS], vb[SP_MAX_BANDS];
    const int knb = (cfg->k_n_bands > 0 && cfg->k_n_bands <= SP_MAX_BANDS) ? cfg->k_n_bands : 5;
    const int vnb = (cfg->v_n_bands > 0 && cfg->v_n_bands <= SP_MAX_BANDS) ? cfg->v_n_bands : 5;
    for (int i = 0; i < knb; i++) kb[i] = cfg->k_band_bits[i] > 0 ? cfg->k_band_bits[i] : defb[i % 5];
    for (int i = 0; i < vnb; i++) vb[i] = cfg->v_band_bits[i] > 0 ? cfg->v_band_bits[i] : defb[i % 5];
    if (sp_band_config_init(&cc->k_bands, sk_k, knb, kb) || sp_band_config_init(&cc->v_bands, sk_k, vnb, vb))
        return sp_set_error(SP_ERR_ARG, "sqfree_cache_init: bad band configuration");
    // Knight mask: squarefree-first ranking, Möbius CSR over proper divisors.
    std::vector<int> rank, skel(sk_k), res, off, term;
    for (int i = 0; i < pd; i++) if (sq_squarefree(i + 1)) rank.push_back(i);
    for (int i = 0; i < pd; i++) if (!sq_squarefree(i + 1)) rank.push_back(i);
    std::vector<int> slot_of(pd, -1);
    for (int s = 0; s < sk_k; s++) { skel[s] = rank[s]; slot_of[rank[s]] = s; }
    for (int i = 0; i < pd; i++) if (slot_of[i] < 0) res.push_back(i);
    std::vector<int> csr_slot, csr_sign;
    for (int r = 0; r < (int)res.size(); r++) {
        off.push_back((int)term.size());
        const int n = res[r] + 1;
        for (int d = 1; d < n; d++) {
            if (n % d) continue;
            const int mu = sq_mu(n / d);
            if (!mu || slot_of[d - 1] < 0) continue;
            term.push_back((slot_of[d - 1] << 1) | (mu < 0 ? 1 : 0));
            csr_slot.push_back(slot_of[d - 1]);
            csr_sign.push_back(mu);
        }
    }
    off.push_back((int)term.size());
    cc->n_terms = (int)term.size();
    for (size_t r = 0; r + 1 < off.size(); r++)
        if (off[r + 1] - off[r] > cc->csr_max_terms) cc->csr_max_terms = off[r + 1] - off[r];
    std::vector<int> tables;
    tables.insert(tables.end(), skel.begin(), skel.end());
    tables.insert(tables.end(), res.begin(), res.end());
    tables.insert(tables.end(), off.begin(), off.end());
    tables.insert(tables.end(), term.begin(), term.end());
    // Residual -> lane assignment of the blocked decode: residuals by
    // decreasing term count, each to the least-loaded lane holding fewer than
    // kSq3LaneRes of them (ties: lower lane).  Table: [32][kSq3LaneRes], -1 free.
    {
        std::vector<int> lane_res(32 * kSq3LaneRes, -1), load(32, 0), cnt(32, 0), order(res.size());
        for (size_t r = 0; r < res.size(); r++) order[r] = (int)r;
        std::stable_sort(order.begin(), order.end(), [&](int x, int y) {
            return off[x + 1] - off[x] > off[y + 1] - off[y];
        });
        bool fits = true;
        for (int r : order) {
            int best = -1;
            for (int ln = 0; ln < 32; ln++)
                if (cnt[ln] < kSq3LaneRes && (best < 0 || load[ln] < load[best])) best = ln;
            if (best < 0) { fits = false; break; }
            lane_res[kSq3LaneRes * best + cnt[best]++] = r;
            load[best] += off[r + 1] - off[r];
        }
        cc->lane_max_terms = 0;
        if (fits)
            for (int ln = 0; ln < 32; ln++) cc->lane_max_terms = std::max(cc->lane_max_terms, std::max(load[ln], 1));
        tables.insert(tables.end(), lane_res.begin(), lane_res.end());
    }
    int factors[kSqMaxStages], nf = 0;
    {
        int r = pd;
        for (int p : {2, 3, 5, 7, 11}) while (r % p == 0) { factors[nf++] = p; r /= p; }
    }
    cc->n_factors = nf;
    SpSqDev tk;
    const size_t k_total = (size_t)cc->n_slots * max_seq_len;
    int rc = SP_OK;
    auto up = [&](void **dst, const void *src, size_t bytes, const char *what) {
        if (rc) return;
        if ((rc = sp_check_cuda(cudaMalloc(dst, bytes > 0 ? bytes : 4), what))) return;
        if (bytes) rc = sp_check_cuda(cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice), what);
    };
    up(&cc->d_tables, tables.data(), tables.size() * 4, "sqfree tables");
    up((void **)&cc->d_skeleton_idx, skel.data(), skel.size() * 4, "skeleton idx");
    up((void **)&cc->d_residual_idx, res.data(), res.size() * 4, "residual idx");
    up((void **)&cc->d_csr_offsets, off.data(), off.size() * 4, "csr offsets");
    up((void **)&cc->d_csr_skel_slot, csr_slot.data(), csr_slot.size() * 4, "csr slots");
    up((void **)&cc->d_csr_mu_sign, csr_sign.data(), csr_sign.size() * 4, "csr signs");
    up((void **)&cc->d_vilenkin_factors, factors, (size_t)nf * 4, "factors");
    if (rc) { sp_cuda_sqfree_cache_free(cc); return rc; }
    if (sq_build_desc(tk, cfg->head_dim, pd, sk_k, cc->n_res, cc->n_terms, cc->k_bands, residual_bits,
                      cc->use_spinor, 0, (const int *)cc->d_tables)) {
        sp_cuda_sqfree_cache_free(cc);
        return sp_set_error(SP_ERR_UNSUPPORTED, "sqfree_cache_init: slot too large");
    }
    cc->bytes_per_pos_k = tk.bytes_per_pos;
    cc->bytes_per_pos_v = sq_desc(cc, 1).bytes_per_pos;
    if ((rc = sp_check_cuda(cudaMalloc(&cc->d_k_cache, k_total * cc->bytes_per_pos_k), "cudaMalloc K cache")) ||
        (rc = sp_check_cuda(cudaMalloc(&cc->d_v_cache, k_total * cc->bytes_per_pos_v), "cudaMalloc V cache"))) {
        sp_cuda_sqfree_cache_free(cc);
        return rc;
    }
    cudaMemset(cc->d_k_cache, 0, k_total * cc->bytes_per_pos_k);
    cudaMemset(cc->d_v_cache, 0, k_total * cc->bytes_per_pos_v);
    cc->attn_ws_bytes = (size_t)cfg->n_layers * 8 * cfg->n_heads_kv * kSqMaxSplits * (pd + 4) * sizeof(float);
    // + 16 bytes: the decode's status word follows the partials
    if ((rc = sq_upload_constants()) ||
        (rc = sp_check_cuda(cudaMalloc(&cc->d_attn_ws, cc->attn_ws_bytes + 16 + sq_qws_bytes(cfg)),
                            "cudaMalloc sqfree workspace")) ||
        (rc = sp_check_cuda(cudaMemset(cc->d_attn_ws, 0, cc->attn_ws_bytes + 16 + sq_qws_bytes(cfg)),
                            "sqfree workspace")) ||
        (rc = sp_check_cuda(cudaDeviceSynchronize(), "sqfree_cache_init"))) {
        sp_cuda_sqfree_cache_free(cc);
        return rc;
    }
    return SP_OK;
}

int sp_cuda_sqfree_cache_init(sp_cuda_sqfree_cache_t *cc, const sp_config_t *cfg, int max_seq_len,
                              int residual_bits, int use_spinor, void *stream)
{
    return sp_cuda_sqfree_cache_init_ex(cc, cfg, max_seq_len, residual_bits, use_spinor, 0.0f, stream);
}

void sp_cuda_sqfree_cache_free(sp_cuda_sqfree_cache_t *cc)
{
    if (!cc) return;
    cudaFree(cc->d_tables);
    cudaFree(cc->d_skeleton_idx);
    cudaFree(cc->d_residual_idx);
    cudaFree(cc->d_csr_offsets);
    cudaFree(cc->d_csr_skel_slot);
    cudaFree(cc->d_csr_mu_sign);
    cudaFree(cc->d_vilenkin_factors);
    cudaFree(cc->d_k_cache);
    cudaFree(cc->d_v_cache);
    cudaFree(cc->d_attn_ws);
    memset(cc, 0, sizeof(*cc));
}

static int sq_check(const sp_cuda_sqfree_cache_t *cc, int layer, int n_layers, int head, int pos, int n)
{
    if (!cc || !cc->d_k_cache) return sp_set_error(SP_ERR_ARG, "sqfree cache not initialised");
    if (layer < 0 || n_layers < 0 || layer + n_layers > cc->config.n_layers || head < 0 ||
        head >= cc->config.n_heads_kv)
        return sp_set_error(SP_ERR_ARG, "sqfree: layer/head out of range");
    if (pos < 0 || n < 0 || (long long)pos + n > cc->max_seq_len)
        return sp_set_error(SP_ERR_ARG, "sqfree: positions [%d,%d) outside the cache", pos, pos + n);
    return SP_OK;
}

static int sq_write_io(sp_cuda_sqfree_cache_t *cc, int which, int layer0, int n_layers, int head0, int nh,
                       int start_pos, int n_tok, const void *d_in, const SpSqDev &t, SqIo &io)
{
    memset(&io, 0, sizeof(io));
    io.in = d_in;
    io.cache = which ? cc->d_v_cache : cc->d_k_cache;
    io.slot_stride = (long long)cc->max_seq_len * t.bytes_per_pos;
    // a single-head write addresses slot (layer0*H + head0): shift the base
    io.cache += (long long)head0 * io.slot_stride;
    io.layer0 = layer0;
    io.n_layers = n_layers;
    io.nh = nh;
    io.start_pos = start_pos;
    io.n_tok = n_tok;
    if (nh != cc->config.n_heads_kv) {
        // one head: slot index (layer0 + li) * nh + h must map to layer*H + head0
        io.layer0 = 0;
        io.cache += (long long)layer0 * cc->config.n_heads_kv * io.slot_stride;
        if (n_layers != 1) return sp_set_error(SP_ERR_ARG, "sqfree: per-head writes take one layer");
    }
    return SP_OK;
}

static unsigned int *sq_status(const sp_cuda_sqfree_cache_t *cc)
{
    return reinterpret_cast<unsigned int *>(reinterpret_cast<char *>(cc->d_attn_ws) + cc->attn_ws_bytes);
}

static int sq_write(sp_cuda_sqfree_cache_t *cc, int which, int layer0, int n_layers, int head0, int nh,
                    int start_pos, int n_tok, const void *d_in, int dtype)
{
    SpSqDev t = sq_desc(cc, which);
    SqIo io;
    int rc = sq_write_io(cc, which, layer0, n_layers, head0, nh, start_pos, n_tok, d_in, t, io);
    if (rc) return rc;
    return sq_launch_encode(t, io, dtype, (cudaStream_t)cc->stream, sq_status(cc));
}

// The lane read of the config-2 slot over a grid of slots; d_out is
// [n_layers][n_pos][n_heads][128] fp32 (one slot: [n_pos][128]).  Returns 1
// when the driver has no tensor-map encoder (the caller takes another path),
// -1 on a launch error, 0 when launched.
static int sq_read_lane(const uint8_t *slab, const SlGrid &g, int n_pos, float *d_out, unsigned int *status,
                        cudaStream_t s)
{
    auto fn = sq_encode_fn();
    if (!fn) return 1;
    SlOutMap map;
    memset(&map, 0, sizeof(map));
    const cuuint64_t row = (cuuint64_t)kSlHD * g.n_heads;
    const cuuint64_t dims[3] = {row, (cuuint64_t)n_pos, (cuuint64_t)g.n_layers};
    const cuuint64_t strides[2] = {row * 4, row * 4 * (cuuint64_t)n_pos};
    const cuuint32_t box[3] = {32, 32, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (fn(&map.m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, d_out, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
        return 1;
    const size_t smem = sizeof(SlReadSmem);
    // Per device: attribute set and occupancy looked up once (atomics, so
    // host threads driving any devices race harmlessly).
    constexpr int kMaxDev = 64;
    static std::atomic<int> occ_tab[kMaxDev], sms_tab[kMaxDev];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDev) return -1;
    int occ = occ_tab[dev].load(std::memory_order_acquire);
    if (occ == 0) {
        if (cudaFuncSetAttribute(k_sq_decode_lane, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess) {
            sp_check_cuda(cudaGetLastError(), "sqfree lane read smem attribute");
            return -1;
        }
        int o = 0, sms = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, k_sq_decode_lane, kSlWarps * 32, smem);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        sms_tab[dev].store(sms > 0 ? sms : 148, std::memory_order_relaxed);
        occ = o > 0 ? o : 1;
        occ_tab[dev].store(occ, std::memory_order_release);
    }
    const int sms = sms_tab[dev].load(std::memory_order_relaxed);
    const long long n_b = (long long)((n_pos + 31) / 32) * g.n_heads * g.n_layers;
    long long blocks = (n_b + kSlWarps - 1) / kSlWarps;
    if (blocks > (long long)sms * occ) blocks = (long long)sms * occ;
    k_sq_decode_lane<<<(unsigned)blocks, kSlWarps * 32, smem, s>>>(slab, g, n_pos, status, map);
    return sp_check_cuda(cudaGetLastError(), "sqfree lane read launch") ? -1 : 0;
}

static int sq_read(const sp_cuda_sqfree_cache_t *cc, int which, int layer, int head, int start_pos, int n_pos,
                   float *d_out)
{
    int rc = sq_check(cc, layer, 1, head, start_pos, n_pos);
    if (rc) return rc;
    SpSqDev t = sq_desc(cc, which);
    SqIo io;
    memset(&io, 0, sizeof(io));
    io.out = d_out;
    io.slot_stride = (long long)cc->max_seq_len * t.bytes_per_pos;
    io.cache = (uint8_t *)(which ? cc->d_v_cache : cc->d_k_cache) +
               ((long long)layer * cc->config.n_heads_kv + head) * io.slot_stride;
    io.layer0 = 0;
    io.n_layers = 1;
    io.nh = 1;
    io.start_pos = start_pos;
    io.n_tok = n_pos;
    io.single_slot = 1;
    if (sq_lane_fits(t, io) && !getenv("SHANNON_PRIME_SQFREE_DECODE_WARP") && !((uintptr_t)d_out & 15) &&
        !(((uintptr_t)io.cache + (uintptr_t)start_pos * t.bytes_per_pos) & 3)) {
        const SlGrid g{0, 0, 1, 1, 0};
        const int r = sq_read_lane(io.cache + (long long)start_pos * t.bytes_per_pos, g, n_pos, d_out, sq_status(cc),
                                   (cudaStream_t)cc->stream);
        if (r <= 0) return r ? sp_set_error(SP_ERR_CUDA, "sqfree lane read failed") : SP_OK;
    }
    return sq_launch_decode(t, io, (cudaStream_t)cc->stream);
}

void sp_cuda_sqfree_write_k(sp_cuda_sqfree_cache_t *cc, int layer, int head, int pos, const float *d_k_vec)
{
    sp_clear_error();
    if (sq_check(cc, layer, 1, head, pos, 1) || !d_k_vec) { if (!d_k_vec) sp_set_error(SP_ERR_ARG, "NULL vector"); return; }
    sq_write(cc, 0, layer, 1, head, 1, pos, 1, d_k_vec, SP_DTYPE_F32);
}

void sp_cuda_sqfree_write_v(sp_cuda_sqfree_cache_t *cc, int layer, int head, int pos, const float *d_v_vec)
{
    sp_clear_error();
    if (sq_check(cc, layer, 1, head, pos, 1) || !d_v_vec) { if (!d_v_vec) sp_set_error(SP_ERR_ARG, "NULL vector"); return; }
    sq_write(cc, 1, layer, 1, head, 1, pos, 1, d_v_vec, SP_DTYPE_F32);
}

void sp_cuda_sqfree_read_k(const sp_cuda_sqfree_cache_t *cc, int layer, int head, int pos, float *d_k_out)
{
    sp_clear_error();
    sq_read(cc, 0, layer, head, pos, 1, d_k_out);
}

void sp_cuda_sqfree_read_v(const sp_cuda_sqfree_cache_t *cc, int layer, int head, int pos, float *d_v_out)
{
    sp_clear_error();
    sq_read(cc, 1, layer, head, pos, 1, d_v_out);
}

void sp_cuda_sqfree_read_k_batch(const sp_cuda_sqfree_cache_t *cc, int layer, int head, int start_pos,
                                 int n_pos, float *d_k_out)
{
    sp_clear_error();
    sq_read(cc, 0, layer, head, start_pos, n_pos, d_k_out);
}

void sp_cuda_sqfree_read_v_batch(const sp_cuda_sqfree_cache_t *cc, int layer, int head, int start_pos,
                                 int n_pos, float *d_v_out)
{
    sp_clear_error();
    sq_read(cc, 1, layer, head, start_pos, n_pos, d_v_out);
}

int sp_cuda_sqfree_write_kv_tokens(sp_cuda_sqfree_cache_t *cc, int layer0, int n_layers, int start_pos,
                                   int n_tokens, const void *d_k, const void *d_v, int dtype)
{
    sp_clear_error();
    int rc = sq_check(cc, layer0, n_layers, 0, start_pos, n_tokens);
    if (rc) return rc;
    const int H = cc->config.n_heads_kv;
    if (d_k && d_v && n_tokens > 0) {
        // both halves in one launch when the lane encoder takes them
        SpSqDev tk = sq_desc(cc, 0), tv = sq_desc(cc, 1);
        SqIo ik, iv;
        if ((rc = sq_write_io(cc, 0, layer0, n_layers, 0, H, start_pos, n_tokens, d_k, tk, ik)) ||
            (rc = sq_write_io(cc, 1, layer0, n_layers, 0, H, start_pos, n_tokens, d_v, tv, iv)))
            return rc;
        const SpSqDev *tt[2] = {&tk, &tv};
        const SqIo *ii[2] = {&ik, &iv};
        if (sq_lane_try(tt, ii, dtype, sq_status(cc), (cudaStream_t)cc->stream, &rc)) return rc;
    }
    if (d_k && (rc = sq_write(cc, 0, layer0, n_layers, 0, H, start_pos, n_tokens, d_k, dtype))) return rc;
    if (d_v && (rc = sq_write(cc, 1, layer0, n_layers, 0, H, start_pos, n_tokens, d_v, dtype))) return rc;
    return SP_OK;
}

int sp_cuda_sqfree_attn_decode(const sp_cuda_sqfree_cache_t *cc, int layer0, int n_layers, const void *d_q,
                               int n_q_heads, int kv_len, float logit_scale, void *d_out, void *stream)
{
    sp_clear_error();
    if (!cc || !cc->d_k_cache || !d_q || !d_out) return sp_set_error(SP_ERR_ARG, "sqfree_attn_decode: NULL argument");
    const int H = cc->config.n_heads_kv;
    if (layer0 < 0 || n_layers <= 0 || layer0 + n_layers > cc->config.n_layers)
        return sp_set_error(SP_ERR_ARG, "sqfree_attn_decode: layers out of range");
    if (n_q_heads <= 0 || n_q_heads % H || n_q_heads / H > 8)
        return sp_set_error(SP_ERR_ARG, "sqfree_attn_decode: n_q_heads %d must be a multiple of %d with <= 8 per KV head",
                            n_q_heads, H);
    if (kv_len < 0 || kv_len > cc->max_seq_len)
        return sp_set_error(SP_ERR_ARG, "sqfree_attn_decode: kv_len %d outside [0,%d]", kv_len, cc->max_seq_len);
    SpSqDev tk = sq_desc(cc, 0), tv = sq_desc(cc, 1);
    SqAttn a;
    memset(&a, 0, sizeof(a));
    a.k_cache = cc->d_k_cache;
    a.v_cache = cc->d_v_cache;
    a.k_slot_stride = (long long)cc->max_seq_len * tk.bytes_per_pos;
    a.v_slot_stride = (long long)cc->max_seq_len * tv.bytes_per_pos;
    a.q = (const __half *)d_q;
    a.out = (__half *)d_out;
    a.ws = (float *)cc->d_attn_ws;
    a.layer0 = layer0;
    a.n_layers = n_layers;
    a.n_kv_heads = H;
    a.n_q_heads = n_q_heads;
    a.group = n_q_heads / H;
    a.kv_len = kv_len;
    a.logit_scale = logit_scale;
    a.store_width_k = store_width_for(tk.bytes_per_pos, a.k_slot_stride, a.k_cache);
    a.store_width_v = store_width_for(tv.bytes_per_pos, a.v_slot_stride, a.v_cache);
    const int units = n_layers * H;
    int splits = (148 * 8 + units - 1) / units;
    const int max_by_len = (kv_len + 63) / 64;
    if (splits > max_by_len) splits = max_by_len;
    if (splits > kSqMaxSplits) splits = kSqMaxSplits;
    if (splits < 1) splits = 1;
    a.chunk = (kv_len + splits - 1) / splits;
    a.n_splits = kv_len == 0 ? 0 : (kv_len + a.chunk - 1) / a.chunk;
    cudaStream_t s = (cudaStream_t)stream;
    a.status = reinterpret_cast<unsigned int *>(reinterpret_cast<char *>(cc->d_attn_ws) + cc->attn_ws_bytes);
    // Blocked kernel: up to 4 queries per KV head, 4 skeleton slots and 2
    // residuals per lane, 8 Möbius terms per lane, 4-byte rows, and 16-byte
    // aligned 4-position blocks for the bulk copies.
    bool same_layout = tk.bytes_per_pos == tv.bytes_per_pos && tk.bl.n_bands == tv.bl.n_bands &&
                       tk.res_off == tv.res_off && tk.sheet_off == tv.sheet_off && tk.mag_off == tv.mag_off &&
                       tk.res_bits == tv.res_bits && tk.use_spinor == tv.use_spinor;
    for (int b = 0; same_layout && b < tk.bl.n_bands; b++)
        same_layout = tk.bl.bits[b] == tv.bl.bits[b] && tk.bl.off[b] == tv.bl.off[b] &&
                      tk.bl.size[b] == tv.bl.size[b] && tk.bl.byte_off[b] == tv.bl.byte_off[b];
    const bool blocked = same_layout && a.group <= 4 && tk.n_skel <= 128 && cc->lane_max_terms > 0 &&
                         cc->lane_max_terms <= 8 &&
                         tk.bytes_per_pos % 4 == 0 && tv.bytes_per_pos % 4 == 0 &&
                         a.k_slot_stride % 16 == 0 && a.v_slot_stride % 16 == 0 &&
                         ((uintptr_t)a.k_cache & 15) == 0 && ((uintptr_t)a.v_cache & 15) == 0 &&
                         getenv("SHANNON_PRIME_SQFREE_DECODE_REG") == nullptr;
    // Lane-per-slot tensor-core kernel: the compiled config-2 layout for K
    // and V, up to 4 queries per KV head, 16-byte aligned 32-position tiles.
    const bool lane_tc = a.group <= 4 && sa_fits(tk) && sa_fits(tv) && a.k_slot_stride % 16 == 0 &&
                         a.v_slot_stride % 16 == 0 && ((uintptr_t)a.k_cache & 15) == 0 &&
                         ((uintptr_t)a.v_cache & 15) == 0 && getenv("SHANNON_PRIME_SQFREE_DECODE_BLOCKED") == nullptr &&
                         getenv("SHANNON_PRIME_SQFREE_DECODE_REG") == nullptr;
    if (lane_tc && kv_len > 0) {
        static std::atomic<int> occ_dev{-1}, occ_val{0}, occ_sms{0};
        int dev = 0;
        cudaGetDevice(&dev);
        const size_t sm = sizeof(SaSmem);
        if (occ_dev.load() != dev) {
            if (cudaFuncSetAttribute(k_sq_attn_lane, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
                return sp_check_cuda(cudaGetLastError(), "sqfree lane attention smem attribute");
            int occ = 0, sms = 0;
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_sq_attn_lane, kSaWarps * 32, sm);
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            occ_val = occ < 1 ? 1 : occ;
            occ_sms = sms < 1 ? 148 : sms;
            occ_dev = dev;
        }
        // Splits: the count (at most one tile per warp's worth of positions
        // per split and kSqMaxSplits) with the least modelled time: waves of
        // resident CTAs times (32-position tiles of the busiest warp + a
        // fixed cost per CTA of about two tiles: query fragments, the warp
        // merge and the partial stores).  Long CTAs amortise that cost and
        // keep a CTA's four warps balanced.
        const long long slots = (long long)occ_val.load() * occ_sms.load();
        const int max_s = std::max(1, std::min(kSqMaxSplits, (kv_len + 32 * kSaWarps - 1) / (32 * kSaWarps)));
        constexpr double kCtaFixedTiles = 2.0;
        int best = 1;
        double best_cost = 1e300;
        for (int sp = 1; sp <= max_s; sp++) {
            const long long ctas = (long long)units * sp;
            const long long waves = (ctas + slots - 1) / slots;
            const int chunk = ((kv_len + sp - 1) / sp + 31) / 32 * 32;
            const int tiles = (chunk + 31) / 32;
            const double cost = (double)waves * ((tiles + kSaWarps - 1) / kSaWarps + kCtaFixedTiles);
            if (cost < best_cost - 1e-9) { best_cost = cost; best = sp; }
        }
        a.chunk = ((kv_len + best - 1) / best + 31) / 32 * 32;
        a.n_splits = (kv_len + a.chunk - 1) / a.chunk;
        a.qws = reinterpret_cast<float *>(reinterpret_cast<char *>(cc->d_attn_ws) + cc->attn_ws_bytes + 16);
        k_sa_query<<<(n_layers * n_q_heads + 3) / 4, 128, 0, s>>>(a);
        k_sq_attn_lane<<<dim3(a.n_splits, H, n_layers), kSaWarps * 32, sm, s>>>(a);
        int rc = sp_check_cuda(cudaGetLastError(), "sqfree lane attention launch");
        if (rc) return rc;
        k_sq_attn_combine<<<dim3(n_q_heads, n_layers), kSqCombineThreads, sq_combine_smem(tk), s>>>(tk, a);
        return sp_check_cuda(cudaGetLastError(), "sqfree attention combine launch");
    }
    if (blocked && a.n_splits > 0) {
        a.chunk = (a.chunk + 15) / 16 * 16;
        a.n_splits = (kv_len + a.chunk - 1) / a.chunk;
        const size_t sm = sq_attn3_smem(tk, tv);
        auto k3 = k_sq_attn3<4, 2, 8>;
        cudaFuncSetAttribute(k3, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        k3<<<dim3(a.n_splits, H, n_layers), kSq3Warps * 32, sm, s>>>(tk, tv, a);
        int rc = sp_check_cuda(cudaGetLastError(), "sqfree attention launch");
        if (rc) return rc;
        k_sq_attn_combine<<<dim3(n_q_heads, n_layers), kSqCombineThreads, sq_combine_smem(tk), s>>>(tk, a);
        return sp_check_cuda(cudaGetLastError(), "sqfree attention combine launch");
    }
    int GT = 0;
    SqAttnKernel kreg = sq_attn_reg_kernel(a.group, (tk.n_skel + 31) / 32, (tk.n_res + 31) / 32, &GT);
    // the prefetch ring copies rows in 4-byte pieces; Möbius terms live in registers
    if (a.store_width_k != 4 || a.store_width_v != 4 || cc->csr_max_terms > kSqMaxTerms) kreg = nullptr;
    if (a.n_splits > 0 && kreg) {
        const size_t sm = sq_attn_reg_smem(tk, tv, GT);
        cudaFuncSetAttribute(kreg, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        kreg<<<dim3(a.n_splits, H, n_layers), kSqAttnWarps * 32, sm, s>>>(tk, tv, a);
        int rc = sp_check_cuda(cudaGetLastError(), "sqfree attention launch");
        if (rc) return rc;
    } else if (a.n_splits > 0) {
        const size_t sm = sq_attn_smem(tk, a.group);
        cudaFuncSetAttribute(k_sq_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        k_sq_attn<<<dim3(a.n_splits, H, n_layers), kSqAttnWarps * 32, sm, s>>>(tk, tv, a);
        int rc = sp_check_cuda(cudaGetLastError(), "sqfree attention launch");
        if (rc) return rc;
    }
    k_sq_attn_combine<<<dim3(n_q_heads, n_layers), kSqCombineThreads, sq_combine_smem(tk), s>>>(tk, a);
    return sp_check_cuda(cudaGetLastError(), "sqfree attention combine launch");
}

// ------------------------------------------------------------------ hier --

int sp_cuda_hier_cache_init(sp_cuda_hier_cache_t *hc, const sp_config_t *cfg, int pad_dim, int n_skeleton,
                            int n_target, int target_res_bits, const int *skeleton_idx, const int *target_idx,
                            const sp_band_config_t *skel_bands, int max_seq_len, int n_slots, void *stream)
{
    sp_clear_error();
    if (!hc || !cfg || !skeleton_idx || !target_idx || !skel_bands)
        return sp_set_error(SP_ERR_ARG, "hier_cache_init: NULL argument");
    memset(hc, 0, sizeof(*hc));
    if (pad_dim < cfg->head_dim || pad_dim > kSqMaxPd || n_skeleton < 1 || n_target < 0 ||
        n_skeleton + n_target > pad_dim || max_seq_len <= 0 || n_slots <= 0 ||
        target_res_bits < 1 || target_res_bits > 8 || skel_bands->head_dim != n_skeleton)
        return sp_set_error(SP_ERR_ARG, "hier_cache_init: bad dims");
    hc->config = *cfg;
    hc->pad_dim = pad_dim;
    hc->n_skeleton = n_skeleton;
    hc->n_target = n_target;
    hc->target_res_bits = target_res_bits;
    hc->n_slots = n_slots;
    hc->max_seq_len = max_seq_len;
    hc->skel_bands = *skel_bands;
    hc->stream = stream;
    cudaGetDevice(&hc->device);
    std::vector<int> tables(skeleton_idx, skeleton_idx + n_skeleton);
    tables.insert(tables.end(), target_idx, target_idx + n_target);
    for (int r = 0; r <= n_target; r++) tables.push_back(0);      // empty CSR
    for (int i = 0; i < n_skeleton + n_target; i++) {
        const int v = tables[i];
        if (v < 0 || v >= pad_dim) return sp_set_error(SP_ERR_ARG, "hier_cache_init: index %d outside pad_dim", v);
    }
    int factors[kSqMaxStages], nf = 0;
    {
        int r = pad_dim;
        for (int p : {2, 3, 5, 7, 11}) while (r % p == 0 && nf < kSqMaxStages) { factors[nf++] = p; r /= p; }
        if (r != 1) return sp_set_error(SP_ERR_UNSUPPORTED, "hier_cache_init: pad_dim %d not {2,3,5,7,11}-smooth", pad_dim);
    }
    hc->n_factors = nf;
    int rc = SP_OK;
    auto up = [&](void **dst, const void *src, size_t bytes, const char *what) {
        if (rc) return;
        if ((rc = sp_check_cuda(cudaMalloc(dst, bytes > 0 ? bytes : 4), what))) return;
        if (bytes && src) rc = sp_check_cuda(cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice), what);
    };
    up(&hc->d_tables, tables.data(), tables.size() * 4, "hier tables");
    up((void **)&hc->d_skeleton_idx, skeleton_idx, (size_t)n_skeleton * 4, "skeleton idx");
    up((void **)&hc->d_target_idx, target_idx, (size_t)n_target * 4, "target idx");
    up((void **)&hc->d_vilenkin_factors, factors, (size_t)nf * 4, "factors");
    up((void **)&hc->d_skel_band_bits, skel_bands->band_bits, (size_t)skel_bands->n_bands * 4, "band bits");
    if (rc) { sp_cuda_hier_cache_free(hc); return rc; }
    SpSqDev t = hier_desc(hc);
    if ((t.bytes_per_pos + 3) / 4 + 2 > kSqRowWords || sq_smem_bytes(t) > 220 * 1024) {
        sp_cuda_hier_cache_free(hc);
        return sp_set_error(SP_ERR_UNSUPPORTED, "hier_cache_init: slot or predictor too large");
    }
    hc->bytes_per_pos_k = hc->bytes_per_pos_v = t.bytes_per_pos;
    const size_t total = (size_t)n_slots * max_seq_len * t.bytes_per_pos;
    up((void **)&hc->d_k_cache, nullptr, total, "cudaMalloc K cache");
    up((void **)&hc->d_v_cache, nullptr, total, "cudaMalloc V cache");
    up((void **)&hc->d_W, nullptr, (size_t)n_slots * n_target * n_skeleton * 2, "cudaMalloc W");
    if (rc) { sp_cuda_hier_cache_free(hc); return rc; }
    cudaMemset(hc->d_k_cache, 0, total);
    cudaMemset(hc->d_v_cache, 0, total);
    cudaMemset(hc->d_W, 0, (size_t)n_slots * n_target * n_skeleton * 2);
    up((void **)&hc->d_status, nullptr, 16, "cudaMalloc hier status");
    if (!rc) cudaMemset(hc->d_status, 0, 16);
    if (hr_kernel(t)) {      // tensor-core batched read: transform rows + per-slot matrices
        const std::vector<float> vr = hr_transform_rows(pad_dim, cfg->head_dim);
        up((void **)&hc->d_vrows, vr.data(), vr.size() * 4, "hier transform rows");
        up(&hc->d_recon, nullptr,
           (size_t)n_slots * cfg->head_dim * hr_stride(t.bl.n_bands, n_target) * 2, "hier reconstruction");
        if (!rc) rc = hr_build(hc);
        if (rc) { sp_cuda_hier_cache_free(hc); return rc; }
    }
    if ((rc = sq_upload_constants()) || (rc = sp_check_cuda(cudaDeviceSynchronize(), "hier_cache_init"))) {
        sp_cuda_hier_cache_free(hc);
        return rc;
    }
    return SP_OK;
}

void sp_cuda_hier_cache_free(sp_cuda_hier_cache_t *hc)
{
    if (!hc) return;
    cudaFree(hc->d_tables);
    cudaFree(hc->d_skeleton_idx);
    cudaFree(hc->d_target_idx);
    cudaFree(hc->d_vilenkin_factors);
    cudaFree(hc->d_skel_band_bits);
    cudaFree(hc->d_k_cache);
    cudaFree(hc->d_v_cache);
    cudaFree(hc->d_W);
    cudaFree(hc->d_vrows);
    cudaFree(hc->d_recon);
    cudaFree(hc->d_status);
    memset(hc, 0, sizeof(*hc));
}

int sp_cuda_hier_cache_upload_W(sp_cuda_hier_cache_t *hc, const uint16_t *W_all)
{
    sp_clear_error();
    if (!hc || !hc->d_W || !W_all) return sp_set_error(SP_ERR_ARG, "hier_upload_W: NULL argument");
    const size_t bytes = (size_t)hc->n_slots * hc->n_target * hc->n_skeleton * 2;
    int rc = sp_check_cuda(cudaMemcpy(hc->d_W, W_all, bytes, cudaMemcpyHostToDevice), "hier_upload_W");
    return rc ? rc : hr_build(hc);
}

static int hier_check(const sp_cuda_hier_cache_t *hc, int layer, int n_layers, int head, int pos, int n)
{
    if (!hc || !hc->d_k_cache) return sp_set_error(SP_ERR_ARG, "hier cache not initialised");
    const int H = hc->config.n_heads_kv;
    if (layer < 0 || n_layers < 0 || head < 0 || head >= H || (long long)(layer + n_layers) * H > hc->n_slots)
        return sp_set_error(SP_ERR_ARG, "hier: layer/head out of range");
    if (pos < 0 || n < 0 || (long long)pos + n > hc->max_seq_len)
        return sp_set_error(SP_ERR_ARG, "hier: positions [%d,%d) outside the cache", pos, pos + n);
    return SP_OK;
}

static int hier_io(const sp_cuda_hier_cache_t *hc, int which, int layer0, int n_layers, int head, int nh,
                   int start_pos, int n_tok, SqIo &io)
{
    memset(&io, 0, sizeof(io));
    const int H = hc->config.n_heads_kv;
    io.slot_stride = (long long)hc->max_seq_len * hc->bytes_per_pos_k;
    io.cache = which ? hc->d_v_cache : hc->d_k_cache;
    io.W = (const __half *)hc->d_W;
    io.layer0 = layer0;
    io.n_layers = n_layers;
    io.nh = nh;
    io.start_pos = start_pos;
    io.n_tok = n_tok;
    if (nh != H) {            // single head: slot = layer0 * H + head
        if (n_layers != 1) return sp_set_error(SP_ERR_ARG, "hier: per-head calls take one layer");
        io.layer0 = layer0 * H + head;
        io.nh = 1;
    }
    return SP_OK;
}

int sp_cuda_hier_write_kv_tokens(sp_cuda_hier_cache_t *hc, int layer0, int n_layers, int start_pos,
                                 int n_tokens, const void *d_k, const void *d_v, int dtype)
{
    sp_clear_error();
    int rc = hier_check(hc, layer0, n_layers, 0, start_pos, n_tokens);
    if (rc) return rc;
    SpSqDev t = hier_desc(hc);
    const int H = hc->config.n_heads_kv;
    for (int which = 0; which < 2; which++) {
        const void *in = which ? d_v : d_k;
        if (!in) continue;
        SqIo io;
        if ((rc = hier_io(hc, which, layer0, n_layers, 0, H, start_pos, n_tokens, io))) return rc;
        io.in = in;
        if ((rc = sq_launch_encode(t, io, dtype, (cudaStream_t)hc->stream))) return rc;
    }
    return SP_OK;
}

int sp_cuda_hier_read_kv_tokens(const sp_cuda_hier_cache_t *hc, int layer0, int n_layers, int start_pos,
                                int n_pos, float *d_k_out, float *d_v_out)
{
    sp_clear_error();
    int rc = hier_check(hc, layer0, n_layers, 0, start_pos, n_pos);
    if (rc) return rc;
    SpSqDev t = hier_desc(hc);
    const int H = hc->config.n_heads_kv;
    for (int which = 0; which < 2; which++) {
        float *out = which ? d_v_out : d_k_out;
        if (!out) continue;
        SqIo io;
        if ((rc = hier_io(hc, which, layer0, n_layers, 0, H, start_pos, n_pos, io))) return rc;
        io.out = out;
        HrKernel hk = hc->d_recon && !getenv("SHANNON_PRIME_HIER_READ_SIMT") ? hr_kernel(t) : nullptr;
        if (hk && n_pos > 0 && hr_tc_supported(t) && !getenv("SHANNON_PRIME_HIER_READ_MMA_SYNC")) {
            HrTcArgs ta;
            ta.h.cache = io.cache;
            ta.h.slot_stride = io.slot_stride;
            ta.h.cache_end = io.cache + (long long)hc->n_slots * io.slot_stride;
            ta.h.recon = (const __half *)hc->d_recon;
            ta.h.out = out;
            ta.h.layer0 = layer0; ta.h.n_layers = n_layers; ta.h.nh = H; ta.h.start_pos = start_pos;
            ta.h.n_tok = n_pos; ta.h.tokens_per_cta = 0;
            ta.status = hc->d_status;
            ta.tiles_per_slot = (n_pos + tc::kM - 1) / tc::kM;
            ta.total_tiles = (long long)n_layers * H * ta.tiles_per_slot;
            int sms = 148;
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, hc->device);
            const long long grid = ta.total_tiles < sms ? ta.total_tiles : sms;
            const size_t sm = hr_tc_smem_bytes();
            cudaFuncSetAttribute(k_hier_recon_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
            k_hier_recon_tc<<<(unsigned)grid, tc::kThreads, sm, (cudaStream_t)hc->stream>>>(t, ta);
            if ((rc = sp_check_cuda(cudaGetLastError(), "hier tcgen05 read launch"))) return rc;
            continue;
        }
        if (hk && n_pos > 0) {
            HrArgs a;
            a.cache = io.cache;
            a.slot_stride = io.slot_stride;
            a.cache_end = io.cache + (long long)hc->n_slots * io.slot_stride;
            a.recon = (const __half *)hc->d_recon;
            a.out = out;
            a.layer0 = layer0; a.n_layers = n_layers; a.nh = H; a.start_pos = start_pos; a.n_tok = n_pos;
            const int slots = n_layers * H;
            int chunks = (148 * 2 + slots - 1) / slots;
            const int max_chunks = (n_pos + 16 * kHrWarps - 1) / (16 * kHrWarps);
            if (chunks > max_chunks) chunks = max_chunks;
            if (chunks < 1) chunks = 1;
            a.tokens_per_cta = ((n_pos + chunks - 1) / chunks + 15) / 16 * 16;
            chunks = (n_pos + a.tokens_per_cta - 1) / a.tokens_per_cta;
            const size_t sm = hr_smem_bytes(t, t.hd);
            cudaFuncSetAttribute(hk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
            hk<<<dim3(chunks, slots), kHrWarps * 32, sm, (cudaStream_t)hc->stream>>>(t, a);
            if ((rc = sp_check_cuda(cudaGetLastError(), "hier tensor-core read launch"))) return rc;
            continue;
        }
        if ((rc = sq_launch_decode(t, io, (cudaStream_t)hc->stream))) return rc;
    }
    return SP_OK;
}

static void hier_one(sp_cuda_hier_cache_t *hc, int which, int layer, int head, int pos, const float *in, float *out)
{
    sp_clear_error();
    if (hier_check(hc, layer, 1, head, pos, 1)) return;
    if (!in && !out) { sp_set_error(SP_ERR_ARG, "hier: NULL vector"); return; }
    SpSqDev t = hier_desc(hc);
    SqIo io;
    if (hier_io(hc, which, layer, 1, head, 1, pos, 1, io)) return;
    if (in) {
        io.in = in;
        sq_launch_encode(t, io, SP_DTYPE_F32, (cudaStream_t)hc->stream);
    } else {
        io.out = out;
        io.single_slot = 1;
        sq_launch_decode(t, io, (cudaStream_t)hc->stream);
    }
}

void sp_cuda_hier_write_k(sp_cuda_hier_cache_t *hc, int layer, int head, int pos, const float *d_k_vec)
{ hier_one(hc, 0, layer, head, pos, d_k_vec, nullptr); }
void sp_cuda_hier_write_v(sp_cuda_hier_cache_t *hc, int layer, int head, int pos, const float *d_v_vec)
{ hier_one(hc, 1, layer, head, pos, d_v_vec, nullptr); }
void sp_cuda_hier_read_k(const sp_cuda_hier_cache_t *hc, int layer, int head, int pos, float *d_k_out)
{ hier_one((sp_cuda_hier_cache_t *)hc, 0, layer, head, pos, nullptr, d_k_out); }
void sp_cuda_hier_read_v(const sp_cuda_hier_cache_t *hc, int layer, int head, int pos, float *d_v_out)
{ hier_one((sp_cuda_hier_cache_t *)hc, 1, layer, head, pos, nullptr, d_v_out); }

}  // extern "C"

// Token-major read of every KV head of a layer range in one launch (the
// per-head read loop of a cache's read_gpu), config-2 slot layout only:
// which 0 = K, 1 = V; d_out [n_layers][n_tok][n_heads_kv][head_dim] fp32.
int sp_cuda_sqfree_read_kv_tokens(const sp_cuda_sqfree_cache_t *cc, int which, int layer0, int n_layers,
                                  int start_pos, int n_tok, float *d_out)
{
    sp_clear_error();
    if (!cc || !d_out || (which != 0 && which != 1))
        return sp_set_error(SP_ERR_ARG, "sqfree read_kv_tokens: bad arguments");
    if (n_layers == 0 || n_tok == 0) return SP_OK;
    int rc = sq_check(cc, layer0, n_layers, 0, start_pos, n_tok);
    if (rc) return rc;
    if (cudaSetDevice(cc->device) != cudaSuccess) return sp_set_error(SP_ERR_CUDA, "sqfree read_kv_tokens: cudaSetDevice");
    const SpSqDev t = sq_desc(cc, which);
    SqIo io;
    memset(&io, 0, sizeof(io));
    io.slot_stride = (long long)cc->max_seq_len * t.bytes_per_pos;
    io.cache = (uint8_t *)(which ? cc->d_v_cache : cc->d_k_cache);
    const int H = cc->config.n_heads_kv;
    if (!sq_lane_fits(t, io) || ((uintptr_t)d_out & 15) || (((uintptr_t)start_pos * t.bytes_per_pos) & 3))
        return sp_set_error(SP_ERR_UNSUPPORTED, "sqfree read_kv_tokens: the head_dim-128 spinor layout "
                                                "(pad 154, 5 skeleton bands, 3-bit residuals) with a 16-byte "
                                                "aligned output");
    const SlGrid g{io.slot_stride, (long long)layer0 * H, H, n_layers, start_pos};
    const int r = sq_read_lane(io.cache, g, n_tok, d_out, sq_status(cc), (cudaStream_t)cc->stream);
    if (r > 0) return sp_set_error(SP_ERR_UNSUPPORTED, "sqfree read_kv_tokens: no tensor-map encoder in this driver");
    return r ? sp_set_error(SP_ERR_CUDA, "sqfree read_kv_tokens: launch failed") : SP_OK;
}
