// sp_ship_lane.cu — lane-per-vector ship encoder for head_dim 128.
//
// The write path (VHT2 -> Möbius reorder -> band quantise -> pack, reference
// sp_cuda_write_k/_v, shannon_prime_cuda.cu:474-521, 565-620) for the two
// ship layouts at head_dim 128: K bands 4 x 32 at 5/5/4/3 bits with the
// squarefree-first order (76-byte rows), V one 128-code band at 3 bits
// (50-byte rows).
//
// One thread owns one whole vector.  A warp takes 32 consecutive positions
// of one head:
//   - one elected lane fetches the batch's 32 input rows with tiled TMA
//     copies (cp.async.bulk.tensor over a [tokens][heads][128] tensor map,
//     128-byte column slices, no multicast) into shared memory with the
//     128-byte swizzle, so each lane's 16-byte reads of its own row fall in
//     distinct banks for the 8 lanes of a phase; the copy of the next batch
//     is issued as soon as the current one sits in registers, so it
//     streams under the arithmetic;
//   - the 128-point Hartley butterfly runs entirely in the thread's
//     registers (896 IEEE adds, no shuffles);
//   - the Möbius order and the band layout are compile-time, so the
//     reorder is register renaming and every code's bit position is a
//     constant: one shift-add per code into the row's words;
//   - the 32 packed rows of the batch are contiguous in the slot, so they
//     are staged in shared memory and written back by one bulk store.
// That is about 60 warp instructions per vector, against ~190 for the
// lane-group kernel in sp_ship.cu, which remains the path for every other
// layout and for a caller-supplied Möbius table.
//
// Bit-exactness: the arithmetic is the same sequence of single IEEE
// operations as the CPU restatement (ascending butterfly lengths, then
// x * (1/sqrt(n)); band absmax skipping NaN; IEEE amax / m; fp16 RNE scale;
// IEEE 1/stored; rint; clamp), so codes equal those of the lane-group
// kernel and of the oracle.
#include "sp_internal.cuh"
#include "sp_bulk.cuh"

#include <atomic>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdlib.h>
#include <string.h>

namespace {

constexpr int kLN = 128;              // coefficients per vector
constexpr int kLaneWarps = 4;         // warps per CTA
constexpr int kLaneMinBlocks = 3;     // CTAs per SM (12 warps, <= 170 registers)

// Compile-time ship layouts.  KS: K (4 bands of 32, 5/5/4/3 bits, Möbius
// order); otherwise V (1 band of 128 at 3 bits, natural order).
template <bool KS> struct LaneLayout;
template <> struct LaneLayout<true> {
    static constexpr int NB = 4, TB = 76, SIZE = 32;
    __host__ __device__ static constexpr int bits(int b) { return b < 2 ? 5 : (b == 2 ? 4 : 3); }
    __host__ __device__ static constexpr int byte_off(int b) { return b == 0 ? 0 : b == 1 ? 22 : b == 2 ? 44 : 62; }
};
template <> struct LaneLayout<false> {
    static constexpr int NB = 1, TB = 50, SIZE = 128;
    __host__ __device__ static constexpr int bits(int) { return 3; }
    __host__ __device__ static constexpr int byte_off(int) { return 0; }
};

__host__ __device__ constexpr bool lane_squarefree(int n)
{
    for (int p = 2; p * p <= n; p++)
        if (n % (p * p) == 0) return false;
    return true;
}

// Squarefree-first order of 0..127 (indices i with i+1 squarefree,
// ascending, then the rest ascending): the table sp_mobius_mask_init
// builds for every cache.
struct LaneOrder { int v[kLN]; };
__host__ __device__ constexpr LaneOrder lane_order()
{
    LaneOrder o{};
    int k = 0;
    for (int i = 0; i < kLN; i++)
        if (lane_squarefree(i + 1)) o.v[k++] = i;
    for (int i = 0; i < kLN; i++)
        if (!lane_squarefree(i + 1)) o.v[k++] = i;
    return o;
}

struct LaneHalf {
    const void *in;            // [n_tokens][nh][128]
    uint8_t *out_base;         // slab base
    long long slot0;           // slot of head 0
    long long slot_stride;     // bytes per slot
};

// One launch encodes the K half (half 0, K layout) and/or the V half
// (half 1, V layout) of the same tokens.
struct LaneArgs {
    LaneHalf half[2];
    int first;                 // first half present (0 = K, 1 = V)
    int n_halves;              // 1 or 2
    int n_tokens;
    int nh;
    int start_pos;
    int nb;                    // batches per half: nh * ceil(n_tokens / 32)
    float inv_sqrt_n;
    unsigned int *status;      // bit 0: a bulk copy did not land in time
};

// Tensor maps of the two halves' inputs ([n_tokens][nh][128], 128-byte
// boxes of 32 tokens x 1 head, 128-byte swizzle).
struct alignas(64) LaneMaps {
    CUtensorMap m[2];
};

template <typename Tin>
struct LaneSmem {
    static constexpr int RB = kLN * (int)sizeof(Tin);          // input row bytes
    static constexpr int OB = 32 * 76;                         // packed rows of a batch (K is the larger)
    alignas(1024) unsigned char in[kLaneWarps][32][RB];
    unsigned char out[kLaneWarps][OB];
    unsigned long long bar[kLaneWarps];
};

__device__ __forceinline__ void bulk_s2g(void *dst, uint32_t src, uint32_t bytes)
{
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src), "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read()
{
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all()
{
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

template <typename Tin>
__device__ __forceinline__ void lane_unpack16(const uint4 &w, float *x)
{
    if constexpr (sizeof(Tin) == 4) {
        x[0] = __uint_as_float(w.x); x[1] = __uint_as_float(w.y);
        x[2] = __uint_as_float(w.z); x[3] = __uint_as_float(w.w);
    } else {
        const Tin *h = reinterpret_cast<const Tin *>(&w);
#pragma unroll
        for (int i = 0; i < 8; i++) x[i] = sp_load_as_float(h, i);
    }
}

// Initial row words: the offset mv << s of every code that starts in the
// word (the codes are then added as signed q << s).
template <bool KS> struct LaneRowInit { uint32_t w[(LaneLayout<KS>::TB + 3) / 4]; };
template <bool KS>
__host__ __device__ constexpr LaneRowInit<KS> lane_row_init()
{
    using L = LaneLayout<KS>;
    LaneRowInit<KS> r{};
    for (int b = 0; b < L::NB; b++) {
        const int bits = L::bits(b), mv = (1 << (bits - 1)) - 1;
        for (int k = 0; k < L::SIZE; k++) {
            const int p = 8 * L::byte_off(b) + 16 + k * bits;
            r.w[p >> 5] += (uint32_t)mv << (p & 31);
        }
    }
    return r;
}

// Quantise and pack the lane's transformed vector into its row, stage the
// warp's 32 rows in shared memory and write them back (one bulk store when
// the batch's rows are 16-byte aligned in the slot, else plain stores).
template <bool KS>
__device__ __forceinline__ void lane_pack_store(const float (&x)[kLN], unsigned char *stage, uint8_t *dst,
                                                int live, int lane)
{
    using L = LaneLayout<KS>;
    constexpr int TB = L::TB;
    constexpr int W = (TB + 3) / 4;             // row words (the last may be partial)
    constexpr LaneOrder ord = lane_order();
    constexpr LaneRowInit<KS> init = lane_row_init<KS>();
    uint32_t row[W];
#pragma unroll
    for (int k = 0; k < W; k++) row[k] = init.w[k];
#pragma unroll
    for (int b = 0; b < L::NB; b++) {
        const int bits = L::bits(b);
        const int mv = (1 << (bits - 1)) - 1;
        // 8 independent partial maxima (each starts at 0, so none is ever
        // NaN and the tree gives the sequential result), not one chain of
        // SIZE dependent fmaxf.
        float am[8];
#pragma unroll
        for (int j = 0; j < 8; j++) am[j] = 0.0f;
#pragma unroll
        for (int k = 0; k < L::SIZE; k++) {
            const int i = KS ? ord.v[b * L::SIZE + k] : k;
            am[k & 7] = fmaxf(am[k & 7], fabsf(x[i]));
        }
#pragma unroll
        for (int j = 0; j < 4; j++) am[j] = fmaxf(am[j], am[j + 4]);
        const float amax = fmaxf(fmaxf(am[0], am[2]), fmaxf(am[1], am[3]));
        const float scale = amax > 0.0f ? __fdiv_rn(amax, (float)mv) : 0.0f;
        const __half hs = __float2half_rn(scale);
        const float stored = __half2float(hs);
        const float inv = stored > 0.0f ? __frcp_rn(stored) : 0.0f;
        const int sbit = 8 * L::byte_off(b);
        row[sbit >> 5] |= (uint32_t)__half_as_ushort(hs) << (sbit & 31);
        // With a normal (or infinite, or zero) fp16 scale every |x * inv| is
        // below mv * (1 + 2^-11) < mv + 0.5, so rint never leaves [-mv, mv]
        // and the clamp is a no-op; only a subnormal scale (amax below
        // ~1e-3 * mv) can round far enough down to need it.
        const bool clamp = __any_sync(0xffffffffu, stored > 0.0f && stored < 6.103515625e-05f);
        // Codes go in as q << s with the offset mv << s of every code
        // already in the row's initial words (exact modulo 2^32); a code that
        // straddles two words adds its high bits from u = q + mv.
        auto put = [&](int k, int q) {
            const int p = sbit + 16 + k * bits;
            row[p >> 5] += (uint32_t)q << (p & 31);
            if ((p & 31) + bits > 32) row[(p >> 5) + 1] += (uint32_t)(q + mv) >> (32 - (p & 31));
        };
        if (clamp) {
#pragma unroll
            for (int k = 0; k < L::SIZE; k++) {
                const int i = KS ? ord.v[b * L::SIZE + k] : k;
                const int q = __float2int_rn(__fmul_rn(x[i], inv));     // NaN -> 0, saturating
                put(k, min(max(q, -mv), mv));
            }
        } else {
#pragma unroll
            for (int k = 0; k < L::SIZE; k++) {
                const int i = KS ? ord.v[b * L::SIZE + k] : k;
                put(k, __float2int_rn(__fmul_rn(x[i], inv)));
            }
        }
    }

    if (lane == 0) bulk_wait_read();            // the previous batch's store has read the stage
    __syncwarp();
    if constexpr ((TB & 3) == 0) {
        uint32_t *r32 = reinterpret_cast<uint32_t *>(stage + lane * TB);
#pragma unroll
        for (int k = 0; k < W; k++) r32[k] = row[k];
    } else {
        uint16_t *r16 = reinterpret_cast<uint16_t *>(stage + lane * TB);
#pragma unroll
        for (int k = 0; k < TB / 2; k++) r16[k] = (uint16_t)(row[k >> 1] >> (16 * (k & 1)));
    }
    spb::fence_proxy_async();
    __syncwarp();
    const uint32_t bytes = (uint32_t)(live * TB);
    if ((((uintptr_t)dst | bytes) & 15) == 0) {
        if (lane == 0) bulk_s2g(dst, spb::smem_u32(stage), bytes);
    } else if ((((uintptr_t)dst | TB) & 3) == 0) {
        const uint32_t *s32 = reinterpret_cast<const uint32_t *>(stage);
        for (uint32_t i = lane; i < bytes / 4; i += 32) reinterpret_cast<uint32_t *>(dst)[i] = s32[i];
    } else if ((((uintptr_t)dst | TB) & 1) == 0) {
        const uint16_t *s16 = reinterpret_cast<const uint16_t *>(stage);
        for (uint32_t i = lane; i < bytes / 2; i += 32) reinterpret_cast<uint16_t *>(dst)[i] = s16[i];
    } else {
        for (uint32_t i = lane; i < bytes; i += 32) dst[i] = stage[i];
    }
    __syncwarp();
}

template <typename Tin>
__global__ void __launch_bounds__(kLaneWarps * 32, kLaneMinBlocks)
k_encode_lane(LaneArgs a, const __grid_constant__ LaneMaps maps)
{
    using S = LaneSmem<Tin>;
    constexpr int RB = S::RB;
    constexpr int C = RB / 16;                  // 16-byte chunks per input row
    constexpr int EPC = 16 / (int)sizeof(Tin);  // elements per chunk
    extern __shared__ __align__(128) unsigned char smem_raw[];
    S &sm = *reinterpret_cast<S *>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int NQ = RB / 128;                // 128-byte column slices per row
    const uint32_t bar = spb::smem_u32(&sm.bar[warp]);
    const uint32_t in0 = spb::smem_u32(&sm.in[warp][0][0]);
    const int gw = blockIdx.x * kLaneWarps + warp, n_w = gridDim.x * kLaneWarps;
    const int n_total = a.nb * a.n_halves;

    // The 128-byte swizzle needs 1024-byte aligned slices.
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

    // Batch g: half first + g / nb; within it head gl % nh, positions
    // 32 * (gl / nh) ...; lane = position.  Rows past n_tokens are filled
    // with zeros by the copy (and never stored).
    auto issue = [&](int g) {
        if (lane == 0) {
            const int hx = a.first + g / a.nb, gl = g % a.nb;
            const int h = gl % a.nh, t0 = (gl / a.nh) * 32;
            const CUtensorMap *tm = hx ? &maps.m[1] : &maps.m[0];
            spb::mbar_expect_tx(bar, (uint32_t)(32 * RB));
#pragma unroll
            for (int q = 0; q < NQ; q++)
                asm volatile(
                    "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                    ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(in0 + q * 4096),
                    "l"(tm), "r"(q * (128 / (int)sizeof(Tin))), "r"(h), "r"(t0), "r"(bar), "l"(policy)
                    : "memory");
        }
    };

    uint32_t parity = 0;
    if (gw < n_total) issue(gw);
    for (int g = gw; g < n_total; g += n_w) {
        const int hx = a.first + g / a.nb, gl = g % a.nb;
        const int h = gl % a.nh, t0 = (gl / a.nh) * 32;
        const int live = min(32, a.n_tokens - t0);
        if (!spb::wait_stage(bar, parity, a.status)) {
            spb::wait_stage(bar, parity, nullptr);   // the late copy, bounded, before the CTA exits
            break;
        }
        parity ^= 1u;

        // ---- row -> registers, then the next batch's copy -----------------
        float x[kLN];
#pragma unroll
        for (int j = 0; j < C; j++) {
            // chunk j = slice j / 8, 16-byte chunk j % 8, swizzled by row
            const int off = (j >> 3) * 4096 + lane * 128 + (((j & 7) ^ (lane & 7)) << 4);
            const uint4 w = *reinterpret_cast<const uint4 *>(&sm.in[warp][0][0] + off);
            lane_unpack16<Tin>(w, &x[j * EPC]);
        }
        __syncwarp();
        spb::fence_proxy_async();
        if (g + n_w < n_total) issue(g + n_w);

        // ---- VHT2: ascending butterfly lengths, then x * (1/sqrt(n)) -------
#pragma unroll
        for (int len = 1; len < kLN; len <<= 1) {
#pragma unroll
            for (int i = 0; i < kLN; i += len << 1) {
#pragma unroll
                for (int j = 0; j < len; j++) {
                    const float u = x[i + j], v = x[i + j + len];
                    x[i + j] = __fadd_rn(u, v);
                    x[i + j + len] = __fsub_rn(u, v);
                }
            }
        }
#pragma unroll
        for (int e = 0; e < kLN; e++) x[e] = __fmul_rn(x[e], a.inv_sqrt_n);

        const LaneHalf &hf = hx ? a.half[1] : a.half[0];
        uint8_t *dst = hf.out_base + (hf.slot0 + h) * hf.slot_stride +
                       (long long)(a.start_pos + t0) * (hx ? LaneLayout<false>::TB : LaneLayout<true>::TB);
        if (hx == 0) lane_pack_store<true>(x, sm.out[warp], dst, live, lane);
        else lane_pack_store<false>(x, sm.out[warp], dst, live, lane);
    }
    if (lane == 0) bulk_wait_all();
}

template <typename Tin>
int launch_lane(const LaneArgs &a, const LaneMaps &maps, cudaStream_t s)
{
    auto k = k_encode_lane<Tin>;
    const size_t smem = sizeof(LaneSmem<Tin>);
    // per device: attribute set and occupancy looked up once (atomics, so
    // host threads driving any devices race harmlessly)
    constexpr int kMaxDev = 64;
    static std::atomic<int> occ_tab[kMaxDev], sms_tab[kMaxDev];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDev) return sp_set_error(SP_ERR_CUDA, "lane encoder: device %d", dev);
    int occ = occ_tab[dev].load(std::memory_order_acquire);
    if (occ == 0) {
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return sp_check_cuda(cudaGetLastError(), "lane encoder smem attribute");
        int o = 0, sm = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, k, kLaneWarps * 32, smem);
        cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev);
        sms_tab[dev].store(sm > 0 ? sm : 148, std::memory_order_relaxed);
        occ = o > 0 ? o : 1;
        occ_tab[dev].store(occ, std::memory_order_release);
    }
    const int sms = sms_tab[dev].load(std::memory_order_relaxed);
    long long blocks = ((long long)a.nb * a.n_halves + kLaneWarps - 1) / kLaneWarps;
    if (blocks > (long long)sms * occ) blocks = (long long)sms * occ;
    k<<<(unsigned)blocks, kLaneWarps * 32, smem, s>>>(a, maps);
    return sp_check_cuda(cudaGetLastError(), "lane encoder launch");
}

// Which half a layout is for the lane encoder: 0 = K ship layout with the
// standard order, 1 = V ship layout without reorder, -1 = not eligible.
int lane_half_of(const SpBandLayout &bl, const int *d_order, bool std_order)
{
    if (bl.n != kLN) return -1;
    if (bl.n_bands == 4 && bl.total_bytes == 76 && d_order && std_order) {
        for (int b = 0; b < 4; b++)
            if (bl.off[b] != 32 * b || bl.size[b] != 32 || bl.bits[b] != LaneLayout<true>::bits(b) ||
                bl.byte_off[b] != LaneLayout<true>::byte_off(b))
                return -1;
        return 0;
    }
    if (bl.n_bands == 1 && bl.total_bytes == 50 && !d_order && bl.bits[0] == 3 && bl.size[0] == 128 &&
        bl.byte_off[0] == 0)
        return 1;
    return -1;
}

}  // namespace

// cuTensorMapEncodeTiled through the runtime's driver entry point (no
// libcuda link); null if the driver does not provide it.
PFN_cuTensorMapEncodeTiled_v12000 lane_encode_fn()
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

// Map of [n_tokens][nh][128] elements: box = 128 bytes of one row x 1 head
// x 32 tokens, 128-byte swizzle.
bool lane_map(CUtensorMap *m, const void *in, int dtype, int n_tokens, int nh)
{
    auto fn = lane_encode_fn();
    if (!fn) return false;
    const int es = dtype == SP_DTYPE_F32 ? 4 : 2;
    const CUtensorMapDataType dt = dtype == SP_DTYPE_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == SP_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                         : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const cuuint64_t dims[3] = {(cuuint64_t)kLN, (cuuint64_t)nh, (cuuint64_t)n_tokens};
    const cuuint64_t strides[2] = {(cuuint64_t)kLN * es, (cuuint64_t)kLN * es * nh};
    const cuuint32_t box[3] = {(cuuint32_t)(128 / es), 1, 32};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, dt, 3, const_cast<void *>(in), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Lane-per-vector encode of the K and/or V half of n_tokens tokens
// ([n_tokens][nh][128] inputs; a null input skips its half).  Returns 1 and
// sets *rc when it takes the call: both present halves must have the ship
// layouts at head_dim 128 (K with the standard squarefree-first order) and
// 16-byte aligned inputs.  Otherwise 0 (nothing launched).
int sp_encode_lane_kv(const void *d_k, const void *d_v, int dtype, int n_tokens, int nh, int start_pos,
                      uint8_t *k_base, long long k_slot0, long long k_slot_stride, const SpBandLayout &kbl,
                      const int *d_order, bool std_order,
                      uint8_t *v_base, long long v_slot0, long long v_slot_stride, const SpBandLayout &vbl,
                      unsigned int *d_status, cudaStream_t s, int *rc)
{
    if (n_tokens <= 0 || nh <= 0 || (!d_k && !d_v)) return 0;
    if (getenv("SHANNON_PRIME_ENCODE_LANEGROUP")) return 0;
    if (d_k && (lane_half_of(kbl, d_order, std_order) != 0 || ((uintptr_t)d_k & 15))) return 0;
    if (d_v && (lane_half_of(vbl, nullptr, false) != 1 || ((uintptr_t)d_v & 15))) return 0;
    if (dtype != SP_DTYPE_F32 && dtype != SP_DTYPE_F16 && dtype != SP_DTYPE_BF16) return 0;
    if (2LL * nh * ((n_tokens + 31) / 32) > 0x7fffffffLL) return 0;
    LaneArgs a;
    a.half[0] = LaneHalf{d_k, k_base, k_slot0, k_slot_stride};
    a.half[1] = LaneHalf{d_v, v_base, v_slot0, v_slot_stride};
    a.first = d_k ? 0 : 1;
    a.n_halves = (d_k && d_v) ? 2 : 1;
    a.n_tokens = n_tokens; a.nh = nh; a.start_pos = start_pos;
    a.nb = nh * ((n_tokens + 31) / 32);
    a.inv_sqrt_n = sp_inv_sqrt_n(kLN);
    a.status = d_status;
    LaneMaps maps;
    memset(&maps, 0, sizeof(maps));
    if ((d_k && !lane_map(&maps.m[0], d_k, dtype, n_tokens, nh)) ||
        (d_v && !lane_map(&maps.m[1], d_v, dtype, n_tokens, nh)))
        return 0;
    switch (dtype) {
    case SP_DTYPE_F32:  *rc = launch_lane<float>(a, maps, s); break;
    case SP_DTYPE_F16:  *rc = launch_lane<__half>(a, maps, s); break;
    default:            *rc = launch_lane<__nv_bfloat16>(a, maps, s); break;
    }
    return 1;
}

// One half through the lane encoder (the sp_launch_encode hook).
int sp_encode_lane_try(const void *d_in, int dtype, int n_tokens, int nh, uint8_t *d_out_base,
                       long long slot0, long long slot_stride, int start_pos, bool std_order,
                       const int *d_order, bool do_wht, const SpBandLayout &bl, unsigned int *d_status,
                       cudaStream_t s, int *rc)
{
    if (!do_wht) return 0;
    const int hx = lane_half_of(bl, d_order, std_order);
    if (hx < 0) return 0;
    if (hx == 0)
        return sp_encode_lane_kv(d_in, nullptr, dtype, n_tokens, nh, start_pos, d_out_base, slot0, slot_stride, bl,
                                 d_order, std_order, nullptr, 0, 0, bl, d_status, s, rc);
    return sp_encode_lane_kv(nullptr, d_in, dtype, n_tokens, nh, start_pos, nullptr, 0, 0, bl, nullptr, false,
                             d_out_base, slot0, slot_stride, bl, d_status, s, rc);
}

// ------------------------------------------------ fused decompress-KQ op --
// GPU counterpart of the reference's CPU ggml op llama_sp_kq_compute
// (src/engine/llama_sp_fused_kq.cpp:82-165): for one head's packed rows
// (k_packed_buf_per_head, total_bytes_per_pos, is_v of its userdata) and
// n_head_q query rows, dst[qh][kv] = dot(decompress(row kv), q[qh]) in fp32.
// The dot is taken in the coefficient domain (q' = perm(H q) / sqrt(n), the
// transform being orthonormal and symmetric), so no row is reconstructed.
// One thread owns one position: its row is staged through shared memory with
// coalesced loads, its 128 coefficients are dequantised into registers with
// the compile-time layout, and the transformed queries are read from shared
// memory as broadcast 16-byte loads (4 heads per load).
namespace {

constexpr int kKqThreads = 128;       // positions per CTA
constexpr int kKqMaxHeads = 64;

// blockIdx.y selects the slot: packed, q and dst advance by their slot
// strides (bytes), so one launch serves every (layer, KV head) of a call.
template <bool KS>
__global__ void __launch_bounds__(kKqThreads)
k_kq_scores_lane(const uint8_t *packed, int n_kv, const void *q, int q_f16, long long q_stride, int n_head_q,
                 float *dst, long long dst_stride, float inv_sqrt_n, long long packed_slot, long long q_slot,
                 long long dst_slot)
{
    packed += (long long)blockIdx.y * packed_slot;
    q = reinterpret_cast<const uint8_t *>(q) + (long long)blockIdx.y * q_slot;
    dst = reinterpret_cast<float *>(reinterpret_cast<char *>(dst) + (long long)blockIdx.y * dst_slot);
    using L = LaneLayout<KS>;
    constexpr int TB = L::TB, TH = TB / 2;     // row bytes, halfwords
    constexpr LaneOrder ord = lane_order();
    __shared__ __align__(16) float qs[kLN][kKqMaxHeads];   // q'[coefficient][head]
    __shared__ uint16_t rows[kKqThreads * TH];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nq4 = (n_head_q + 3) & ~3;

    // ---- q' = perm(H q) / sqrt(n), one warp per head ----
    for (int g = warp; g < nq4; g += kKqThreads / 32) {
        float x[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int i = lane * 4 + e;
            float v = 0.0f;
            if (g < n_head_q) {
                const uint8_t *qr = reinterpret_cast<const uint8_t *>(q) + g * q_stride;
                v = q_f16 ? __half2float(reinterpret_cast<const __half *>(qr)[i])
                          : reinterpret_cast<const float *>(qr)[i];
            }
            x[e] = v;
        }
        sp_warp_wht<4>(x, lane);
        __shared__ float tmp[kKqThreads / 32][kLN];
#pragma unroll
        for (int e = 0; e < 4; e++) tmp[warp][lane * 4 + e] = x[e] * inv_sqrt_n;
        __syncwarp();
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int j = lane * 4 + e;
            qs[j][g] = tmp[warp][KS ? ord.v[j] : j];
        }
        __syncwarp();
    }
    // ---- this CTA's rows, coalesced, into shared memory ----
    const long long kv0 = (long long)blockIdx.x * kKqThreads;
    const int n_here = (int)min((long long)kKqThreads, n_kv - kv0);
    const uint16_t *src = reinterpret_cast<const uint16_t *>(packed + kv0 * TB);
    for (int i = tid; i < n_here * TH; i += kKqThreads) rows[i] = src[i];
    __syncthreads();
    if (tid >= n_here) return;

    // ---- dequantise the thread's row (stored order) ----
    const uint16_t *r16 = rows + tid * TH;
    auto bits_at = [&](int p, int nb) -> uint32_t {          // nb <= 16 bits at bit p of the row
        const int h = p >> 4, sh = p & 15;
        uint32_t w = r16[h];
        if (sh + nb > 16) w |= (uint32_t)r16[h + 1] << 16;
        return (w >> sh) & ((1u << nb) - 1u);
    };
    float c[kLN];
#pragma unroll
    for (int b = 0; b < L::NB; b++) {
        const int bits = L::bits(b), mv = (1 << (bits - 1)) - 1;
        const int sbit = 8 * L::byte_off(b);
        float scale = __half2float(__ushort_as_half((unsigned short)bits_at(sbit, 16)));
        if (!isfinite(scale)) scale = 0.0f;
#pragma unroll
        for (int k = 0; k < L::SIZE; k++)
            c[b * L::SIZE + k] = (float)((int)bits_at(sbit + 16 + k * bits, bits) - mv) * scale;
    }
    // ---- dots, 4 heads per pass ----
    float *out = dst + (kv0 + tid);
    for (int g0 = 0; g0 < n_head_q; g0 += 4) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int j = 0; j < kLN; j++) {
            const float4 w = *reinterpret_cast<const float4 *>(&qs[j][g0]);
            acc[0] = fmaf(c[j], w.x, acc[0]);
            acc[1] = fmaf(c[j], w.y, acc[1]);
            acc[2] = fmaf(c[j], w.z, acc[2]);
            acc[3] = fmaf(c[j], w.w, acc[3]);
        }
#pragma unroll
        for (int e = 0; e < 4; e++)
            if (g0 + e < n_head_q)
                *reinterpret_cast<float *>(reinterpret_cast<char *>(out) + (long long)(g0 + e) * dst_stride) = acc[e];
    }
}

}  // namespace

// tcgen05 form for K rows (sp_attn_tc.cu): 1 and *rc set if it took the call.
int sp_kq_scores_tc_try(const uint8_t *packed, long long packed_slot, int n_slots, int n_kv, const void *q,
                        int q_f16, long long q_stride, long long q_slot, int n_head_q, float *dst,
                        long long dst_stride, long long dst_slot, float inv_sqrt_n, cudaStream_t s, int *rc);

extern "C" int sp_cuda_kq_scores_strided(const void *d_packed, long long packed_slot_stride, int n_slots,
                                         int total_bytes_per_pos, int is_v, int head_dim, int n_kv, const void *d_q,
                                         int q_dtype, long long q_row_stride, long long q_slot_stride, int n_head_q,
                                         float *d_dst, long long dst_row_stride, long long dst_slot_stride,
                                         void *stream)
{
    sp_clear_error();
    if (n_kv < 0 || n_head_q < 1 || n_slots < 0 || !d_packed || !d_q || !d_dst)
        return sp_set_error(SP_ERR_ARG, "kq_scores: bad arguments");
    if (n_kv == 0 || n_slots == 0) return SP_OK;
    if (n_slots > 65535) return sp_set_error(SP_ERR_ARG, "kq_scores: at most 65535 slots per call");
    if (head_dim != kLN || n_head_q > kKqMaxHeads ||
        total_bytes_per_pos != (is_v ? LaneLayout<false>::TB : LaneLayout<true>::TB))
        return sp_set_error(SP_ERR_UNSUPPORTED,
                            "kq_scores: head_dim 128 ship rows (K 76 B, V 50 B), at most %d query rows",
                            kKqMaxHeads);
    if (q_dtype != SP_DTYPE_F32 && q_dtype != SP_DTYPE_F16)
        return sp_set_error(SP_ERR_ARG, "kq_scores: q must be f32 or f16");
    const int es = q_dtype == SP_DTYPE_F32 ? 4 : 2;
    if (((uintptr_t)d_packed & 1) || ((uintptr_t)d_q % es) || (q_row_stride % es) || ((uintptr_t)d_dst & 3) ||
        (dst_row_stride & 3) || q_row_stride < (long long)es * head_dim || dst_row_stride < 4LL * n_kv ||
        (packed_slot_stride & 1) || (q_slot_stride % es) || (dst_slot_stride & 3))
        return sp_set_error(SP_ERR_ARG, "kq_scores: misaligned pointer or stride");
    cudaStream_t s = (cudaStream_t)stream;
    const float isn = sp_inv_sqrt_n(kLN);
    int rc = SP_OK;
    if (!is_v && sp_kq_scores_tc_try((const uint8_t *)d_packed, packed_slot_stride, n_slots, n_kv, d_q,
                                     q_dtype == SP_DTYPE_F16, q_row_stride, q_slot_stride, n_head_q, d_dst,
                                     dst_row_stride, dst_slot_stride, isn, s, &rc))
        return rc;
    const dim3 grid((unsigned)((n_kv + kKqThreads - 1) / kKqThreads), (unsigned)n_slots);
    if (is_v)
        k_kq_scores_lane<false><<<grid, kKqThreads, 0, s>>>((const uint8_t *)d_packed, n_kv, d_q,
                                                            q_dtype == SP_DTYPE_F16, q_row_stride, n_head_q, d_dst,
                                                            dst_row_stride, isn, packed_slot_stride, q_slot_stride,
                                                            dst_slot_stride);
    else
        k_kq_scores_lane<true><<<grid, kKqThreads, 0, s>>>((const uint8_t *)d_packed, n_kv, d_q,
                                                           q_dtype == SP_DTYPE_F16, q_row_stride, n_head_q, d_dst,
                                                           dst_row_stride, isn, packed_slot_stride, q_slot_stride,
                                                           dst_slot_stride);
    return sp_check_cuda(cudaGetLastError(), "kq_scores launch");
}

extern "C" int sp_cuda_kq_scores(const void *d_packed, int total_bytes_per_pos, int is_v, int head_dim, int n_kv,
                                 const void *d_q, int q_dtype, long long q_row_stride, int n_head_q,
                                 float *d_dst, long long dst_row_stride, void *stream)
{
    return sp_cuda_kq_scores_strided(d_packed, 0, 1, total_bytes_per_pos, is_v, head_dim, n_kv, d_q, q_dtype,
                                     q_row_stride, 0, n_head_q, d_dst, dst_row_stride, 0, stream);
}

// ------------------------------------------------- lane-per-vector read --
// The ship read (reference sp_cuda_read_k/_v[_batch], shannon_prime_cuda.cu:
// 524-559, 622-657: dequantise -> Möbius unreorder -> VHT2 -> fp32 rows) for
// the head_dim-128 ship layouts, one thread per position: the warp's 32
// packed rows are loaded coalesced into shared memory, each thread
// dequantises its row with the compile-time layout (bands at or beyond
// max_bands read as zero), unreorders by register renaming, runs the
// butterfly in registers, and writes its fp32 row into a 128-byte-swizzled
// shared-memory tile that one elected lane stores with tiled TMA copies.
// Same IEEE operations in the same order as k_decode, so rows are
// bit-identical.
namespace {

struct alignas(64) ReadMap { CUtensorMap m; };

template <bool KS>
struct ReadSmem {
    alignas(1024) unsigned char out[kLaneWarps][4][4096];      // 4 column slices x 32 rows x 128 B
    alignas(16) uint16_t rows[kLaneWarps][32 * LaneLayout<KS>::TB / 2];
    unsigned long long bar[kLaneWarps];
};

// Slots a read covers: n_layers x n_heads slots, slot (l, h) at
// packed + (slot0 + l * n_heads + h) * slot_stride + pos0 * row bytes; its
// rows go to the output tensor at coordinates (h * 128, t, l).
struct ReadGrid {
    long long slot_stride;
    long long slot0;
    int n_heads, n_layers, pos0;
};

template <bool KS>
__global__ void __launch_bounds__(kLaneWarps * 32, kLaneMinBlocks)
k_decode_lane(const uint8_t *packed, ReadGrid rg, int n_pos, int nb_use, float inv_sqrt_n, unsigned int *status,
              const __grid_constant__ ReadMap map)
{
    using L = LaneLayout<KS>;
    constexpr int TB = L::TB, TH = TB / 2;
    constexpr LaneOrder ord = lane_order();
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    ReadSmem<KS> &sm = *reinterpret_cast<ReadSmem<KS> *>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t out0 = spb::smem_u32(&sm.out[warp][0][0]);
    if (out0 & 1023) {
        if (threadIdx.x == 0 && status) atomicOr(status, 4u);
        return;
    }
    const int n_bs = (n_pos + 31) >> 5;                 // batches per slot
    const long long n_b = (long long)n_bs * rg.n_heads * rg.n_layers;
    const long long b_step = (long long)gridDim.x * kLaneWarps;
    // The 32 packed rows of a full batch are contiguous (32 x TB bytes, a
    // multiple of 16): when their start is 16-byte aligned one bulk copy
    // fetches them into the warp's row buffer, issued as soon as the
    // previous batch's rows are in registers, so the load streams under that
    // batch's butterfly and stores.  Ragged or unaligned batches are loaded
    // by the lanes.
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
        return packed + (rg.slot0 + sl) * rg.slot_stride + (long long)(rg.pos0 + t0) * TB;
    };
    auto bulkable = [&](const uint8_t *src, int live) { return live == 32 && ((uintptr_t)src & 15) == 0; };
    uint32_t par = 0u;                                  // parity of the next wait
    bool pending = false;                               // a copy was issued into the buffer
    // Next batch's source, or null when the lanes load it.
    auto next_src = [&](long long bt) -> const uint8_t * {
        if (bt >= n_b) return nullptr;
        int sl, t0, live;
        const uint8_t *src = batch_src(bt, sl, t0, live);
        return bulkable(src, live) ? src : nullptr;
    };
    auto issue = [&](const uint8_t *src) {
        if (!src) return;
        pending = true;                                 // warp-uniform bookkeeping
        if (lane == 0) {
            spb::fence_proxy_async();
            spb::mbar_expect_tx(bar0, 32 * TB);
            spb::bulk_g2s(rows0, src, 32 * TB, bar0, policy);
        }
    };
    long long bt = (long long)blockIdx.x * kLaneWarps + warp;
    issue(next_src(bt));
    bool failed = false;
    for (; bt < n_b; bt += b_step) {
        const uint8_t *nsrc = next_src(bt + b_step);
        int sl, t0, live;
        const uint8_t *srcb = batch_src(bt, sl, t0, live);
        const int l = sl / rg.n_heads, hh = sl - l * rg.n_heads;
        uint16_t *rows = sm.rows[warp];
        if (pending) {
            if (!spb::wait_stage(bar0, par, status)) {
                failed = true;                  // the copy may still land: waited for below
                break;
            }
            pending = false;
            par ^= 1u;
        } else {
            const uint16_t *src = reinterpret_cast<const uint16_t *>(srcb);
            for (int i = lane; i < live * TH; i += 32) rows[i] = src[i];
            __syncwarp();
        }
        const uint16_t *r16 = rows + lane * TH;
        auto bits_at = [&](int p, int nb) -> uint32_t {
            const int h = p >> 4, sh = p & 15;
            uint32_t w = r16[h];
            if (sh + nb > 16) w |= (uint32_t)r16[h + 1] << 16;
            return (w >> sh) & ((1u << nb) - 1u);
        };
        float x[kLN];
#pragma unroll
        for (int b = 0; b < L::NB; b++) {
            const int bits = L::bits(b), mv = (1 << (bits - 1)) - 1;
            const int sbit = 8 * L::byte_off(b);
            float scale = __half2float(__ushort_as_half((unsigned short)bits_at(sbit, 16)));
            if (!isfinite(scale)) scale = 0.0f;
            const bool on = b < nb_use;
#pragma unroll
            for (int k = 0; k < L::SIZE; k++) {
                const int j = b * L::SIZE + k;                 // stored index
                const float v = on ? __fmul_rn((float)((int)bits_at(sbit + 16 + k * bits, bits) - mv), scale)
                                   : 0.0f;
                x[KS ? ord.v[j] : j] = v;                      // unreorder
            }
        }
        __syncwarp();                           // every lane's row is in registers
        issue(nsrc);
#pragma unroll
        for (int len = 1; len < kLN; len <<= 1) {
#pragma unroll
            for (int i = 0; i < kLN; i += len << 1) {
#pragma unroll
                for (int j = 0; j < len; j++) {
                    const float u = x[i + j], v = x[i + j + len];
                    x[i + j] = __fadd_rn(u, v);
                    x[i + j + len] = __fsub_rn(u, v);
                }
            }
        }
        if (lane == 0) bulk_wait_read();        // the previous batch's stores have read the tile
        __syncwarp();
#pragma unroll
        for (int c = 0; c < kLN / 4; c++) {
            const int off = (c >> 3) * 4096 + lane * 128 + (((c & 7) ^ (lane & 7)) << 4);
            *reinterpret_cast<float4 *>(&sm.out[warp][0][0] + off) =
                make_float4(__fmul_rn(x[4 * c], inv_sqrt_n), __fmul_rn(x[4 * c + 1], inv_sqrt_n),
                            __fmul_rn(x[4 * c + 2], inv_sqrt_n), __fmul_rn(x[4 * c + 3], inv_sqrt_n));
        }
        spb::fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
#pragma unroll
            for (int q = 0; q < 4; q++)
                asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
                                 &map.m),
                             "r"(hh * kLN + q * 32), "r"(t0), "r"(l), "r"(out0 + q * 4096)
                             : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
        (void)live;
    }
    // After a timed-out wait: bounded waits for the copies still in flight
    // before the CTA's shared memory is released.
    if (failed && pending) spb::wait_stage(bar0, par, nullptr);
    if (lane == 0) bulk_wait_all();
}

// Output d_out: [n_layers][n_pos][n_heads][128] fp32 (one slot: [n_pos][128]).
template <bool KS>
int launch_read_lane(const uint8_t *packed, const ReadGrid &rg, int n_pos, int nb_use, float *d_out,
                     unsigned int *status, cudaStream_t s)
{
    auto fn = lane_encode_fn();
    if (!fn) return 1;
    ReadMap map;
    memset(&map, 0, sizeof(map));
    const cuuint64_t row = (cuuint64_t)kLN * rg.n_heads;
    const cuuint64_t dims[3] = {row, (cuuint64_t)n_pos, (cuuint64_t)rg.n_layers};
    const cuuint64_t strides[2] = {row * 4, row * 4 * (cuuint64_t)n_pos};
    const cuuint32_t box[3] = {32, 32, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (fn(&map.m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, d_out, dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return 1;
    auto k = k_decode_lane<KS>;
    const size_t smem = sizeof(ReadSmem<KS>);
    // Per device: attribute set and occupancy looked up once (atomics, so
    // host threads driving any devices race harmlessly).
    constexpr int kMaxDev = 64;
    static std::atomic<int> occ_tab[kMaxDev], sms_tab[kMaxDev];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDev) return -1;
    int occ = occ_tab[dev].load(std::memory_order_acquire);
    if (occ == 0) {
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
            sp_check_cuda(cudaGetLastError(), "lane read smem attribute");
            return -1;
        }
        int o = 0, sms = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, k, kLaneWarps * 32, smem);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        sms_tab[dev].store(sms > 0 ? sms : 148, std::memory_order_relaxed);
        occ = o > 0 ? o : 1;
        occ_tab[dev].store(occ, std::memory_order_release);
    }
    const int sms = sms_tab[dev].load(std::memory_order_relaxed);
    const long long n_b = (long long)((n_pos + 31) / 32) * rg.n_heads * rg.n_layers;
    long long blocks = (n_b + kLaneWarps - 1) / kLaneWarps;
    if (blocks > (long long)sms * occ) blocks = (long long)sms * occ;
    k<<<(unsigned)blocks, kLaneWarps * 32, smem, s>>>(packed, rg, n_pos, nb_use, sp_inv_sqrt_n(kLN), status, map);
    return sp_check_cuda(cudaGetLastError(), "lane read launch") ? -1 : 0;
}

}  // namespace

// The lane-per-vector read for the head_dim-128 ship layouts (K with the
// standard order): 1 and *rc set if it took the call.
int sp_decode_lane_try(const uint8_t *d_rows, int n_pos, float *d_out, const int *d_order, bool std_order,
                       bool do_wht, int max_bands, const SpBandLayout &bl, unsigned int *d_status, cudaStream_t s,
                       int *rc)
{
    if (!do_wht || n_pos <= 0 || getenv("SHANNON_PRIME_DECODE_WARP")) return 0;
    const int hx = lane_half_of(bl, d_order, std_order);
    if (hx < 0 || ((uintptr_t)d_rows & 1) || ((uintptr_t)d_out & 15)) return 0;
    const int nb_use = (max_bands < 0 || max_bands >= bl.n_bands) ? bl.n_bands : max_bands;
    const ReadGrid rg{0, 0, 1, 1, 0};
    const int r = hx == 0 ? launch_read_lane<true>(d_rows, rg, n_pos, nb_use, d_out, d_status, s)
                          : launch_read_lane<false>(d_rows, rg, n_pos, nb_use, d_out, d_status, s);
    if (r > 0) return 0;                        // no tensor-map encoder: the warp kernel reads
    *rc = r ? sp_set_error(SP_ERR_CUDA, "lane read failed") : SP_OK;
    return 1;
}

// Token-major read of every head of a layer range in one launch (the B200
// form of the reference's KvCache::read_gpu, kv_cache.cpp:1100-1228, which
// decompresses head by head into [kv_len][H][hd]): which 0 = K, 1 = V.
extern "C" int sp_cuda_read_kv_tokens(const sp_cuda_cache_t *cc, int which, int layer0, int n_layers,
                                      int start_pos, int n_tok, float *d_out, int max_bands)
{
    sp_clear_error();
    if (!cc || !d_out || (which != 0 && which != 1)) return sp_set_error(SP_ERR_ARG, "read_kv_tokens: bad arguments");
    const int H = cc->config.n_heads_kv;
    if (layer0 < 0 || n_layers < 0 || layer0 + n_layers > cc->config.n_layers || start_pos < 0 || n_tok < 0 ||
        (long long)start_pos + n_tok > cc->max_seq_len)
        return sp_set_error(SP_ERR_ARG, "read_kv_tokens: range out of bounds");
    if (n_layers == 0 || n_tok == 0) return SP_OK;
    if (cudaSetDevice(cc->device) != cudaSuccess) return sp_set_error(SP_ERR_CUDA, "read_kv_tokens: cudaSetDevice");
    const sp_band_config_t &bc = which ? cc->v_bands : cc->k_bands;
    const SpBandLayout bl = sp_layout_from(bc);
    const int *order = which ? nullptr : (cc->config.use_mobius_mask ? cc->d_mobius_order : nullptr);
    const int hx = lane_half_of(bl, order, true);
    const uint8_t *base = (const uint8_t *)(which ? cc->d_v_cache : cc->d_k_cache);
    if (hx < 0 || hx != which || ((uintptr_t)base & 1) || ((uintptr_t)d_out & 15))
        return sp_set_error(SP_ERR_UNSUPPORTED,
                            "read_kv_tokens: head_dim 128 ship layouts (K 5/5/4/3 with the standard order, V 3-bit), "
                            "16-byte aligned output");
    const int nb_use = (max_bands < 0 || max_bands >= bl.n_bands) ? bl.n_bands : max_bands;
    const ReadGrid rg{(long long)cc->max_seq_len * bc.total_bytes, (long long)layer0 * H, H, n_layers, start_pos};
    cudaStream_t s = (cudaStream_t)cc->stream;
    const int r = hx == 0 ? launch_read_lane<true>(base, rg, n_tok, nb_use, d_out, cc->d_status, s)
                          : launch_read_lane<false>(base, rg, n_tok, nb_use, d_out, cc->d_status, s);
    if (r > 0) return sp_set_error(SP_ERR_UNSUPPORTED, "read_kv_tokens: no tensor-map encoder in this driver");
    return r ? sp_set_error(SP_ERR_CUDA, "read_kv_tokens: launch failed") : SP_OK;
}
