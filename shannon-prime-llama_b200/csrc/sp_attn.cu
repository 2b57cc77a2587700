// sp_attn.cu — fused decompress-KQ / decompress-V decode attention.
//
// Math (no K or V row is ever reconstructed):
//   K_hat_t = H * unreorder(c_t)          (H = orthonormal, symmetric VHT2)
//   q . K_hat_t = (H q) . unreorder(c_t) = sum_i q'[i] c_t[i],
//                 q'[i] = (H q)[order[i]]
//   sum_t p_t V_hat_t = H (sum_t p_t cv_t)
// so scores are dot products of the transformed query with the dequantised
// codes, V is accumulated in the coefficient domain, and one VHT2 per
// (layer, query head) finishes the output.
//
// Work split: flash-decoding.  A CTA owns one (layer, KV head, token chunk)
// and all query heads of that KV head's GQA group; it writes an unnormalised
// partial (running max m, denominator l, coefficient accumulator) to the
// cache's workspace, and a combine kernel merges the chunks with
// log-sum-exp weights, applies the VHT2 and writes fp16.
//
// This file holds the generic SIMT kernel (any power-of-two head_dim, any
// band layout, 1..8 queries per KV head), the combine kernel and the
// dispatcher.  sp_attn_mma.cu holds the tensor-core kernel for the ship
// layout (head_dim 128, K bands 5/5/4/3, V 3-bit).
#include "sp_internal.cuh"
#include "sp_attn.cuh"

#include <math.h>
#include <string.h>

#include <atomic>

namespace {

constexpr int kAttnWarps = 4;

__device__ __forceinline__ int band_of_i(const SpBandLayout &bl, int i)
{
    int b = 0;
#pragma unroll 1
    for (int k = 1; k < bl.n_bands; k++)
        if (i >= bl.off[k]) b = k;
    return b;
}

// Dequantised coefficient i of a packed row (partial-band rule applied).
__device__ __forceinline__ float coeff_at(const SpBandLayout &bl, const uint8_t *row, int i,
                                          int nb_use)
{
    const int b = band_of_i(bl, i);
    if (b >= nb_use) return 0.0f;
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
    return (float)(u - max_val) * scale;
}

}  // namespace

// Transformed, permuted, scaled query of one (layer, q head) into s_out[n]
// (one warp).  s_tmp is n floats of warp-private shared memory.
template <int E>
__device__ void sp_attn_prepare_query(const __half *q, const int *order, float scale_all,
                                      float *s_tmp, float *s_out, int lane)
{
    constexpr int n = 32 * E;
    float x[E];
#pragma unroll
    for (int e = 0; e < E; e++) x[e] = __half2float(q[lane * E + e]);
    sp_warp_wht<E>(x, lane);
#pragma unroll
    for (int e = 0; e < E; e++) s_tmp[lane * E + e] = x[e] * scale_all;
    __syncwarp();
#pragma unroll
    for (int e = 0; e < E; e++) {
        const int i = lane * E + e;
        s_out[i] = order ? s_tmp[order[i]] : s_tmp[i];
    }
    __syncwarp();
    (void)n;
}

namespace {

template <int E>
__global__ void __launch_bounds__(kAttnWarps * 32)
k_attn_generic(SpAttnArgs a)
{
    constexpr int n = 32 * E;
    extern __shared__ __align__(16) float sm[];
    const int G = a.group;
    float *s_q = sm;                                   // [G][n]
    float *s_tmp = s_q + G * n;                        // [warps][n]
    float *s_acc = s_tmp + kAttnWarps * n;             // [warps][G][n]
    float *s_ml = s_acc + kAttnWarps * G * n;          // [warps][G][2]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x;
    const int h = blockIdx.y;
    const int li = blockIdx.z;                  // layer index within the call
    const int layer = a.layer0 + li;
    const int t_begin = split * a.chunk;
    const int t_end = min(a.kv_len, t_begin + a.chunk);
    const long long slot = (long long)layer * a.n_kv_heads + h;
    const float kLog2e = 1.4426950408889634f;

    for (int g = warp; g < G; g += kAttnWarps) {
        const __half *qg = a.q + ((long long)li * a.n_q_heads + h * G + g) * n;
        sp_attn_prepare_query<E>(qg, a.order, a.logit_scale * kLog2e * a.inv_sqrt_n, s_tmp + warp * n,
                                 s_q + g * n, lane);
    }
    float *acc = s_acc + warp * G * n;
    for (int j = lane; j < G * n; j += 32) acc[j] = 0.0f;
    __syncthreads();

    float m[8], l[8];
#pragma unroll
    for (int g = 0; g < 8; g++) { m[g] = -INFINITY; l[g] = 0.0f; }

    const uint8_t *kbase = a.k_cache + slot * a.k_slot_stride;
    const uint8_t *vbase = a.v_cache + slot * a.v_slot_stride;
    for (int t = t_begin + warp; t < t_end; t += kAttnWarps) {
        const uint8_t *krow = kbase + (long long)t * a.kl.total_bytes;
        const uint8_t *vrow = vbase + (long long)t * a.vl.total_bytes;
        float ck[E], cv[E];
#pragma unroll
        for (int e = 0; e < E; e++) {
            ck[e] = coeff_at(a.kl, krow, lane * E + e, a.nb_k);
            cv[e] = coeff_at(a.vl, vrow, lane * E + e, a.nb_v);
        }
#pragma unroll 1
        for (int g = 0; g < G; g++) {
            float s = 0.0f;
#pragma unroll
            for (int e = 0; e < E; e++) s += ck[e] * s_q[g * n + lane * E + e];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            // s is the base-2 logit (log2e folded into the query).
            float mg = m[0], lg = l[0];
#pragma unroll
            for (int k = 1; k < 8; k++) if (k == g) { mg = m[k]; lg = l[k]; }
            const float mn = fmaxf(mg, s);
            const float alpha = exp2f(mg - mn);
            const float p = exp2f(s - mn);
            lg = lg * alpha + p;
#pragma unroll
            for (int k = 0; k < 8; k++) if (k == g) { m[k] = mn; l[k] = lg; }
            float *ag = acc + g * n;
#pragma unroll
            for (int e = 0; e < E; e++) {
                const int i = lane * E + e;
                ag[i] = ag[i] * alpha + p * cv[e];
            }
        }
    }
    if (lane == 0) {
        for (int g = 0; g < G; g++) {
            float mg = m[0], lg = l[0];
            for (int k = 1; k < 8; k++) if (k == g) { mg = m[k]; lg = l[k]; }
            s_ml[(warp * G + g) * 2] = mg;
            s_ml[(warp * G + g) * 2 + 1] = lg;
        }
    }
    __syncthreads();
    // Merge the warps and write the CTA's partial.
    for (int g = 0; g < G; g++) {
        float M = -INFINITY;
        for (int w = 0; w < kAttnWarps; w++) M = fmaxf(M, s_ml[(w * G + g) * 2]);
        float wsc[kAttnWarps], L = 0.0f;
        for (int w = 0; w < kAttnWarps; w++) {
            const float mw = s_ml[(w * G + g) * 2];
            wsc[w] = (mw == -INFINITY) ? 0.0f : exp2f(mw - M);
            L += wsc[w] * s_ml[(w * G + g) * 2 + 1];
        }
        float *part = sp_attn_partial(a, li, h * G + g, split);
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            float v = 0.0f;
            for (int w = 0; w < kAttnWarps; w++) v += wsc[w] * s_acc[(w * G + g) * n + i];
            part[4 + i] = v;
        }
        if (threadIdx.x == 0) { part[0] = M; part[1] = L; }
    }
}

// Merge the split partials of one (layer, q head), transform, write fp16.
template <int E>
__global__ void k_attn_combine(SpAttnArgs a)
{
    constexpr int n = 32 * E;
    const int lane = threadIdx.x & 31;
    const int qh = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int li = blockIdx.y;
    if (qh < a.n_q_heads) {
        float M = -INFINITY;
        for (int s = 0; s < a.n_splits; s++) M = fmaxf(M, sp_attn_partial(a, li, qh, s)[0]);
        float x[E];
#pragma unroll
        for (int e = 0; e < E; e++) x[e] = 0.0f;
        float L = 0.0f;
        for (int s = 0; s < a.n_splits; s++) {
            const float *p = sp_attn_partial(a, li, qh, s);
            if (p[0] == -INFINITY) continue;
            const float w = exp2f(p[0] - M);
            L += w * p[1];
#pragma unroll
            for (int e = 0; e < E; e++) x[e] += w * p[4 + lane * E + e];
        }
        const float inv = L > 0.0f ? 1.0f / L : 0.0f;
        sp_warp_wht<E>(x, lane);
        __half h[E];
#pragma unroll
        for (int e = 0; e < E; e++) h[e] = __float2half_rn(x[e] * a.inv_sqrt_n * inv);
        sp_attn_store_row<E>(a, li, qh, lane, h);
    }
    sp_attn_gather_signal(a);
}

template <int E>
int launch_generic(const SpAttnArgs &a, cudaStream_t s)
{
    constexpr int n = 32 * E;
    const size_t sm = sizeof(float) * ((size_t)a.group * n + kAttnWarps * n +
                                       (size_t)kAttnWarps * a.group * n + kAttnWarps * a.group * 2);
    auto k = k_attn_generic<E>;
    if (sm > 48 * 1024)
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    dim3 grid(a.n_splits, a.n_kv_heads, a.n_layers);
    k<<<grid, kAttnWarps * 32, sm, s>>>(a);
    return sp_check_cuda(cudaGetLastError(), "attention launch");
}

template <int E>
int launch_combine(const SpAttnArgs &a, cudaStream_t s)
{
    const int per_block = 4;
    dim3 grid((a.n_q_heads + per_block - 1) / per_block, a.n_layers);
    k_attn_combine<E><<<grid, per_block * 32, 0, s>>>(a);
    return sp_check_cuda(cudaGetLastError(), "attention combine launch");
}

}  // namespace

// ------------------------------------------------------------ dispatch --

size_t sp_attn_workspace_bytes(const sp_cuda_cache_t *cc)
{
    return (size_t)cc->attn_ws_layers * cc->attn_max_q_heads * kAttnMaxSplits *
           sp_attn_partial_stride(cc->config.head_dim) * sizeof(float);
}

// Diagnostic kernel choice, process-wide (tests use it to compare the two
// kernels): 0 auto, 1 generic SIMT, 2 mma.sync tensor-core, 3 tcgen05.  Atomic, so host threads
// may read it while another sets it.
static std::atomic<int> g_force_impl{0};

extern "C" void sp_cuda_attn_force_impl(int impl) { g_force_impl.store(impl, std::memory_order_relaxed); }

// Optional timing of the main (non-combine) kernel with CUDA events recorded
// on the caller's stream, for the benchmark's roofline figure.  Per host
// thread: a thread enables it and reads back its own last call.
static thread_local bool g_prof = false;
static thread_local cudaEvent_t g_ev[2] = {nullptr, nullptr};
static thread_local int g_prof_splits = 0;

extern "C" void sp_cuda_attn_profile(int enable)
{
    g_prof = enable != 0;
    if (g_prof && !g_ev[0]) {
        cudaEventCreate(&g_ev[0]);
        cudaEventCreate(&g_ev[1]);
    }
}

extern "C" float sp_cuda_attn_last_kernel_ms(void)
{
    if (!g_ev[0]) return -1.0f;
    float ms = -1.0f;
    if (cudaEventSynchronize(g_ev[1]) != cudaSuccess) return -1.0f;
    cudaEventElapsedTime(&ms, g_ev[0], g_ev[1]);
    return ms;
}

extern "C" int sp_cuda_attn_last_splits(void) { return g_prof_splits; }

// Kernel choice and split chunking of a filled SpAttnArgs, shared by every
// decode entry point.  `aligned`: the caches and their slot stride allow the
// tensor-core kernel's 16-byte aligned bulk copies of 16-position tiles.
static int attn_plan(SpAttnArgs &a, bool aligned, bool &use_mma)
{
    use_mma = aligned && g_force_impl != 1 && sp_attn_mma_supported(a) == SP_OK;
    if (g_force_impl == 2 && !use_mma)
        return sp_set_error(SP_ERR_UNSUPPORTED, "attn_decode: tensor-core path does not support this layout");
    if (g_force_impl == 3 && !(use_mma && sp_attn_tc_supported(a) == SP_OK))
        return sp_set_error(SP_ERR_UNSUPPORTED, "attn_decode: tcgen05 path does not support this layout");

    // Chunking: enough CTAs to fill the 148 SMs several times over, chunks of
    // at least kAttnMinChunk tokens, at most kAttnMaxSplits chunks.
    const int units = a.n_layers * a.n_kv_heads;
    const int target_ctas = use_mma ? 148 * 4 : 148 * 8;
    int splits = (target_ctas + units - 1) / units;
    const int max_by_len = (a.kv_len + kAttnMinChunk - 1) / kAttnMinChunk;
    if (splits > max_by_len) splits = max_by_len;
    if (splits > kAttnMaxSplits) splits = kAttnMaxSplits;
    if (splits < 1) splits = 1;
    int chunk = (a.kv_len + splits - 1) / splits;
    chunk = (chunk + 15) & ~15;
    if (chunk < 16) chunk = 16;
    a.chunk = chunk;
    a.n_splits = a.kv_len == 0 ? 0 : (a.kv_len + chunk - 1) / chunk;
    if (a.n_splits > kAttnMaxSplits)
        return sp_set_error(SP_ERR_ARG, "attn_decode: too many splits");
    return SP_OK;
}

// Validate a decode call and fill its kernel arguments and split chunking.
static int attn_prepare(const sp_cuda_cache_t *cc, int layer0, int n_layers, const void *d_q, int n_q_heads,
                        int kv_len, float logit_scale, int max_bands, SpAttnArgs &a, bool &use_mma)
{
    if (!cc || !cc->d_k_cache || !d_q)
        return sp_set_error(SP_ERR_ARG, "attn_decode: NULL argument");
    const int H = cc->config.n_heads_kv;
    if (layer0 < 0 || n_layers <= 0 || layer0 + n_layers > cc->config.n_layers)
        return sp_set_error(SP_ERR_ARG, "attn_decode: layers [%d,%d) out of range", layer0, layer0 + n_layers);
    if (n_q_heads <= 0 || n_q_heads % H || n_q_heads / H > 8)
        return sp_set_error(SP_ERR_ARG, "attn_decode: n_q_heads %d must be a multiple of %d with <= 8 per KV head", n_q_heads, H);
    if (n_layers > cc->attn_ws_layers || n_q_heads > cc->attn_max_q_heads)
        return sp_set_error(SP_ERR_ARG, "attn_decode: workspace too small");
    if (kv_len < 0 || kv_len > cc->max_seq_len)
        return sp_set_error(SP_ERR_ARG, "attn_decode: kv_len %d outside [0,%d]", kv_len, cc->max_seq_len);
    if (cudaSetDevice(cc->device) != cudaSuccess)
        return sp_set_error(SP_ERR_CUDA, "attn_decode: cudaSetDevice");

    memset(&a, 0, sizeof(a));
    a.k_cache = (const uint8_t *)cc->d_k_cache;
    a.v_cache = (const uint8_t *)cc->d_v_cache;
    a.k_slot_stride = (long long)cc->max_seq_len * cc->k_bands.total_bytes;
    a.v_slot_stride = (long long)cc->max_seq_len * cc->v_bands.total_bytes;
    a.order = cc->config.use_mobius_mask ? cc->d_mobius_order : nullptr;
    a.q = (const __half *)d_q;
    a.ws = (float *)cc->d_attn_ws;
    a.layer0 = layer0; a.n_layers = n_layers; a.n_kv_heads = H;
    a.n_q_heads = n_q_heads; a.group = n_q_heads / H;
    a.kv_len = kv_len;
    a.kl = sp_layout_from(cc->k_bands);
    a.vl = sp_layout_from(cc->v_bands);
    a.nb_k = (max_bands < 0 || max_bands >= a.kl.n_bands) ? a.kl.n_bands : max_bands;
    a.nb_v = (max_bands < 0 || max_bands >= a.vl.n_bands) ? a.vl.n_bands : max_bands;
    a.logit_scale = logit_scale;
    a.inv_sqrt_n = sp_inv_sqrt_n(cc->config.head_dim);
    a.status = cc->d_status;

    return attn_plan(a, true, use_mma);
}

// Main kernel(s) and the combine of a prepared call.
static int attn_launch(const SpAttnArgs &a, bool use_mma, cudaStream_t s)
{
    int rc = SP_OK;
    const int n = a.kl.n;
    g_prof_splits = a.n_splits;
    if (use_mma && a.kv_len > 0) {
        // mma.sync kernel; the tcgen05 kernel on request (impl 3: measured
        // slower on the ship layout, 471 vs 345 us for config 1)
        if (g_force_impl == 3)
            return sp_attn_tc_launch(a, s, g_prof ? g_ev[0] : nullptr, g_prof ? g_ev[1] : nullptr);
        return sp_attn_mma_launch(a, s, g_prof ? g_ev[0] : nullptr, g_prof ? g_ev[1] : nullptr);
    }
    if (a.n_splits > 0) {
        if (g_prof) cudaEventRecord(g_ev[0], s);
        {
            switch (n) {
            case 32:  rc = launch_generic<1>(a, s); break;
            case 64:  rc = launch_generic<2>(a, s); break;
            case 128: rc = launch_generic<4>(a, s); break;
            case 256: rc = launch_generic<8>(a, s); break;
            case 512: rc = launch_generic<16>(a, s); break;
            default: return sp_set_error(SP_ERR_UNSUPPORTED, "attn_decode: head_dim %d", n);
            }
        }
        if (g_prof) cudaEventRecord(g_ev[1], s);
        if (rc) return rc;
    }
    switch (n) {
    case 32:  return launch_combine<1>(a, s);
    case 64:  return launch_combine<2>(a, s);
    case 128: return launch_combine<4>(a, s);
    case 256: return launch_combine<8>(a, s);
    case 512: return launch_combine<16>(a, s);
    }
    return sp_set_error(SP_ERR_UNSUPPORTED, "attn_decode: head_dim %d", n);
}

extern "C" int sp_cuda_attn_decode(const sp_cuda_cache_t *cc, int layer0, int n_layers,
                                   const void *d_q, int n_q_heads, int kv_len,
                                   float logit_scale, void *d_out, int max_bands, void *stream)
{
    sp_clear_error();
    if (!d_out) return sp_set_error(SP_ERR_ARG, "attn_decode: NULL argument");
    SpAttnArgs a;
    bool use_mma = false;
    int rc = attn_prepare(cc, layer0, n_layers, d_q, n_q_heads, kv_len, logit_scale, max_bands, a, use_mma);
    if (rc) return rc;
    a.out = (__half *)d_out;
    return attn_launch(a, use_mma, (cudaStream_t)stream);
}

// ----------------------------------------------- fused decode + all-gather --

extern "C" int sp_cuda_attn_decode_allgather(const sp_cuda_cache_t *cc, int layer0, int n_layers,
                                             const void *d_q, int n_q_heads, int kv_len, float logit_scale,
                                             int max_bands, void *d_local_buf, void *const *d_peer_bufs,
                                             const int *d_dst_layer, const int *d_dst_qhead, int n_q_heads_total,
                                             long long flags_offset, long long epoch_stride, int rank, int world,
                                             unsigned int epoch, void *stream)
{
    sp_clear_error();
    if (!d_local_buf || !d_peer_bufs || !d_dst_layer || !d_dst_qhead)
        return sp_set_error(SP_ERR_ARG, "attn_decode_allgather: NULL argument");
    if (world < 1 || rank < 0 || rank >= world || world > 32 || n_q_heads_total < n_q_heads)
        return sp_set_error(SP_ERR_ARG, "attn_decode_allgather: rank %d / world %d / heads %d of %d", rank, world,
                            n_q_heads, n_q_heads_total);
    if (flags_offset < 0 || (flags_offset & 3))
        return sp_set_error(SP_ERR_ARG, "attn_decode_allgather: flags_offset must be a non-negative multiple of 4");
    if (epoch_stride < 0 || (epoch_stride & 15))
        return sp_set_error(SP_ERR_ARG, "attn_decode_allgather: epoch_stride must be a non-negative multiple of 16");
    SpAttnArgs a;
    bool use_mma = false;
    int rc = attn_prepare(cc, layer0, n_layers, d_q, n_q_heads, kv_len, logit_scale, max_bands, a, use_mma);
    if (rc) return rc;
    a.g.peers = d_peer_bufs;
    a.g.dst_layer = d_dst_layer;
    a.g.dst_qhead = d_dst_qhead;
    a.g.n_q_total = n_q_heads_total;
    a.g.flags_offset = flags_offset;
    a.g.rows_offset = (epoch & 1u) ? epoch_stride : 0;
    a.g.rank = rank;
    a.g.world = world;
    a.g.epoch = epoch;
    a.g.block_count = cc->d_status + 1;          // zero between calls
    a.g.n_blocks = (unsigned)(((n_q_heads + 3) / 4) * n_layers);   // both combine grids: 4 rows per block
    a.g.own_flags = reinterpret_cast<const unsigned int *>(static_cast<const unsigned char *>(d_local_buf) +
                                                           flags_offset);
    // The combine's last block waits for every rank's flag, so the call's
    // kernels end only once the gathered rows are all in place.
    return attn_launch(a, use_mma, (cudaStream_t)stream);
}

// ------------------------------------------------ allocation-free variant --
//
// Some callers cannot call cudaMalloc: an engine that owns all device
// memory through its own allocator and hands the attention op only the
// buffers it needs (llama.cpp's ggml backend buffers work this way), or a
// plugin host that forbids a library from growing the process's device
// footprint after start-up.  Such a caller keeps the compressed cache,
// queries and outputs in memory it already owns, and has no
// sp_cuda_cache_t workspace to offer.  sp_cuda_attn_decode_noalloc runs the
// same fused decode with its split partials in the fixed device array below.
//
// The array is file-scope device memory: every GPU that loads this library
// holds SP_ATTN_STATIC_SCRATCH_BYTES of it until the process exits.  In host
// code its name is only a host-side stand-in, not a device address, so the
// first call on each device looks the real address up with
// cudaGetSymbolAddress (that device current) and keeps it; make that first
// call before any stream capture.  Every call shares the array: a call
// writes each partial it reads before reading it, so nothing has to start
// at zero, but calls that overlap on the GPU (two streams, two threads)
// race on it and must be serialised by the caller.

#define SP_ATTN_STATIC_SCRATCH_BYTES (16u << 20)

static __device__ __align__(256) unsigned char g_attn_static_scratch[SP_ATTN_STATIC_SCRATCH_BYTES];

// Error word of the allocation-free decode, shared by every call on a device
// like the scratch: bit 0 is set when a bounded copy wait of the tensor-core
// kernel ran out (that warp's tiles are then missing from the output).
// sp_cuda_attn_decode_noalloc_status reads and optionally clears it.
static __device__ unsigned int g_attn_static_status;

static void *g_static_ws_addr[128];       // per-device addresses, set once
static void *g_static_status_addr[128];

// The device addresses are looked up once per device and kept for the life
// of the process; a cudaDeviceReset after the first call on a device is not
// supported (the module's memory, and so the cached addresses, go away).
static int static_scratch_address(void **out, unsigned int **status)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128)
        return sp_set_error(SP_ERR_CUDA, "attn_decode_noalloc: no current CUDA device");
    void *p = __atomic_load_n(&g_static_ws_addr[dev], __ATOMIC_ACQUIRE);
    void *st = __atomic_load_n(&g_static_status_addr[dev], __ATOMIC_ACQUIRE);
    if (!p || !st) {
        cudaError_t e = cudaGetSymbolAddress(&p, g_attn_static_scratch);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&st, g_attn_static_status);
        if (e != cudaSuccess || !p || !st)
            return sp_set_error(SP_ERR_CUDA, "attn_decode_noalloc: cudaGetSymbolAddress: %s",
                                cudaGetErrorString(e));
        __atomic_store_n(&g_static_status_addr[dev], st, __ATOMIC_RELEASE);
        __atomic_store_n(&g_static_ws_addr[dev], p, __ATOMIC_RELEASE);
    }
    *out = p;
    *status = (unsigned int *)st;
    return SP_OK;
}

extern "C" int sp_cuda_attn_decode_noalloc_status(unsigned int *status_out, int clear, void *stream)
{
    sp_clear_error();
    if (!status_out) return sp_set_error(SP_ERR_ARG, "attn_decode_noalloc_status: NULL argument");
    void *ws = nullptr;
    unsigned int *st = nullptr;
    int rc = static_scratch_address(&ws, &st);
    if (rc) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t e = cudaMemcpyAsync(status_out, st, sizeof(unsigned int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && clear) e = cudaMemsetAsync(st, 0, sizeof(unsigned int), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return sp_check_cuda(e, "attn_decode_noalloc_status");
}

extern "C" int sp_cuda_attn_decode_noalloc(const void *d_k_cache, const void *d_v_cache,
                                           int max_seq_len, const sp_band_config_t *k_bands,
                                           const sp_band_config_t *v_bands,
                                           const int *d_mobius_order, int n_heads_kv,
                                           int layer0, int n_layers, const void *d_q,
                                           int n_q_heads, int kv_len, float logit_scale,
                                           void *d_out, int max_bands, void *stream)
{
    sp_clear_error();
    if (!d_k_cache || !d_v_cache || !k_bands || !v_bands || !d_q || !d_out)
        return sp_set_error(SP_ERR_ARG, "attn_decode_noalloc: NULL argument");
    const int n = k_bands->head_dim;
    if (v_bands->head_dim != n || n < 32 || n > SP_MAX_HEAD_DIM || (n & (n - 1)))
        return sp_set_error(SP_ERR_UNSUPPORTED, "attn_decode_noalloc: head_dim %d", n);
    if (max_seq_len <= 0 || n_heads_kv <= 0 || layer0 < 0 || n_layers <= 0)
        return sp_set_error(SP_ERR_ARG, "attn_decode_noalloc: bad dims");
    if (n_q_heads <= 0 || n_q_heads % n_heads_kv || n_q_heads / n_heads_kv > 8)
        return sp_set_error(SP_ERR_ARG, "attn_decode_noalloc: n_q_heads %d must be a multiple of %d with <= 8 per KV head",
                            n_q_heads, n_heads_kv);
    if (kv_len < 0 || kv_len > max_seq_len)
        return sp_set_error(SP_ERR_ARG, "attn_decode_noalloc: kv_len %d outside [0,%d]", kv_len, max_seq_len);
    const unsigned long long need = (unsigned long long)n_layers * n_q_heads * kAttnMaxSplits *
                                    sp_attn_partial_stride(n) * sizeof(float);
    if (need > SP_ATTN_STATIC_SCRATCH_BYTES)
        return sp_set_error(SP_ERR_ARG,
                            "attn_decode_noalloc: n_layers*n_q_heads=%d needs %llu bytes of scratch, more than "
                            "the fixed %u (at most %llu layer x q-head pairs at head_dim %d)",
                            n_layers * n_q_heads, need, SP_ATTN_STATIC_SCRATCH_BYTES,
                            (unsigned long long)SP_ATTN_STATIC_SCRATCH_BYTES /
                                (kAttnMaxSplits * sp_attn_partial_stride(n) * sizeof(float)), n);
    void *ws = nullptr;
    unsigned int *status = nullptr;
    int rc = static_scratch_address(&ws, &status);
    if (rc) return rc;

    SpAttnArgs a;
    memset(&a, 0, sizeof(a));
    a.k_cache = (const uint8_t *)d_k_cache;
    a.v_cache = (const uint8_t *)d_v_cache;
    a.k_slot_stride = (long long)max_seq_len * k_bands->total_bytes;
    a.v_slot_stride = (long long)max_seq_len * v_bands->total_bytes;
    a.order = d_mobius_order;
    a.q = (const __half *)d_q;
    a.out = (__half *)d_out;
    a.ws = (float *)ws;
    a.layer0 = layer0; a.n_layers = n_layers; a.n_kv_heads = n_heads_kv;
    a.n_q_heads = n_q_heads; a.group = n_q_heads / n_heads_kv;
    a.kv_len = kv_len;
    a.kl = sp_layout_from(*k_bands);
    a.vl = sp_layout_from(*v_bands);
    a.nb_k = (max_bands < 0 || max_bands >= a.kl.n_bands) ? a.kl.n_bands : max_bands;
    a.nb_v = (max_bands < 0 || max_bands >= a.vl.n_bands) ? a.vl.n_bands : max_bands;
    a.logit_scale = logit_scale;
    a.inv_sqrt_n = sp_inv_sqrt_n(n);
    a.status = status;

    // The tensor-core kernel stages 16-position tiles with bulk copies, which
    // need 16-byte aligned tile starts; other layouts take the generic kernel.
    const bool aligned = ((uintptr_t)d_k_cache % 16 == 0) && ((uintptr_t)d_v_cache % 16 == 0) &&
                         (max_seq_len % 16 == 0);
    bool use_mma = false;
    if ((rc = attn_plan(a, aligned, use_mma))) return rc;
    return attn_launch(a, use_mma, (cudaStream_t)stream);
}
