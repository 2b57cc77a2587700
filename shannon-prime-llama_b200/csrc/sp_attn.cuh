// sp_attn.cuh — arguments and workspace layout shared by the fused decode
// attention kernels (sp_attn.cu, sp_attn_mma.cu).
#pragma once

#include "sp_internal.cuh"

// Split-K workspace: one partial per (layer in call, query head, split):
// [m, l, pad, pad, acc[n]] floats, m and l in base-2 logit units.
constexpr int kAttnMaxSplits = 128;
constexpr int kAttnMinChunk = 64;       // tokens; multiple of 16

// Fused all-gather epilogue of the combine kernels (world == 0: off, the
// outputs go to SpAttnArgs::out).  Each output row is stored straight into
// every rank's gather buffer (peer addresses mapped into this process), at
// row dst_layer[li] * n_q_total + dst_qhead[qh]; the last combine block then
// writes `epoch` into slot `rank` of every rank's flag array.
struct SpGather {
    void *const *peers;                 // device array [world]
    const int *dst_layer;               // [n_layers] destination layer row
    const int *dst_qhead;               // [n_q_heads] destination query-head column
    int n_q_total;                      // query heads per destination layer row
    long long flags_offset;             // bytes: [world] uint32 flags in each buffer
    long long rows_offset;              // bytes: this call's copy of the rows in each buffer
    int rank, world;
    unsigned int epoch;
    unsigned int *block_count;          // device counter, zero between calls
    unsigned int n_blocks;              // combine blocks in the call
    const unsigned int *own_flags;      // [world] flags in this rank's own buffer
};

// Programmatic dependent launch: a main decode kernel lets its combine
// kernel launch early (sp_pdl_trigger at its start); the combine waits for
// the main grid's completion and memory (sp_pdl_wait) before it reads any
// partial.
__device__ __forceinline__ void sp_pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void sp_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

struct SpAttnArgs {
    const uint8_t *k_cache;
    const uint8_t *v_cache;
    long long k_slot_stride;            // bytes per slot
    long long v_slot_stride;
    const int *order;                   // Möbius order (K) or nullptr
    const __half *q;                    // [n_layers][n_q_heads][n]
    __half *out;                        // [n_layers][n_q_heads][n]
    float *ws;                          // partials
    int layer0, n_layers, n_kv_heads, n_q_heads, group;
    int kv_len, chunk, n_splits;
    int nb_k, nb_v;                     // bands used (partial reads)
    float logit_scale;
    float inv_sqrt_n;
    unsigned int *status;               // device error word
    SpBandLayout kl, vl;
    SpGather g;
};

// Store one lane's E output halves of row (li, qh): locally, or into every
// rank's gather buffer.
template <int E>
__device__ __forceinline__ void sp_attn_store_row(const SpAttnArgs &a, int li, int qh, int lane, const __half (&h)[E])
{
    const int n = 32 * E;
    if (a.g.world == 0) {
        __half *o = a.out + ((long long)li * a.n_q_heads + qh) * n + lane * E;
        if constexpr (E == 4) {
            if (((uintptr_t)o & 7) == 0) {      // one 8-byte store per lane (the output may be host memory)
                uint2 w;
                w.x = (uint32_t)__half_as_ushort(h[0]) | ((uint32_t)__half_as_ushort(h[1]) << 16);
                w.y = (uint32_t)__half_as_ushort(h[2]) | ((uint32_t)__half_as_ushort(h[3]) << 16);
                *reinterpret_cast<uint2 *>(o) = w;
                return;
            }
        }
#pragma unroll
        for (int e = 0; e < E; e++) o[e] = h[e];
        return;
    }
    const long long off = ((long long)a.g.dst_layer[li] * a.g.n_q_total + a.g.dst_qhead[qh]) * n + lane * E;
    for (int p = 0; p < a.g.world; p++) {
        __half *o = reinterpret_cast<__half *>(reinterpret_cast<unsigned char *>(a.g.peers[p]) +
                                               a.g.rows_offset) + off;
        if constexpr (E == 4) {
            uint2 w;
            w.x = (uint32_t)__half_as_ushort(h[0]) | ((uint32_t)__half_as_ushort(h[1]) << 16);
            w.y = (uint32_t)__half_as_ushort(h[2]) | ((uint32_t)__half_as_ushort(h[3]) << 16);
            *reinterpret_cast<uint2 *>(o) = w;
        } else {
#pragma unroll
            for (int e = 0; e < E; e++) o[e] = h[e];
        }
    }
}

// After a combine block's rows are stored: the last block of the call
// raises this rank's flag in every rank's buffer, then waits (bounded at
// 2 s by %globaltimer; bit 1 of *status on timeout) until every rank's flag
// in this rank's own buffer shows the epoch (wrap-safe), so the kernel ends
// only when the whole gathered output is in place.  Called by every thread.
__device__ __forceinline__ void sp_attn_gather_signal(const SpAttnArgs &a)
{
    if (a.g.world == 0) return;
    __threadfence_system();             // this thread's peer stores before the count
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int prev = atomicAdd(a.g.block_count, 1u);
        if (prev == a.g.n_blocks - 1) {
            __threadfence_system();
            *a.g.block_count = 0u;
            for (int p = 0; p < a.g.world; p++) {
                unsigned int *f = reinterpret_cast<unsigned int *>(
                    reinterpret_cast<unsigned char *>(a.g.peers[p]) + a.g.flags_offset) + a.g.rank;
                asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(a.g.epoch) : "memory");
            }
            unsigned long long t0;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
            for (int p = 0; p < a.g.world; p++) {
                for (;;) {
                    unsigned int v;
                    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a.g.own_flags + p) : "memory");
                    if ((int)(v - a.g.epoch) >= 0) break;
                    unsigned long long t;
                    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
                    if (t - t0 > 2000000000ull) {
                        atomicOr(a.status, 2u);
                        return;
                    }
                    __nanosleep(64);
                }
            }
        }
    }
}

__host__ __device__ inline long long sp_attn_partial_stride(int n) { return n + 4; }

__device__ inline float *sp_attn_partial(const SpAttnArgs &a, int li, int qh, int split)
{
    const long long idx = ((long long)li * a.n_q_heads + qh) * kAttnMaxSplits + split;
    return a.ws + idx * sp_attn_partial_stride(a.kl.n);
}

// Tensor-core kernel for the ship layout (sp_attn_mma.cu).  Returns
// SP_ERR_UNSUPPORTED (without launching) when the layout does not match.
int sp_attn_mma_supported(const SpAttnArgs &a);
// Launches the main kernel and its own segment combine.  ev_begin/ev_end
// (optional) are recorded around the main kernel on stream s.
int sp_attn_mma_launch(const SpAttnArgs &a, cudaStream_t s, cudaEvent_t ev_begin = nullptr,
                       cudaEvent_t ev_end = nullptr);

// Work split of the tensor-core decode kernels: the flattened (layer, KV
// head, tile) space is cut into n_ctas equal contiguous ranges, one per CTA;
// a CTA writes one partial per (layer, KV head) segment it touches.
struct SpSched {
    long long total_tiles;   // units * tiles_per_unit
    int tiles_per_unit;      // ceil(kv_len / tile)
    int n_ctas;
};

__host__ __device__ inline long long sp_tile_begin(long long i, const SpSched &s)
{
    return i * s.total_tiles / s.n_ctas;
}
// Index of the CTA whose range holds tile g.
__host__ __device__ inline int sp_cta_of_tile(long long g, const SpSched &s)
{
    return (int)(((g + 1) * s.n_ctas + s.total_tiles - 1) / s.total_tiles) - 1;
}

// Segment combine of a tensor-core decode (sp_attn_mma.cu): merges the
// partials the schedule wrote, applies the inverse VHT2, writes fp16 rows
// (locally or into the gather buffers).
int sp_attn_seg_combine_launch(const SpAttnArgs &a, const SpSched &sc, cudaStream_t s);

// tcgen05 kernel for the ship layout (sp_attn_tc.cu).
int sp_attn_tc_supported(const SpAttnArgs &a);
int sp_attn_tc_launch(const SpAttnArgs &a, cudaStream_t s, cudaEvent_t ev_begin = nullptr,
                      cudaEvent_t ev_end = nullptr);
