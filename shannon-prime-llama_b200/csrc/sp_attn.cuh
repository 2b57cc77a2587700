// sp_attn.cuh — arguments and workspace layout shared by the fused decode
// attention kernels (sp_attn.cu, sp_attn_mma.cu).
#pragma once

#include "sp_internal.cuh"

// Split-K workspace: one partial per (layer in call, query head, split):
// [m, l, pad, pad, acc[n]] floats, m and l in base-2 logit units.
constexpr int kAttnMaxSplits = 128;
constexpr int kAttnMinChunk = 64;       // tokens; multiple of 16

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
};

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
