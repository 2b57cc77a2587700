// sp_internal.cuh — shared device/host helpers of the B200 Shannon-Prime
// kernels (not part of the public C-ABI).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "shannon_prime.h"
#include "shannon_prime_cuda.h"

// Band layout of one packed vector, passed to kernels by value.
struct SpBandLayout {
    int n;                       // coefficients per vector
    int n_bands;
    int total_bytes;
    int off[SP_MAX_BANDS];       // first coefficient of band b
    int size[SP_MAX_BANDS];      // coefficients in band b
    int bits[SP_MAX_BANDS];
    int byte_off[SP_MAX_BANDS];  // byte offset of band b's fp16 scale
};

// Built from a reference-style sp_band_config_t (spans as sp_band_span).
SpBandLayout sp_layout_from(const sp_band_config_t &bc);

// Per-host-thread status used by the void entry points.
int  sp_set_error(int code, const char *fmt, ...);
void sp_clear_error();
int  sp_check_cuda(cudaError_t e, const char *what);

// Bytes of sp_cuda_cache_t::d_scratch: the staging rows of the ggml-shaped
// decode (sp_ggml.cu): fp16 queries and fp16 outputs of one token, up to 8
// query heads per KV head, and never less than the reference's [head_dim]
// floats.
inline size_t sp_io_scratch_bytes(const sp_config_t *cfg)
{
    const size_t io = 2ull * 8 * cfg->n_heads_kv * cfg->head_dim * 2;
    const size_t ref = (size_t)cfg->head_dim * 4;
    return io > ref ? io : ref;
}

// 1/sqrt(n) exactly as the CPU path computes it (IEEE sqrt, IEEE divide).
float sp_inv_sqrt_n(int n);

// Launch helpers implemented in sp_ship.cu, shared with the bridge.
int sp_launch_encode(const void *d_in, int dtype, int n_tokens, int nh,
                     uint8_t *d_out_base, long long slot0, long long slot_stride_bytes,
                     int start_pos, const int *d_order, bool do_wht,
                     const SpBandLayout &bl, cudaStream_t s, bool std_order = false,
                     unsigned int *d_status = nullptr);
// Lane-per-vector ship encoder (sp_ship_lane.cu): returns 1 and sets *rc
// when it takes the call (head_dim 128 ship layouts, standard order).
int sp_encode_lane_try(const void *d_in, int dtype, int n_tokens, int nh, uint8_t *d_out_base,
                       long long slot0, long long slot_stride, int start_pos, bool std_order,
                       const int *d_order, bool do_wht, const SpBandLayout &bl, unsigned int *d_status,
                       cudaStream_t s, int *rc);
// Both halves of one layer's tokens in one lane-encoder launch (null input =
// half skipped); 0 when the layouts or inputs do not qualify.
int sp_encode_lane_kv(const void *d_k, const void *d_v, int dtype, int n_tokens, int nh, int start_pos,
                      uint8_t *k_base, long long k_slot0, long long k_slot_stride, const SpBandLayout &kbl,
                      const int *d_order, bool std_order,
                      uint8_t *v_base, long long v_slot0, long long v_slot_stride, const SpBandLayout &vbl,
                      unsigned int *d_status, cudaStream_t s, int *rc);
int sp_launch_decode(const uint8_t *d_in_base, long long slot, long long slot_stride_bytes,
                     int start_pos, int n_pos, float *d_out, const int *d_order,
                     bool do_wht, int max_bands, const SpBandLayout &bl, cudaStream_t s,
                     bool std_order = false, unsigned int *d_status = nullptr);
// Lane-per-vector ship read (sp_ship_lane.cu): 1 and *rc set if it took the call.
int sp_decode_lane_try(const uint8_t *d_rows, int n_pos, float *d_out, const int *d_order, bool std_order,
                       bool do_wht, int max_bands, const SpBandLayout &bl, unsigned int *d_status, cudaStream_t s,
                       int *rc);

// ---------------------------------------------------------------- device --

static __device__ __forceinline__ float sp_load_as_float(const float *p, long long i) { return p[i]; }
static __device__ __forceinline__ float sp_load_as_float(const __half *p, long long i) { return __half2float(p[i]); }
static __device__ __forceinline__ float sp_load_as_float(const __nv_bfloat16 *p, long long i) { return __bfloat162float(p[i]); }

// In-register p=2 Hartley butterfly over a warp-distributed vector of
// 32*E floats: lane L holds elements L*E .. L*E+E-1.  The pair (i, i+len)
// becomes (x_i + x_{i+len}, x_i - x_{i+len}) for len = 1, 2, 4, ... exactly
// as the CPU form (shannon_prime_adreno.c:281-296), so every output is the
// same sequence of IEEE adds; the caller applies the 1/sqrt(n) scale.
template <int E>
static __device__ __forceinline__ void sp_warp_wht(float (&x)[E], int lane)
{
#pragma unroll
    for (int len = 1; len < E; len <<= 1) {
#pragma unroll
        for (int i = 0; i < E; i += len << 1) {
#pragma unroll
            for (int j = 0; j < len; j++) {
                float u = x[i + j], v = x[i + j + len];
                x[i + j] = __fadd_rn(u, v);
                x[i + j + len] = __fsub_rn(u, v);
            }
        }
    }
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const bool upper = (lane & m) != 0;
#pragma unroll
        for (int e = 0; e < E; e++) {
            float o = __shfl_xor_sync(0xffffffffu, x[e], m);
            // lower element keeps u + v, upper keeps u - v (u = lower).
            x[e] = upper ? __fsub_rn(o, x[e]) : __fadd_rn(x[e], o);
        }
    }
}
