// sp_dual.cu — the GPU merge of the System 1 <-> 2 dual cache
// (DualKvCache::read_merged_gpu, src/engine/kv_cache.cpp:1832-1860).  The
// reference reads System 1 for every position and leaves the System 2
// positions unmerged on the GPU (its comment plans "a single merge kernel
// that takes both device buffers + a route bitset and scatters in one
// pass"); its host path selects row by row (kv_cache.cpp:1817-1828).  This
// is that kernel: row p of the output comes from System 2 when bit p of the
// route bitset is set, else from System 1.
#include "sp_internal.cuh"

namespace {

// One warp per row; rows move as float4 when both buffers allow it.
__global__ void k_dual_merge(const float *sys1, const float *sys2, const uint32_t *route, int n_pos, int row,
                             float *out, bool vec4)
{
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= n_pos) return;
    const bool s2 = (route[warp >> 5] >> (warp & 31)) & 1u;
    const float *src = (s2 ? sys2 : sys1) + (long long)warp * row;
    float *dst = out + (long long)warp * row;
    if (src == dst) return;                     // in place: the row is already there
    if (vec4) {
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        float4 *d4 = reinterpret_cast<float4 *>(dst);
        for (int i = lane; i < row / 4; i += 32) d4[i] = s4[i];
    } else {
        for (int i = lane; i < row; i += 32) dst[i] = src[i];
    }
}

}  // namespace

extern "C" int sp_cuda_dual_merge(const float *d_sys1, const float *d_sys2, const uint32_t *d_route_bits,
                                  int n_pos, int row_floats, float *d_out, void *stream)
{
    sp_clear_error();
    if (!d_sys1 || !d_sys2 || !d_route_bits || !d_out) return sp_set_error(SP_ERR_ARG, "dual_merge: NULL argument");
    if (n_pos < 0 || row_floats <= 0) return sp_set_error(SP_ERR_ARG, "dual_merge: bad sizes");
    if (n_pos == 0) return SP_OK;
    const bool vec4 = row_floats % 4 == 0 && ((uintptr_t)d_sys1 | (uintptr_t)d_sys2 | (uintptr_t)d_out) % 16 == 0;
    const long long threads = (long long)n_pos * 32;
    k_dual_merge<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        d_sys1, d_sys2, d_route_bits, n_pos, row_floats, d_out, vec4);
    return sp_check_cuda(cudaGetLastError(), "dual_merge launch");
}
