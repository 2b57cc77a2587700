// sp_cold.cu — cold storage: per-layer page-locked host mirrors of cache
// slabs (the warm tier of the reference's tiered offload; interface and
// semantics of shannon_prime_cuda.h:233-286 / shannon_prime_cuda.cu:680-785,
// as the engine drives them in kv_cache.cpp:1385-1530).
//
// Host code only: page-locked allocation and async copies on the caller's
// stream.  Errors are returned (-1) as in the reference, and also recorded
// for sp_cuda_last_error().
#include "shannon_prime_cuda.h"
#include "sp_internal.cuh"

#include <cuda_runtime.h>
#include <string.h>

extern "C" {

void sp_cuda_d2h_async(void *dst_host, const void *src_device, int64_t n_bytes, void *stream)
{
    sp_clear_error();
    if (n_bytes <= 0) return;
    sp_check_cuda(cudaMemcpyAsync(dst_host, src_device, (size_t)n_bytes, cudaMemcpyDeviceToHost,
                                  (cudaStream_t)stream),
                  "sp_cuda_d2h_async");
}

void sp_cuda_h2d_async(void *dst_device, const void *src_host, int64_t n_bytes, void *stream)
{
    sp_clear_error();
    if (n_bytes <= 0) return;
    sp_check_cuda(cudaMemcpyAsync(dst_device, src_host, (size_t)n_bytes, cudaMemcpyHostToDevice,
                                  (cudaStream_t)stream),
                  "sp_cuda_h2d_async");
}

int sp_cuda_cold_layer_init(sp_cuda_cold_layer_t *cl, int64_t cap_bytes, int packed_stride, int n_heads)
{
    sp_clear_error();
    if (!cl || cap_bytes <= 0 || packed_stride <= 0 || n_heads <= 0) {
        sp_set_error(SP_ERR_ARG, "cold_layer_init: bad arguments");
        return -1;
    }
    memset(cl, 0, sizeof(*cl));
    void *p = nullptr;
    if (sp_check_cuda(cudaHostAlloc(&p, (size_t)cap_bytes, cudaHostAllocDefault), "cold_layer_init cudaHostAlloc"))
        return -1;
    cl->h_pinned = static_cast<uint8_t *>(p);
    cl->capacity = cap_bytes;
    cl->packed_stride = packed_stride;
    cl->n_heads = n_heads;
    cl->write_head = 0;
    cl->oldest_pos = -1;
    cl->newest_pos = -1;
    cl->ring_mode = false;
    cl->initialized = true;
    return 0;
}

void sp_cuda_cold_layer_free(sp_cuda_cold_layer_t *cl)
{
    sp_clear_error();
    if (!cl) return;
    if (cl->h_pinned) sp_check_cuda(cudaFreeHost(cl->h_pinned), "cold_layer_free");
    cl->h_pinned = nullptr;
    cl->initialized = false;
}

int sp_cuda_cold_writeback(sp_cuda_cold_layer_t *cl, const void *d_packed, int start_pos, int n_pos,
                           void *stream)
{
    sp_clear_error();
    if (!cl || !cl->initialized || !d_packed || n_pos <= 0 || start_pos < 0) {
        sp_set_error(SP_ERR_ARG, "cold_writeback: bad arguments");
        return -1;
    }
    const int64_t per_pos = (int64_t)cl->n_heads * cl->packed_stride;
    const int64_t bytes = (int64_t)n_pos * per_pos;
    if (bytes > cl->capacity) {
        sp_set_error(SP_ERR_ARG, "cold_writeback: %lld bytes exceed the buffer (%lld)", (long long)bytes,
                     (long long)cl->capacity);
        return -1;
    }
    if (cl->write_head + bytes > cl->capacity) {   // wrap: the ring restarts at offset 0
        cl->write_head = 0;
        cl->ring_mode = true;
    }
    if (sp_check_cuda(cudaMemcpyAsync(cl->h_pinned + cl->write_head,
                                      static_cast<const uint8_t *>(d_packed) + (int64_t)start_pos * per_pos,
                                      (size_t)bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream),
                      "cold_writeback"))
        return -1;
    cl->write_head += bytes;
    cl->newest_pos = (int64_t)start_pos + n_pos - 1;
    if (cl->ring_mode) {
        const int64_t held = cl->capacity / per_pos;   // positions the buffer holds
        cl->oldest_pos = cl->newest_pos - held + 1;
        if (cl->oldest_pos < 0) cl->oldest_pos = 0;
    } else if (cl->oldest_pos < 0) {
        cl->oldest_pos = 0;
    }
    return 0;
}

int sp_cuda_cold_restore(const sp_cuda_cold_layer_t *cl, void *d_packed, int n_pos, void *stream)
{
    sp_clear_error();
    if (!cl || !cl->initialized || !d_packed || n_pos <= 0) {
        sp_set_error(SP_ERR_ARG, "cold_restore: bad arguments");
        return -1;
    }
    if (cl->ring_mode) {
        sp_set_error(SP_ERR_UNSUPPORTED, "cold_restore: the buffer has wrapped (ring mode)");
        return -1;
    }
    const int64_t bytes = (int64_t)n_pos * cl->n_heads * cl->packed_stride;
    if (bytes > cl->capacity) {
        sp_set_error(SP_ERR_ARG, "cold_restore: %lld bytes exceed the buffer (%lld)", (long long)bytes,
                     (long long)cl->capacity);
        return -1;
    }
    if (sp_check_cuda(cudaMemcpyAsync(d_packed, cl->h_pinned, (size_t)bytes, cudaMemcpyHostToDevice,
                                      (cudaStream_t)stream),
                      "cold_restore"))
        return -1;
    return 0;
}

}  // extern "C"
