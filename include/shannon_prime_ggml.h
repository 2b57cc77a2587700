/*
 * shannon_prime_ggml.h — the B200 fused decode behind ggml's tensor
 * conventions (no ggml types in the signature: a tensor is passed as its
 * data pointer, its ggml type id and its ne[4] / nb[4] arrays, so a
 * ggml-cuda backend op can call it with tensor->data, tensor->type,
 * tensor->ne and tensor->nb unchanged).
 *
 * Replaces, for decode, the attention subgraph the reference builds in
 * llama.cpp's build_attn_mha (patches/llama-cpp-b8861-full-engine.patch:
 * 393-410): ggml_map_custom2(q, k, llama_sp_kq_compute) (the CPU op of
 * src/engine/llama_sp_fused_kq.cpp:82-165, scores only, K decompressed per
 * row), then ggml_soft_max_ext(kq, kq_mask, kq_scale) and
 * ggml_mul_mat(v, kq).  Here one call reads the compressed K and V slots of
 * layer il of a ship cache and returns softmax(kq_scale * q.K^T) V for every
 * query head.
 */
#ifndef SHANNON_PRIME_GGML_H
#define SHANNON_PRIME_GGML_H

#include <stddef.h>
#include <stdint.h>

#include "shannon_prime_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids accepted for q and dst (ggml.h: GGML_TYPE_F32, GGML_TYPE_F16) */
#define SP_GGML_TYPE_F32 0
#define SP_GGML_TYPE_F16 1

/* One decode token of layer il:
 *   q    ne = {head_dim, 1, n_head_q, 1}, nb in bytes (the permuted Q view)
 *   dst  ne = {head_dim, n_head_q, 1, 1}, nb in bytes (kqv before cont_2d)
 * n_head_q a multiple of the cache's n_heads_kv, at most 8 per KV head;
 * query head g reads KV head g / (n_head_q / n_heads_kv).  n_kv: cached
 * positions attended ([0, n_kv)); max_bands < 0 reads every band.
 * Stream-ordered on `stream`; allocates nothing (the fp16 staging rows live
 * in cc->d_scratch, so calls on one cache must not overlap on the GPU).
 * Returns 0 or an SP_ERR_* code. */
int sp_ggml_attn_decode(const sp_cuda_cache_t *cc, int il, const void *q_data, int q_type,
                        const int64_t q_ne[4], const size_t q_nb[4], void *dst_data, int dst_type,
                        const int64_t dst_ne[4], const size_t dst_nb[4], float kq_scale, int n_kv,
                        int max_bands, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* SHANNON_PRIME_GGML_H */
