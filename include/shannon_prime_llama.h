/*
 * shannon_prime_llama.h — the llama.cpp bridge (sp_llama_*) of the B200
 * build.  Drop-in for the reference bridge src/tools/shannon_prime_llama.h:
 * same types, names, argument meaning, environment variables and NULL/void
 * error behaviour.  Vectors are HOST float pointers of head_dim (batches
 * [n_pos][head_dim] contiguous), as in the reference.
 *
 * Differences a caller can see:
 *   - one backend: the CUDA sm_100a cache of shannon_prime_cuda.h.  params->
 *     backend and SHANNON_PRIME_BACKEND are accepted and ignored (the
 *     reference's CPU/Adreno/Hexagon backends are not built; there is no
 *     CPU fallback).  Init returns NULL when no CUDA device is usable.
 *   - SHANNON_PRIME_{K,V}_TERNARY_BANDS (and the DRAFT_ forms) set the
 *     ternary band masks (shannon_prime_llama.c:142-166, 283-285).
 *     SHANNON_PRIME_FP8 is recognised and answered with a one-line warning
 *     (integer bands are used), as the reference bridge does on backends
 *     without an fp8 path (shannon_prime_llama.c:313-326).
 *   - PrimePE factors (core sp_prime_pe_freq_factors, absent from the
 *     reference checkout) are not computed: sp_llama_get_freq_factors()
 *     returns NULL and sp_llama_get_n_freqs() 0, the reference's
 *     "PrimePE disabled" answer.
 *   - The Hexagon archive getters return NULL / 0 (reference behaviour when
 *     that backend is not active, shannon_prime_llama.c:941-965).
 *   - Additions at the end: device-side access and the fused decode
 *     attention over host buffers.
 */
#ifndef SHANNON_PRIME_LLAMA_H
#define SHANNON_PRIME_LLAMA_H

#include "shannon_prime.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Reference shannon_prime_llama.h:97-123. */
typedef struct {
    int head_dim;
    int n_layers;
    int n_heads_kv;
    int max_seq_len;
    enum {
        SP_BACKEND_CPU     = 0,
        SP_BACKEND_CUDA    = 1,
        SP_BACKEND_VULKAN  = 2,
        SP_BACKEND_ADRENO  = 3,
        SP_BACKEND_HEXAGON = 4,
    } backend;
    void *gpu_context;          /* cudaStream_t to run on (NULL: a private stream) */
    const char *arch_name;
} sp_llama_params_t;

typedef struct sp_llama_ctx_s sp_llama_ctx_t;

/* Reference shannon_prime_llama.h:148-152. */
typedef enum {
    SP_LLAMA_ROLE_DEFAULT = 0,
    SP_LLAMA_ROLE_TARGET  = 1,
    SP_LLAMA_ROLE_DRAFT   = 2,
} sp_llama_role_t;

/* Lifecycle — reference shannon_prime_llama.h:161-182. */
sp_llama_ctx_t *sp_llama_init(const sp_llama_params_t *params);
sp_llama_ctx_t *sp_llama_init_with_role(const sp_llama_params_t *params,
                                        sp_llama_role_t role);
sp_llama_ctx_t *sp_llama_init_config(const sp_llama_params_t *params,
                                     const sp_config_t *cfg);
void sp_llama_free(sp_llama_ctx_t *ctx);

/* Write path — reference shannon_prime_llama.h:196-219. */
void sp_llama_write_kv(sp_llama_ctx_t *ctx, int layer, int head, int pos,
                       const float *k_vec, const float *v_vec);
void sp_llama_write_k(sp_llama_ctx_t *ctx, int layer, int head, int pos,
                      const float *k_vec);
void sp_llama_write_v(sp_llama_ctx_t *ctx, int layer, int head, int pos,
                      const float *v_vec);
void sp_llama_write_k_batch(sp_llama_ctx_t *ctx, int layer, int head,
                            int start_pos, int n_pos, const float *k_vecs);
void sp_llama_write_v_batch(sp_llama_ctx_t *ctx, int layer, int head,
                            int start_pos, int n_pos, const float *v_vecs);

/* Read path — reference shannon_prime_llama.h:229-266. */
void sp_llama_read_k(const sp_llama_ctx_t *ctx, int layer, int head, int pos,
                     float *k_out);
void sp_llama_read_v(const sp_llama_ctx_t *ctx, int layer, int head, int pos,
                     float *v_out);
void sp_llama_read_k_partial(const sp_llama_ctx_t *ctx, int layer, int head,
                             int pos, float *k_out, int max_bands);
void sp_llama_read_v_partial(const sp_llama_ctx_t *ctx, int layer, int head,
                             int pos, float *v_out, int max_bands);
void sp_llama_read_k_batch(const sp_llama_ctx_t *ctx, int layer, int head,
                           int start_pos, int n_pos, float *k_out);
void sp_llama_read_v_batch(const sp_llama_ctx_t *ctx, int layer, int head,
                           int start_pos, int n_pos, float *v_out);

/* Cache management — reference shannon_prime_llama.h:273-287. */
void sp_llama_clear_range(sp_llama_ctx_t *ctx, int start_pos, int end_pos);

typedef struct {
    size_t compressed_bytes;
    size_t baseline_bytes;
    float  compression_ratio;
    int    n_positions;
} sp_llama_memory_t;

sp_llama_memory_t sp_llama_memory(const sp_llama_ctx_t *ctx);

/* Diagnostics — reference shannon_prime_llama.h:294-298. */
float sp_llama_validate_k(sp_llama_ctx_t *ctx, const float *k_vec, int head_dim);
void  sp_llama_print_config(const sp_llama_ctx_t *ctx);

/* PrimePE — reference shannon_prime_llama.h:318-321 (see above). */
const float *sp_llama_get_freq_factors(const sp_llama_ctx_t *ctx);
int          sp_llama_get_n_freqs(const sp_llama_ctx_t *ctx);

/* Hexagon archive — reference shannon_prime_llama.h:340-342 (see above). */
const void *sp_llama_get_hexagon_k_buf(const sp_llama_ctx_t *ctx, int layer, int head);
int          sp_llama_get_hexagon_k_total_bytes(const sp_llama_ctx_t *ctx);

/* ----------------------------------------------------- B200 additions -- */

/* The device cache behind the context (a const sp_cuda_cache_t *, see
 * shannon_prime_cuda.h), for callers that keep K/V and queries on the GPU. */
const void *sp_llama_get_cuda_cache(const sp_llama_ctx_t *ctx);

/* Fused decode attention over HOST buffers: q_f16 and out_f16 are fp16 bit
 * patterns [n_layers][n_q_heads][head_dim].  Copies q in, runs
 * sp_cuda_attn_decode, copies the output back and waits for it.  Replaces
 * the CPU ggml op llama_sp_kq_compute (src/engine/llama_sp_fused_kq.cpp:
 * 82-165) plus the softmax and V product after it.  Returns 0 or SP_ERR_*. */
int sp_llama_attn_decode(sp_llama_ctx_t *ctx, int layer0, int n_layers,
                         const uint16_t *q_f16, int n_q_heads, int kv_len,
                         float logit_scale, uint16_t *out_f16, int max_bands);

/* Token-major write of every head of one layer from HOST buffers
 * [n_tokens][n_heads_kv][head_dim] fp32 (NULL skips K or V). */
int sp_llama_write_kv_tokens(sp_llama_ctx_t *ctx, int layer, int start_pos,
                             int n_tokens, const float *k, const float *v);

#ifdef __cplusplus
}
#endif

#endif /* SHANNON_PRIME_LLAMA_H */
