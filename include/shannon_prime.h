/*
 * shannon_prime.h — core configuration types and host utilities of the
 * Shannon-Prime KV-cache codec, restated for the B200 build.
 *
 * The reference keeps these in its core library (lib/shannon-prime/core/
 * shannon_prime.h), a git submodule that is empty in the reference checkout
 * (.gitmodules:1-3).  Every reference call site that this build replaces
 * includes it (src/backends/cuda/shannon_prime_cuda.h:12,
 * src/tools/shannon_prime_llama.h:87), so the same names are restated here
 * from how those call sites use them:
 *
 *   sp_config_t        fields read at src/tools/shannon_prime_llama.c:219-286
 *                      (head_dim, n_layers, n_heads_kv, k_n_bands,
 *                      k_band_bits, v_n_bands, v_band_bits, use_mobius_mask,
 *                      k_ternary_mask, v_ternary_mask, use_fp8)
 *   sp_band_config_t   fields read at src/backends/cuda/shannon_prime_cuda.cu:
 *                      358-377 (head_dim, n_bands, band_bits, band_size,
 *                      total_bytes)
 *   sp_band_span       src/backends/vulkan/shannon_prime_vulkan.c:563-576
 *                      (last band absorbs the remainder)
 *   sp_mobius_mask_t   .order[] used at shannon_prime_cuda.cu:427-446
 *
 * Byte layout of one packed vector (reference kernel
 * shannon_prime_cuda.cu:131-204): for each band b in order, a 2-byte
 * little-endian IEEE fp16 scale, then ceil(size_b * bits_b / 8) bytes of
 * offset codes u = q + (2^(bits_b-1) - 1) packed LSB-first; every band starts
 * on a byte boundary.
 */
#ifndef SHANNON_PRIME_H
#define SHANNON_PRIME_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SP_MAX_BANDS 16     /* Vulkan push constant carries bits[16] (shannon_prime_vulkan.c:540-546) */
#define SP_MAX_HEAD_DIM 512 /* largest power-of-two head_dim the ship kernels accept */

typedef struct {
    int head_dim;
    int n_layers;
    int n_heads_kv;

    int k_n_bands;
    int k_band_bits[SP_MAX_BANDS];
    int v_n_bands;
    int v_band_bits[SP_MAX_BANDS];

    int use_mobius_mask;        /* squarefree-first reorder of K coefficients */

    /* Bit b of a ternary mask stores band b as {-1, 0, +1} at 2 bits per
     * code whatever its band_bits (the band quantiser at m = 1).  use_fp8 is
     * rejected by sp_cuda_cache_init; the bridge treats it as advisory and
     * uses integer bands, as the reference bridge does. */
    uint32_t k_ternary_mask;
    uint32_t v_ternary_mask;
    int use_fp8;
} sp_config_t;

typedef struct {
    int head_dim;
    int n_bands;
    int band_bits[SP_MAX_BANDS];
    int band_size;              /* head_dim / n_bands; last band takes the remainder */
    int total_bytes;            /* packed bytes per vector */
} sp_band_config_t;

typedef struct {
    int  n;
    int *order;                 /* order[i] = source coefficient for reordered slot i */
} sp_mobius_mask_t;

/* Defaults follow the bridge's head-dim-adaptive choice
 * (shannon_prime_llama.c:235-252): hd >= 128 -> K 5,5,4,3 and V 3;
 * hd < 128 -> K 5,4,4 and V 5.  Möbius on. */
void sp_config_init(sp_config_t *cfg, int head_dim, int n_layers, int n_heads_kv);

/* Returns 0 on success, -1 on invalid arguments (bits outside 1..8,
 * n_bands outside 1..SP_MAX_BANDS or > head_dim). */
int  sp_band_config_init(sp_band_config_t *bc, int head_dim, int n_bands,
                         const int *band_bits);
void sp_band_span(const sp_band_config_t *bc, int band, int *offset, int *size);

/* Squarefree-first permutation: indices i in [0,n) with i+1 squarefree,
 * ascending, then the others ascending.  Returns 0 / -1 (allocation). */
int  sp_mobius_mask_init(sp_mobius_mask_t *mask, int n);
void sp_mobius_mask_free(sp_mobius_mask_t *mask);

/* Pearson correlation of two float vectors (accumulated in double). */
float sp_correlation_f32(const float *a, const float *b, int n);

void sp_config_print(const sp_config_t *cfg);

#ifdef __cplusplus
}
#endif

#endif /* SHANNON_PRIME_H */
