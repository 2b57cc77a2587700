/*
 * sp_oracle.h — CPU restatement of the Shannon-Prime KV-cache hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this code; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline legs use it, as the checker and as the timed CPU baseline.
 *
 * Parity status: PINNED to the reference's own CUDA code, run on a B200.
 * The reference CPU path (sp_shadow_*, sp_band_*, sp_vht2_forward_f32,
 * sp_mobius_mask_init in the core library lib/shannon-prime) is an empty git
 * submodule in the reference checkout (.gitmodules:1-3), so it cannot run.
 * The reference's CUDA sources src/backends/cuda/shannon_prime_{cuda,sqfree,
 * hier}.cu do build, unmodified, against include/shannon_prime.h
 * (oracle/ref/Makefile -> oracle/_ref); tests/golden/make_ref_fixtures.py
 * ran them and tests/test_ref_fixtures.py checks this oracle against what
 * they computed:
 *   - band quantiser (shannon_prime_cuda.cu:131-204): bit-exact on 65,536
 *     config-0 rows and 128 edge rows;
 *   - the reference's whole write (:565-620) equals this quantiser on the
 *     reference CUDA form of the VHT2 (per-stage x1/sqrt2, :37-75) bit for
 *     bit; this oracle's VHT2 follows the CPU core's form (NEON restatement
 *     shannon_prime_adreno.c:270-309, reported bit-equal to the core at
 *     hd 32/64/128 in android_build/test_adreno_phone.log:44-46), and the
 *     two forms differ in about 1e-4 of bands (fp16-scale midpoints and
 *     half-integer ties, each checked);
 *   - sqfree Möbius prediction, spinor choice, residual levels, packing and
 *     dequantisation, and the hier W.skeleton product, levels and
 *     dequantisation: bit-exact; the hier magnitude differs by <= 2 ulp (sum
 *     order) with no level changed.
 * Choices of the absent core that no reference code fixes (tables): the
 * Möbius order (squarefree-first, ascending), the Knight skeleton ranking
 * and CSR, the sqfree pad mean (true mean; the reference kernel sums warp 0
 * only), cas tables in double (the reference uses __cosf/__sinf; agreement
 * within 5e-5 is checked).
 */
#ifndef SP_ORACLE_H
#define SP_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OR_MAX_BANDS 16

typedef struct {
    int n;                     /* vector length */
    int n_bands;
    int bits[OR_MAX_BANDS];
    int off[OR_MAX_BANDS];     /* first coefficient of band b */
    int size[OR_MAX_BANDS];    /* coefficients in band b */
    int byte_off[OR_MAX_BANDS];/* byte offset of band b's fp16 scale */
    int total_bytes;
} or_bands_t;

uint16_t or_f32_to_f16(float f);
float    or_f16_to_f32(uint16_t h);

int  or_band_config(or_bands_t *bc, int n, int n_bands, const int *bits);
void or_vht2(float *x, int n);
void or_mobius_order(int n, int *order);

void or_band_quantize(const float *coeffs, uint8_t *out, const or_bands_t *bc);
void or_band_dequantize(const uint8_t *in, float *coeffs, const or_bands_t *bc,
                        int max_bands);

void or_ship_write(const float *vec, uint8_t *out, const or_bands_t *bc,
                   const int *order);
void or_ship_read(const uint8_t *in, float *vec, const or_bands_t *bc,
                  const int *order, int max_bands);

/* Batched forms (OpenMP over vectors when n_threads > 1).  vec i is read
 * from vecs + i * vec_stride (floats); packed row i goes to out + i * bytes. */
void or_ship_write_batch(int n_vecs, const float *vecs, size_t vec_stride,
                         uint8_t *out, const or_bands_t *bc, const int *order,
                         int n_threads);
void or_ship_read_batch(int n_vecs, const uint8_t *in, float *vecs,
                        const or_bands_t *bc, const int *order, int max_bands,
                        int n_threads);

/* Decode attention over one compressed (layer) cache, the reference's fused
 * decompress-KQ algorithm (llama_sp_fused_kq.cpp:82-165: decompress a row,
 * dot it with every query of the group) extended with softmax and the
 * decompressed V rows, accumulated in double.
 *   k_slots: [n_kv_heads][slot_stride_k bytes], token t of head h at
 *            k_slots + h*slot_stride_k + t*kb.total_bytes (same for V)
 *   q:       [n_q_heads][n] fp16 bits; q head g uses kv head g / (n_q/n_kv)
 *   out:     [n_q_heads][n] float
 */
void or_attn_decode(const uint8_t *k_slots, size_t slot_stride_k,
                    const uint8_t *v_slots, size_t slot_stride_v,
                    const or_bands_t *kb, const or_bands_t *vb,
                    const int *order, int n_kv_heads, int n_q_heads,
                    int kv_len, const uint16_t *q, float logit_scale,
                    float *out, int n_threads);

/* ---- sqfree+spinor and hierarchical Vilenkin (sp_oracle_sqfree.c) ---- */

#define OR_SQ_MAX_PD 512
#define OR_SQ_MAX_TERMS 16384

typedef struct {
    int hd, pd, sk_k, n_res, n_terms, res_bits, use_spinor;
    int skel_idx[OR_SQ_MAX_PD];      /* skeleton slot -> coefficient index */
    int res_idx[OR_SQ_MAX_PD];       /* residual slot -> coefficient index */
    int csr_off[OR_SQ_MAX_PD + 1];
    int csr_slot[OR_SQ_MAX_TERMS];
    int csr_sign[OR_SQ_MAX_TERMS];
    or_bands_t bands;                /* band layout over the sk_k skeleton values */
    int res_bytes, sheet_bytes, bytes_per_pos;
} or_sqfree_t;

typedef struct {
    int hd, pd, n_skel, n_target, res_bits;
    or_bands_t bands;                /* over the n_skel skeleton values (indices 0..n_skel) */
    int res_bytes, bytes_per_pos;
} or_hier_t;

float or_lane_tree_sum(const float *v, int n);
int   or_sqfree_pad_dim(int hd);
int   or_vilenkin_factors(int pd, int *factors);
void  or_cas_table(int p, float *cas, float *inv_sqrt_p);
void  or_vilenkin(float *x, int pd);

int  or_sqfree_layout(or_sqfree_t *L, int hd, int sk_k, int n_bands, const int *bits,
                      int residual_bits, int use_spinor);
void or_sqfree_write(const float *vec, uint8_t *out, const or_sqfree_t *L);
void or_sqfree_coeffs(const uint8_t *in, float *coeffs, const or_sqfree_t *L);
void or_sqfree_read(const uint8_t *in, float *vec, const or_sqfree_t *L);
void or_sqfree_write_batch(int n_vecs, const float *vecs, uint8_t *out, const or_sqfree_t *L,
                           int n_threads);
void or_sqfree_read_batch(int n_vecs, const uint8_t *in, float *vecs, const or_sqfree_t *L,
                          int n_threads);
void or_sqfree_attn_decode(const uint8_t *k_slots, size_t stride_k, const uint8_t *v_slots,
                           size_t stride_v, const or_sqfree_t *LK, const or_sqfree_t *LV,
                           int n_kv_heads, int n_q_heads, int kv_len, const uint16_t *q,
                           float logit_scale, float *out, int n_threads);

int  or_hier_layout(or_hier_t *L, int hd, int n_bands, const int *bits, int residual_bits);
void or_hier_write(const float *vec, uint8_t *out, const or_hier_t *L, const uint16_t *W);
void or_hier_read(const uint8_t *in, float *vec, const or_hier_t *L, const uint16_t *W);
void or_hier_write_batch(int n_vecs, const float *vecs, uint8_t *out, const or_hier_t *L,
                         const uint16_t *W, int n_threads);
void or_hier_read_batch(int n_vecs, const uint8_t *in, float *vecs, const or_hier_t *L,
                        const uint16_t *W, int n_threads);

/* Residual stages (each checked against the reference's own kernel). */
void  or_sq_predict(const or_sqfree_t *L, const float *sk, float *pred);
void  or_hier_predict(const or_hier_t *L, const uint16_t *W, const float *sk, float *pred);
void  or_sq_spinor(const float *actual, const float *pred, int n, float *dev, uint8_t *sheet);
float or_residual_mag(const float *dev, int n);
void  or_sq_levels(const float *dev, int n, int bits, float mag, uint8_t *lv);
void  or_sq_unlevels(const uint8_t *lv, int n, int bits, float mag, float *dev);
void  or_hier_levels(const float *dev, int n, int bits, float mag, uint8_t *lv);
void  or_hier_unlevels(const uint8_t *lv, int n, int bits, float mag, float *dev);

/* Pearson correlation accumulated in double. */
double or_correlation(const float *a, const float *b, int n);

#ifdef __cplusplus
}
#endif

#endif
