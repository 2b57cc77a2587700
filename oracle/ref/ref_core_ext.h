/*
 * ref_core_ext.h -- TEST INFRASTRUCTURE (the reference-run checker).
 *
 * Force-included (nvcc -include) when the unmodified reference source
 * src/backends/cuda/shannon_prime_sqfree.cu is compiled into oracle/_ref.
 * That file calls four sqfree helpers of the absent core library
 * (sp_sqfree_pad_dim, sp_knight_mask_t/_init/_free at
 * shannon_prime_sqfree.cu:600-657).  The checker only launches the
 * self-contained residual, prediction and spinor kernels of that file, never
 * its cache init, so the helpers are declared here with the field names the
 * file reads and defined in ref_glue.cu as "not provided" (init returns -1).
 */
#ifndef SP_REF_CORE_EXT_H
#define SP_REF_CORE_EXT_H
#include "shannon_prime.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int     sk_k, n_res, n_terms;
    int    *skeleton_idx;
    int    *residual_idx;
    int    *csr_offsets;
    int    *csr_skel_slot;
    int8_t *csr_mu_sign;
} sp_knight_mask_t;

int  sp_sqfree_pad_dim(int head_dim);
int  sp_knight_mask_init(sp_knight_mask_t *m, int pad_dim, int sk_k, const float *variance);
void sp_knight_mask_free(sp_knight_mask_t *m);

#ifdef __cplusplus
}
#endif
#endif
