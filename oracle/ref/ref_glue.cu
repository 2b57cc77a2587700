/*
 * ref_glue.cu -- TEST INFRASTRUCTURE: host-buffer entry points into the
 * reference's own CUDA code, compiled unmodified from the reference checkout
 * into oracle/_ref/libsp_ref_cuda.so by oracle/ref/Makefile.
 *
 * Nothing in the shipped library links or loads this.  It exists so the
 * tests can pin the CPU oracle and the B200 kernels to outputs that the
 * reference's code computed:
 *
 *   ship path   src/backends/cuda/shannon_prime_cuda.cu
 *               sp_cuda_vht2_forward (:303-327), sp_cuda_mobius_(un)reorder
 *               (:329-350), sp_cuda_band_(de)quantize (:352-401),
 *               sp_cuda_cache_init + sp_cuda_write_{k,v}_batch +
 *               sp_cuda_read_{k,v}_batch (:407-462, :565-657)
 *   sqfree      src/backends/cuda/shannon_prime_sqfree.cu
 *               sp_cuda_vilenkin_inplace (:282-290), sp_cuda_mobius_predict,
 *               sp_cuda_spinor_extract (:300-345), kernel_mean_abs,
 *               kernel_quantize_residual, kernel_dequantize_residual,
 *               kernel_pack_levels (:490-548)
 *   hier        src/backends/cuda/shannon_prime_hier.cu
 *               kernel_hier_predict (:74-92), kernel_residual_magnitude,
 *               kernel_quantize_residual, kernel_dequantize_residual
 *               (:112-206)
 *
 * The reference kernels are launched exactly as the reference's own write
 * paths launch them (block sizes from shannon_prime_sqfree.cu:750-853 and
 * shannon_prime_hier.cu:399-489).  Every function returns 0, or the CUDA
 * error code of the first failing call.
 */
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "shannon_prime_cuda.h"   /* the reference's own header */

/* Kernels defined (with external linkage) in the reference sqfree TU. */
__global__ void kernel_mean_abs(const float *dev, int n_res, float *d_mag);
__global__ void kernel_quantize_residual(const float *dev, int n_res, int bits,
                                         const float *d_mag, uint8_t *levels);
__global__ void kernel_dequantize_residual(const uint8_t *levels, int n_res, int bits,
                                           const float *d_mag, float *dev);
__global__ void kernel_pack_levels(const uint8_t *levels, int n_res, int bits,
                                   uint8_t *packed, int packed_bytes);
/* ... and in the reference hier TU (overloads, different parameter lists). */
__global__ void kernel_hier_predict(const uint16_t *W, const float *skeleton,
                                    float *target_out, int n_target, int n_skeleton);
__global__ void kernel_residual_magnitude(const float *deviation, float *mag_out,
                                          int n_target);
__global__ void kernel_quantize_residual(const float *deviation, const float *mag,
                                         unsigned char *levels, int n_target, int nbits);
__global__ void kernel_dequantize_residual(const unsigned char *levels, const float *mag,
                                           float *output, int n_target, int nbits);

extern "C" {
void sp_cuda_vilenkin_inplace(float *d_data, int pad_dim, int n_vecs,
                              int *d_factors, int n_factors, cudaStream_t stream);
void sp_cuda_mobius_predict(const float *d_skel, float *d_pred,
                            const int *d_offsets, const int *d_slots,
                            const int *d_signs, int sk_k, int n_res, int n_vecs,
                            cudaStream_t stream);
void sp_cuda_spinor_extract(const float *d_actual, const float *d_pred,
                            float *d_deviation, uint8_t *d_sheet,
                            int n_res, int n_vecs, cudaStream_t stream);

/* Core helpers the sqfree TU references from its cache init, which the
 * checker never calls (ref_core_ext.h). */
int sp_sqfree_pad_dim(int head_dim) { (void)head_dim; return -1; }
int sp_knight_mask_init(sp_knight_mask_t *m, int pad_dim, int sk_k, const float *variance)
{
    (void)pad_dim; (void)sk_k; (void)variance;
    memset(m, 0, sizeof(*m));
    fprintf(stderr, "[ref-glue] sp_knight_mask_init is not provided by the checker\n");
    return -1;
}
void sp_knight_mask_free(sp_knight_mask_t *m) { (void)m; }
}

#define CK(x) do { cudaError_t e_ = (x); if (e_ != cudaSuccess) { rc = (int)e_; goto done; } } while (0)

template <class T> static cudaError_t up(T **d, const T *h, size_t n)
{
    cudaError_t e = cudaMalloc((void **)d, n * sizeof(T) + 16);
    if (e != cudaSuccess) return e;
    return h ? cudaMemcpy(*d, h, n * sizeof(T), cudaMemcpyHostToDevice)
             : cudaMemset(*d, 0, n * sizeof(T) + 16);
}

extern "C" {

int refg_vht2(float *h, int n, int n_vecs)
{
    int rc = 0;
    float *d = nullptr;
    CK(up(&d, h, (size_t)n * n_vecs));
    sp_cuda_vht2_forward(d, n, n_vecs, nullptr);
    CK(cudaGetLastError());
    CK(cudaMemcpy(h, d, sizeof(float) * n * n_vecs, cudaMemcpyDeviceToHost));
done:
    cudaFree(d);
    return rc;
}

int refg_mobius(float *h, const int *order, int n, int n_vecs, int inverse)
{
    int rc = 0;
    float *d = nullptr;
    int *d_o = nullptr;
    CK(up(&d, h, (size_t)n * n_vecs));
    CK(up(&d_o, order, (size_t)n));
    if (inverse) sp_cuda_mobius_unreorder(d, d_o, n, n_vecs, nullptr);
    else sp_cuda_mobius_reorder(d, d_o, n, n_vecs, nullptr);
    CK(cudaGetLastError());
    CK(cudaMemcpy(h, d, sizeof(float) * n * n_vecs, cudaMemcpyDeviceToHost));
done:
    cudaFree(d);
    cudaFree(d_o);
    return rc;
}

int refg_band_quantize(const float *h_in, int n, int n_vecs, int n_bands, const int *bits,
                       uint8_t *h_out)
{
    int rc = 0;
    sp_band_config_t bc;
    float *d_in = nullptr;
    uint8_t *d_out = nullptr;
    if (sp_band_config_init(&bc, n, n_bands, bits) != 0) return -1;
    CK(up(&d_in, h_in, (size_t)n * n_vecs));
    CK(up(&d_out, (const uint8_t *)nullptr, (size_t)bc.total_bytes * n_vecs));
    sp_cuda_band_quantize(d_in, d_out, &bc, n_vecs, nullptr);
    CK(cudaGetLastError());
    CK(cudaMemcpy(h_out, d_out, (size_t)bc.total_bytes * n_vecs, cudaMemcpyDeviceToHost));
done:
    cudaFree(d_in);
    cudaFree(d_out);
    return rc;
}

int refg_band_dequantize(const uint8_t *h_in, int n, int n_vecs, int n_bands, const int *bits,
                         float *h_out)
{
    int rc = 0;
    sp_band_config_t bc;
    uint8_t *d_in = nullptr;
    float *d_out = nullptr;
    if (sp_band_config_init(&bc, n, n_bands, bits) != 0) return -1;
    CK(up(&d_in, h_in, (size_t)bc.total_bytes * n_vecs));
    CK(up(&d_out, (const float *)nullptr, (size_t)n * n_vecs));
    sp_cuda_band_dequantize(d_in, d_out, &bc, n_vecs, nullptr);
    CK(cudaGetLastError());
    CK(cudaMemcpy(h_out, d_out, sizeof(float) * n * n_vecs, cudaMemcpyDeviceToHost));
done:
    cudaFree(d_in);
    cudaFree(d_out);
    return rc;
}

/* One (layer 0, head 0) slot of n_pos positions through the reference's own
 * cache: sp_cuda_cache_init, then the batch write (or, for read, the packed
 * rows uploaded into the slab and the batch read).  K and V are separate
 * calls so either half can be checked alone. */
static int ship_cache(sp_cuda_cache_t *cc, int n, int n_pos, int n_bands_k, const int *k_bits,
                      int n_bands_v, const int *v_bits, int mobius)
{
    sp_config_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.head_dim = n;
    cfg.n_layers = 1;
    cfg.n_heads_kv = 1;
    cfg.k_n_bands = n_bands_k;
    cfg.v_n_bands = n_bands_v;
    for (int b = 0; b < n_bands_k; b++) cfg.k_band_bits[b] = k_bits[b];
    for (int b = 0; b < n_bands_v; b++) cfg.v_band_bits[b] = v_bits[b];
    cfg.use_mobius_mask = mobius;
    memset(cc, 0, sizeof(*cc));
    return sp_cuda_cache_init(cc, &cfg, n_pos, nullptr);
}

int refg_ship_write(int is_v, const float *h_in, int n, int n_pos, int n_bands_k,
                    const int *k_bits, int n_bands_v, const int *v_bits, int mobius,
                    uint8_t *h_out)
{
    int rc = 0;
    sp_cuda_cache_t cc;
    float *d_in = nullptr;
    if (ship_cache(&cc, n, n_pos, n_bands_k, k_bits, n_bands_v, v_bits, mobius) != 0) return -1;
    CK(up(&d_in, h_in, (size_t)n * n_pos));
    if (is_v) sp_cuda_write_v_batch(&cc, 0, 0, 0, n_pos, d_in);
    else sp_cuda_write_k_batch(&cc, 0, 0, 0, n_pos, d_in);
    CK(cudaGetLastError());
    CK(cudaDeviceSynchronize());
    {
        int tb = is_v ? cc.v_bands.total_bytes : cc.k_bands.total_bytes;
        CK(cudaMemcpy(h_out, is_v ? cc.d_v_cache : cc.d_k_cache, (size_t)tb * n_pos,
                      cudaMemcpyDeviceToHost));
    }
done:
    cudaFree(d_in);
    sp_cuda_cache_free(&cc);
    return rc;
}

int refg_ship_read(int is_v, const uint8_t *h_in, int n, int n_pos, int n_bands_k,
                   const int *k_bits, int n_bands_v, const int *v_bits, int mobius,
                   float *h_out)
{
    int rc = 0;
    sp_cuda_cache_t cc;
    float *d_out = nullptr;
    if (ship_cache(&cc, n, n_pos, n_bands_k, k_bits, n_bands_v, v_bits, mobius) != 0) return -1;
    {
        int tb = is_v ? cc.v_bands.total_bytes : cc.k_bands.total_bytes;
        CK(cudaMemcpy(is_v ? cc.d_v_cache : cc.d_k_cache, h_in, (size_t)tb * n_pos,
                      cudaMemcpyHostToDevice));
    }
    CK(up(&d_out, (const float *)nullptr, (size_t)n * n_pos));
    if (is_v) sp_cuda_read_v_batch(&cc, 0, 0, 0, n_pos, d_out);
    else sp_cuda_read_k_batch(&cc, 0, 0, 0, n_pos, d_out);
    CK(cudaGetLastError());
    CK(cudaMemcpy(h_out, d_out, sizeof(float) * n * n_pos, cudaMemcpyDeviceToHost));
done:
    cudaFree(d_out);
    sp_cuda_cache_free(&cc);
    return rc;
}

int refg_vilenkin(float *h, int pd, int n_vecs)
{
    int rc = 0, nf = 0, f[16], r = pd;
    static const int primes[5] = {2, 3, 5, 7, 11};   /* factor order of shannon_prime_sqfree.cu:662-671 */
    float *d = nullptr;
    int *d_f = nullptr;
    for (int p = 0; p < 5; p++)
        while (r % primes[p] == 0) { f[nf++] = primes[p]; r /= primes[p]; }
    if (r != 1) return -1;
    CK(up(&d, h, (size_t)pd * n_vecs));
    CK(up(&d_f, f, (size_t)nf));
    sp_cuda_vilenkin_inplace(d, pd, n_vecs, d_f, nf, nullptr);
    CK(cudaGetLastError());
    CK(cudaMemcpy(h, d, sizeof(float) * pd * n_vecs, cudaMemcpyDeviceToHost));
done:
    cudaFree(d);
    cudaFree(d_f);
    return rc;
}

int refg_sq_predict(const float *h_skel, int n_vecs, int sk_k, int n_res, const int *off,
                    const int *slot, const int *sign, float *h_pred)
{
    int rc = 0;
    float *d_s = nullptr, *d_p = nullptr;
    int *d_off = nullptr, *d_slot = nullptr, *d_sign = nullptr;
    int nt = off[n_res];
    CK(up(&d_s, h_skel, (size_t)sk_k * n_vecs));
    CK(up(&d_p, (const float *)nullptr, (size_t)n_res * n_vecs));
    CK(up(&d_off, off, (size_t)n_res + 1));
    CK(up(&d_slot, slot, (size_t)(nt > 0 ? nt : 1)));
    CK(up(&d_sign, sign, (size_t)(nt > 0 ? nt : 1)));
    sp_cuda_mobius_predict(d_s, d_p, d_off, d_slot, d_sign, sk_k, n_res, n_vecs, nullptr);
    CK(cudaGetLastError());
    CK(cudaMemcpy(h_pred, d_p, sizeof(float) * n_res * n_vecs, cudaMemcpyDeviceToHost));
done:
    cudaFree(d_s); cudaFree(d_p); cudaFree(d_off); cudaFree(d_slot); cudaFree(d_sign);
    return rc;
}

int refg_sq_spinor(const float *h_actual, const float *h_pred, int n_vecs, int n_res,
                   float *h_dev, uint8_t *h_sheet)
{
    int rc = 0;
    int sb = (n_res + 7) / 8;
    float *d_a = nullptr, *d_p = nullptr, *d_d = nullptr;
    uint8_t *d_sh = nullptr;
    CK(up(&d_a, h_actual, (size_t)n_res * n_vecs));
    CK(up(&d_p, h_pred, (size_t)n_res * n_vecs));
    CK(up(&d_d, (const float *)nullptr, (size_t)n_res * n_vecs));
    CK(up(&d_sh, (const uint8_t *)nullptr, (size_t)sb * n_vecs));
    sp_cuda_spinor_extract(d_a, d_p, d_d, d_sh, n_res, n_vecs, nullptr);
    CK(cudaGetLastError());
    CK(cudaMemcpy(h_dev, d_d, sizeof(float) * n_res * n_vecs, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(h_sheet, d_sh, (size_t)sb * n_vecs, cudaMemcpyDeviceToHost));
done:
    cudaFree(d_a); cudaFree(d_p); cudaFree(d_d); cudaFree(d_sh);
    return rc;
}

/* The sqfree residual stage of one write, per vector: mag = kernel_mean_abs
 * (one 256-thread block), then levels, then LSB-first packing
 * (shannon_prime_sqfree.cu:820-842).  Also returns the magnitude. */
int refg_sq_residual(const float *h_dev, int n_vecs, int n_res, int bits, float *h_mag,
                     uint8_t *h_levels, uint8_t *h_packed)
{
    int rc = 0;
    int rb = (n_res * bits + 7) / 8;
    float *d_dev = nullptr, *d_mag = nullptr;
    uint8_t *d_lv = nullptr, *d_pk = nullptr;
    CK(up(&d_dev, h_dev, (size_t)n_res * n_vecs));
    CK(up(&d_mag, (const float *)nullptr, (size_t)n_vecs));
    CK(up(&d_lv, (const uint8_t *)nullptr, (size_t)n_res * n_vecs));
    CK(up(&d_pk, (const uint8_t *)nullptr, (size_t)rb * n_vecs));
    for (int v = 0; v < n_vecs; v++) {
        const float *dv = d_dev + (size_t)v * n_res;
        kernel_mean_abs<<<1, 256>>>(dv, n_res, d_mag + v);
        kernel_quantize_residual<<<(n_res + 127) / 128, 128>>>(dv, n_res, bits, d_mag + v,
                                                               d_lv + (size_t)v * n_res);
        kernel_pack_levels<<<1, 1>>>(d_lv + (size_t)v * n_res, n_res, bits,
                                     d_pk + (size_t)v * rb, rb);
    }
    CK(cudaGetLastError());
    CK(cudaMemcpy(h_mag, d_mag, sizeof(float) * n_vecs, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(h_levels, d_lv, (size_t)n_res * n_vecs, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(h_packed, d_pk, (size_t)rb * n_vecs, cudaMemcpyDeviceToHost));
done:
    cudaFree(d_dev); cudaFree(d_mag); cudaFree(d_lv); cudaFree(d_pk);
    return rc;
}

/* Levels -> deviations with a given per-vector magnitude (sqfree form). */
int refg_sq_dequant(const uint8_t *h_levels, const float *h_mag, int n_vecs, int n_res,
                    int bits, float *h_dev)
{
    int rc = 0;
    float *d_dev = nullptr, *d_mag = nullptr;
    uint8_t *d_lv = nullptr;
    CK(up(&d_lv, h_levels, (size_t)n_res * n_vecs));
    CK(up(&d_mag, h_mag, (size_t)n_vecs));
    CK(up(&d_dev, (const float *)nullptr, (size_t)n_res * n_vecs));
    for (int v = 0; v < n_vecs; v++)
        kernel_dequantize_residual<<<(n_res + 127) / 128, 128>>>(
            d_lv + (size_t)v * n_res, n_res, bits, d_mag + v, d_dev + (size_t)v * n_res);
    CK(cudaGetLastError());
    CK(cudaMemcpy(h_dev, d_dev, sizeof(float) * n_res * n_vecs, cudaMemcpyDeviceToHost));
done:
    cudaFree(d_dev); cudaFree(d_mag); cudaFree(d_lv);
    return rc;
}

/* The hier target stage of one write, per vector: pred = W·skeleton
 * (kernel_hier_predict), then the caller's dev, then magnitude and levels
 * (shannon_prime_hier.cu:435-482).  W is [n_target][n_skel] fp16 bits. */
int refg_hier_predict(const uint16_t *h_W, const float *h_skel, int n_vecs, int n_target,
                      int n_skel, float *h_pred)
{
    int rc = 0;
    uint16_t *d_W = nullptr;
    float *d_s = nullptr, *d_p = nullptr;
    CK(up(&d_W, h_W, (size_t)n_target * n_skel));
    CK(up(&d_s, h_skel, (size_t)n_skel * n_vecs));
    CK(up(&d_p, (const float *)nullptr, (size_t)n_target * n_vecs));
    for (int v = 0; v < n_vecs; v++)
        kernel_hier_predict<<<(n_target + 127) / 128, 128>>>(
            d_W, d_s + (size_t)v * n_skel, d_p + (size_t)v * n_target, n_target, n_skel);
    CK(cudaGetLastError());
    CK(cudaMemcpy(h_pred, d_p, sizeof(float) * n_target * n_vecs, cudaMemcpyDeviceToHost));
done:
    cudaFree(d_W); cudaFree(d_s); cudaFree(d_p);
    return rc;
}

int refg_hier_residual(const float *h_dev, int n_vecs, int n_target, int bits, float *h_mag,
                       uint8_t *h_levels)
{
    int rc = 0;
    float *d_dev = nullptr, *d_mag = nullptr;
    uint8_t *d_lv = nullptr;
    CK(up(&d_dev, h_dev, (size_t)n_target * n_vecs));
    CK(up(&d_mag, (const float *)nullptr, (size_t)n_vecs));
    CK(up(&d_lv, (const uint8_t *)nullptr, (size_t)n_target * n_vecs));
    for (int v = 0; v < n_vecs; v++) {
        const float *dv = d_dev + (size_t)v * n_target;
        kernel_residual_magnitude<<<1, 256, 256 * sizeof(float)>>>(dv, d_mag + v, n_target);
        kernel_quantize_residual<<<(n_target + 127) / 128, 128>>>(
            dv, d_mag + v, d_lv + (size_t)v * n_target, n_target, bits);
    }
    CK(cudaGetLastError());
    CK(cudaMemcpy(h_mag, d_mag, sizeof(float) * n_vecs, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(h_levels, d_lv, (size_t)n_target * n_vecs, cudaMemcpyDeviceToHost));
done:
    cudaFree(d_dev); cudaFree(d_mag); cudaFree(d_lv);
    return rc;
}

int refg_hier_dequant(const uint8_t *h_levels, const float *h_mag, int n_vecs, int n_target,
                      int bits, float *h_dev)
{
    int rc = 0;
    float *d_dev = nullptr, *d_mag = nullptr;
    uint8_t *d_lv = nullptr;
    CK(up(&d_lv, h_levels, (size_t)n_target * n_vecs));
    CK(up(&d_mag, h_mag, (size_t)n_vecs));
    CK(up(&d_dev, (const float *)nullptr, (size_t)n_target * n_vecs));
    for (int v = 0; v < n_vecs; v++)
        kernel_dequantize_residual<<<(n_target + 127) / 128, 128>>>(
            d_lv + (size_t)v * n_target, d_mag + v, d_dev + (size_t)v * n_target, n_target, bits);
    CK(cudaGetLastError());
    CK(cudaMemcpy(h_dev, d_dev, sizeof(float) * n_target * n_vecs, cudaMemcpyDeviceToHost));
done:
    cudaFree(d_dev); cudaFree(d_mag); cudaFree(d_lv);
    return rc;
}

}  /* extern "C" */
