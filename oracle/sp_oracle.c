/*
 * sp_oracle.c — CPU restatement of the Shannon-Prime ship path (test
 * infrastructure; see sp_oracle.h for what pins it and what does not).
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -fopenmp).  FMA
 * contraction must stay off: every float operation below is one IEEE
 * single-precision operation, in the order the reference performs it, so
 * the packed codes can be compared bit for bit with the CUDA kernels.
 */
#include "sp_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- fp16 -- */

/* IEEE binary32 -> binary16, round to nearest even (the rounding of CUDA's
 * __float2half used at shannon_prime_cuda.cu:171). */
uint16_t or_f32_to_f16(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7fffffffu;
    if (ax > 0x7f800000u) return sign | 0x7e00u;          /* NaN */
    if (ax >= 0x477ff000u) return sign | 0x7c00u;         /* >= 65520 -> inf */
    if (ax < 0x38800000u) {                               /* below 2^-14: subnormal */
        float a;
        memcpy(&a, &ax, 4);
        double r = rint((double)a * 16777216.0);          /* exact scale, RNE */
        return sign | (uint16_t)r;                        /* 1024 -> smallest normal */
    }
    uint32_t e = (ax >> 23) - 127 + 15;
    uint32_t m = ax & 0x7fffffu;
    uint32_t h = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return sign | (uint16_t)h;
}

float or_f16_to_f32(uint16_t h)
{
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {                                          /* subnormal: normalise */
            int sh = 0;
            while (!(m & 0x400u)) { m <<= 1; sh++; }
            m &= 0x3ffu;
            x = sign | ((uint32_t)(127 - 15 + 1 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 127 - 15) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* ------------------------------------------------------- band layout -- */

/* Band spans as sp_band_span (shannon_prime_vulkan.c:563-576, cuda.cu:149-151):
 * band_size = n / n_bands, the last band absorbs the remainder. */
int or_band_config(or_bands_t *bc, int n, int n_bands, const int *bits)
{
    if (!bc || n <= 0 || n_bands < 1 || n_bands > OR_MAX_BANDS || n_bands > n)
        return -1;
    memset(bc, 0, sizeof(*bc));
    bc->n = n;
    bc->n_bands = n_bands;
    int bs = n / n_bands;
    int byte = 0;
    for (int b = 0; b < n_bands; b++) {
        if (bits[b] < 1 || bits[b] > 8) return -1;
        bc->bits[b] = bits[b];
        bc->off[b] = b * bs;
        bc->size[b] = (b == n_bands - 1) ? (n - b * bs) : bs;
        bc->byte_off[b] = byte;
        byte += 2 + (bc->size[b] * bits[b] + 7) / 8;
    }
    bc->total_bytes = byte;
    return 0;
}

/* ----------------------------------------------------------------- VHT2 -- */

/* p=2 Vilenkin-Hartley transform as the NEON restatement
 * (shannon_prime_adreno.c:270-309): unnormalised butterfly with pairs
 * (i+j, i+j+len) for len = 1, 2, 4, ..., then one multiply by 1.0f/sqrtf(n).
 * Orthonormal and self-inverse. n must be a power of two. */
void or_vht2(float *x, int n)
{
    for (int len = 1; len < n; len <<= 1) {
        for (int i = 0; i < n; i += len << 1) {
            for (int j = 0; j < len; j++) {
                float u = x[i + j];
                float v = x[i + j + len];
                x[i + j] = u + v;
                x[i + j + len] = u - v;
            }
        }
    }
    const float s = 1.0f / sqrtf((float)n);
    for (int i = 0; i < n; i++) x[i] *= s;
}

/* ---------------------------------------------------------- Möbius -- */

static int or_squarefree(int m)
{
    for (int p = 2; p * p <= m; p++)
        if (m % (p * p) == 0) return 0;
    return 1;
}

/* Squarefree-first order (the reference describes the permutation at
 * shannon_prime_cuda.cu:79-83; the table itself comes from the absent core
 * sp_mobius_mask_init): slots 0.. hold the indices i whose 1-based index
 * i+1 is squarefree, ascending, then the remaining indices ascending. */
void or_mobius_order(int n, int *order)
{
    int k = 0;
    for (int i = 0; i < n; i++)
        if (or_squarefree(i + 1)) order[k++] = i;
    for (int i = 0; i < n; i++)
        if (!or_squarefree(i + 1)) order[k++] = i;
}

/* ------------------------------------------------------ quantisation -- */

/* Band quantiser, step for step as kernel_band_quantize_simple
 * (shannon_prime_cuda.cu:131-204). */
void or_band_quantize(const float *x, uint8_t *out, const or_bands_t *bc)
{
    for (int b = 0; b < bc->n_bands; b++) {
        const float *band = x + bc->off[b];
        const int sz = bc->size[b];
        const int bits = bc->bits[b];
        const int max_val = (1 << (bits - 1)) - 1;
        uint8_t *o = out + bc->byte_off[b];

        float amax = 0.0f;
        for (int i = 0; i < sz; i++) {
            float a = fabsf(band[i]);
            if (a > amax) amax = a;
        }
        /* max_val is 0 for 1-bit bands: scale is then inf or nan and every
         * code is the offset 0, exactly as the reference kernel behaves. */
        float scale = (amax > 0.0f) ? amax / (float)max_val : 0.0f;
        uint16_t sh = or_f32_to_f16(scale);
        o[0] = (uint8_t)(sh & 0xff);
        o[1] = (uint8_t)(sh >> 8);
        float stored = or_f16_to_f32(sh);
        float inv = (stored > 0.0f) ? 1.0f / stored : 0.0f;

        uint64_t acc = 0;
        int nb = 0, ob = 2;
        for (int i = 0; i < sz; i++) {
            float p = band[i] * inv;
            int q;
            if (p != p) {
                q = 0;                         /* cvt.rni of NaN is 0 */
            } else {
                float r = rintf(p);            /* round half to even */
                if (r > (float)max_val) q = max_val;
                else if (r < (float)-max_val) q = -max_val;
                else q = (int)r;
            }
            uint32_t u = (uint32_t)(q + max_val);
            acc |= (uint64_t)u << nb;
            nb += bits;
            while (nb >= 8) {
                o[ob++] = (uint8_t)(acc & 0xff);
                acc >>= 8;
                nb -= 8;
            }
        }
        if (nb > 0) o[ob++] = (uint8_t)(acc & 0xff);
    }
}

/* Dequantiser as kernel_band_dequantize_simple (shannon_prime_cuda.cu:210-270)
 * with the partial-read rule of sp_llama_read_k_partial
 * (shannon_prime_llama.h:240-255): bands >= max_bands are zero when
 * 0 <= max_bands < n_bands. */
void or_band_dequantize(const uint8_t *in, float *x, const or_bands_t *bc,
                        int max_bands)
{
    int nb_use = (max_bands < 0 || max_bands >= bc->n_bands) ? bc->n_bands : max_bands;
    for (int b = 0; b < bc->n_bands; b++) {
        float *band = x + bc->off[b];
        const int sz = bc->size[b];
        if (b >= nb_use) {
            for (int i = 0; i < sz; i++) band[i] = 0.0f;
            continue;
        }
        const int bits = bc->bits[b];
        const int max_val = (1 << (bits - 1)) - 1;
        const uint32_t mask = (1u << bits) - 1u;
        const uint8_t *p = in + bc->byte_off[b];
        float scale = or_f16_to_f32((uint16_t)(p[0] | (p[1] << 8)));
        if (!isfinite(scale)) scale = 0.0f;
        uint64_t acc = 0;
        int nbits = 0, ib = 2;
        for (int i = 0; i < sz; i++) {
            while (nbits < bits) {
                acc |= (uint64_t)p[ib++] << nbits;
                nbits += 8;
            }
            uint32_t u = (uint32_t)(acc & mask);
            acc >>= bits;
            nbits -= bits;
            band[i] = (float)((int)u - max_val) * scale;
        }
    }
}

/* ------------------------------------------------------ ship path -- */

/* Write: VHT2 -> Möbius reorder (K only) -> band quantise, the order of
 * sp_adreno_write_k (shannon_prime_adreno.c:696-716) and sp_cuda_write_k
 * (shannon_prime_cuda.cu:474-500). order == NULL skips the reorder (V). */
void or_ship_write(const float *vec, uint8_t *out, const or_bands_t *bc,
                   const int *order)
{
    float t[1024], r[1024];
    const int n = bc->n;
    memcpy(t, vec, sizeof(float) * (size_t)n);
    or_vht2(t, n);
    if (order) {
        for (int i = 0; i < n; i++) r[i] = t[order[i]];
        or_band_quantize(r, out, bc);
    } else {
        or_band_quantize(t, out, bc);
    }
}

/* Read: dequantise -> Möbius unreorder (out[order[i]] = in[i]) -> VHT2,
 * as sp_adreno_read_k (shannon_prime_adreno.c:790-806). */
void or_ship_read(const uint8_t *in, float *vec, const or_bands_t *bc,
                  const int *order, int max_bands)
{
    float c[1024];
    const int n = bc->n;
    or_band_dequantize(in, c, bc, max_bands);
    if (order) {
        for (int i = 0; i < n; i++) vec[order[i]] = c[i];
    } else {
        memcpy(vec, c, sizeof(float) * (size_t)n);
    }
    or_vht2(vec, n);
}

void or_ship_write_batch(int n_vecs, const float *vecs, size_t vec_stride,
                         uint8_t *out, const or_bands_t *bc, const int *order,
                         int n_threads)
{
#ifdef _OPENMP
    if (n_threads < 1) n_threads = 1;
#pragma omp parallel for num_threads(n_threads) schedule(static)
#endif
    for (int i = 0; i < n_vecs; i++)
        or_ship_write(vecs + (size_t)i * vec_stride,
                      out + (size_t)i * (size_t)bc->total_bytes, bc, order);
}

void or_ship_read_batch(int n_vecs, const uint8_t *in, float *vecs,
                        const or_bands_t *bc, const int *order, int max_bands,
                        int n_threads)
{
#ifdef _OPENMP
    if (n_threads < 1) n_threads = 1;
#pragma omp parallel for num_threads(n_threads) schedule(static)
#endif
    for (int i = 0; i < n_vecs; i++)
        or_ship_read(in + (size_t)i * (size_t)bc->total_bytes,
                     vecs + (size_t)i * (size_t)bc->n, bc, order, max_bands);
}

/* ------------------------------------------------------- attention -- */

/* One (KV head, token chunk) task: scores of every query of the group over
 * tokens [t0, t1), the chunk's max per query, and exp-weighted sums relative
 * to that max (double). */
typedef struct {
    double mx[8];
    double den[8];
    double *acc;               /* [group][n] */
} or_attn_part_t;

static void or_attn_chunk(const uint8_t *ks, const uint8_t *vs, const or_bands_t *kb,
                          const or_bands_t *vb, const int *order, const double (*qd)[1024],
                          int group, int t0, int t1, float logit_scale, or_attn_part_t *pt)
{
    const int n = kb->n;
    float kr[1024], vr[1024];
    double *score = (double *)malloc(sizeof(double) * (size_t)(t1 - t0) * (size_t)group);
    for (int g = 0; g < group; g++) { pt->mx[g] = -INFINITY; pt->den[g] = 0.0; }
    for (int t = t0; t < t1; t++) {
        or_ship_read(ks + (size_t)t * kb->total_bytes, kr, kb, order, -1);
        for (int g = 0; g < group; g++) {
            double sc = 0.0;
            for (int d = 0; d < n; d++) sc += (double)kr[d] * qd[g][d];
            sc *= (double)logit_scale;
            score[(size_t)(t - t0) * group + g] = sc;
            if (sc > pt->mx[g]) pt->mx[g] = sc;
        }
    }
    for (int t = t0; t < t1; t++) {
        or_ship_read(vs + (size_t)t * vb->total_bytes, vr, vb, NULL, -1);
        for (int g = 0; g < group; g++) {
            double pr = exp(score[(size_t)(t - t0) * group + g] - pt->mx[g]);
            pt->den[g] += pr;
            double *a = pt->acc + (size_t)g * n;
            for (int d = 0; d < n; d++) a[d] += pr * (double)vr[d];
        }
    }
    free(score);
}

void or_attn_decode(const uint8_t *k_slots, size_t slot_stride_k,
                    const uint8_t *v_slots, size_t slot_stride_v,
                    const or_bands_t *kb, const or_bands_t *vb,
                    const int *order, int n_kv_heads, int n_q_heads,
                    int kv_len, const uint16_t *q, float logit_scale,
                    float *out, int n_threads)
{
    const int n = kb->n;
    const int group = n_q_heads / n_kv_heads;
    if (n_threads < 1) n_threads = 1;
    /* Token chunks per head: enough tasks for every thread (the result is
     * the same softmax, merged with log-sum-exp weights in double). */
    int chunks = (2 * n_threads + n_kv_heads - 1) / n_kv_heads;
    if (chunks > kv_len) chunks = kv_len > 0 ? kv_len : 1;
    const int n_tasks = n_kv_heads * chunks;
    or_attn_part_t *parts = (or_attn_part_t *)calloc((size_t)n_tasks, sizeof(or_attn_part_t));
    double *accs = (double *)calloc((size_t)n_tasks * (size_t)group * (size_t)n, sizeof(double));
#ifdef _OPENMP
#pragma omp parallel for num_threads(n_threads) schedule(dynamic)
#endif
    for (int task = 0; task < n_tasks; task++) {
        const int h = task / chunks, c = task % chunks;
        const int t0 = (int)((long long)kv_len * c / chunks), t1 = (int)((long long)kv_len * (c + 1) / chunks);
        double qd[8][1024];
        for (int g = 0; g < group && g < 8; g++)
            for (int d = 0; d < n; d++)
                qd[g][d] = (double)or_f16_to_f32(q[(size_t)(h * group + g) * n + d]);
        parts[task].acc = accs + (size_t)task * group * n;
        or_attn_chunk(k_slots + (size_t)h * slot_stride_k, v_slots + (size_t)h * slot_stride_v, kb, vb,
                      order, (const double (*)[1024])qd, group, t0, t1, logit_scale, &parts[task]);
    }
    for (int h = 0; h < n_kv_heads; h++) {
        for (int g = 0; g < group; g++) {
            double M = -INFINITY;
            for (int c = 0; c < chunks; c++) if (parts[h * chunks + c].mx[g] > M) M = parts[h * chunks + c].mx[g];
            double den = 0.0;
            double *o = (double *)calloc((size_t)n, sizeof(double));
            for (int c = 0; c < chunks; c++) {
                const or_attn_part_t *pt = &parts[h * chunks + c];
                if (pt->mx[g] == -INFINITY) continue;
                const double w = exp(pt->mx[g] - M);
                den += w * pt->den[g];
                for (int d = 0; d < n; d++) o[d] += w * pt->acc[(size_t)g * n + d];
            }
            for (int d = 0; d < n; d++)
                out[(size_t)(h * group + g) * n + d] = den > 0.0 ? (float)(o[d] / den) : 0.0f;
            free(o);
        }
    }
    free(accs);
    free(parts);
}

double or_correlation(const float *a, const float *b, int n)
{
    double ma = 0, mb = 0;
    for (int i = 0; i < n; i++) { ma += a[i]; mb += b[i]; }
    ma /= n; mb /= n;
    double sab = 0, saa = 0, sbb = 0;
    for (int i = 0; i < n; i++) {
        double x = a[i] - ma, y = b[i] - mb;
        sab += x * y; saa += x * x; sbb += y * y;
    }
    if (saa <= 0 || sbb <= 0) return 0.0;
    return sab / sqrt(saa * sbb);
}
