/*
 * sp_oracle_sqfree.c — CPU restatement of the sqfree+spinor and the
 * hierarchical-Vilenkin paths (test infrastructure; see sp_oracle.h).
 *
 * The reference keeps the definitions of these paths in its core library
 * (core/shannon_prime_sqfree.c), an empty submodule in the reference
 * checkout, so what is restated here follows the reference's CUDA
 * restatements operation by operation and fixes the points they leave
 * open (every choice is a data table or a named reduction order, so the
 * GPU kernels can reproduce it bit for bit):
 *
 *   pad_dim      smallest squarefree {2,3,5,7,11}-smooth number >= head_dim
 *                (66, 154, 330 at 64, 128, 256: patches/README.md:105);
 *   pad fill     the mean of the head_dim inputs (the reference kernel's
 *                sum reduces only warp 0, shannon_prime_sqfree.cu:132-144;
 *                the true mean is used), summed in the "lane tree" order
 *                below;
 *   Vilenkin     stages per prime factor, ascending, stride ascending
 *                (shannon_prime_sqfree.cu:66-106); each output
 *                acc = fma(cas[k][j], x[j], acc) over j ascending, then
 *                acc * (float)(1/sqrt(p)); cas[k][j] = (float)(cos + sin of
 *                2 pi kj / p) computed in double (the reference kernel uses
 *                __cosf/__sinf, which are not reproducible on a CPU);
 *   Knight mask  ranking = indices i whose i+1 is squarefree ascending, then
 *                the rest ascending; skeleton = the first sk_k of the
 *                ranking (in ranking order), residual = the rest ascending;
 *                CSR predictor of residual i (n = i+1): every proper divisor
 *                d of n whose index d-1 is a skeleton slot, d ascending,
 *                sign mu(n/d), terms with mu = 0 dropped;
 *   predict      pred = pred +/- skel[slot], CSR order, fp32
 *                (kernel_mobius_predict, shannon_prime_sqfree.cu:179-203);
 *   spinor       dev = |a+p| < |a-p| ? a+p : a-p, sheet bit set for a+p
 *                (shannon_prime_sqfree.cu:212-240);
 *   sqfree quant mag = max(sum|dev| / n_res, 1e-12); sat = mag*bits;
 *                step = 2*sat/(L-1); level = (int)(fma(dev, 1/step, c) + 0.5)
 *                clamped to [0, L-1], c = (L-1)/2
 *                (shannon_prime_sqfree.cu:493-548);
 *   hier quant   step = 2*mag/(L-1); level = rint(fma(dev, 1/step, c))
 *                clamped (shannon_prime_hier.cu:148-196);
 *   hier predict pred[t] = fma(W[t][s] (fp16), skel[s], acc), s ascending
 *                (kernel_hier_predict, shannon_prime_hier.cu:74-92);
 *   slot layouts [skeleton bands][fp32 mag][levels LSB-first][sheet bits]
 *                (shannon_prime_sqfree.cu:683-686, shannon_prime_hier.cu:
 *                331-335).
 *
 * Lane-tree sum of v[0..n): s_l = v[l] + v[l+32] + ... (sequential, l < 32),
 * then for off = 16, 8, 4, 2, 1: s_l = s_l + s_(l ^ off); the result is s_0.
 */
#include "sp_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

float or_lane_tree_sum(const float *v, int n)
{
    float s[32];
    for (int l = 0; l < 32; l++) {
        float a = 0.0f;
        for (int i = l; i < n; i += 32) a = a + v[i];
        s[l] = a;
    }
    for (int off = 16; off >= 1; off >>= 1) {
        float t[32];
        for (int l = 0; l < 32; l++) t[l] = s[l] + s[l ^ off];
        memcpy(s, t, sizeof(s));
    }
    return s[0];
}

static int or_is_squarefree(int m)
{
    for (int p = 2; p * p <= m; p++)
        if (m % (p * p) == 0) return 0;
    return 1;
}

static int or_mu(int m)
{
    int k = 0;
    for (int p = 2; p * p <= m; p++) {
        if (m % p == 0) {
            m /= p;
            if (m % p == 0) return 0;
            k++;
        }
    }
    if (m > 1) k++;
    return (k & 1) ? -1 : 1;
}

int or_sqfree_pad_dim(int hd)
{
    for (int m = hd > 1 ? hd : 2;; m++) {
        if (!or_is_squarefree(m)) continue;
        int r = m;
        const int pr[5] = {2, 3, 5, 7, 11};
        for (int i = 0; i < 5; i++)
            if (r % pr[i] == 0) r /= pr[i];
        if (r == 1) return m;
    }
}

int or_vilenkin_factors(int pd, int *factors)
{
    int nf = 0, r = pd;
    const int pr[5] = {2, 3, 5, 7, 11};
    for (int i = 0; i < 5; i++)
        while (r % pr[i] == 0) { factors[nf++] = pr[i]; r /= pr[i]; }
    return r == 1 ? nf : -1;
}

void or_cas_table(int p, float *cas /* [p*p] */, float *inv_sqrt_p)
{
    for (int k = 0; k < p; k++)
        for (int j = 0; j < p; j++) {
            const double a = 2.0 * 3.14159265358979323846 * (double)((k * j) % p) / (double)p;
            cas[k * p + j] = (float)(cos(a) + sin(a));
        }
    *inv_sqrt_p = (float)(1.0 / sqrt((double)p));
}

void or_vilenkin(float *x, int pd)
{
    int f[16];
    const int nf = or_vilenkin_factors(pd, f);
    int stride = 1;
    for (int s = 0; s < nf; s++) {
        const int p = f[s];
        float cas[121], isp, g[11];
        or_cas_table(p, cas, &isp);
        const int bs = stride * p;
        for (int blk = 0; blk < pd / bs; blk++)
            for (int o = 0; o < stride; o++) {
                const int base = blk * bs + o;
                for (int j = 0; j < p; j++) g[j] = x[base + j * stride];
                for (int k = 0; k < p; k++) {
                    float acc = 0.0f;
                    for (int j = 0; j < p; j++) acc = fmaf(cas[k * p + j], g[j], acc);
                    x[base + k * stride] = acc * isp;
                }
            }
        stride *= p;
    }
}

int or_sqfree_layout(or_sqfree_t *L, int hd, int sk_k, int n_bands, const int *bits,
                     int residual_bits, int use_spinor)
{
    memset(L, 0, sizeof(*L));
    L->hd = hd;
    L->pd = or_sqfree_pad_dim(hd);
    if (L->pd > OR_SQ_MAX_PD) return -1;
    if (sk_k < 1 || sk_k > L->pd) return -1;
    L->sk_k = sk_k;
    L->n_res = L->pd - sk_k;
    L->res_bits = residual_bits;
    L->use_spinor = use_spinor;
    /* ranking: squarefree (1-based) first */
    int rank[OR_SQ_MAX_PD], nr = 0;
    for (int i = 0; i < L->pd; i++) if (or_is_squarefree(i + 1)) rank[nr++] = i;
    for (int i = 0; i < L->pd; i++) if (!or_is_squarefree(i + 1)) rank[nr++] = i;
    int slot_of[OR_SQ_MAX_PD];
    for (int i = 0; i < L->pd; i++) slot_of[i] = -1;
    for (int s = 0; s < sk_k; s++) { L->skel_idx[s] = rank[s]; slot_of[rank[s]] = s; }
    int r = 0;
    for (int i = 0; i < L->pd; i++) if (slot_of[i] < 0) L->res_idx[r++] = i;
    int t = 0;
    for (r = 0; r < L->n_res; r++) {
        L->csr_off[r] = t;
        const int n = L->res_idx[r] + 1;
        for (int d = 1; d < n; d++) {
            if (n % d) continue;
            const int m = or_mu(n / d);
            if (!m || slot_of[d - 1] < 0) continue;
            if (t >= OR_SQ_MAX_TERMS) return -1;
            L->csr_slot[t] = slot_of[d - 1];
            L->csr_sign[t] = m;
            t++;
        }
    }
    L->csr_off[L->n_res] = t;
    L->n_terms = t;
    if (or_band_config(&L->bands, sk_k, n_bands, bits)) return -1;
    L->res_bytes = (L->n_res * residual_bits + 7) / 8;
    L->sheet_bytes = use_spinor ? (L->n_res + 7) / 8 : 0;
    L->bytes_per_pos = L->bands.total_bytes + 4 + L->res_bytes + L->sheet_bytes;
    return 0;
}

static void or_pack_levels(const uint8_t *lv, int n, int bits, uint8_t *out, int nbytes)
{
    memset(out, 0, (size_t)nbytes);
    for (int i = 0; i < n; i++) {
        const int b = i * bits;
        out[b >> 3] |= (uint8_t)(lv[i] << (b & 7));
        if ((b & 7) + bits > 8 && (b >> 3) + 1 < nbytes)
            out[(b >> 3) + 1] |= (uint8_t)(lv[i] >> (8 - (b & 7)));
    }
}

static void or_unpack_levels(const uint8_t *in, int n, int bits, uint8_t *lv, int nbytes)
{
    for (int i = 0; i < n; i++) {
        const int b = i * bits;
        uint32_t w = (uint32_t)in[b >> 3] >> (b & 7);
        if ((b & 7) + bits > 8 && (b >> 3) + 1 < nbytes) w |= (uint32_t)in[(b >> 3) + 1] << (8 - (b & 7));
        lv[i] = (uint8_t)(w & ((1u << bits) - 1u));
    }
}

static void or_pad(const float *vec, int hd, int pd, float *out)
{
    const float mean = or_lane_tree_sum(vec, hd) / (float)hd;
    for (int i = 0; i < pd; i++) out[i] = i < hd ? vec[i] : mean;
}

void or_sq_predict(const or_sqfree_t *L, const float *sk, float *pred)
{
    for (int r = 0; r < L->n_res; r++) {
        float p = 0.0f;
        for (int t = L->csr_off[r]; t < L->csr_off[r + 1]; t++)
            p = L->csr_sign[t] > 0 ? p + sk[L->csr_slot[t]] : p - sk[L->csr_slot[t]];
        pred[r] = p;
    }
}

/* Residual stages, exported so the tests can check each one against the
 * reference's own kernels (shannon_prime_sqfree.cu:212-240, 490-530;
 * shannon_prime_hier.cu:112-190) on identical inputs. */

/* Spinor sheet choice (shannon_prime_sqfree.cu:212-240): dev = a - p unless
 * |a + p| < |a - p|, in which case dev = a + p and the sheet bit is set.
 * sheet[] must start zeroed. */
void or_sq_spinor(const float *actual, const float *pred, int n, float *dev, uint8_t *sheet)
{
    for (int r = 0; r < n; r++) {
        const float vp = actual[r] - pred[r], vm = actual[r] + pred[r];
        const int use_minus = fabsf(vm) < fabsf(vp);
        dev[r] = use_minus ? vm : vp;
        if (use_minus) sheet[r >> 3] |= (uint8_t)(1u << (r & 7));
    }
}

/* mean |dev| with the 1e-12 floor (shannon_prime_sqfree.cu:490-508,
 * shannon_prime_hier.cu:112-140).  The sum runs in the lane-tree order of
 * the B200 kernels, which may differ from the reference's 256-thread
 * shared-memory tree in the last bit. */
float or_residual_mag(const float *dev, int n)
{
    float ad[OR_SQ_MAX_PD];
    for (int r = 0; r < n; r++) ad[r] = fabsf(dev[r]);
    float mag = or_lane_tree_sum(ad, n) / (float)n;
    return mag < 1e-12f ? 1e-12f : mag;
}

/* Sqfree levels (shannon_prime_sqfree.cu:514-532): sat = mag*bits,
 * step = 2 sat/(L-1), level = (int)(dev*(1/step) + center + 0.5) with the
 * product and sum contracted into one fma, clamped to [0, L). */
void or_sq_levels(const float *dev, int n, int bits, float mag, uint8_t *lv)
{
    const int Lv = 1 << bits;
    const float center = 0.5f * (float)(Lv - 1);
    const float sat = mag * (float)bits;
    const float step = (2.0f * sat) / (float)(Lv - 1);
    const float inv = 1.0f / step;
    for (int r = 0; r < n; r++) {
        int level = (int)(fmaf(dev[r], inv, center) + 0.5f);
        if (level < 0) level = 0;
        if (level >= Lv) level = Lv - 1;
        lv[r] = (uint8_t)level;
    }
}

/* Sqfree deviations from levels (shannon_prime_sqfree.cu:535-548). */
void or_sq_unlevels(const uint8_t *lv, int n, int bits, float mag, float *dev)
{
    const int Lv = 1 << bits;
    const float center = 0.5f * (float)(Lv - 1);
    const float sat = mag * (float)bits;
    const float step = Lv > 1 ? (2.0f * sat / (float)(Lv - 1)) : 0.0f;
    for (int r = 0; r < n; r++) dev[r] = ((float)lv[r] - center) * step;
}

/* Hier levels (shannon_prime_hier.cu:150-172): step = 2 mag/(L-1),
 * q = rint(fma(dev, 1/step, center)), clamped. */
void or_hier_levels(const float *dev, int n, int bits, float mag, uint8_t *lv)
{
    const int Lv = 1 << bits;
    const float step = 2.0f * mag / (float)(Lv - 1);
    const float center = (float)(Lv - 1) / 2.0f;
    const float inv = step > 0.0f ? 1.0f / step : 0.0f;
    for (int t = 0; t < n; t++) {
        int q = (int)rintf(fmaf(dev[t], inv, center));
        if (q < 0) q = 0;
        if (q >= Lv) q = Lv - 1;
        lv[t] = (uint8_t)q;
    }
}

/* Hier deviations from levels (shannon_prime_hier.cu:178-192). */
void or_hier_unlevels(const uint8_t *lv, int n, int bits, float mag, float *dev)
{
    const int Lv = 1 << bits;
    const float step = 2.0f * mag / (float)(Lv - 1);
    const float center = (float)(Lv - 1) / 2.0f;
    for (int t = 0; t < n; t++) dev[t] = ((float)lv[t] - center) * step;
}

void or_sqfree_write(const float *vec, uint8_t *out, const or_sqfree_t *L)
{
    float c[OR_SQ_MAX_PD], sk[OR_SQ_MAX_PD], pred[OR_SQ_MAX_PD], act[OR_SQ_MAX_PD], dev[OR_SQ_MAX_PD];
    uint8_t lv[OR_SQ_MAX_PD];
    or_pad(vec, L->hd, L->pd, c);
    or_vilenkin(c, L->pd);
    for (int s = 0; s < L->sk_k; s++) sk[s] = c[L->skel_idx[s]];
    memset(out, 0, (size_t)L->bytes_per_pos);
    or_band_quantize(sk, out, &L->bands);
    if (L->n_res == 0) return;
    or_sq_predict(L, sk, pred);
    for (int r = 0; r < L->n_res; r++) act[r] = c[L->res_idx[r]];
    if (L->use_spinor)
        or_sq_spinor(act, pred, L->n_res, dev, out + L->bands.total_bytes + 4 + L->res_bytes);
    else
        for (int r = 0; r < L->n_res; r++) dev[r] = act[r] - pred[r];
    const float mag = or_residual_mag(dev, L->n_res);
    memcpy(out + L->bands.total_bytes, &mag, 4);
    or_sq_levels(dev, L->n_res, L->res_bits, mag, lv);
    or_pack_levels(lv, L->n_res, L->res_bits, out + L->bands.total_bytes + 4, L->res_bytes);
}

/* Coefficient-domain reconstruction (before the inverse transform). */
void or_sqfree_coeffs(const uint8_t *in, float *c, const or_sqfree_t *L)
{
    float sk[OR_SQ_MAX_PD], pred[OR_SQ_MAX_PD];
    uint8_t lv[OR_SQ_MAX_PD];
    or_band_dequantize(in, sk, &L->bands, -1);
    for (int i = 0; i < L->pd; i++) c[i] = 0.0f;
    for (int s = 0; s < L->sk_k; s++) c[L->skel_idx[s]] = sk[s];
    if (L->n_res == 0) return;
    or_sq_predict(L, sk, pred);
    float mag;
    memcpy(&mag, in + L->bands.total_bytes, 4);
    or_unpack_levels(in + L->bands.total_bytes + 4, L->n_res, L->res_bits, lv, L->res_bytes);
    const uint8_t *sheet = in + L->bands.total_bytes + 4 + L->res_bytes;
    float dev[OR_SQ_MAX_PD];
    or_sq_unlevels(lv, L->n_res, L->res_bits, mag, dev);
    for (int r = 0; r < L->n_res; r++) {
        float p = pred[r];
        if (L->use_spinor && (sheet[r >> 3] >> (r & 7) & 1)) p = -p;
        c[L->res_idx[r]] = p + dev[r];
    }
}

void or_sqfree_read(const uint8_t *in, float *vec, const or_sqfree_t *L)
{
    float c[OR_SQ_MAX_PD];
    or_sqfree_coeffs(in, c, L);
    or_vilenkin(c, L->pd);
    memcpy(vec, c, sizeof(float) * (size_t)L->hd);
}

void or_sqfree_write_batch(int n_vecs, const float *vecs, uint8_t *out, const or_sqfree_t *L,
                           int n_threads)
{
#ifdef _OPENMP
    if (n_threads < 1) n_threads = 1;
#pragma omp parallel for num_threads(n_threads) schedule(static)
#endif
    for (int i = 0; i < n_vecs; i++)
        or_sqfree_write(vecs + (size_t)i * L->hd, out + (size_t)i * L->bytes_per_pos, L);
}

void or_sqfree_read_batch(int n_vecs, const uint8_t *in, float *vecs, const or_sqfree_t *L,
                          int n_threads)
{
#ifdef _OPENMP
    if (n_threads < 1) n_threads = 1;
#pragma omp parallel for num_threads(n_threads) schedule(static)
#endif
    for (int i = 0; i < n_vecs; i++)
        or_sqfree_read(in + (size_t)i * L->bytes_per_pos, vecs + (size_t)i * L->hd, L);
}

/* Decode attention over sqfree-compressed K/V of n_kv_heads slots (each
 * slot stride bytes apart), double accumulation; q fp16 bits
 * [n_q_heads][hd], query head g uses KV head g / (n_q / n_kv). */
void or_sqfree_attn_decode(const uint8_t *k_slots, size_t stride_k, const uint8_t *v_slots,
                           size_t stride_v, const or_sqfree_t *LK, const or_sqfree_t *LV,
                           int n_kv_heads, int n_q_heads, int kv_len, const uint16_t *q,
                           float logit_scale, float *out, int n_threads)
{
    const int hd = LK->hd;
    const int group = n_q_heads / n_kv_heads;
#ifdef _OPENMP
    if (n_threads < 1) n_threads = 1;
#pragma omp parallel for num_threads(n_threads) schedule(dynamic)
#endif
    for (int task = 0; task < n_q_heads; task++) {
        const int h = task / group;
        float kr[OR_SQ_MAX_PD], vr[OR_SQ_MAX_PD];
        double qd[OR_SQ_MAX_PD];
        for (int d = 0; d < hd; d++) qd[d] = (double)or_f16_to_f32(q[(size_t)task * hd + d]);
        double *sc = (double *)malloc(sizeof(double) * (size_t)(kv_len > 0 ? kv_len : 1));
        double mx = -INFINITY;
        for (int t = 0; t < kv_len; t++) {
            or_sqfree_read(k_slots + (size_t)h * stride_k + (size_t)t * LK->bytes_per_pos, kr, LK);
            double s = 0.0;
            for (int d = 0; d < hd; d++) s += (double)kr[d] * qd[d];
            sc[t] = s * (double)logit_scale;
            if (sc[t] > mx) mx = sc[t];
        }
        double den = 0.0, acc[OR_SQ_MAX_PD];
        for (int d = 0; d < hd; d++) acc[d] = 0.0;
        for (int t = 0; t < kv_len; t++) {
            or_sqfree_read(v_slots + (size_t)h * stride_v + (size_t)t * LV->bytes_per_pos, vr, LV);
            const double p = exp(sc[t] - mx);
            den += p;
            for (int d = 0; d < hd; d++) acc[d] += p * (double)vr[d];
        }
        for (int d = 0; d < hd; d++) out[(size_t)task * hd + d] = den > 0.0 ? (float)(acc[d] / den) : 0.0f;
        free(sc);
    }
}

/* ------------------------------------------------------------------ hier -- */

int or_hier_layout(or_hier_t *L, int hd, int n_bands, const int *bits, int residual_bits)
{
    memset(L, 0, sizeof(*L));
    L->hd = hd;
    L->pd = or_sqfree_pad_dim(hd);
    if (L->pd > OR_SQ_MAX_PD) return -1;
    int f[16];
    const int nf = or_vilenkin_factors(L->pd, f);
    if (nf < 1) return -1;
    L->n_skel = L->pd / f[nf - 1];
    L->n_target = L->pd - L->n_skel;
    L->res_bits = residual_bits;
    if (or_band_config(&L->bands, L->n_skel, n_bands, bits)) return -1;
    L->res_bytes = (L->n_target * residual_bits + 7) / 8;
    L->bytes_per_pos = L->bands.total_bytes + 4 + L->res_bytes;
    return 0;
}

void or_hier_predict(const or_hier_t *L, const uint16_t *W, const float *sk, float *pred)
{
    for (int t = 0; t < L->n_target; t++) {
        float acc = 0.0f;
        for (int s = 0; s < L->n_skel; s++)
            acc = fmaf(or_f16_to_f32(W[(size_t)t * L->n_skel + s]), sk[s], acc);
        pred[t] = acc;
    }
}

void or_hier_write(const float *vec, uint8_t *out, const or_hier_t *L, const uint16_t *W)
{
    float c[OR_SQ_MAX_PD], pred[OR_SQ_MAX_PD], dev[OR_SQ_MAX_PD];
    uint8_t lv[OR_SQ_MAX_PD];
    or_pad(vec, L->hd, L->pd, c);
    or_vilenkin(c, L->pd);
    memset(out, 0, (size_t)L->bytes_per_pos);
    or_band_quantize(c, out, &L->bands);              /* skeleton = c[0 .. n_skel) */
    or_hier_predict(L, W, c, pred);
    for (int t = 0; t < L->n_target; t++) dev[t] = c[L->n_skel + t] - pred[t];
    const float mag = or_residual_mag(dev, L->n_target);
    memcpy(out + L->bands.total_bytes, &mag, 4);
    or_hier_levels(dev, L->n_target, L->res_bits, mag, lv);
    or_pack_levels(lv, L->n_target, L->res_bits, out + L->bands.total_bytes + 4, L->res_bytes);
}

void or_hier_read(const uint8_t *in, float *vec, const or_hier_t *L, const uint16_t *W)
{
    float c[OR_SQ_MAX_PD], pred[OR_SQ_MAX_PD];
    uint8_t lv[OR_SQ_MAX_PD];
    or_band_dequantize(in, c, &L->bands, -1);
    or_hier_predict(L, W, c, pred);
    float mag;
    memcpy(&mag, in + L->bands.total_bytes, 4);
    or_unpack_levels(in + L->bands.total_bytes + 4, L->n_target, L->res_bits, lv, L->res_bytes);
    float dev[OR_SQ_MAX_PD];
    or_hier_unlevels(lv, L->n_target, L->res_bits, mag, dev);
    for (int t = 0; t < L->n_target; t++) c[L->n_skel + t] = pred[t] + dev[t];
    or_vilenkin(c, L->pd);
    memcpy(vec, c, sizeof(float) * (size_t)L->hd);
}

void or_hier_write_batch(int n_vecs, const float *vecs, uint8_t *out, const or_hier_t *L,
                         const uint16_t *W, int n_threads)
{
#ifdef _OPENMP
    if (n_threads < 1) n_threads = 1;
#pragma omp parallel for num_threads(n_threads) schedule(static)
#endif
    for (int i = 0; i < n_vecs; i++)
        or_hier_write(vecs + (size_t)i * L->hd, out + (size_t)i * L->bytes_per_pos, L, W);
}

void or_hier_read_batch(int n_vecs, const uint8_t *in, float *vecs, const or_hier_t *L,
                        const uint16_t *W, int n_threads)
{
#ifdef _OPENMP
    if (n_threads < 1) n_threads = 1;
#pragma omp parallel for num_threads(n_threads) schedule(static)
#endif
    for (int i = 0; i < n_vecs; i++)
        or_hier_read(in + (size_t)i * L->bytes_per_pos, vecs + (size_t)i * L->hd, L, W);
}
