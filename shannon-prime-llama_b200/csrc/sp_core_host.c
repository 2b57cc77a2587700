/*
 * sp_core_host.c — host-side configuration utilities of the codec (the
 * subset of the absent core library lib/shannon-prime/core that the CUDA
 * C-ABI and the llama bridge need; see include/shannon_prime.h).
 */
#include "shannon_prime.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

void sp_config_init(sp_config_t *cfg, int head_dim, int n_layers, int n_heads_kv)
{
    memset(cfg, 0, sizeof(*cfg));
    cfg->head_dim = head_dim;
    cfg->n_layers = n_layers;
    cfg->n_heads_kv = n_heads_kv;
    if (head_dim >= 128) {          /* shannon_prime_llama.c:241-245 */
        static const int k[4] = {5, 5, 4, 3};
        cfg->k_n_bands = 4;
        memcpy(cfg->k_band_bits, k, sizeof(k));
        cfg->v_band_bits[0] = 3;
    } else {                        /* shannon_prime_llama.c:246-250 */
        static const int k[3] = {5, 4, 4};
        cfg->k_n_bands = 3;
        memcpy(cfg->k_band_bits, k, sizeof(k));
        cfg->v_band_bits[0] = 5;
    }
    cfg->v_n_bands = 1;
    cfg->use_mobius_mask = 1;
}

int sp_band_config_init(sp_band_config_t *bc, int head_dim, int n_bands,
                        const int *band_bits)
{
    if (!bc || !band_bits || head_dim <= 0 || n_bands < 1 ||
        n_bands > SP_MAX_BANDS || n_bands > head_dim)
        return -1;
    memset(bc, 0, sizeof(*bc));
    bc->head_dim = head_dim;
    bc->n_bands = n_bands;
    bc->band_size = head_dim / n_bands;
    int total = 0;
    for (int b = 0; b < n_bands; b++) {
        if (band_bits[b] < 1 || band_bits[b] > 8) return -1;
        bc->band_bits[b] = band_bits[b];
        int off, sz;
        sp_band_span(bc, b, &off, &sz);
        total += 2 + (sz * band_bits[b] + 7) / 8;
    }
    bc->total_bytes = total;
    return 0;
}

void sp_band_span(const sp_band_config_t *bc, int band, int *offset, int *size)
{
    int off = band * bc->band_size;
    *offset = off;
    *size = (band == bc->n_bands - 1) ? (bc->head_dim - off) : bc->band_size;
}

static int is_squarefree(int m)
{
    for (int p = 2; p * p <= m; p++)
        if (m % (p * p) == 0) return 0;
    return 1;
}

int sp_mobius_mask_init(sp_mobius_mask_t *mask, int n)
{
    mask->n = n;
    mask->order = (int *)malloc(sizeof(int) * (size_t)n);
    if (!mask->order) return -1;
    int k = 0;
    for (int i = 0; i < n; i++)
        if (is_squarefree(i + 1)) mask->order[k++] = i;
    for (int i = 0; i < n; i++)
        if (!is_squarefree(i + 1)) mask->order[k++] = i;
    return 0;
}

void sp_mobius_mask_free(sp_mobius_mask_t *mask)
{
    if (!mask) return;
    free(mask->order);
    mask->order = NULL;
}

float sp_correlation_f32(const float *a, const float *b, int n)
{
    if (n <= 0) return 0.0f;
    double ma = 0, mb = 0;
    for (int i = 0; i < n; i++) { ma += a[i]; mb += b[i]; }
    ma /= n; mb /= n;
    double sab = 0, saa = 0, sbb = 0;
    for (int i = 0; i < n; i++) {
        double x = a[i] - ma, y = b[i] - mb;
        sab += x * y; saa += x * x; sbb += y * y;
    }
    if (saa <= 0 || sbb <= 0) return 0.0f;
    return (float)(sab / sqrt(saa * sbb));
}

void sp_config_print(const sp_config_t *cfg)
{
    fprintf(stderr, "  head_dim=%d layers=%d kv_heads=%d mobius=%d\n",
            cfg->head_dim, cfg->n_layers, cfg->n_heads_kv, cfg->use_mobius_mask);
    fprintf(stderr, "  K bits:");
    for (int b = 0; b < cfg->k_n_bands; b++) fprintf(stderr, " %d", cfg->k_band_bits[b]);
    fprintf(stderr, "\n  V bits:");
    for (int b = 0; b < cfg->v_n_bands; b++) fprintf(stderr, " %d", cfg->v_band_bits[b]);
    fprintf(stderr, "\n");
}
