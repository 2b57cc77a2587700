// sp_api.cu — cache lifecycle and the reference-named write/read entry
// points of shannon_prime_cuda.h, plus the per-thread status of the C-ABI.
#include "sp_internal.cuh"

#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

size_t sp_attn_workspace_bytes(const sp_cuda_cache_t *cc);   // sp_attn.cu

// ------------------------------------------------------------- status --

static thread_local int t_err = SP_OK;
static thread_local char t_msg[256] = "ok";

int sp_set_error(int code, const char *fmt, ...)
{
    t_err = code;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
    va_end(ap);
    return code;
}

void sp_clear_error()
{
    t_err = SP_OK;
    t_msg[0] = 'o'; t_msg[1] = 'k'; t_msg[2] = 0;
}

int sp_check_cuda(cudaError_t e, const char *what)
{
    if (e == cudaSuccess) return SP_OK;
    return sp_set_error(SP_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

float sp_inv_sqrt_n(int n)
{
    volatile float fn = (float)n;          // IEEE sqrtf and divide, as the CPU path
    return 1.0f / sqrtf(fn);
}

SpBandLayout sp_layout_from(const sp_band_config_t &bc)
{
    SpBandLayout l;
    memset(&l, 0, sizeof(l));
    l.n = bc.head_dim;
    l.n_bands = bc.n_bands;
    int byte = 0;
    for (int b = 0; b < bc.n_bands; b++) {
        int off, sz;
        sp_band_span(&bc, b, &off, &sz);
        l.off[b] = off;
        l.size[b] = sz;
        l.bits[b] = bc.band_bits[b];
        l.byte_off[b] = byte;
        byte += 2 + (sz * bc.band_bits[b] + 7) / 8;
    }
    l.total_bytes = byte;
    return l;
}

extern "C" int sp_cuda_last_error(void) { return t_err; }
extern "C" const char *sp_cuda_last_error_string(void) { return t_msg; }

// ---------------------------------------------------------- lifecycle --

static bool pow2_in_range(int n) { return n >= 32 && n <= SP_MAX_HEAD_DIM && (n & (n - 1)) == 0; }

extern "C" int sp_cuda_cache_init(sp_cuda_cache_t *cc, const sp_config_t *cfg,
                                  int max_seq_len, void *stream)
{
    sp_clear_error();
    if (!cc || !cfg) return sp_set_error(SP_ERR_ARG, "cache_init: NULL argument");
    memset(cc, 0, sizeof(*cc));
    if (cfg->n_layers <= 0 || cfg->n_heads_kv <= 0 || max_seq_len <= 0)
        return sp_set_error(SP_ERR_ARG, "cache_init: bad dims");
    if (!pow2_in_range(cfg->head_dim))
        return sp_set_error(SP_ERR_UNSUPPORTED, "cache_init: head_dim %d not a power of two in [32,512]", cfg->head_dim);
    if (cfg->use_fp8)
        return sp_set_error(SP_ERR_UNSUPPORTED, "cache_init: fp8 bands are not implemented (the bridge falls "
                            "back to integer bands, as the reference bridge does)");
    cc->config = *cfg;
    // Ternary noise-tail bands (the core's sp_band_config_init_ext ternary
    // mask, CHANGELOG.md:107-114): bit b set stores band b as {-1, 0, +1}
    // at 2 bits per code whatever its band_bits, i.e. the band quantiser at
    // 2 bits (m = 1, scale = max|x|).
    int kbits[SP_MAX_BANDS], vbits[SP_MAX_BANDS];
    for (int b = 0; b < SP_MAX_BANDS; b++) {
        kbits[b] = (cfg->k_ternary_mask >> b) & 1u ? 2 : cfg->k_band_bits[b];
        vbits[b] = (cfg->v_ternary_mask >> b) & 1u ? 2 : cfg->v_band_bits[b];
    }
    if (sp_band_config_init(&cc->k_bands, cfg->head_dim, cfg->k_n_bands, kbits) ||
        sp_band_config_init(&cc->v_bands, cfg->head_dim, cfg->v_n_bands, vbits))
        return sp_set_error(SP_ERR_ARG, "cache_init: bad band configuration");
    cc->max_seq_len = (max_seq_len + 15) & ~15;
    cc->stream = stream;
    cc->n_slots = cfg->n_layers * cfg->n_heads_kv;
    cudaGetDevice(&cc->device);

    const size_t k_total = (size_t)cc->n_slots * cc->max_seq_len * cc->k_bands.total_bytes;
    const size_t v_total = (size_t)cc->n_slots * cc->max_seq_len * cc->v_bands.total_bytes;
    int rc = SP_OK;
    if ((rc = sp_check_cuda(cudaMalloc(&cc->d_k_cache, k_total), "cudaMalloc K cache")) ||
        (rc = sp_check_cuda(cudaMalloc(&cc->d_v_cache, v_total), "cudaMalloc V cache")) ||
        (rc = sp_check_cuda(cudaMalloc(&cc->d_scratch, sp_io_scratch_bytes(cfg)), "cudaMalloc scratch")) ||
        (rc = sp_check_cuda(cudaMalloc(&cc->d_status, 16), "cudaMalloc status"))) {
        sp_cuda_cache_free(cc);
        return rc;
    }
    cudaMemset(cc->d_k_cache, 0, k_total);
    cudaMemset(cc->d_v_cache, 0, v_total);
    cudaMemset(cc->d_status, 0, 16);

    if (cfg->use_mobius_mask) {
        sp_mobius_mask_t m;
        if (sp_mobius_mask_init(&m, cfg->head_dim)) {
            sp_cuda_cache_free(cc);
            return sp_set_error(SP_ERR_ARG, "cache_init: mobius table");
        }
        int *inv = (int *)malloc(sizeof(int) * cfg->head_dim);
        for (int i = 0; i < cfg->head_dim; i++) inv[m.order[i]] = i;
        if ((rc = sp_check_cuda(cudaMalloc(&cc->d_mobius_order, cfg->head_dim * sizeof(int)), "cudaMalloc order")) ||
            (rc = sp_check_cuda(cudaMalloc(&cc->d_mobius_inv, cfg->head_dim * sizeof(int)), "cudaMalloc inv"))) {
            free(inv);
            sp_mobius_mask_free(&m);
            sp_cuda_cache_free(cc);
            return rc;
        }
        cudaMemcpy(cc->d_mobius_order, m.order, cfg->head_dim * sizeof(int), cudaMemcpyHostToDevice);
        cudaMemcpy(cc->d_mobius_inv, inv, cfg->head_dim * sizeof(int), cudaMemcpyHostToDevice);
        free(inv);
        sp_mobius_mask_free(&m);
    }

    cc->attn_max_q_heads = 8 * cfg->n_heads_kv;
    cc->attn_ws_layers = cfg->n_layers;
    cc->attn_ws_bytes = sp_attn_workspace_bytes(cc);
    if ((rc = sp_check_cuda(cudaMalloc(&cc->d_attn_ws, cc->attn_ws_bytes), "cudaMalloc attention workspace"))) {
        sp_cuda_cache_free(cc);
        return rc;
    }
    if ((rc = sp_check_cuda(cudaDeviceSynchronize(), "cache_init"))) {
        sp_cuda_cache_free(cc);
        return rc;
    }
    if (getenv("SHANNON_PRIME_VERBOSE") && getenv("SHANNON_PRIME_VERBOSE")[0] == '1')
        sp_cuda_print_memory(cc);
    return SP_OK;
}

extern "C" void sp_cuda_cache_free(sp_cuda_cache_t *cc)
{
    if (!cc) return;
    cudaFree(cc->d_k_cache);
    cudaFree(cc->d_v_cache);
    cudaFree(cc->d_scratch);
    cudaFree(cc->d_mobius_order);
    cudaFree(cc->d_mobius_inv);
    cudaFree(cc->d_attn_ws);
    cudaFree(cc->d_status);
    cc->d_k_cache = cc->d_v_cache = nullptr;
    cc->d_scratch = nullptr;
    cc->d_mobius_order = cc->d_mobius_inv = nullptr;
    cc->d_attn_ws = nullptr;
    cc->d_status = nullptr;
}

extern "C" void sp_cuda_print_memory(const sp_cuda_cache_t *cc)
{
    const double mb = 1024.0 * 1024.0;
    size_t k = (size_t)cc->n_slots * cc->max_seq_len * cc->k_bands.total_bytes;
    size_t v = (size_t)cc->n_slots * cc->max_seq_len * cc->v_bands.total_bytes;
    size_t base = (size_t)cc->n_slots * cc->max_seq_len * cc->config.head_dim * 2 * 2;
    fprintf(stderr, "[Shannon-Prime B200] Memory:\n");
    fprintf(stderr, "  Compressed: %.2f MB (K: %.2f + V: %.2f)\n", (k + v) / mb, k / mb, v / mb);
    fprintf(stderr, "  Baseline:   %.2f MB\n", base / mb);
    fprintf(stderr, "  Ratio:      %.2fx\n", (double)base / (double)(k + v));
}

// ---------------------------------------------------------- write / read --

static int check_pos(const sp_cuda_cache_t *cc, int layer, int head, int pos, int n)
{
    if (!cc || !cc->d_k_cache) return sp_set_error(SP_ERR_ARG, "cache not initialised");
    if (layer < 0 || layer >= cc->config.n_layers || head < 0 || head >= cc->config.n_heads_kv)
        return sp_set_error(SP_ERR_ARG, "layer/head out of range (%d,%d)", layer, head);
    if (pos < 0 || n < 0 || (long long)pos + n > cc->max_seq_len)
        return sp_set_error(SP_ERR_ARG, "positions [%d,%d) outside the cache", pos, pos + n);
    return SP_OK;
}

static int write_one_half(sp_cuda_cache_t *cc, int which, int layer, int head0, int nh,
                          int start_pos, int n_tokens, const void *d_in, int dtype)
{
    const sp_band_config_t &bc = which ? cc->v_bands : cc->k_bands;
    SpBandLayout bl = sp_layout_from(bc);
    uint8_t *base = (uint8_t *)(which ? cc->d_v_cache : cc->d_k_cache);
    const int *order = which ? nullptr : (cc->config.use_mobius_mask ? cc->d_mobius_order : nullptr);
    return sp_launch_encode(d_in, dtype, n_tokens, nh, base,
                            (long long)layer * cc->config.n_heads_kv + head0,
                            (long long)cc->max_seq_len * bc.total_bytes, start_pos, order, true,
                            bl, (cudaStream_t)cc->stream, true, cc->d_status);
}

extern "C" int sp_cuda_write_kv_tokens(sp_cuda_cache_t *cc, int layer, int start_pos,
                                       int n_tokens, const void *d_k, const void *d_v, int dtype)
{
    sp_clear_error();
    int rc = check_pos(cc, layer, 0, start_pos, n_tokens);
    if (rc) return rc;
    const int H = cc->config.n_heads_kv;
    // Both halves in one launch when the lane encoder takes them.
    if (d_k && d_v && n_tokens > 0) {
        const SpBandLayout kbl = sp_layout_from(cc->k_bands), vbl = sp_layout_from(cc->v_bands);
        const long long slot0 = (long long)layer * H;
        if (sp_encode_lane_kv(d_k, d_v, dtype, n_tokens, H, start_pos, (uint8_t *)cc->d_k_cache, slot0,
                              (long long)cc->max_seq_len * cc->k_bands.total_bytes, kbl,
                              cc->config.use_mobius_mask ? cc->d_mobius_order : nullptr, true,
                              (uint8_t *)cc->d_v_cache, slot0,
                              (long long)cc->max_seq_len * cc->v_bands.total_bytes, vbl, cc->d_status,
                              (cudaStream_t)cc->stream, &rc))
            return rc;
    }
    if (d_k && (rc = write_one_half(cc, 0, layer, 0, H, start_pos, n_tokens, d_k, dtype))) return rc;
    if (d_v && (rc = write_one_half(cc, 1, layer, 0, H, start_pos, n_tokens, d_v, dtype))) return rc;
    return SP_OK;
}

static void write_batch(sp_cuda_cache_t *cc, int which, int layer, int head, int start_pos,
                        int n_pos, const float *d_vecs)
{
    sp_clear_error();
    if (check_pos(cc, layer, head, start_pos, n_pos)) return;
    write_one_half(cc, which, layer, head, 1, start_pos, n_pos, d_vecs, SP_DTYPE_F32);
}

extern "C" void sp_cuda_write_k(sp_cuda_cache_t *cc, int layer, int head, int pos, const float *d_k_vec)
{ write_batch(cc, 0, layer, head, pos, 1, d_k_vec); }
extern "C" void sp_cuda_write_v(sp_cuda_cache_t *cc, int layer, int head, int pos, const float *d_v_vec)
{ write_batch(cc, 1, layer, head, pos, 1, d_v_vec); }
extern "C" void sp_cuda_write_k_batch(sp_cuda_cache_t *cc, int layer, int head, int start_pos,
                                      int n_pos, const float *d_k_vecs)
{ write_batch(cc, 0, layer, head, start_pos, n_pos, d_k_vecs); }
extern "C" void sp_cuda_write_v_batch(sp_cuda_cache_t *cc, int layer, int head, int start_pos,
                                      int n_pos, const float *d_v_vecs)
{ write_batch(cc, 1, layer, head, start_pos, n_pos, d_v_vecs); }

extern "C" int sp_cuda_read_batch_partial(const sp_cuda_cache_t *cc, int which, int layer, int head,
                                          int start_pos, int n_pos, float *d_out, int max_bands)
{
    sp_clear_error();
    int rc = check_pos(cc, layer, head, start_pos, n_pos);
    if (rc) return rc;
    if (which != 0 && which != 1) return sp_set_error(SP_ERR_ARG, "which must be 0 (K) or 1 (V)");
    const sp_band_config_t &bc = which ? cc->v_bands : cc->k_bands;
    SpBandLayout bl = sp_layout_from(bc);
    const uint8_t *base = (const uint8_t *)(which ? cc->d_v_cache : cc->d_k_cache);
    const int *order = which ? nullptr : (cc->config.use_mobius_mask ? cc->d_mobius_order : nullptr);
    return sp_launch_decode(base, (long long)layer * cc->config.n_heads_kv + head,
                            (long long)cc->max_seq_len * bc.total_bytes, start_pos, n_pos, d_out,
                            order, true, max_bands, bl, (cudaStream_t)cc->stream, true, cc->d_status);
}

extern "C" void sp_cuda_read_k(const sp_cuda_cache_t *cc, int layer, int head, int pos, float *d_k_out)
{ sp_cuda_read_batch_partial(cc, 0, layer, head, pos, 1, d_k_out, -1); }
extern "C" void sp_cuda_read_v(const sp_cuda_cache_t *cc, int layer, int head, int pos, float *d_v_out)
{ sp_cuda_read_batch_partial(cc, 1, layer, head, pos, 1, d_v_out, -1); }
extern "C" void sp_cuda_read_k_batch(const sp_cuda_cache_t *cc, int layer, int head, int start_pos,
                                     int n_pos, float *d_k_out)
{ sp_cuda_read_batch_partial(cc, 0, layer, head, start_pos, n_pos, d_k_out, -1); }
extern "C" void sp_cuda_read_v_batch(const sp_cuda_cache_t *cc, int layer, int head, int start_pos,
                                     int n_pos, float *d_v_out)
{ sp_cuda_read_batch_partial(cc, 1, layer, head, start_pos, n_pos, d_v_out, -1); }

// sizeof of the public structs, so bindings in other languages can check
// their mirror of the layout (0 = sp_config_t, 1 = sp_band_config_t,
// 2 = sp_cuda_cache_t).
extern "C" int sp_cuda_abi_struct_size(int which)
{
    switch (which) {
    case 0: return (int)sizeof(sp_config_t);
    case 1: return (int)sizeof(sp_band_config_t);
    case 2: return (int)sizeof(sp_cuda_cache_t);
    case 3: return (int)sizeof(sp_cuda_sqfree_cache_t);
    case 4: return (int)sizeof(sp_cuda_hier_cache_t);
    case 5: return (int)sizeof(sp_cuda_cold_layer_t);
    }
    return -1;
}
