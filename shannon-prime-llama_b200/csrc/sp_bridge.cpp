// sp_bridge.cpp — the sp_llama_* bridge over the sm_100a CUDA cache.
//
// Follows the reference bridge src/tools/shannon_prime_llama.c: the same
// environment variables, role-aware lookups (SHANNON_PRIME_DRAFT_<X> first
// for draft contexts, :101-140), head-dim-adaptive defaults (:235-252),
// draft presets (:177-199), position tracking for sp_llama_memory and the
// memory formula (:874-908).  Host vectors go through pinned staging
// buffers allocated once at init, so no call allocates afterwards.
#include "shannon_prime_llama.h"
#include "shannon_prime_cuda.h"

#include <cuda_runtime.h>

#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <algorithm>

namespace {

constexpr int kStageVecs = 8192;     // vectors per staged chunk

int parse_env_bool(const char *name, int default_val)
{
    const char *v = getenv(name);
    if (!v) return default_val;
    return (v[0] == '1' || v[0] == 'y' || v[0] == 'Y');
}

const char *role_name(const char *base, sp_llama_role_t role, char *out, size_t n)
{
    if (role == SP_LLAMA_ROLE_DRAFT) {
        snprintf(out, n, "SHANNON_PRIME_DRAFT_%s", base);
        const char *v = getenv(out);
        if (v && *v) return out;
    }
    snprintf(out, n, "SHANNON_PRIME_%s", base);
    return out;
}

const char *role_getenv(const char *base, sp_llama_role_t role)
{
    char name[160];
    return getenv(role_name(base, role, name, sizeof(name)));
}

int role_bool(const char *base, sp_llama_role_t role, int def)
{
    char name[160];
    return parse_env_bool(role_name(base, role, name, sizeof(name)), def);
}

// Comma-separated bit list; returns the count parsed (0 when unset).
int role_bits(const char *base, sp_llama_role_t role, int *bits, int max_n)
{
    const char *v = role_getenv(base, role);
    if (!v || !*v) return 0;
    int i = 0;
    const char *p = v;
    while (i < max_n && *p) {
        bits[i++] = atoi(p);
        while (*p && *p != ',') p++;
        if (*p == ',') p++;
    }
    return i;
}

// Band indices (comma-separated, e.g. "3" or "2,3") -> bit mask for
// sp_config_t::{k,v}_ternary_mask, as the reference bridge builds it
// (shannon_prime_llama.c:142-166): indices outside [0, 32) and tokens that
// do not start with a digit are ignored; unset or empty gives 0.
uint32_t role_ternary_mask(const char *base, sp_llama_role_t role)
{
    const char *v = role_getenv(base, role);
    uint32_t mask = 0u;
    if (!v) return mask;
    for (const char *p = v; *p;) {
        while (*p == ' ' || *p == '\t') p++;
        if (*p >= '0' && *p <= '9') {
            char *end = nullptr;
            const long idx = strtol(p, &end, 10);
            if (idx >= 0 && idx < 32) mask |= 1u << idx;
            p = end;
        }
        while (*p && *p != ',') p++;        // rest of this token
        if (*p == ',') p++;
        while (*p == ' ' || *p == '\t') p++;
    }
    return mask;
}

void apply_draft_preset(sp_config_t *cfg)
{
    const char *preset = getenv("SHANNON_PRIME_DRAFT_PRESET");
    if (!preset || !*preset) return;
    if (!strcmp(preset, "aggressive")) {
        cfg->k_band_bits[0] = 2; cfg->k_band_bits[1] = 1; cfg->k_n_bands = 2;
        cfg->v_band_bits[0] = 1; cfg->v_n_bands = 1;
    } else if (!strcmp(preset, "ternary")) {
        cfg->k_band_bits[0] = 2; cfg->k_band_bits[1] = 2; cfg->k_n_bands = 2;
        cfg->v_band_bits[0] = 2; cfg->v_n_bands = 1;
    } else if (strcmp(preset, "ship")) {
        fprintf(stderr, "[Shannon-Prime] unknown SHANNON_PRIME_DRAFT_PRESET '%s' "
                        "(known: aggressive, ternary, ship); ignoring\n", preset);
    }
}

}  // namespace

struct sp_llama_ctx_s {
    sp_llama_params_t params;
    sp_config_t config;
    sp_cuda_cache_t cache;
    cudaStream_t stream;
    bool own_stream;
    int n_positions;
    float *h_stage;            // pinned [kStageVecs][hd]
    float *d_stage;            // device [kStageVecs][hd]
    uint16_t *h_q, *h_out;     // pinned fp16 [n_layers][8*H][hd]
    void *d_q, *d_out;
    size_t qo_elems;
};

extern "C" {

sp_llama_ctx_t *sp_llama_init(const sp_llama_params_t *params)
{
    return sp_llama_init_with_role(params, SP_LLAMA_ROLE_DEFAULT);
}

sp_llama_ctx_t *sp_llama_init_with_role(const sp_llama_params_t *params, sp_llama_role_t role)
{
    if (!params || !role_bool("ENABLED", role, 0)) return nullptr;
    sp_config_t cfg;
    sp_config_init(&cfg, params->head_dim, params->n_layers, params->n_heads_kv);
    if (role == SP_LLAMA_ROLE_DRAFT) apply_draft_preset(&cfg);
    int n = role_bits("K_BITS", role, cfg.k_band_bits, SP_MAX_BANDS);
    if (n > 0) cfg.k_n_bands = n;
    n = role_bits("V_BITS", role, cfg.v_band_bits, SP_MAX_BANDS);
    if (n > 0) cfg.v_n_bands = n;
    cfg.use_mobius_mask = role_bool("MOBIUS", role, 1);
    cfg.k_ternary_mask = role_ternary_mask("K_TERNARY_BANDS", role);
    cfg.v_ternary_mask = role_ternary_mask("V_TERNARY_BANDS", role);
    // FP8 is advisory at the bridge, as in the reference
    // (shannon_prime_llama.c:287-326): no backend behind this bridge has an
    // fp8 path, so the request is logged and integer bands are used.
    if (role_bool("FP8", role, 0))
        fprintf(stderr, "[Shannon-Prime] SHANNON_PRIME_FP8=1 requested but this backend has no fp8 "
                        "band path; falling back to int\n");
    return sp_llama_init_config(params, &cfg);
}

sp_llama_ctx_t *sp_llama_init_config(const sp_llama_params_t *params, const sp_config_t *cfg)
{
    if (!params || !cfg) return nullptr;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        fprintf(stderr, "[Shannon-Prime] no CUDA device: the B200 bridge has no CPU backend\n");
        return nullptr;
    }
    sp_llama_ctx_t *ctx = (sp_llama_ctx_t *)calloc(1, sizeof(*ctx));
    if (!ctx) return nullptr;
    ctx->params = *params;
    ctx->config = *cfg;
    if (params->gpu_context) {
        ctx->stream = (cudaStream_t)params->gpu_context;
    } else {
        cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
        ctx->own_stream = true;
    }
    sp_config_t c = *cfg;
    c.use_fp8 = 0;
    if (sp_cuda_cache_init(&ctx->cache, &c, params->max_seq_len, ctx->stream) != SP_OK) {
        fprintf(stderr, "[Shannon-Prime] cache init failed: %s\n", sp_cuda_last_error_string());
        if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
        free(ctx);
        return nullptr;
    }
    const int hd = cfg->head_dim;
    ctx->qo_elems = (size_t)cfg->n_layers * 8 * cfg->n_heads_kv * hd;
    bool ok = cudaMallocHost(&ctx->h_stage, sizeof(float) * kStageVecs * hd) == cudaSuccess &&
              cudaMalloc(&ctx->d_stage, sizeof(float) * kStageVecs * hd) == cudaSuccess &&
              cudaMallocHost(&ctx->h_q, 2 * ctx->qo_elems) == cudaSuccess &&
              cudaMallocHost(&ctx->h_out, 2 * ctx->qo_elems) == cudaSuccess &&
              cudaMalloc(&ctx->d_q, 2 * ctx->qo_elems) == cudaSuccess &&
              cudaMalloc(&ctx->d_out, 2 * ctx->qo_elems) == cudaSuccess;
    if (!ok) {
        fprintf(stderr, "[Shannon-Prime] staging allocation failed\n");
        sp_llama_free(ctx);
        return nullptr;
    }
    if (parse_env_bool("SHANNON_PRIME_VERBOSE", 0)) sp_llama_print_config(ctx);
    return ctx;
}

void sp_llama_free(sp_llama_ctx_t *ctx)
{
    if (!ctx) return;
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    sp_cuda_cache_free(&ctx->cache);
    cudaFreeHost(ctx->h_stage);
    cudaFree(ctx->d_stage);
    cudaFreeHost(ctx->h_q);
    cudaFreeHost(ctx->h_out);
    cudaFree(ctx->d_q);
    cudaFree(ctx->d_out);
    if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
    free(ctx);
}

}  // extern "C"

// ------------------------------------------------------------ data path --

namespace {

bool valid(const sp_llama_ctx_t *ctx, int layer, int head, int pos, int n)
{
    return ctx && layer >= 0 && layer < ctx->config.n_layers && head >= 0 &&
           head < ctx->config.n_heads_kv && pos >= 0 && n >= 0 &&
           (long long)pos + n <= ctx->params.max_seq_len;
}

void track(sp_llama_ctx_t *ctx, int last_pos_excl)
{
    if (last_pos_excl > ctx->n_positions) ctx->n_positions = last_pos_excl;
}

// Host vectors -> pinned -> device -> encode, in chunks of kStageVecs.
void write_host(sp_llama_ctx_t *ctx, int which, int layer, int head, int start_pos, int n_pos,
                const float *vecs)
{
    if (!valid(ctx, layer, head, start_pos, n_pos) || !vecs) return;
    const int hd = ctx->config.head_dim;
    for (int done = 0; done < n_pos; done += kStageVecs) {
        const int cnt = std::min(kStageVecs, n_pos - done);
        memcpy(ctx->h_stage, vecs + (size_t)done * hd, sizeof(float) * cnt * hd);
        cudaMemcpyAsync(ctx->d_stage, ctx->h_stage, sizeof(float) * cnt * hd,
                        cudaMemcpyHostToDevice, ctx->stream);
        if (which == 0) sp_cuda_write_k_batch(&ctx->cache, layer, head, start_pos + done, cnt, ctx->d_stage);
        else sp_cuda_write_v_batch(&ctx->cache, layer, head, start_pos + done, cnt, ctx->d_stage);
        cudaStreamSynchronize(ctx->stream);   // staging is reused by the next chunk
    }
    if (which == 0) track(ctx, start_pos + n_pos);
}

void read_host(const sp_llama_ctx_t *cctx, int which, int layer, int head, int start_pos, int n_pos,
               float *out, int max_bands)
{
    sp_llama_ctx_t *ctx = const_cast<sp_llama_ctx_t *>(cctx);
    if (!valid(ctx, layer, head, start_pos, n_pos) || !out) return;
    const int hd = ctx->config.head_dim;
    for (int done = 0; done < n_pos; done += kStageVecs) {
        const int cnt = std::min(kStageVecs, n_pos - done);
        sp_cuda_read_batch_partial(&ctx->cache, which, layer, head, start_pos + done, cnt,
                                   ctx->d_stage, max_bands);
        cudaMemcpyAsync(ctx->h_stage, ctx->d_stage, sizeof(float) * cnt * hd,
                        cudaMemcpyDeviceToHost, ctx->stream);
        cudaStreamSynchronize(ctx->stream);
        memcpy(out + (size_t)done * hd, ctx->h_stage, sizeof(float) * cnt * hd);
    }
}

}  // namespace

extern "C" {

void sp_llama_write_kv(sp_llama_ctx_t *ctx, int layer, int head, int pos,
                       const float *k_vec, const float *v_vec)
{
    sp_llama_write_k(ctx, layer, head, pos, k_vec);
    sp_llama_write_v(ctx, layer, head, pos, v_vec);
}

void sp_llama_write_k(sp_llama_ctx_t *ctx, int layer, int head, int pos, const float *k_vec)
{ write_host(ctx, 0, layer, head, pos, 1, k_vec); }
void sp_llama_write_v(sp_llama_ctx_t *ctx, int layer, int head, int pos, const float *v_vec)
{ write_host(ctx, 1, layer, head, pos, 1, v_vec); }
void sp_llama_write_k_batch(sp_llama_ctx_t *ctx, int layer, int head, int start_pos, int n_pos,
                            const float *k_vecs)
{ write_host(ctx, 0, layer, head, start_pos, n_pos, k_vecs); }
void sp_llama_write_v_batch(sp_llama_ctx_t *ctx, int layer, int head, int start_pos, int n_pos,
                            const float *v_vecs)
{ write_host(ctx, 1, layer, head, start_pos, n_pos, v_vecs); }

void sp_llama_read_k(const sp_llama_ctx_t *ctx, int layer, int head, int pos, float *k_out)
{ read_host(ctx, 0, layer, head, pos, 1, k_out, -1); }
void sp_llama_read_v(const sp_llama_ctx_t *ctx, int layer, int head, int pos, float *v_out)
{ read_host(ctx, 1, layer, head, pos, 1, v_out, -1); }
void sp_llama_read_k_partial(const sp_llama_ctx_t *ctx, int layer, int head, int pos,
                             float *k_out, int max_bands)
{ read_host(ctx, 0, layer, head, pos, 1, k_out, max_bands); }
void sp_llama_read_v_partial(const sp_llama_ctx_t *ctx, int layer, int head, int pos,
                             float *v_out, int max_bands)
{ read_host(ctx, 1, layer, head, pos, 1, v_out, max_bands); }
void sp_llama_read_k_batch(const sp_llama_ctx_t *ctx, int layer, int head, int start_pos,
                           int n_pos, float *k_out)
{ read_host(ctx, 0, layer, head, start_pos, n_pos, k_out, -1); }
void sp_llama_read_v_batch(const sp_llama_ctx_t *ctx, int layer, int head, int start_pos,
                           int n_pos, float *v_out)
{ read_host(ctx, 1, layer, head, start_pos, n_pos, v_out, -1); }

int sp_llama_write_kv_tokens(sp_llama_ctx_t *ctx, int layer, int start_pos, int n_tokens,
                             const float *k, const float *v)
{
    if (!valid(ctx, layer, 0, start_pos, n_tokens)) return SP_ERR_ARG;
    const int hd = ctx->config.head_dim, H = ctx->config.n_heads_kv;
    const int tok_per_chunk = std::max(1, kStageVecs / H);
    for (int done = 0; done < n_tokens; done += tok_per_chunk) {
        const int cnt = std::min(tok_per_chunk, n_tokens - done);
        const size_t elems = (size_t)cnt * H * hd;
        for (int half = 0; half < 2; half++) {
            const float *src = half ? v : k;
            if (!src) continue;
            memcpy(ctx->h_stage, src + (size_t)done * H * hd, sizeof(float) * elems);
            cudaMemcpyAsync(ctx->d_stage, ctx->h_stage, sizeof(float) * elems,
                            cudaMemcpyHostToDevice, ctx->stream);
            int rc = sp_cuda_write_kv_tokens(&ctx->cache, layer, start_pos + done, cnt,
                                             half ? nullptr : ctx->d_stage,
                                             half ? ctx->d_stage : nullptr, SP_DTYPE_F32);
            if (rc) return rc;
            if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) return SP_ERR_CUDA;
        }
    }
    track(ctx, start_pos + n_tokens);
    return SP_OK;
}

// True if p is page-locked host memory known to the CUDA runtime.
static bool host_pinned(const void *p)
{
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeHost;
}

// Device address of a page-locked host buffer that the GPU can address
// directly (mapped, as every cudaHostAlloc / cudaMallocHost buffer is under
// unified addressing), or null.
static void *host_mapped(const void *p)
{
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return at.type == cudaMemoryTypeHost ? at.devicePointer : nullptr;
}

int sp_llama_attn_decode(sp_llama_ctx_t *ctx, int layer0, int n_layers, const uint16_t *q_f16,
                         int n_q_heads, int kv_len, float logit_scale, uint16_t *out_f16,
                         int max_bands)
{
    if (!ctx || !q_f16 || !out_f16 || n_layers <= 0) return SP_ERR_ARG;
    const size_t elems = (size_t)n_layers * n_q_heads * ctx->config.head_dim;
    if (elems > ctx->qo_elems) return SP_ERR_ARG;
    // Page-locked caller buffers that the GPU maps are read and written by
    // the decode kernels in place over the host link (the queries at each
    // block's set-up, the output rows by the combine), which takes the two
    // copy-engine transfers and their latencies off the call.  Other
    // page-locked buffers are copied from / to directly; pageable ones go
    // through the context's pinned staging buffers.
    const void *q_dev = host_mapped(q_f16);
    void *out_dev = host_mapped(out_f16);
    const bool q_pinned = q_dev || host_pinned(q_f16), out_pinned = out_dev || host_pinned(out_f16);
    if (!q_dev) {
        if (!q_pinned) memcpy(ctx->h_q, q_f16, 2 * elems);
        cudaMemcpyAsync(ctx->d_q, q_pinned ? (const void *)q_f16 : ctx->h_q, 2 * elems, cudaMemcpyHostToDevice,
                        ctx->stream);
    }
    int rc = sp_cuda_attn_decode(&ctx->cache, layer0, n_layers, q_dev ? q_dev : ctx->d_q, n_q_heads, kv_len,
                                 logit_scale, out_dev ? out_dev : ctx->d_out, max_bands, ctx->stream);
    if (rc) return rc;
    if (!out_dev)
        cudaMemcpyAsync(out_pinned ? (void *)out_f16 : ctx->h_out, ctx->d_out, 2 * elems, cudaMemcpyDeviceToHost,
                        ctx->stream);
    if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) return SP_ERR_CUDA;
    if (!out_pinned) memcpy(out_f16, ctx->h_out, 2 * elems);
    return SP_OK;
}

const void *sp_llama_get_cuda_cache(const sp_llama_ctx_t *ctx)
{
    return ctx ? (const void *)&ctx->cache : nullptr;
}

// ------------------------------------------------------------- management --

void sp_llama_clear_range(sp_llama_ctx_t *ctx, int start_pos, int end_pos)
{
    if (!ctx || start_pos < 0 || end_pos <= start_pos || end_pos > ctx->cache.max_seq_len) return;
    const sp_cuda_cache_t &c = ctx->cache;
    for (int half = 0; half < 2; half++) {
        const size_t tb = half ? c.v_bands.total_bytes : c.k_bands.total_bytes;
        char *base = (char *)(half ? c.d_v_cache : c.d_k_cache) + (size_t)start_pos * tb;
        cudaMemset2DAsync(base, (size_t)c.max_seq_len * tb, 0, (size_t)(end_pos - start_pos) * tb,
                          c.n_slots, ctx->stream);
    }
    cudaStreamSynchronize(ctx->stream);
}

sp_llama_memory_t sp_llama_memory(const sp_llama_ctx_t *ctx)
{
    sp_llama_memory_t m;
    memset(&m, 0, sizeof(m));
    if (!ctx) return m;
    const size_t slots = (size_t)ctx->config.n_layers * ctx->config.n_heads_kv;
    const size_t n = ctx->n_positions;
    m.compressed_bytes = slots * n * (ctx->cache.k_bands.total_bytes + ctx->cache.v_bands.total_bytes);
    m.baseline_bytes = slots * n * ctx->config.head_dim * 2 * 2;
    m.compression_ratio = m.compressed_bytes ? (float)m.baseline_bytes / (float)m.compressed_bytes : 0.0f;
    m.n_positions = ctx->n_positions;
    return m;
}

float sp_llama_validate_k(sp_llama_ctx_t *ctx, const float *k_vec, int head_dim)
{
    if (!ctx || !k_vec || head_dim != ctx->config.head_dim) return 0.0f;
    float *recon = (float *)malloc(sizeof(float) * head_dim);
    sp_llama_write_k(ctx, 0, 0, 0, k_vec);
    sp_llama_read_k(ctx, 0, 0, 0, recon);
    float c = sp_correlation_f32(k_vec, recon, head_dim);
    free(recon);
    return c;
}

void sp_llama_print_config(const sp_llama_ctx_t *ctx)
{
    if (!ctx) return;
    fprintf(stderr, "[Shannon-Prime] llama.cpp integration\n  Backend:  CUDA (sm_100a)\n");
    sp_config_print(&ctx->config);
}

const float *sp_llama_get_freq_factors(const sp_llama_ctx_t *) { return nullptr; }
int sp_llama_get_n_freqs(const sp_llama_ctx_t *) { return 0; }
const void *sp_llama_get_hexagon_k_buf(const sp_llama_ctx_t *, int, int) { return nullptr; }
int sp_llama_get_hexagon_k_total_bytes(const sp_llama_ctx_t *) { return 0; }

}  // extern "C"
