/*
 * ggml_decode_check.c — a C client of the public headers (built by
 * tests/test_gpu_ggml_op.py with gcc against the headers in include/ and the in-tree
 * library).  It plays the ggml-cuda side of the fused attention op: builds
 * a ship cache through the C-ABI, fills it from host K/V, then calls
 * sp_ggml_attn_decode with ggml-style tensor views — an F32 query view with
 * padded row strides, as build_attn_mha's permuted Q is, and an F32 output
 * view with padded strides — and writes the cache slabs, the queries and
 * the outputs to a file for the Python test to check against the oracle.
 *
 *   ggml_decode_check <out.bin>
 */
#include <cuda_runtime_api.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "shannon_prime.h"
#include "shannon_prime_cuda.h"
#include "shannon_prime_ggml.h"

#define L 2
#define H 4
#define G 4
#define HD 128
#define T 600
#define NQ (H * G)

static uint64_t rng = 88172645463325252ull;
static float nrand(void)
{
    /* sum of 4 uniforms, centred: a cheap bell-shaped value */
    float s = 0.0f;
    for (int i = 0; i < 4; i++) {
        rng ^= rng << 13; rng ^= rng >> 7; rng ^= rng << 17;
        s += (float)(rng >> 40) / (float)(1ull << 24);
    }
    return (s - 2.0f) * 1.7f;
}

#define CK(x) do { if ((x) != 0) { fprintf(stderr, "%s failed at line %d\n", #x, __LINE__); return 1; } } while (0)

int main(int argc, char **argv)
{
    if (argc < 2) return 2;
    sp_config_t cfg;
    sp_config_init(&cfg, HD, L, H);
    sp_cuda_cache_t cc;
    memset(&cc, 0, sizeof cc);
    CK(sp_cuda_cache_init(&cc, &cfg, T, NULL));

    const size_t kv_n = (size_t)T * H * HD;
    float *hk = malloc(kv_n * 4), *hv = malloc(kv_n * 4);
    void *dk, *dv;
    CK(cudaMalloc(&dk, kv_n * 4));
    CK(cudaMalloc(&dv, kv_n * 4));
    for (int l = 0; l < L; l++) {
        for (size_t i = 0; i < kv_n; i++) { hk[i] = nrand(); hv[i] = nrand(); }
        CK(cudaMemcpy(dk, hk, kv_n * 4, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(dv, hv, kv_n * 4, cudaMemcpyHostToDevice));
        CK(sp_cuda_write_kv_tokens(&cc, l, 0, T, dk, dv, SP_DTYPE_F32));
    }

    /* Q view: ne {HD, 1, NQ, 1}, element stride 4, head stride padded to 160 floats */
    const size_t q_row = 160;
    float *hq = calloc(q_row * NQ, 4);
    for (int g = 0; g < NQ; g++)
        for (int d = 0; d < HD; d++) hq[g * q_row + d] = nrand() * 0.09f;
    void *dq, *dout;
    CK(cudaMalloc(&dq, q_row * NQ * 4));
    CK(cudaMemcpy(dq, hq, q_row * NQ * 4, cudaMemcpyHostToDevice));
    const int64_t q_ne[4] = {HD, 1, NQ, 1};
    const size_t q_nb[4] = {4, q_row * 4 * NQ, q_row * 4, q_row * 4 * NQ};
    /* output view: ne {HD, NQ, 1, 1}, rows padded to 136 floats */
    const size_t o_row = 136;
    CK(cudaMalloc(&dout, o_row * NQ * 4));
    CK(cudaMemset(dout, 0, o_row * NQ * 4));
    const int64_t o_ne[4] = {HD, NQ, 1, 1};
    const size_t o_nb[4] = {4, o_row * 4, o_row * 4 * NQ, o_row * 4 * NQ};
    const int il = 1;
    const float scale = 0.8f;
    CK(sp_ggml_attn_decode(&cc, il, dq, SP_GGML_TYPE_F32, q_ne, q_nb, dout, SP_GGML_TYPE_F32, o_ne, o_nb,
                           scale, T, -1, NULL));
    CK(cudaDeviceSynchronize());
    float *ho = malloc(o_row * NQ * 4);
    CK(cudaMemcpy(ho, dout, o_row * NQ * 4, cudaMemcpyDeviceToHost));

    /* layer il's slabs */
    const size_t kb = cc.k_bands.total_bytes, vb = cc.v_bands.total_bytes;
    const size_t ks = (size_t)H * cc.max_seq_len * kb, vs = (size_t)H * cc.max_seq_len * vb;
    unsigned char *hks = malloc(ks), *hvs = malloc(vs);
    CK(cudaMemcpy(hks, (unsigned char *)cc.d_k_cache + il * ks, ks, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(hvs, (unsigned char *)cc.d_v_cache + il * vs, vs, cudaMemcpyDeviceToHost));

    FILE *f = fopen(argv[1], "wb");
    if (!f) return 3;
    const int32_t hdr[8] = {L, H, G, HD, T, cc.max_seq_len, (int32_t)kb, (int32_t)vb};
    fwrite(hdr, 4, 8, f);
    fwrite(&scale, 4, 1, f);
    for (int g = 0; g < NQ; g++) fwrite(hq + g * q_row, 4, HD, f);
    for (int g = 0; g < NQ; g++) fwrite(ho + g * o_row, 4, HD, f);
    fwrite(hks, 1, ks, f);
    fwrite(hvs, 1, vs, f);
    fclose(f);
    sp_cuda_cache_free(&cc);
    printf("GGML_DECODE_OK\n");
    return 0;
}
