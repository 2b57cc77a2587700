// sp_ggml.cu — the fused decode behind ggml's tensor conventions, for a
// ggml-cuda backend op that replaces the attention subgraph the reference
// patches (patches/llama-cpp-b8861-full-engine.patch:393-410: kq =
// ggml_map_custom2(q, k, llama_sp_kq_compute) in build_attn_mha, then
// ggml's soft_max_ext(kq_scale) and mul_mat(v, kq)).
//
// The reference op runs on the CPU inside ggml's graph and produces scores
// only; here one call produces the attention output of every query head of
// one layer for one decode token, straight from the compressed slots: the
// queries are read through the Q view's byte strides (F32 or F16), staged
// as fp16 in the cache's scratch, attended by the fused decode
// (sp_cuda_attn_decode), and written through the output view's strides in
// its type.  Tensor shapes follow build_attn_mha after its permutes:
//   q    ne = {head_dim, n_tokens = 1, n_head_q, 1}     (q->nb in bytes)
//   dst  ne = {head_dim, n_head_q,     n_tokens = 1, 1} (kqv before cont_2d)
// GQA maps query head g to KV head g / (n_head_q / n_heads_kv), as ggml's
// broadcasting mul_mat does.
#include "sp_internal.cuh"
#include "shannon_prime_ggml.h"

namespace {

constexpr int kGgmlF32 = 0;   // GGML_TYPE_F32
constexpr int kGgmlF16 = 1;   // GGML_TYPE_F16

__global__ void k_ggml_gather_q(const unsigned char *q, int type, long long nb0, long long nb2, int hd, int nq,
                                __half *out)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= hd * nq) return;
    const int g = i / hd, d = i - g * hd;
    const unsigned char *p = q + (long long)g * nb2 + (long long)d * nb0;
    out[i] = type == kGgmlF32 ? __float2half_rn(*reinterpret_cast<const float *>(p))
                              : *reinterpret_cast<const __half *>(p);
}

__global__ void k_ggml_scatter_out(const __half *in, int type, long long nb0, long long nb1, int hd, int nq,
                                   unsigned char *dst)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= hd * nq) return;
    const int g = i / hd, d = i - g * hd;
    unsigned char *p = dst + (long long)g * nb1 + (long long)d * nb0;
    if (type == kGgmlF32) *reinterpret_cast<float *>(p) = __half2float(in[i]);
    else *reinterpret_cast<__half *>(p) = in[i];
}

bool aligned_view(const void *data, int type, long long nb0, long long nbx)
{
    const long long el = type == kGgmlF32 ? 4 : 2;
    return ((uintptr_t)data % el) == 0 && nb0 % el == 0 && nbx % el == 0;
}

}  // namespace

extern "C" int sp_ggml_attn_decode(const sp_cuda_cache_t *cc, int il, const void *q_data, int q_type,
                                   const int64_t q_ne[4], const size_t q_nb[4], void *dst_data, int dst_type,
                                   const int64_t dst_ne[4], const size_t dst_nb[4], float kq_scale, int n_kv,
                                   int max_bands, void *stream)
{
    sp_clear_error();
    if (!cc || !cc->d_scratch || !q_data || !dst_data || !q_ne || !q_nb || !dst_ne || !dst_nb)
        return sp_set_error(SP_ERR_ARG, "ggml_attn_decode: NULL argument");
    const int hd = cc->config.head_dim;
    if ((q_type != kGgmlF32 && q_type != kGgmlF16) || (dst_type != kGgmlF32 && dst_type != kGgmlF16))
        return sp_set_error(SP_ERR_UNSUPPORTED, "ggml_attn_decode: q/dst types must be F32 or F16");
    if (q_ne[0] != hd || q_ne[1] != 1 || q_ne[3] != 1)
        return sp_set_error(SP_ERR_ARG, "ggml_attn_decode: q must be {head_dim, 1 token, n_head_q, 1}");
    const int nq = (int)q_ne[2];
    if (dst_ne[0] != hd || dst_ne[1] != nq || dst_ne[2] != 1 || dst_ne[3] != 1)
        return sp_set_error(SP_ERR_ARG, "ggml_attn_decode: dst must be {head_dim, n_head_q, 1, 1}");
    if (nq <= 0 || nq > 8 * cc->config.n_heads_kv)
        return sp_set_error(SP_ERR_ARG, "ggml_attn_decode: %d query heads", nq);
    if (!aligned_view(q_data, q_type, (long long)q_nb[0], (long long)q_nb[2]) ||
        !aligned_view(dst_data, dst_type, (long long)dst_nb[0], (long long)dst_nb[1]))
        return sp_set_error(SP_ERR_ARG, "ggml_attn_decode: misaligned view");
    if (cudaSetDevice(cc->device) != cudaSuccess) return sp_set_error(SP_ERR_CUDA, "ggml_attn_decode: cudaSetDevice");
    cudaStream_t s = (cudaStream_t)stream;
    __half *sq = reinterpret_cast<__half *>(cc->d_scratch);
    __half *so = sq + (size_t)8 * cc->config.n_heads_kv * hd;
    const int n = hd * nq;
    k_ggml_gather_q<<<(n + 255) / 256, 256, 0, s>>>((const unsigned char *)q_data, q_type, (long long)q_nb[0],
                                                     (long long)q_nb[2], hd, nq, sq);
    int rc = sp_check_cuda(cudaGetLastError(), "ggml_attn_decode gather");
    if (rc) return rc;
    rc = sp_cuda_attn_decode(cc, il, 1, sq, nq, n_kv, kq_scale, so, max_bands, stream);
    if (rc) return rc;
    k_ggml_scatter_out<<<(n + 255) / 256, 256, 0, s>>>(so, dst_type, (long long)dst_nb[0], (long long)dst_nb[1],
                                                        hd, nq, (unsigned char *)dst_data);
    return sp_check_cuda(cudaGetLastError(), "ggml_attn_decode scatter");
}
