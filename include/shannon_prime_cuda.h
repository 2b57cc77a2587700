/*
 * shannon_prime_cuda.h — C-ABI of the B200 (sm_100a) Shannon-Prime KV-cache
 * hot path.
 *
 * Drop-in for the reference's CUDA C-ABI src/backends/cuda/shannon_prime_cuda.h
 * (names, argument meaning and the caller-visible struct fields are kept:
 * k_bands.total_bytes, stream, d_k_cache, d_v_cache, d_mobius_order,
 * max_seq_len are read by the reference engine at src/engine/kv_cache.cpp:
 * 638, 1034, 1378-1383, 1457-1459).  The reference functions return void and
 * fail silently; here every void entry point records its status, readable
 * with sp_cuda_last_error(), and every new entry point returns it (0 = ok).
 *
 * All device pointers are plain CUDA device addresses; "stream" is a
 * cudaStream_t passed as void*.  Work is stream-ordered; no entry point
 * below allocates device memory after sp_cuda_cache_init, and none
 * synchronises the stream unless it says so.
 *
 * Cache layout (as the reference, shannon_prime_cuda.cu:494-497): slot-major
 * [n_layers * n_heads_kv][max_seq_len][total_bytes], slot = layer*H + head.
 * sp_cuda_cache_init rounds max_seq_len up to a multiple of 16 and stores the
 * rounded value, so every 16-position tile of every slot starts on a 16-byte
 * boundary (the fused decode kernels stage tiles with bulk copies).
 */
#ifndef SHANNON_PRIME_CUDA_H
#define SHANNON_PRIME_CUDA_H

#include "shannon_prime.h"

#include <stdbool.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by the int entry points / sp_cuda_last_error(). */
#define SP_OK              0
#define SP_ERR_ARG        -1   /* invalid argument, shape or range */
#define SP_ERR_CUDA       -2   /* a CUDA runtime call failed */
#define SP_ERR_UNSUPPORTED -3  /* configuration this build does not implement */
#define SP_ERR_TIMEOUT    -4   /* a bounded device-side wait gave up */

/* Element types for the token-major write entry point. */
#define SP_DTYPE_F32  0
#define SP_DTYPE_F16  1
#define SP_DTYPE_BF16 2

typedef struct {
    /* --- fields of the reference struct (shannon_prime_cuda.h:29-46) --- */
    sp_config_t      config;
    sp_band_config_t k_bands;
    sp_band_config_t v_bands;
    void            *d_k_cache;      /* [n_slots][max_seq_len][k_bands.total_bytes] */
    void            *d_v_cache;      /* [n_slots][max_seq_len][v_bands.total_bytes] */
    int              max_seq_len;
    int             *d_mobius_order; /* [head_dim] forward permutation (NULL: Möbius off) */
    int             *d_mobius_inv;   /* [head_dim] inverse permutation */
    float           *d_scratch;      /* at least [head_dim] floats (the reference's size); here the
                                        fp16 query/output staging of sp_ggml_attn_decode */
    void            *stream;

    /* --- B200 build additions --- */
    int              n_slots;        /* n_layers * n_heads_kv */
    int              device;         /* CUDA device the cache lives on */
    void            *d_attn_ws;      /* split-K partials of the fused decode */
    size_t           attn_ws_bytes;
    int              attn_max_q_heads; /* q heads per layer the workspace is sized for */
    int              attn_ws_layers;   /* layers per call the workspace is sized for */
    unsigned int    *d_status;       /* device-side error word: bit 0 a bounded copy wait ran
                                        out, bit 1 the cross-GPU gather wait ran out, bit 2 a
                                        lane kernel found its shared memory misaligned for the
                                        128-byte swizzle and wrote nothing */
} sp_cuda_cache_t;

/* ------------------------------------------------------------ lifecycle -- */

/* Replaces reference sp_cuda_cache_init (shannon_prime_cuda.h:50-51,
 * shannon_prime_cuda.cu:407-463).  Allocates the cache slabs, the Möbius
 * tables and the fused-decode workspace (sized for up to 8 query heads per
 * KV head and all layers).  Returns 0 or an SP_ERR_* code. */
int  sp_cuda_cache_init(sp_cuda_cache_t *cc, const sp_config_t *cfg,
                        int max_seq_len, void *stream);
/* Replaces reference sp_cuda_cache_free (shannon_prime_cuda.h:52). */
void sp_cuda_cache_free(sp_cuda_cache_t *cc);

/* ------------------------------------------------------------ write path -- */
/* VHT2 -> Möbius reorder (K) -> band quantise -> store.  Packed codes are
 * bit-identical to the CPU restatement of the core path. */

/* Reference shannon_prime_cuda.h:60-66 (single vector, device pointer). */
void sp_cuda_write_k(sp_cuda_cache_t *cc, int layer, int head, int pos,
                     const float *d_k_vec);
void sp_cuda_write_v(sp_cuda_cache_t *cc, int layer, int head, int pos,
                     const float *d_v_vec);

/* Reference shannon_prime_cuda.h:89-97: d_vecs is [n_pos][head_dim]. */
void sp_cuda_write_k_batch(sp_cuda_cache_t *cc, int layer, int head,
                           int start_pos, int n_pos, const float *d_k_vecs);
void sp_cuda_write_v_batch(sp_cuda_cache_t *cc, int layer, int head,
                           int start_pos, int n_pos, const float *d_v_vecs);

/* New: one launch for every head of a layer, K and V together, in the
 * engine's token-major layout [n_tokens][n_heads_kv][head_dim] (the layout
 * KvCache::write_gpu walks vector by vector, kv_cache.cpp:1045-1091).
 * d_k or d_v may be NULL to skip that half.  dtype is SP_DTYPE_*. */
int  sp_cuda_write_kv_tokens(sp_cuda_cache_t *cc, int layer, int start_pos,
                             int n_tokens, const void *d_k, const void *d_v,
                             int dtype);

/* ------------------------------------------------------------- read path -- */
/* dequantise -> Möbius unreorder (K) -> VHT2 -> fp32. */

/* Reference shannon_prime_cuda.h:75-81. */
void sp_cuda_read_k(const sp_cuda_cache_t *cc, int layer, int head, int pos,
                    float *d_k_out);
void sp_cuda_read_v(const sp_cuda_cache_t *cc, int layer, int head, int pos,
                    float *d_v_out);

/* Reference shannon_prime_cuda.h:100-108: output [n_pos][head_dim]. */
void sp_cuda_read_k_batch(const sp_cuda_cache_t *cc, int layer, int head,
                          int start_pos, int n_pos, float *d_k_out);
void sp_cuda_read_v_batch(const sp_cuda_cache_t *cc, int layer, int head,
                          int start_pos, int n_pos, float *d_v_out);

/* New: partial-band read (semantics of sp_llama_read_k_partial,
 * shannon_prime_llama.h:240-255: bands >= max_bands read as zero;
 * max_bands < 0 or >= n_bands is a full read).  which: 0 = K, 1 = V. */
int  sp_cuda_read_batch_partial(const sp_cuda_cache_t *cc, int which,
                                int layer, int head, int start_pos, int n_pos,
                                float *d_out, int max_bands);

/* New: token-major read of every KV head of a layer range in one launch
 * (replaces the per-head loop of KvCache::read_gpu,
 * src/engine/kv_cache.cpp:1100-1228): which 0 = K, 1 = V; positions
 * [start_pos, start_pos + n_tok) of layers [layer0, layer0 + n_layers) go
 * to d_out as fp32 [n_layers][n_tok][n_heads_kv][head_dim], rows equal to
 * those of sp_cuda_read_batch_partial (same max_bands meaning).  The
 * head_dim-128 ship layouts only (K 5/5/4/3 with the squarefree-first
 * order, V 3-bit; d_out 16-byte aligned); other caches return
 * SP_ERR_UNSUPPORTED.  Stream-ordered on cc->stream, allocates nothing. */
int  sp_cuda_read_kv_tokens(const sp_cuda_cache_t *cc, int which, int layer0, int n_layers,
                            int start_pos, int n_tok, float *d_out, int max_bands);

/* -------------------------------------------------- fused decode attention -- */
/* New (no reference GPU counterpart; replaces the CPU ggml op
 * llama_sp_kq_compute, src/engine/llama_sp_fused_kq.cpp:82-165, plus the
 * softmax and V product that ggml runs after it).
 *
 * For layers [layer0, layer0+n_layers) and every query head g (KV head
 * g / (n_q_heads / n_heads_kv)):
 *     out[l][g] = softmax(logit_scale * q[l][g] . K_hat[l][h][0:kv_len]) . V_hat[l][h]
 * where K_hat, V_hat are the decompressed cache rows.  Neither K_hat nor
 * V_hat is materialised: scores are taken in the VHT2 coefficient domain
 * against the packed codes and V is accumulated in that domain and
 * transformed once per head.
 *   d_q   : fp16 [n_layers][n_q_heads][head_dim]
 *   d_out : fp16 [n_layers][n_q_heads][head_dim]
 * n_q_heads must be a multiple of n_heads_kv with at most 8 queries per KV
 * head.  max_bands limits the K and V bands read (-1 = all; the partial-read
 * rule above).  kv_len == 0 writes zeros. */
int  sp_cuda_attn_decode(const sp_cuda_cache_t *cc, int layer0, int n_layers,
                         const void *d_q, int n_q_heads, int kv_len,
                         float logit_scale, void *d_out, int max_bands,
                         void *stream);

/* Replaces the CPU ggml custom2 op llama_sp_kq_compute
 * (src/engine/llama_sp_fused_kq.cpp:82-165, userdata llama_sp_kq_userdata,
 * src/engine/llama_sp_fused_kq.h:45-56) on the GPU: for one head's packed
 * rows (d_packed = k_packed_buf_per_head, [n_kv][total_bytes_per_pos];
 * is_v selects the V layout) and n_head_q query rows (d_q, f32 or f16,
 * q_row_stride bytes apart = Q's nb[1]), writes the fp32 scores
 * dst[qh][kv] = dot(decompressed row kv, q row qh) at d_dst + qh *
 * dst_row_stride bytes (= dst's nb[1]), as the reference op does for all of
 * its ith/nth slices at once.  Ship rows at head_dim 128 only (K 76 B with
 * the squarefree-first order, V 50 B), at most 64 query rows; other shapes
 * return SP_ERR_UNSUPPORTED.  Stream-ordered, allocates nothing. */
int  sp_cuda_kq_scores(const void *d_packed, int total_bytes_per_pos, int is_v, int head_dim,
                       int n_kv, const void *d_q, int q_dtype, long long q_row_stride,
                       int n_head_q, float *d_dst, long long dst_row_stride, void *stream);

/* New: the same op over n_slots slots in one launch (slot i reads
 * d_packed + i * packed_slot_stride, its query rows at d_q + i *
 * q_slot_stride and writes dst rows at d_dst + i * dst_slot_stride, all in
 * bytes), e.g. every (layer, KV head) of a cache with the slot stride
 * max_seq_len * total_bytes_per_pos.  The reference calls its op once per
 * head; one launch per step avoids a launch per slot.  At most 65535 slots. */
int  sp_cuda_kq_scores_strided(const void *d_packed, long long packed_slot_stride, int n_slots,
                               int total_bytes_per_pos, int is_v, int head_dim, int n_kv,
                               const void *d_q, int q_dtype, long long q_row_stride,
                               long long q_slot_stride, int n_head_q, float *d_dst,
                               long long dst_row_stride, long long dst_slot_stride, void *stream);

/* New; no counterpart in the reference.  The fused decode above for callers
 * that cannot allocate device memory (an engine that owns every device
 * buffer through its own allocator, such as llama.cpp's ggml backend
 * buffers, or a plugin host that forbids a library from growing its device
 * footprint).  Same arguments and results as sp_cuda_attn_decode, but the
 * cache is described by plain pointers the caller owns (layout as above:
 * slot = layer * n_heads_kv + head, slot stride max_seq_len * total_bytes;
 * d_mobius_order = head_dim ints on the device, or NULL for no reorder) and
 * the split partials live in a fixed 16 MiB device array inside this
 * library instead of a cudaMalloc'd workspace.  Nothing is allocated.
 *   Limit: n_layers * n_q_heads * 128 * (head_dim + 4) * 4 bytes must fit in
 *   16 MiB (at head_dim 128: n_layers * n_q_heads <= 248, e.g. one layer of a
 *   32-head model per call); larger requests return SP_ERR_ARG.
 *   The first call on each device looks up the array's device address
 *   (cudaGetSymbolAddress); make it before any stream capture.  All calls
 *   share the array, so calls that overlap on the GPU race: serialise them.
 *   The addresses are kept for the life of the process: a cudaDeviceReset
 *   after the first call on a device is not supported.
 *   Failures inside the kernels (a bounded copy wait that ran out) set bit 0
 *   of a status word that all calls on the device share, like the array;
 *   read it with sp_cuda_attn_decode_noalloc_status. */
int  sp_cuda_attn_decode_noalloc(const void *d_k_cache, const void *d_v_cache,
                                 int max_seq_len, const sp_band_config_t *k_bands,
                                 const sp_band_config_t *v_bands,
                                 const int *d_mobius_order, int n_heads_kv,
                                 int layer0, int n_layers, const void *d_q,
                                 int n_q_heads, int kv_len, float logit_scale,
                                 void *d_out, int max_bands, void *stream);
/* New: the shared status word of sp_cuda_attn_decode_noalloc on the current
 * device, read after the stream's work (synchronises `stream`); clear != 0
 * resets it to 0 afterwards.  Allocates nothing. */
int  sp_cuda_attn_decode_noalloc_status(unsigned int *status_out, int clear, void *stream);

/* ------------------------------------------------- sqfree + spinor cache -- */
/* Replaces reference sp_cuda_sqfree_cache_t (shannon_prime_cuda.h:153-230,
 * src/backends/cuda/shannon_prime_sqfree.cu:585-1122).  Per position and
 * K/V half the slot holds [skeleton bands][fp32 magnitude][residual levels,
 * LSB-first][spinor sheet bits] (shannon_prime_sqfree.cu:683-686):
 *   pad head_dim -> pad_dim (squarefree, {2,3,5,7,11}-smooth; 154 at 128)
 *   with the mean, Vilenkin (staged prime Hartley) transform, keep sk_k
 *   skeleton coefficients (band-quantised), predict the n_res others from
 *   the skeleton by a Möbius CSR sum, store the (spinor-signed) deviation
 *   with residual_bits per coefficient.
 * The reference's fields are kept; its per-call scratch buffers are not
 * needed (every kernel here keeps its intermediates on chip) and stay NULL. */
typedef struct {
    sp_config_t      config;
    int              pad_dim;
    int              sk_k;
    int              n_res;
    int              n_terms;
    int              residual_bits;
    int              use_spinor;
    int              use_skel_mobius;   /* unused, as in the reference */
    sp_band_config_t k_bands;           /* over the sk_k skeleton values */
    sp_band_config_t v_bands;
    int             *d_skeleton_idx;    /* [sk_k] */
    int             *d_residual_idx;    /* [n_res] */
    int             *d_csr_offsets;     /* [n_res + 1] */
    int             *d_csr_skel_slot;   /* [n_terms] */
    int             *d_csr_mu_sign;     /* [n_terms], +1 / -1 */
    int             *d_vilenkin_factors;
    int              n_factors;
    unsigned char   *d_k_cache;         /* [n_slots][max_seq_len][bytes_per_pos_k] */
    unsigned char   *d_v_cache;
    int              bytes_per_pos_k;
    int              bytes_per_pos_v;
    int              max_seq_len;
    int              n_slots;
    float           *d_pad_scratch;     /* unused (NULL) */
    float           *d_coeff_scratch;
    float           *d_skel_scratch;
    float           *d_pred_scratch;
    float           *d_dev_scratch;
    unsigned char   *d_levels_scratch;
    float           *d_mag_scratch;
    float           *d_actual_scratch;
    unsigned char   *d_sheet_scratch;
    void            *stream;
    /* --- B200 build additions --- */
    int              device;
    void            *d_tables;          /* packed kernel tables (indices, CSR, cas) */
    void            *d_attn_ws;         /* fused-decode partials */
    size_t           attn_ws_bytes;
    int              csr_max_terms;     /* most Möbius terms of one residual */
    int              lane_max_terms;    /* most Möbius terms of one lane under the balanced
                                           residual-to-lane assignment of the blocked decode
                                           (0: the assignment needs more than 2 residuals per lane) */
} sp_cuda_sqfree_cache_t;

/* Reference signature; the skeleton is pad_dim / 2 as in the reference CUDA
 * cache (shannon_prime_sqfree.cu:606).  Returns 0 or SP_ERR_*. */
int  sp_cuda_sqfree_cache_init(sp_cuda_sqfree_cache_t *cc, const sp_config_t *cfg,
                               int max_seq_len, int residual_bits, int use_spinor,
                               void *stream);
/* New: skeleton = floor(sk_frac * pad_dim) (the bridge's SHANNON_PRIME_SK_FRAC,
 * shannon_prime_llama_sqfree.c:68-71, which the reference parses but never
 * passes on). */
int  sp_cuda_sqfree_cache_init_ex(sp_cuda_sqfree_cache_t *cc, const sp_config_t *cfg,
                                  int max_seq_len, int residual_bits, int use_spinor,
                                  float sk_frac, void *stream);
void sp_cuda_sqfree_cache_free(sp_cuda_sqfree_cache_t *cc);
/* Reference shannon_prime_cuda.h:185-220 (device vectors of head_dim). */
void sp_cuda_sqfree_write_k(sp_cuda_sqfree_cache_t *cc, int layer, int head, int pos,
                            const float *d_k_vec);
void sp_cuda_sqfree_write_v(sp_cuda_sqfree_cache_t *cc, int layer, int head, int pos,
                            const float *d_v_vec);
void sp_cuda_sqfree_read_k(const sp_cuda_sqfree_cache_t *cc, int layer, int head, int pos,
                           float *d_k_out);
void sp_cuda_sqfree_read_v(const sp_cuda_sqfree_cache_t *cc, int layer, int head, int pos,
                           float *d_v_out);
void sp_cuda_sqfree_read_k_batch(const sp_cuda_sqfree_cache_t *cc, int layer, int head,
                                 int start_pos, int n_pos, float *d_k_out);
void sp_cuda_sqfree_read_v_batch(const sp_cuda_sqfree_cache_t *cc, int layer, int head,
                                 int start_pos, int n_pos, float *d_v_out);

/* New: token-major read of every KV head of a layer range in one launch
 * (which 0 = K, 1 = V): positions [start_pos, start_pos + n_tok) of layers
 * [layer0, layer0 + n_layers) to d_out as fp32
 * [n_layers][n_tok][n_heads_kv][head_dim], rows equal to those of the
 * per-slot batch reads.  The head_dim-128 spinor layout with 3-bit
 * residuals (pad 154, skeleton in 5 bands) and a 16-byte aligned d_out;
 * other caches return SP_ERR_UNSUPPORTED.  Allocates nothing. */
int  sp_cuda_sqfree_read_kv_tokens(const sp_cuda_sqfree_cache_t *cc, int which, int layer0,
                                   int n_layers, int start_pos, int n_tok, float *d_out);
/* New: token-major write of every head of layers [layer0, layer0+n_layers):
 * d_k / d_v are [n_layers][n_tokens][n_heads_kv][head_dim] (NULL skips). */
int  sp_cuda_sqfree_write_kv_tokens(sp_cuda_sqfree_cache_t *cc, int layer0, int n_layers,
                                    int start_pos, int n_tokens, const void *d_k,
                                    const void *d_v, int dtype);
/* New: fused decode attention over the sqfree cache, same contract as
 * sp_cuda_attn_decode (fp16 q/out [n_layers][n_q_heads][head_dim], at most
 * 8 query heads per KV head); scores and the V sum are taken in the
 * Vilenkin coefficient domain, one inverse transform per query head. */
int  sp_cuda_sqfree_attn_decode(const sp_cuda_sqfree_cache_t *cc, int layer0, int n_layers,
                                const void *d_q, int n_q_heads, int kv_len, float logit_scale,
                                void *d_out, void *stream);

/* ------------------------------------------- hierarchical Vilenkin cache -- */
/* Replaces reference sp_cuda_hier_cache_t (shannon_prime_cuda.h:300-377,
 * shannon_prime_hier.cu:272-601).  Slot: [skeleton bands][fp32 magnitude]
 * [target residual levels]; targets are predicted as W_slot . skeleton with
 * a per-slot fp16 W [n_target][n_skeleton] uploaded after calibration. */
typedef struct {
    sp_config_t      config;
    int              pad_dim;
    int              n_skeleton;
    int              n_target;
    int              target_res_bits;
    int              n_slots;
    int              max_seq_len;
    uint16_t        *d_W;               /* [n_slots][n_target][n_skeleton] fp16 */
    int             *d_skeleton_idx;    /* [n_skeleton] */
    int             *d_target_idx;      /* [n_target] */
    int             *d_vilenkin_factors;
    int              n_factors;
    sp_band_config_t skel_bands;
    int             *d_skel_band_bits;
    unsigned char   *d_k_cache;
    unsigned char   *d_v_cache;
    int              bytes_per_pos_k;
    int              bytes_per_pos_v;
    float           *d_pad_scratch;     /* unused (NULL) */
    float           *d_coeff_scratch;
    float           *d_skel_scratch;
    float           *d_pred_scratch;
    float           *d_dev_scratch;
    float           *d_mag_scratch;
    unsigned char   *d_levels_scratch;
    void            *stream;
    /* --- B200 build additions --- */
    int              device;
    void            *d_tables;
    float           *d_vrows;           /* [head_dim][pad_dim] rows of the transform matrix */
    void            *d_recon;           /* [n_slots][head_dim][K + 8] fp16 reconstruction matrices
                                           of the tensor-core batched read (NULL: not used) */
    unsigned int    *d_status;          /* device error word: bit 0 a bounded wait of the tcgen05
                                           read ran out (its tiles are missing from the output) */
} sp_cuda_hier_cache_t;

/* Reference shannon_prime_cuda.h:337-349 (caller supplies the index sets and
 * the skeleton band layout). */
int  sp_cuda_hier_cache_init(sp_cuda_hier_cache_t *hc, const sp_config_t *cfg,
                             int pad_dim, int n_skeleton, int n_target, int target_res_bits,
                             const int *skeleton_idx, const int *target_idx,
                             const sp_band_config_t *skel_bands, int max_seq_len, int n_slots,
                             void *stream);
void sp_cuda_hier_cache_free(sp_cuda_hier_cache_t *hc);
/* Reference shannon_prime_cuda.h:354-355: W_all [n_slots][n_target][n_skeleton] fp16. */
int  sp_cuda_hier_cache_upload_W(sp_cuda_hier_cache_t *hc, const uint16_t *W_all);
void sp_cuda_hier_write_k(sp_cuda_hier_cache_t *hc, int layer, int head, int pos,
                          const float *d_k_vec);
void sp_cuda_hier_write_v(sp_cuda_hier_cache_t *hc, int layer, int head, int pos,
                          const float *d_v_vec);
void sp_cuda_hier_read_k(const sp_cuda_hier_cache_t *hc, int layer, int head, int pos,
                         float *d_k_out);
void sp_cuda_hier_read_v(const sp_cuda_hier_cache_t *hc, int layer, int head, int pos,
                         float *d_v_out);
/* New: batched compress of layers [layer0, layer0+n_layers) in one call,
 * inputs [n_layers][n_tokens][n_heads_kv][head_dim] (f32/f16/bf16). */
int  sp_cuda_hier_write_kv_tokens(sp_cuda_hier_cache_t *hc, int layer0, int n_layers,
                                  int start_pos, int n_tokens, const void *d_k,
                                  const void *d_v, int dtype);
/* New: batched decompress, outputs fp32 [n_layers][n_pos][n_heads_kv][head_dim]. */
int  sp_cuda_hier_read_kv_tokens(const sp_cuda_hier_cache_t *hc, int layer0, int n_layers,
                                 int start_pos, int n_pos, float *d_k_out, float *d_v_out);

/* ----------------------------------------- kernel launchers (for tests) -- */

/* New: fused decode + all-gather over peer memory, for a cache sharded over
 * the GPUs of one node (one process per GPU).  Runs the same decode as
 * sp_cuda_attn_decode on this rank's (layer, KV head) slots; the combine
 * kernel then stores every fp16 output row directly into each rank's gather
 * buffer (NVLink peer stores), at row
 *     d_dst_layer[l] * n_q_heads_total + d_dst_qhead[h]   (rows of head_dim fp16)
 * for local layer l and local query head h, and its last block writes `epoch`
 * into uint32 slot `rank` of the flag array at byte flags_offset of every
 * buffer, then waits (bounded, 2 s) until all `world` slots of this rank's
 * own flag array reach `epoch`; stream work after the call sees the whole
 * gathered output.
 *   epoch_stride   bytes between two copies of the gathered rows in each
 *                  buffer: the rows of call `epoch` start at byte
 *                  (epoch & 1) * epoch_stride.  With two copies a rank may
 *                  issue call e+1 while a slower rank still reads call e's
 *                  rows (each rank's reads of call e must be stream-ordered
 *                  before its own call e+1, which is what raises its flag
 *                  for e+1, and no rank passes call e+1's wait before all
 *                  flags show e+1).  0 = one copy: the caller must then keep
 *                  every rank from starting call e+1 until all ranks have
 *                  consumed call e (a barrier).
 *   d_local_buf    this rank's gather buffer
 *   d_peer_bufs    device array [world] of every rank's buffer as mapped in
 *                  this process (its own at index rank), e.g. from CUDA IPC or
 *                  symmetric memory
 *   d_dst_layer    device int [n_layers];  d_dst_qhead: device int [n_q_heads]
 *   epoch          increases by one per call (flags are never reset)
 * A wait that runs out sets bit 1 of the cache's d_status word.  Calls on one
 * cache must not overlap on the GPU. */
int sp_cuda_attn_decode_allgather(const sp_cuda_cache_t *cc, int layer0, int n_layers, const void *d_q,
                                  int n_q_heads, int kv_len, float logit_scale, int max_bands,
                                  void *d_local_buf, void *const *d_peer_bufs, const int *d_dst_layer,
                                  const int *d_dst_qhead, int n_q_heads_total, long long flags_offset,
                                  long long epoch_stride, int rank, int world, unsigned int epoch,
                                  void *stream);

/* ---------------------------------------------------------------------------
 * Cold storage: per-layer pinned host mirror of a cache slab (the warm tier
 * of the reference's GPU <-> CPU <-> disk offload, shannon_prime_cuda.h:233-286,
 * called by src/engine/kv_cache.cpp:1401-1520).
 *
 * A layer slab is the n_heads_kv * max_seq_len * packed_stride bytes of one
 * layer in d_k_cache or d_v_cache.  Writebacks mirror byte ranges of the slab:
 * positions [start_pos, start_pos + n_pos) cover slab bytes
 * [start_pos, start_pos + n_pos) * n_heads * packed_stride, appended at
 * write_head of the pinned buffer; a range that does not fit wraps the buffer
 * to offset 0 (ring mode).  A restore copies the first n_pos * n_heads *
 * packed_stride bytes of the buffer back to the start of the slab, and is
 * refused once the buffer has wrapped.  Copies are async on `stream`.
 * ------------------------------------------------------------------------- */
typedef struct {
    uint8_t *h_pinned;           /* page-locked staging buffer (capacity bytes) */
    int64_t  capacity;
    int      packed_stride;      /* bytes per position per head */
    int      n_heads;
    int64_t  write_head;         /* byte offset of the next writeback */
    int64_t  oldest_pos;         /* oldest position held (-1: none yet) */
    int64_t  newest_pos;         /* newest position written */
    bool     ring_mode;          /* the buffer has wrapped */
    bool     initialized;
} sp_cuda_cold_layer_t;

/* 0 on success, -1 on bad arguments or a failed page-locked allocation. */
int  sp_cuda_cold_layer_init(sp_cuda_cold_layer_t *cl, int64_t cap_bytes, int packed_stride, int n_heads);
void sp_cuda_cold_layer_free(sp_cuda_cold_layer_t *cl);
/* Async device -> host copy of positions [start_pos, start_pos + n_pos) of a
 * layer slab (d_packed = the slab's device address).  0 on success, -1 on bad
 * arguments or a range larger than the buffer. */
int  sp_cuda_cold_writeback(sp_cuda_cold_layer_t *cl, const void *d_packed, int start_pos, int n_pos,
                            void *stream);
/* Async host -> device copy of positions [0, n_pos) back to the slab start.
 * -1 in ring mode, on bad arguments, or for more bytes than the buffer holds. */
int  sp_cuda_cold_restore(const sp_cuda_cold_layer_t *cl, void *d_packed, int n_pos, void *stream);
/* Async copies of arbitrary buffers on `stream`. */
void sp_cuda_d2h_async(void *dst_host, const void *src_device, int64_t n_bytes, void *stream);
void sp_cuda_h2d_async(void *dst_device, const void *src_host, int64_t n_bytes, void *stream);

/* ---------------------------------------------------------------------------
 * System 1 <-> 2 dual cache: merged read on the GPU, replacing
 * DualKvCache::read_merged_gpu (src/engine/kv_cache.cpp:1832-1860), which
 * reads System 1 for every position and leaves the System 2 positions
 * unmerged on the GPU.  Rows of row_floats floats: row p of d_out is row p
 * of d_sys2 when bit p of d_route_bits (uint32 words, bit p%32 of word p/32)
 * is set, else row p of d_sys1.  d_out may be d_sys1 (then only the System 2
 * rows are written).  One launch, stream-ordered; allocates nothing. */
int sp_cuda_dual_merge(const float *d_sys1, const float *d_sys2, const uint32_t *d_route_bits,
                       int n_pos, int row_floats, float *d_out, void *stream);

/* ---------------------------------------------------------------------------
 * Disk tier: save / load of a ship cache's compressed slabs, replacing the
 * engine's KvCache::save_to_disk / load_from_disk / load_from_disk_partial
 * (src/engine/kv_cache.h:133-147, kv_cache.cpp:1535-1585, which call the
 * core's sp_shadow_cache_save / _load / _load_partial, CHANGELOG.md:41-61).
 * One file per layer, {prefix}.L{layer}.bin: a 64-byte header ("VHT2",
 * version, model hash, n_pos, shape and band layout, header checksum), then
 * the layer's K rows and V rows of positions [0, n_pos):
 *   version 2  per-vector interleaved ([head][pos][row bytes]);
 *   version 3  band-major ([band][head][pos][band bytes]), so a partial load
 *              reads only the first max_bands bands from disk.
 * model_hash: the caller's FNV-1a 64 hash of the model path (sp_fnv1a64).
 * Loads check the header against the cache's shape and layout, and the hash
 * strictly unless SP_DISK_HASH_STRICT=0 (then a mismatch only warns).
 * Save returns 0; load returns n_pos; errors return a negative SP_ERR_*.
 * Synchronous on the cache's stream; staging buffers are allocated per call. */
uint64_t sp_fnv1a64(const void *data, size_t n);
int sp_cuda_cache_save(const sp_cuda_cache_t *cc, const char *prefix, int n_pos, uint64_t model_hash,
                       int version);
int sp_cuda_cache_load(sp_cuda_cache_t *cc, const char *prefix, uint64_t expected_hash);
/* Bands at or beyond max_bands are not read (v3) and are stored as zeros, so
 * reads and the fused decode see exactly a partial-band read
 * (shannon_prime_llama.h:240-255); max_bands < 0 loads everything. */
int sp_cuda_cache_load_partial(sp_cuda_cache_t *cc, const char *prefix, uint64_t expected_hash,
                               int max_bands);


/* Reference shannon_prime_cuda.h:116-134.  In-place VHT2 of n_vecs
 * vectors (power-of-two n, 32 <= n <= SP_MAX_HEAD_DIM). */
void sp_cuda_vht2_forward(float *d_data, int n, int n_vecs, void *stream);
void sp_cuda_mobius_reorder(float *d_data, const int *d_order, int n,
                            int n_vecs, void *stream);
void sp_cuda_mobius_unreorder(float *d_data, const int *d_order, int n,
                              int n_vecs, void *stream);
void sp_cuda_band_quantize(const float *d_input, void *d_output,
                           const sp_band_config_t *bc, int n_vecs, void *stream);
void sp_cuda_band_dequantize(const void *d_input, float *d_output,
                             const sp_band_config_t *bc, int n_vecs, void *stream);

/* ----------------------------------------------------------- diagnostics -- */

/* Reference shannon_prime_cuda.h:141. */
void sp_cuda_print_memory(const sp_cuda_cache_t *cc);

/* New: status of the last call made on this host thread (SP_OK or SP_ERR_*)
 * and a message for it.  The void reference entry points report only here. */
int         sp_cuda_last_error(void);
const char *sp_cuda_last_error_string(void);

/* New: sizeof(sp_config_t) (which=0), sizeof(sp_band_config_t) (1),
 * sizeof(sp_cuda_cache_t) (2), sizeof(sp_cuda_sqfree_cache_t) (3),
 * sizeof(sp_cuda_hier_cache_t) (4), sizeof(sp_cuda_cold_layer_t) (5), so
 * bindings can check their mirrors. */
int sp_cuda_abi_struct_size(int which);

/* New, for tests and benchmarks: force the fused-decode kernel family
 * (0 = automatic, 1 = generic SIMT kernel, 2 = mma.sync tensor-core ship
 * kernel, 3 = tcgen05 ship kernel; 0 takes 2 where the layout allows, else
 * 1; 3 needs whole 128-position tiles inside each slot). */
void sp_cuda_attn_force_impl(int impl);

/* New, for benchmarks: when enabled, sp_cuda_attn_decode records CUDA events
 * around its main kernel on the caller's stream; sp_cuda_attn_last_kernel_ms
 * waits for the last one and returns its duration (-1 if none), and
 * sp_cuda_attn_last_splits the number of token chunks it used. */
void  sp_cuda_attn_profile(int enable);
float sp_cuda_attn_last_kernel_ms(void);
int   sp_cuda_attn_last_splits(void);

#ifdef __cplusplus
}
#endif

#endif /* SHANNON_PRIME_CUDA_H */
