// sp_disk.cu — disk tier of the ship cache: save / load of the compressed
// slabs in the reference's per-layer file scheme (src/engine/kv_cache.h:
// 133-147: files {prefix}.L{n}.bin, each with a 64-byte header carrying a
// magic, the format version, an FNV-1a model hash and n_pos; strict hash
// check with the SP_DISK_HASH_STRICT=0 escape, CHANGELOG.md:41-49) and its
// two body layouts (CHANGELOG.md:56-61):
//
//   v2  per-vector interleaved: the slab rows as they sit in HBM,
//       K [n_heads][n_pos][k_total_bytes] then V [n_heads][n_pos][v_total_bytes];
//   v3  band-major: for K then V, band b's bytes (its fp16 scale and codes)
//       of every (head, position) contiguous: [band][n_heads][n_pos][bytes_b],
//       so a partial load reads only the first max_bands regions from disk.
//
// The header's field layout belongs to the absent core library
// (sp_shadow_cache_save); the one here is this build's own (below).  On the
// GPU the band-major transpose and its inverse are one gather / scatter
// kernel over all rows of a layer; the host side is one file read or write
// per K/V region.  Not on the decode hot path: staging buffers are
// allocated per call.
#include "sp_internal.cuh"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

namespace {

// Header (64 bytes, little-endian):
//   0  char[4]  "VHT2"
//   4  u32      version (2 or 3)
//   8  u64      model hash (FNV-1a 64 of the model path, caller-supplied)
//  16  i32      n_pos      20 i32 head_dim   24 i32 n_heads_kv   28 i32 layer
//  32  u8       k_n_bands  33 u8 v_n_bands   34 u8 use_mobius    35 u8 0
//  36  u8[8]    K band bits, 4 bits each (band 2i low nibble)
//  44  u8[8]    V band bits, likewise
//  52  u32      k_total_bytes   56 u32 v_total_bytes
//  60  u32      FNV-1a 32 of bytes 0..59
constexpr int kHdrBytes = 64;

uint32_t fnv1a32(const unsigned char *p, size_t n)
{
    uint32_t h = 2166136261u;
    for (size_t i = 0; i < n; i++) { h ^= p[i]; h *= 16777619u; }
    return h;
}

void put32(unsigned char *p, uint32_t v) { memcpy(p, &v, 4); }
uint32_t get32(const unsigned char *p) { uint32_t v; memcpy(&v, p, 4); return v; }

void pack_header(unsigned char *h, const sp_cuda_cache_t *cc, int version, uint64_t hash, int n_pos, int layer)
{
    memset(h, 0, kHdrBytes);
    memcpy(h, "VHT2", 4);
    put32(h + 4, (uint32_t)version);
    memcpy(h + 8, &hash, 8);
    put32(h + 16, (uint32_t)n_pos);
    put32(h + 20, (uint32_t)cc->config.head_dim);
    put32(h + 24, (uint32_t)cc->config.n_heads_kv);
    put32(h + 28, (uint32_t)layer);
    h[32] = (unsigned char)cc->k_bands.n_bands;
    h[33] = (unsigned char)cc->v_bands.n_bands;
    h[34] = cc->config.use_mobius_mask ? 1 : 0;
    for (int b = 0; b < cc->k_bands.n_bands; b++) h[36 + b / 2] |= (unsigned char)(cc->k_bands.band_bits[b] << (4 * (b & 1)));
    for (int b = 0; b < cc->v_bands.n_bands; b++) h[44 + b / 2] |= (unsigned char)(cc->v_bands.band_bits[b] << (4 * (b & 1)));
    put32(h + 52, (uint32_t)cc->k_bands.total_bytes);
    put32(h + 56, (uint32_t)cc->v_bands.total_bytes);
    put32(h + 60, fnv1a32(h, 60));
}

// Byte span of band b in a packed row: [lo, lo + len).
void band_span(const SpBandLayout &bl, int b, int *lo, int *len)
{
    *lo = bl.byte_off[b];
    *len = 2 + (bl.size[b] * bl.bits[b] + 7) / 8;
}

struct BandSpans {
    int n_bands, row_bytes;
    int lo[SP_MAX_BANDS], len[SP_MAX_BANDS];
    long long region[SP_MAX_BANDS + 1];   // start of band b's region in the band-major buffer, in rows*len units summed
};

BandSpans spans_of(const SpBandLayout &bl, long long rows)
{
    BandSpans s;
    s.n_bands = bl.n_bands;
    s.row_bytes = bl.total_bytes;
    long long off = 0;
    for (int b = 0; b < bl.n_bands; b++) {
        band_span(bl, b, &s.lo[b], &s.len[b]);
        s.region[b] = off;
        off += rows * s.len[b];
    }
    s.region[bl.n_bands] = off;
    return s;
}

// Slab rows of one layer ([H][max_seq][row] with n_pos used) <-> band-major
// buffer ([band][H][n_pos][len_b]).  One thread per (row, band).  On the
// scatter, bands at or beyond max_bands are written as zero bytes (a zero
// fp16 scale reads back as an all-zero band, as a partial read does).
__global__ void k_band_gather(const uint8_t *slab, long long slot_stride, int n_pos, int H, BandSpans s,
                              uint8_t *out)
{
    const long long rows = (long long)H * n_pos;
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= rows * s.n_bands) return;
    const int b = (int)(i / rows);
    const long long r = i - (long long)b * rows;
    const int h = (int)(r / n_pos), p = (int)(r - (long long)h * n_pos);
    const uint8_t *src = slab + h * slot_stride + (long long)p * s.row_bytes + s.lo[b];
    uint8_t *dst = out + s.region[b] + r * s.len[b];
    for (int k = 0; k < s.len[b]; k++) dst[k] = src[k];
}

__global__ void k_band_scatter(const uint8_t *in, long long slot_stride, int n_pos, int H, BandSpans s,
                               int max_bands, uint8_t *slab)
{
    const long long rows = (long long)H * n_pos;
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= rows * s.n_bands) return;
    const int b = (int)(i / rows);
    const long long r = i - (long long)b * rows;
    const int h = (int)(r / n_pos), p = (int)(r - (long long)h * n_pos);
    uint8_t *dst = slab + h * slot_stride + (long long)p * s.row_bytes + s.lo[b];
    if (b >= max_bands) {
        for (int k = 0; k < s.len[b]; k++) dst[k] = 0;
        return;
    }
    const uint8_t *src = in + s.region[b] + r * s.len[b];
    for (int k = 0; k < s.len[b]; k++) dst[k] = src[k];
}

struct HostBuf {
    void *p = nullptr;
    ~HostBuf() { if (p) cudaFreeHost(p); }
};
struct DevBuf {
    void *p = nullptr;
    ~DevBuf() { if (p) cudaFree(p); }
};
struct File {
    FILE *f = nullptr;
    ~File() { if (f) fclose(f); }
};

void layer_path(char *buf, size_t n, const char *prefix, int layer)
{
    snprintf(buf, n, "%s.L%d.bin", prefix, layer);
}

bool hash_strict()
{
    const char *e = getenv("SP_DISK_HASH_STRICT");
    return !(e && e[0] == '0');
}

// One half (K or V) of one layer: device slab rows -> host file region.
int save_half(FILE *f, const uint8_t *slab, long long slot_stride, int n_pos, int H, const SpBandLayout &bl,
              int version, cudaStream_t s)
{
    const long long rows = (long long)H * n_pos;
    const size_t bytes = (size_t)rows * bl.total_bytes;
    HostBuf hb;
    DevBuf db;
    if (cudaMallocHost(&hb.p, bytes) != cudaSuccess) return sp_set_error(SP_ERR_CUDA, "cache_save: host buffer");
    if (version == 3) {
        if (cudaMalloc(&db.p, bytes) != cudaSuccess) return sp_set_error(SP_ERR_CUDA, "cache_save: device buffer");
        const BandSpans sp = spans_of(bl, rows);
        const long long work = rows * bl.n_bands;
        k_band_gather<<<(unsigned)((work + 255) / 256), 256, 0, s>>>(slab, slot_stride, n_pos, H, sp,
                                                                      (uint8_t *)db.p);
        if (int rc = sp_check_cuda(cudaGetLastError(), "cache_save gather")) return rc;
        cudaMemcpyAsync(hb.p, db.p, bytes, cudaMemcpyDeviceToHost, s);
    } else {
        for (int h = 0; h < H; h++)
            cudaMemcpyAsync((uint8_t *)hb.p + (size_t)h * n_pos * bl.total_bytes, slab + h * slot_stride,
                            (size_t)n_pos * bl.total_bytes, cudaMemcpyDeviceToHost, s);
    }
    if (int rc = sp_check_cuda(cudaStreamSynchronize(s), "cache_save copy")) return rc;
    if (fwrite(hb.p, 1, bytes, f) != bytes) return sp_set_error(SP_ERR_ARG, "cache_save: write failed");
    return SP_OK;
}

// One half of one layer from its file region (starting at the current file
// position) into the slab; v3 reads only the first max_bands band regions.
int load_half(FILE *f, long long region_start, uint8_t *slab, long long slot_stride, int n_pos, int H,
              const SpBandLayout &bl, int version, int max_bands, cudaStream_t s)
{
    const long long rows = (long long)H * n_pos;
    const size_t bytes = (size_t)rows * bl.total_bytes;
    HostBuf hb;
    DevBuf db;
    if (cudaMallocHost(&hb.p, bytes) != cudaSuccess) return sp_set_error(SP_ERR_CUDA, "cache_load: host buffer");
    if (cudaMalloc(&db.p, bytes) != cudaSuccess) return sp_set_error(SP_ERR_CUDA, "cache_load: device buffer");
    const BandSpans sp = spans_of(bl, rows);
    size_t want = bytes;
    if (version == 3 && max_bands < bl.n_bands) want = (size_t)sp.region[max_bands];
    if (fseek(f, (long)region_start, SEEK_SET) != 0 || fread(hb.p, 1, want, f) != want)
        return sp_set_error(SP_ERR_ARG, "cache_load: file shorter than its header says");
    cudaMemcpyAsync(db.p, hb.p, want, cudaMemcpyHostToDevice, s);
    const long long work = rows * bl.n_bands;
    if (version == 3) {
        k_band_scatter<<<(unsigned)((work + 255) / 256), 256, 0, s>>>((const uint8_t *)db.p, slot_stride, n_pos,
                                                                       H, sp, max_bands, slab);
    } else {
        // v2 rows are already per-vector; copy them back, then clear the
        // bands a partial load leaves out.
        for (int h = 0; h < H; h++)
            cudaMemcpyAsync(slab + h * slot_stride, (const uint8_t *)db.p + (size_t)h * n_pos * bl.total_bytes,
                            (size_t)n_pos * bl.total_bytes, cudaMemcpyDeviceToDevice, s);
        if (max_bands < bl.n_bands) {
            // gather the just-restored rows into the band-major buffer and
            // scatter them back with the band limit
            k_band_gather<<<(unsigned)((work + 255) / 256), 256, 0, s>>>(slab, slot_stride, n_pos, H, sp,
                                                                          (uint8_t *)db.p);
            k_band_scatter<<<(unsigned)((work + 255) / 256), 256, 0, s>>>((const uint8_t *)db.p, slot_stride,
                                                                           n_pos, H, sp, max_bands, slab);
        }
    }
    if (int rc = sp_check_cuda(cudaGetLastError(), "cache_load scatter")) return rc;
    return sp_check_cuda(cudaStreamSynchronize(s), "cache_load copy");
}

int load_impl(sp_cuda_cache_t *cc, const char *prefix, uint64_t expected_hash, int max_bands)
{
    sp_clear_error();
    if (!cc || !cc->d_k_cache || !prefix) return sp_set_error(SP_ERR_ARG, "cache_load: NULL argument");
    if (cudaSetDevice(cc->device) != cudaSuccess) return sp_set_error(SP_ERR_CUDA, "cache_load: cudaSetDevice");
    const SpBandLayout kl = sp_layout_from(cc->k_bands), vl = sp_layout_from(cc->v_bands);
    const int H = cc->config.n_heads_kv;
    const long long ks = (long long)cc->max_seq_len * kl.total_bytes, vs = (long long)cc->max_seq_len * vl.total_bytes;
    cudaStream_t s = (cudaStream_t)cc->stream;
    int n_pos_all = -1;
    for (int layer = 0; layer < cc->config.n_layers; layer++) {
        char path[4096];
        layer_path(path, sizeof path, prefix, layer);
        File fl;
        fl.f = fopen(path, "rb");
        if (!fl.f) return sp_set_error(SP_ERR_ARG, "cache_load: cannot open %s", path);
        unsigned char h[kHdrBytes], want[kHdrBytes];
        if (fread(h, 1, kHdrBytes, fl.f) != (size_t)kHdrBytes || memcmp(h, "VHT2", 4) != 0)
            return sp_set_error(SP_ERR_ARG, "cache_load: %s has no VHT2 header", path);
        if (get32(h + 60) != fnv1a32(h, 60)) return sp_set_error(SP_ERR_ARG, "cache_load: %s header checksum", path);
        const int version = (int)get32(h + 4);
        if (version != 2 && version != 3) return sp_set_error(SP_ERR_UNSUPPORTED, "cache_load: format v%d", version);
        const int n_pos = (int)get32(h + 16);
        if (n_pos <= 0 || n_pos > cc->max_seq_len)
            return sp_set_error(SP_ERR_ARG, "cache_load: n_pos %d outside (0, %d]", n_pos, cc->max_seq_len);
        if (n_pos_all >= 0 && n_pos != n_pos_all) return sp_set_error(SP_ERR_ARG, "cache_load: layers disagree on n_pos");
        n_pos_all = n_pos;
        uint64_t hash;
        memcpy(&hash, h + 8, 8);
        // Shape fields must match this cache exactly (the hash and n_pos are
        // the file's own).
        pack_header(want, cc, version, hash, n_pos, layer);
        if (memcmp(h + 16, want + 16, 44) != 0)
            return sp_set_error(SP_ERR_ARG, "cache_load: %s was saved from a cache of another shape or layout", path);
        if (hash != expected_hash) {
            if (hash_strict())
                return sp_set_error(SP_ERR_ARG, "cache_load: %s model hash %016llx, expected %016llx "
                                    "(SP_DISK_HASH_STRICT=0 loads anyway)", path, (unsigned long long)hash,
                                    (unsigned long long)expected_hash);
            fprintf(stderr, "[sp-b200] cache_load: %s model hash mismatch, loading anyway (SP_DISK_HASH_STRICT=0)\n",
                    path);
        }
        const long long rows = (long long)H * n_pos;
        const int mk = max_bands < 0 || max_bands > kl.n_bands ? kl.n_bands : max_bands;
        const int mv = max_bands < 0 || max_bands > vl.n_bands ? vl.n_bands : max_bands;
        const long long slot0 = (long long)layer * H;
        int rc = load_half(fl.f, kHdrBytes, (uint8_t *)cc->d_k_cache + slot0 * ks, ks, n_pos, H, kl, version, mk, s);
        if (rc) return rc;
        rc = load_half(fl.f, kHdrBytes + rows * kl.total_bytes, (uint8_t *)cc->d_v_cache + slot0 * vs, vs, n_pos,
                       H, vl, version, mv, s);
        if (rc) return rc;
    }
    return n_pos_all;
}

}  // namespace

extern "C" uint64_t sp_fnv1a64(const void *data, size_t n)
{
    const unsigned char *p = (const unsigned char *)data;
    uint64_t h = 0xcbf29ce484222325ull;
    for (size_t i = 0; i < n; i++) { h ^= p[i]; h *= 0x100000001b3ull; }
    return h;
}

extern "C" int sp_cuda_cache_save(const sp_cuda_cache_t *cc, const char *prefix, int n_pos, uint64_t model_hash,
                                  int version)
{
    sp_clear_error();
    if (!cc || !cc->d_k_cache || !prefix) return sp_set_error(SP_ERR_ARG, "cache_save: NULL argument");
    if (version != 2 && version != 3) return sp_set_error(SP_ERR_ARG, "cache_save: version must be 2 or 3");
    if (n_pos <= 0 || n_pos > cc->max_seq_len)
        return sp_set_error(SP_ERR_ARG, "cache_save: bad n_pos=%d (max_seq=%d)", n_pos, cc->max_seq_len);
    if (cudaSetDevice(cc->device) != cudaSuccess) return sp_set_error(SP_ERR_CUDA, "cache_save: cudaSetDevice");
    const SpBandLayout kl = sp_layout_from(cc->k_bands), vl = sp_layout_from(cc->v_bands);
    const int H = cc->config.n_heads_kv;
    const long long ks = (long long)cc->max_seq_len * kl.total_bytes, vs = (long long)cc->max_seq_len * vl.total_bytes;
    cudaStream_t s = (cudaStream_t)cc->stream;
    for (int layer = 0; layer < cc->config.n_layers; layer++) {
        char path[4096];
        layer_path(path, sizeof path, prefix, layer);
        File fl;
        fl.f = fopen(path, "wb");
        if (!fl.f) return sp_set_error(SP_ERR_ARG, "cache_save: cannot create %s", path);
        unsigned char h[kHdrBytes];
        pack_header(h, cc, version, model_hash, n_pos, layer);
        if (fwrite(h, 1, kHdrBytes, fl.f) != (size_t)kHdrBytes) return sp_set_error(SP_ERR_ARG, "cache_save: write failed");
        const long long slot0 = (long long)layer * H;
        int rc = save_half(fl.f, (const uint8_t *)cc->d_k_cache + slot0 * ks, ks, n_pos, H, kl, version, s);
        if (rc) return rc;
        rc = save_half(fl.f, (const uint8_t *)cc->d_v_cache + slot0 * vs, vs, n_pos, H, vl, version, s);
        if (rc) return rc;
    }
    return SP_OK;
}

extern "C" int sp_cuda_cache_load(sp_cuda_cache_t *cc, const char *prefix, uint64_t expected_hash)
{
    return load_impl(cc, prefix, expected_hash, -1);
}

extern "C" int sp_cuda_cache_load_partial(sp_cuda_cache_t *cc, const char *prefix, uint64_t expected_hash,
                                          int max_bands)
{
    if (max_bands < 0) return load_impl(cc, prefix, expected_hash, -1);
    return load_impl(cc, prefix, expected_hash, max_bands);
}
