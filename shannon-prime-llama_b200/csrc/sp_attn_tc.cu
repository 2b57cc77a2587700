// sp_attn_tc.cu — fused decode attention for the ship layout on the
// 5th-generation tensor cores (tcgen05, tensor memory).
//
// Same mathematics as sp_attn_mma.cu: the attention runs in the VHT2
// coefficient domain (score_t = q' . c_t with q' the transformed, Möbius-
// permuted query; the V sum is taken on dequantised coefficients and
// transformed once per (layer, query head) by the segment combine), and the
// packed codes enter the tensor cores as exact fp16 subnormals u * 2^(d-24).
//
// Layout of the work: a CTA of 8 warps takes 128-position tiles of one
// (layer, KV head) at a time.  Warps 0-3 own the K side, warps 4-7 the V side;
// thread t of either group owns position t of the tile.
//
//   K side  D_S[128 pos x 16] (tensor memory, per tile parity)
//             = A_K[128 pos x 128 codes] (tensor memory, per tile parity;
//               each K thread unpacks its own row, writes it with tcgen05.st)
//             x B_q[128 x 16] (shared memory, K-major; column (band, query
//               head), zero outside the band's rows; q' split into fp16 hi
//               and lo parts that two MMAs add into the same column)
//   V side  D_O[128 coeff x 16] (tensor memory, read back every tile)
//             = A_V[128 coeff x 128 pos] (shared memory, MN-major: each V
//               thread unpacks its own row and stores it with 16-byte stores)
//             x B_P[128 pos x 16] (shared memory, MN-major: p * vscale hi/lo,
//               written by the K thread of each position)
//
// One elected thread issues the MMAs (kind::f16, fp32 accumulation) and
// commits each group to an mbarrier.  The K threads read their scores row
// back with tcgen05.ld and form the softmax weights; the V threads read
// their coefficient row of D_O with tcgen05.ld once per tile and keep the
// running (centred) sums in fp32 registers.  Tiles arrive by cp.async.bulk
// (no multicast) into a 3-deep ring; every wait is bounded by %globaltimer
// and sets status bit 0 instead of hanging.
//
// Measured against the mma.sync decode (sp_attn_mma.cu), CUDA events on a
// B200: config 1 (32 layers, 8 KV heads, 32768 positions) 471 vs 345 us,
// config 3's shape (48 layers x 4 KV heads x 131072, G = 8) 1652 vs 1297 us.
// The unpack costs about one instruction per code in either layout, and
// this layout adds per tile: ~60 issue cycles per M = 128, N = 16 MMA for
// the issuing warp, V operands read from shared memory (4 KB per MMA), the
// tensor-memory round trips of scores and sums, and the barriers between
// the K, softmax and V phases.  So the mma.sync kernel stays the default and
// this one is selected with sp_cuda_attn_force_impl(3).
#include "sp_attn.cuh"
#include "sp_bulk.cuh"

#include <atomic>
#include <utility>
#include <math.h>
#include <stdlib.h>
#include <string.h>

namespace {

constexpr int kTM = 128;                       // positions per tile
constexpr int kThreads = 256;
constexpr int kKRow = 76, kVRow = 50;
constexpr int kKTileB = kTM * kKRow;           // 9728
constexpr int kVTileB = kTM * kVRow;           // 6400
constexpr int kStageB = kKTileB + kVTileB;     // 16128 (multiple of 16)
constexpr int kStages = 3;
constexpr int kN = 128;
constexpr float kEmptyMax = -1.0e30f;

// Ship layout (checked on the host): bit of band b's first code in a K row,
// its code width, and the 32-bit word / half holding its fp16 scale.
__host__ __device__ constexpr int kbit(int b) { return b == 0 ? 16 : b == 1 ? 192 : b == 2 ? 368 : 512; }
__host__ __device__ constexpr int kbits(int b) { return b < 2 ? 5 : (b == 2 ? 4 : 3); }

// Operand registers: each 32-bit A register holds two codes of one row as
// the fp16 subnormals u * 2^(d-24) of its low and high half, code c_lo at
// bits d_lo.. of the low half and c_hi at bits 16 + d_hi.. of the word, both
// taken from ONE funnel-shifted 32-bit window of the packed row with one AND.
// That needs bits * (c_hi - c_lo) = 16 + d_hi - d_lo and d + bits <= 10
// (the code stays in the mantissa).  The tensor cores multiply such
// subnormals exactly for d >= 2 and to ~1e-6 of the product's magnitude at
// d = 1 (3-bit codes); K codes use d >= 1 (a score error of that size is far
// below the softmax's resolution), V codes d >= 4 (their sums run over the
// whole context).  Among the valid choices the table takes windows that
// start on a word boundary or repeat an earlier window, so that shifts are
// shared.  Entries: {c_lo, c_hi, d_lo, d_hi}; register r of band b is K
// column 32 b + 2 r (low half) and 32 b + 2 r + 1 (high half).
constexpr signed char kKPair[4][16][4] = {
    {{0, 3, 2, 1}, {1, 4, 2, 1}, {2, 5, 2, 1}, {6, 9, 2, 1}, {7, 10, 2, 1}, {8, 11, 2, 1}, {12, 15, 2, 1},
     {13, 16, 2, 1}, {14, 17, 2, 1}, {18, 21, 2, 1}, {19, 22, 2, 1}, {20, 23, 2, 1}, {24, 27, 2, 1},
     {25, 29, 1, 5}, {26, 30, 1, 5}, {28, 31, 2, 1}},
    {{0, 3, 2, 1}, {1, 4, 5, 4}, {2, 5, 2, 1}, {6, 9, 2, 1}, {7, 10, 3, 2}, {8, 11, 2, 1}, {12, 15, 2, 1},
     {13, 16, 2, 1}, {14, 17, 2, 1}, {18, 21, 2, 1}, {19, 22, 2, 1}, {20, 23, 4, 3}, {24, 27, 2, 1},
     {25, 29, 1, 5}, {26, 30, 1, 5}, {28, 31, 2, 1}},
    {{0, 3, 5, 1}, {1, 4, 5, 1}, {2, 5, 5, 1}, {6, 9, 5, 1}, {7, 10, 5, 1}, {8, 11, 5, 1}, {12, 15, 5, 1},
     {13, 16, 5, 1}, {14, 17, 5, 1}, {18, 21, 5, 1}, {19, 22, 5, 1}, {20, 23, 5, 1}, {24, 27, 5, 1},
     {25, 29, 1, 1}, {26, 30, 5, 5}, {28, 31, 5, 1}},
    {{0, 4, 5, 1}, {1, 5, 5, 1}, {2, 6, 6, 2}, {3, 7, 5, 1}, {8, 12, 5, 1}, {9, 13, 5, 1}, {10, 14, 5, 1},
     {11, 15, 5, 1}, {16, 20, 5, 1}, {17, 21, 5, 1}, {18, 22, 5, 1}, {19, 23, 5, 1}, {24, 28, 5, 1},
     {25, 29, 5, 1}, {26, 30, 5, 1}, {27, 31, 5, 1}},
};
// V: 128 3-bit codes, register j holds rows m = 2j (low half) and 2j + 1
// (high half) of A_V, i.e. coefficients kVPair[j][0] and kVPair[j][1].
constexpr signed char kVPair[64][4] = {
    {0, 5, 5, 4},     {1, 6, 5, 4},     {2, 7, 6, 5},     {3, 8, 5, 4},     {4, 9, 5, 4},     {10, 15, 5, 4},
    {11, 16, 5, 4},   {12, 17, 5, 4},   {13, 18, 7, 6},   {14, 19, 5, 4},   {20, 25, 5, 4},   {21, 26, 5, 4},
    {22, 27, 5, 4},   {23, 28, 5, 4},   {24, 29, 5, 4},   {30, 35, 5, 4},   {31, 36, 5, 4},   {32, 37, 5, 4},
    {33, 38, 5, 4},   {34, 39, 6, 5},   {40, 45, 5, 4},   {41, 46, 5, 4},   {42, 47, 5, 4},   {43, 48, 5, 4},
    {44, 49, 5, 4},   {50, 55, 5, 4},   {51, 56, 5, 4},   {52, 57, 5, 4},   {53, 58, 5, 4},   {54, 59, 5, 4},
    {60, 65, 5, 4},   {61, 66, 5, 4},   {62, 67, 5, 4},   {63, 68, 5, 4},   {64, 69, 5, 4},   {70, 75, 5, 4},
    {71, 76, 5, 4},   {72, 77, 5, 4},   {73, 78, 5, 4},   {74, 79, 5, 4},   {80, 85, 5, 4},   {81, 86, 5, 4},
    {82, 87, 5, 4},   {83, 88, 5, 4},   {84, 90, 4, 6},   {89, 94, 5, 4},   {91, 96, 5, 4},   {92, 97, 5, 4},
    {93, 98, 5, 4},   {95, 101, 4, 6},  {99, 104, 5, 4},  {100, 105, 5, 4}, {102, 107, 5, 4}, {103, 108, 5, 4},
    {106, 112, 4, 6}, {109, 114, 7, 6}, {110, 115, 5, 4}, {111, 116, 5, 4}, {113, 118, 5, 4}, {117, 123, 4, 6},
    {119, 124, 5, 4}, {120, 125, 5, 4}, {121, 126, 5, 4}, {122, 127, 5, 4},
};

constexpr bool pairs_valid(const signed char (*t)[4], int n_regs, int n_codes, int bits, int dmin)
{
    bool seen[128] = {};
    for (int r = 0; r < n_regs; r++) {
        const int cl = t[r][0], ch = t[r][1], dl = t[r][2], dh = t[r][3];
        if (cl < 0 || ch >= n_codes || cl >= ch || seen[cl] || seen[ch]) return false;
        if (bits * (ch - cl) != 16 + dh - dl) return false;
        if (dl < dmin || dh < dmin || dl + bits > 10 || dh + bits > 10) return false;
        seen[cl] = seen[ch] = true;
    }
    for (int c = 0; c < n_codes; c++)
        if (!seen[c]) return false;
    return true;
}
static_assert(pairs_valid(kKPair[0], 16, 32, 5, 1) && pairs_valid(kKPair[1], 16, 32, 5, 1) &&
                  pairs_valid(kKPair[2], 16, 32, 4, 1) && pairs_valid(kKPair[3], 16, 32, 3, 1),
              "K operand pairing");
static_assert(pairs_valid(kVPair, 64, 128, 3, 4), "V operand pairing");

// Funnel-shifted 32-bit window of packed words starting at bit W.
template <int W, int NW>
__device__ __forceinline__ uint32_t window(const uint32_t (&w)[NW])
{
    if constexpr ((W & 31) == 0) return w[W >> 5];
    else return __funnelshift_r(w[W >> 5], w[(W >> 5) + 1], W & 31);
}

// ------------------------------------------------------------- tcgen05 --

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
                 "%12, %13, %14, %15, %16};" ::"r"(taddr),
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
                 "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
                 : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
                 "%12, %13, %14, %15}, [%16];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                   "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
                   "=r"(v[14]), "=r"(v[15])
                 : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, no swizzle.  K-major operands: lbo =
// bytes between the two 8-element K halves of one MMA, sbo = bytes between
// groups of 8 rows.  MN-major operands: lbo = bytes between K-adjacent core
// matrices (8 K rows x 16 bytes of M or N), sbo = bytes between MN-adjacent
// ones.
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo)
{
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFFu) >> 4);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;                      // descriptor version for sm_100
    return d;
}

// kind::f16 instruction descriptor: f16 A and B, f32 D, M = 128, N = 16;
// a_mn / b_mn select MN-major shared-memory operands.
__host__ __device__ constexpr uint32_t idesc_f16(int a_mn, int b_mn)
{
    return (1u << 4) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) | ((uint32_t)(16 >> 3) << 17) |
           ((uint32_t)(128 >> 4) << 24);
}

// D[tmem] (+)= A[tmem] x B[smem]
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t acc)
{
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %3, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %4, p;\n\t}"
                 ::"r"(d), "r"(a), "l"(b), "r"(acc), "r"(idesc_f16(0, 0)) : "memory");
}

// D[tmem] (+)= A[smem] x B[smem], both MN-major.
__device__ __forceinline__ void mma_ss_mn(uint32_t d, uint64_t a, uint64_t b, uint32_t acc)
{
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %3, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %4, p;\n\t}"
                 ::"r"(d), "l"(a), "l"(b), "r"(acc), "r"(idesc_f16(1, 1)) : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void named_sync(int id, int n)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// OR of `pred` over the n threads meeting at barrier id.
__device__ __forceinline__ bool named_or(int id, int n, bool pred)
{
    uint32_t r;
    asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\t"
                 "barrier.cta.red.or.pred p, %2, %3, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(r) : "r"((uint32_t)pred), "r"(id), "r"(n) : "memory");
    return r != 0;
}

__device__ __forceinline__ float fast_exp2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float finite_or_zero_f(unsigned short bits)
{
    const float f = __half2float(__ushort_as_half(bits));
    return fabsf(f) <= 65504.0f ? f : 0.0f;
}


// Compile-time loop: f(std::integral_constant<int, i>) for i = 0..N-1.
template <class F, int... I>
__device__ __forceinline__ void sfor_impl(F &&f, std::integer_sequence<int, I...>)
{
    (f(std::integral_constant<int, I>{}), ...);
}
template <int N, class F>
__device__ __forceinline__ void static_for(F &&f)
{
    sfor_impl(f, std::make_integer_sequence<int, N>{});
}

// Runtime lookups of the pairing (B_q construction, D_O rows): the same
// tables in constant memory.
struct PairTabs {
    signed char k[4][16][4];
    signed char v[64][4];
};
constexpr PairTabs make_tabs()
{
    PairTabs t{};
    for (int b = 0; b < 4; b++)
        for (int r = 0; r < 16; r++)
            for (int e = 0; e < 4; e++) t.k[b][r][e] = kKPair[b][r][e];
    for (int j = 0; j < 64; j++)
        for (int e = 0; e < 4; e++) t.v[j][e] = kVPair[j][e];
    return t;
}
__constant__ PairTabs c_tabs = make_tabs();

// Sum of v[h] over the warp for GT values at once: log2(GT) halving
// exchanges, then plain butterflies.  Returns the total of head
// `head_of_lane(lane)` (valid on every lane).
template <int GT>
__device__ __forceinline__ float warp_sum_heads(float (&v)[GT], int lane)
{
    constexpr int LG = GT == 8 ? 3 : (GT == 4 ? 2 : (GT == 2 ? 1 : 0));
    float x[GT];
#pragma unroll
    for (int i = 0; i < GT; i++) x[i] = v[i];
#pragma unroll
    for (int j = 0; j < LG; j++) {
        const int M = 16 >> j, n = GT >> (j + 1);
        const bool up = (lane & M) != 0;
#pragma unroll
        for (int i = 0; i < n; i++) {
            const float send = up ? x[i] : x[i + n];
            const float keep = up ? x[i + n] : x[i];
            x[i] = keep + __shfl_xor_sync(0xffffffffu, send, M);
        }
    }
#pragma unroll
    for (int M = 16 >> LG; M > 0; M >>= 1) x[0] += __shfl_xor_sync(0xffffffffu, x[0], M);
    return x[0];
}
template <int GT>
__device__ __forceinline__ int head_of_lane(int lane)
{
    constexpr int LG = GT == 8 ? 3 : (GT == 4 ? 2 : (GT == 2 ? 1 : 0));
    int h = 0;
#pragma unroll
    for (int j = 0; j < LG; j++)
        if (lane & (16 >> j)) h += GT >> (j + 1);
    return h;
}
// Lanes that write the per-head totals: one per head.
template <int GT>
__device__ __forceinline__ bool head_writer(int lane)
{
    constexpr int LG = GT == 8 ? 3 : (GT == 4 ? 2 : (GT == 2 ? 1 : 0));
    return (lane & ((16 >> LG) * 2 - 1)) == 0;
}

// Shared memory of one CTA.
struct alignas(128) TcSmem {
    unsigned char ring[kStages][kStageB];      // 48384
    unsigned char av[kTM * kN * 2];            // A_V, MN-major: (m,k) at m/8*128 + k/8*2048 + k%8*16 + m%8*2
    unsigned char bp[2][16 * kTM * 2];         // B_P per tile parity, MN-major: (k,n) at n/8*128 + k/8*256 + k%8*16 + n%8*2
    unsigned char bq[16 * kN * 2];             // B_q, K-major: (n,k) at n/8*2048 + k/8*128 + n%8*16 + k%8*2
    float q[8][kN];                            // q' of the segment (transformed, permuted, scaled)
    float qt[8][kN];                           // transform scratch
    float qsum[8][4];
    float qmax[8];
    float cin[4][8];                           // per band, per head: -m_b * sum_b(q') * 2^(F-24)
    float sred[2][4][8];                       // per tile parity, K warp, head: sum of p * vscale
    float alpha[2][8];                         // per tile parity, head: rescale of the running sums
    float mx[4][8];                            // per K warp, head: tile maximum (rescale path)
    float lred[4][8];                          // per K warp, head: softmax denominator at segment end
    unsigned long long bar_ring[kStages];
    unsigned long long bar_s, bar_o;
    uint32_t tmem;
    int abort;
};

// Tensor memory (256 columns x 128 lanes).  Score accumulators D_S: one
// 16-column block per band, column h for the hi part of query head h and
// GT + h for its lo part (GT = 4: columns 0-7 used).  The V product is split
// over four D_O blocks (two k-steps each), summed when read back.  Each
// block is written by MMAs that one warp issues, so that the MMAs of
// different blocks are issued by several warps at once (an M = 128, N = 16
// MMA costs a warp ~60 issue cycles; the tensor core takes more in parallel).
constexpr uint32_t kColS = 0;      // D_S: band b at 16 b
constexpr uint32_t kColO = 64;     // D_O: blocks at 64 + 16 i
constexpr uint32_t kColA = 128;    // A_K: band b at 128 + 16 b
constexpr uint32_t kTmemCols = 256;
constexpr int kVIssuers = 4;       // V warps issuing the V MMAs (k-steps 2i, 2i+1 into D_O block i)

__device__ __forceinline__ bool elect_one()
{
    uint32_t e;
    asm volatile("{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}" : "=r"(e));
    return e != 0;
}

// GT query heads per KV head (4 or 8; fewer are padded with zero queries),
// NBK K bands read (4, or fewer for a partial-band read).
template <int GT, int NBK>
__global__ void __launch_bounds__(kThreads, 2)
k_attn_ship_tc(SpAttnArgs a, SpSched sc)
{
    static_assert(GT == 4 || GT == 8, "4 or 8 query heads per KV head");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    TcSmem &sm = *reinterpret_cast<TcSmem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool kside = warp < 4;
    const int t = tid & 127;                       // position (K and V) / coefficient row (V drain)
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    const int cta = blockIdx.x;
    const long long g_begin = sp_tile_begin(cta, sc), g_end = sp_tile_begin(cta + 1, sc);
    const int n_my = (int)(g_end - g_begin);
    const int n_t = sc.tiles_per_unit;
    const int G = a.group, H = a.n_kv_heads;

    if (tid == 0) {
        for (int s = 0; s < kStages; s++) spb::mbar_init(spb::smem_u32(&sm.bar_ring[s]), 1);
        spb::mbar_init(spb::smem_u32(&sm.bar_s), NBK);          // one commit per band's warp
        spb::mbar_init(spb::smem_u32(&sm.bar_o), kVIssuers);
        spb::mbar_init_fence();
        sm.abort = 0;
    }
    // B_P columns a head group leaves unused stay zero.
    for (int i = tid; i < (int)(sizeof(sm.bp) / 16); i += kThreads)
        reinterpret_cast<uint4 *>(&sm.bp[0][0])[i] = make_uint4(0u, 0u, 0u, 0u);
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(spb::smem_u32(&sm.tmem)), "r"(kTmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem;

    // ---- ring: thread 0 fetches tile k of this CTA into stage k % kStages
    uint64_t policy = 0;
    if (tid == 0) policy = spb::evict_first_policy();
    auto issue = [&](int k) {
        const long long g = g_begin + k;
        const long long u = g / n_t;
        const int tt = (int)(g - u * n_t);
        const int li = (int)(u / H), h = (int)(u % H);
        const long long slot = (long long)(a.layer0 + li) * H + h;
        const int st = k % kStages;
        const uint32_t bar = spb::smem_u32(&sm.bar_ring[st]);
        const uint32_t dst = spb::smem_u32(&sm.ring[st][0]);
        spb::fence_proxy_async();
        spb::mbar_expect_tx(bar, kStageB);
        spb::bulk_g2s(dst, a.k_cache + slot * a.k_slot_stride + (long long)tt * kKTileB, kKTileB, bar, policy);
        spb::bulk_g2s(dst + kKTileB, a.v_cache + slot * a.v_slot_stride + (long long)tt * kVTileB, kVTileB, bar,
                      policy);
    };
    if (tid == 0)
        for (int k = 0; k < kStages && k < n_my; k++) issue(k);

    // Bounded waits.  After the first timeout the CTA stops waiting (results
    // are then garbage, status bit 0 is set) but keeps meeting its barriers.
    auto wait_bar = [&](uint32_t bar, uint32_t parity) {
        if (spb::mbar_try_wait(bar, parity)) return;
        if (*(volatile int *)&sm.abort) return;
        if (!spb::wait_stage(bar, parity, a.status)) *(volatile int *)&sm.abort = 1;
    };

    // ---- per-thread segment state
    float kc[GT], m_run[GT], nkm[GT], l_sum[GT];   // K side
    float acc[GT];                                 // V side: centred sum of coefficient row t
    int v_coef = 0;
    float v_scale = 0.0f;                          // 2^(24 - d) of D_O row t
    {
        const int j = t >> 1, hf = t & 1;
        v_coef = c_tabs.v[j][hf];
        v_scale = ldexpf(1.0f, 24 - c_tabs.v[j][2 + hf]);
    }
#pragma unroll
    for (int h = 0; h < GT; h++) { kc[h] = 1.0f; m_run[h] = kEmptyMax; nkm[h] = 0.0f; l_sum[h] = 0.0f; acc[h] = 0.0f; }

    // Queries of unit u (K threads): q' = perm(H q) * scale per head, the
    // B_q operand (hi and lo parts), the band offsets and the score scale.
    auto setup_unit = [&](long long u) {
        const int li = (int)(u / H), h = (int)(u % H);
        for (int g = warp; g < GT; g += 4) {
            if (g < G) {
                const __half *qg = a.q + ((long long)li * a.n_q_heads + h * G + g) * kN;
                float x[4];
#pragma unroll
                for (int e = 0; e < 4; e++) x[e] = __half2float(qg[lane * 4 + e]);
                sp_warp_wht<4>(x, lane);
                const float sc_all = a.logit_scale * 1.4426950408889634f * a.inv_sqrt_n;
#pragma unroll
                for (int e = 0; e < 4; e++) sm.qt[g][lane * 4 + e] = x[e] * sc_all;
                __syncwarp();
                float mxv = 0.0f, bs = 0.0f;
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int i = lane * 4 + e;
                    const float v = sm.qt[g][a.order ? a.order[i] : i];
                    sm.q[g][i] = v;
                    mxv = fmaxf(mxv, fabsf(v));
                    bs += v;
                }
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) bs += __shfl_xor_sync(0xffffffffu, bs, o);
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) mxv = fmaxf(mxv, __shfl_xor_sync(0xffffffffu, mxv, o));
                if ((lane & 7) == 0) sm.qsum[g][lane >> 3] = bs;
                if (lane == 0) sm.qmax[g] = mxv;
            } else {
                for (int i = lane; i < kN; i += 32) sm.q[g][i] = 0.0f;
                if (lane < 4) sm.qsum[g][lane] = 0.0f;
                if (lane == 0) sm.qmax[g] = 0.0f;
            }
        }
        named_sync(1, 128);
        // column k = t of B_q: band b, register r, half hf of the pairing
        const int b = t >> 5, r = (t & 31) >> 1, hf = t & 1;
        const int code = c_tabs.k[b][r][hf], d = c_tabs.k[b][r][2 + hf];
        unsigned char *colbase = sm.bq + (t >> 3) * 128 + (t & 7) * 2;
#pragma unroll
        for (int g = 0; g < GT; g++) {
            const float qm = sm.qmax[g];
            const int F = qm > 1e-30f ? 6 - ilogbf(qm) : 0;
            const float v = (b < a.nb_k) ? ldexpf(sm.q[g][32 * b + code], F - d) : 0.0f;
            const __half hi = __float2half_rn(v);
            const __half lo = __float2half_rn(v - __half2float(hi));
            const int nh = g, nl = GT + g;
            *reinterpret_cast<__half *>(colbase + (nh >> 3) * 2048 + (nh & 7) * 16) = hi;
            *reinterpret_cast<__half *>(colbase + (nl >> 3) * 2048 + (nl & 7) * 16) = lo;
            kc[g] = ldexpf(1.0f, 24 - F);
            if (t < 4) {
                const float m_b = (float)((1 << (kbits(t) - 1)) - 1);
                sm.cin[t][g] = t < a.nb_k ? -ldexpf(m_b * sm.qsum[g][t], F - 24) : 0.0f;
            }
        }
        if (GT == 4) {       // rows n = 8..15 of B_q unused: zero
#pragma unroll
            for (int n = 8; n < 16; n++) *reinterpret_cast<__half *>(colbase + 2048 + (n & 7) * 16) = __float2half_rn(0.0f);
        }
#pragma unroll
        for (int g = 0; g < GT; g++) { m_run[g] = kEmptyMax; nkm[g] = 0.0f; l_sum[g] = 0.0f; }
        spb::fence_proxy_async();      // B_q generic stores before the tensor core reads them
        named_sync(1, 128);            // cin / q reads done before anyone rewrites them
    };

    // D_O row t of tile k into the running sums (V threads).
    auto drain = [&](int k) {
        uint32_t d[16];
        if constexpr (GT == 4) {
            uint32_t d4[kVIssuers][8];
#pragma unroll
            for (int i = 0; i < kVIssuers; i++) tmem_ld8(tmem + lane_base + kColO + 16 * i, d4[i]);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 8; e++) {
                float x = __uint_as_float(d4[0][e]);
#pragma unroll
                for (int i = 1; i < kVIssuers; i++) x += __uint_as_float(d4[i][e]);
                d[e] = __float_as_uint(x);
            }
        } else {
            uint32_t d1[16];
            tmem_ld16(tmem + lane_base + kColO, d);
#pragma unroll
            for (int i = 1; i < kVIssuers; i++) {
                tmem_ld16(tmem + lane_base + kColO + 16 * i, d1);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 16; e++) d[e] = __float_as_uint(__uint_as_float(d[e]) + __uint_as_float(d1[e]));
            }
            tmem_wait_ld();
        }
        const int par = k & 1;
        float S[GT];
#pragma unroll
        for (int h0 = 0; h0 < GT; h0 += 4) {
            float4 s4 = *reinterpret_cast<const float4 *>(&sm.sred[par][0][h0]);
#pragma unroll
            for (int w = 1; w < 4; w++) {
                const float4 x = *reinterpret_cast<const float4 *>(&sm.sred[par][w][h0]);
                s4.x += x.x; s4.y += x.y; s4.z += x.z; s4.w += x.w;
            }
            S[h0] = s4.x; S[h0 + 1] = s4.y; S[h0 + 2] = s4.z; S[h0 + 3] = s4.w;
        }
#pragma unroll
        for (int h = 0; h < GT; h++) {
            const float tile = fmaf(__uint_as_float(d[h]) + __uint_as_float(d[GT + h]), v_scale, -3.0f * S[h]);
            acc[h] = fmaf(acc[h], sm.alpha[par][h], tile);
        }
    };

    // End of the segment of unit u whose last tile is k (all threads).
    auto finish_unit = [&](long long u, int k) {
        const int li = (int)(u / H), h = (int)(u % H);
        const int seg = cta - sp_cta_of_tile(u * (long long)n_t, sc);
        if (kside) {
            const float L = warp_sum_heads<GT>(l_sum, lane);
            if (head_writer<GT>(lane)) sm.lred[warp][head_of_lane<GT>(lane)] = L;
            named_sync(1, 128);
            if (t < G) {
                float *part = sp_attn_partial(a, li, h * G + t, seg);
                float mr = kEmptyMax;
#pragma unroll
                for (int g = 0; g < GT; g++)
                    if (g == t) mr = kc[g] * m_run[g];
                part[0] = fmaxf(mr, kEmptyMax);
                part[1] = sm.lred[0][t] + sm.lred[1][t] + sm.lred[2][t] + sm.lred[3][t];
            }
        } else {
            wait_bar(spb::smem_u32(&sm.bar_o), (uint32_t)(k & 1));
            tc_fence_after();
            drain(k);
#pragma unroll
            for (int g = 0; g < GT; g++) {
                if (g < G) sp_attn_partial(a, li, h * G + g, seg)[4 + v_coef] = acc[g];
                acc[g] = 0.0f;
            }
        }
    };

    // K row t of tile k -> A_K; then the warp of band b issues band b's two
    // score MMAs into D_S block b and commits them to bar_s.  The row's band
    // scales and V scale come back for the epilogue.
    auto k_front = [&](int k, float (&bsc)[4], float &vs) {
        const int st = k % kStages;
        wait_bar(spb::smem_u32(&sm.bar_ring[st]), (uint32_t)((k / kStages) & 1));
        const unsigned char *stg = sm.ring[st];
        uint32_t w[19];
        const uint32_t *kr = reinterpret_cast<const uint32_t *>(stg + kKRow * t);
#pragma unroll
        for (int i = 0; i < 19; i++) w[i] = kr[i];
        vs = finite_or_zero_f(*reinterpret_cast<const unsigned short *>(stg + kKTileB + kVRow * t));
        bsc[0] = finite_or_zero_f((unsigned short)(w[0] & 0xffffu));
        bsc[1] = finite_or_zero_f((unsigned short)(w[5] >> 16));
        bsc[2] = finite_or_zero_f((unsigned short)(w[11] & 0xffffu));
        bsc[3] = finite_or_zero_f((unsigned short)(w[15] >> 16));
        const uint32_t a_base = tmem + lane_base + kColA;
        static_for<NBK>([&](auto B) {
            constexpr int b = decltype(B)::value;
            uint32_t v[16];
            static_for<16>([&](auto R) {
                constexpr int r = decltype(R)::value;
                constexpr int bits = kbits(b);
                constexpr int W = kbit(b) + bits * kKPair[b][r][0] - kKPair[b][r][2];
                constexpr uint32_t M = (((1u << bits) - 1u) << kKPair[b][r][2]) |
                                       (((1u << bits) - 1u) << (16 + kKPair[b][r][3]));
                v[r] = window<W>(w) & M;
            });
            tmem_st16(a_base + 16 * b, v);
        });
        tmem_wait_st();
        tc_fence_before();
        named_sync(1, 128);
        if (warp < NBK) {
            if (elect_one()) {
                tc_fence_after();
                const uint32_t bq = spb::smem_u32(sm.bq);
                const int b = warp;
#pragma unroll
                for (int j = 0; j < 2; j++)
                    mma_ts(tmem + kColS + 16u * b, tmem + kColA + 16u * b + 8u * j,
                           sdesc(bq + (uint32_t)(4 * b + 2 * j) * 128u, 128u, 2048u), (uint32_t)j);
                mma_commit(spb::smem_u32(&sm.bar_s));
            }
            __syncwarp();
        }
    };

    long long cur_u = -1;
    int seg_first = 0;
    float bsc_c[4], vs_c = 0.0f;
    for (int k = 0; k < n_my; k++) {
        const long long g = g_begin + k;
        const long long u = g / n_t;
        const int tt = (int)(g - u * n_t);
        if (u != cur_u) {
            if (cur_u >= 0) finish_unit(cur_u, k - 1);
            if (kside) setup_unit(u);
            cur_u = u;
            seg_first = k;
        }
        const int st = k % kStages, par = k & 1;
        if (kside) {
            k_front(k, bsc_c, vs_c);
            wait_bar(spb::smem_u32(&sm.bar_s), (uint32_t)par);
            tc_fence_after();
            // ---- scores of position t in units of 1/kc --------------------
            float su[GT];
#pragma unroll
            for (int h = 0; h < GT; h++) su[h] = 0.0f;
#pragma unroll
            for (int b = 0; b < NBK; b++) {
                uint32_t d[16];
                if constexpr (GT == 4) tmem_ld8(tmem + lane_base + kColS + 16 * b, *reinterpret_cast<uint32_t (*)[8]>(&d[0]));
                else tmem_ld16(tmem + lane_base + kColS + 16 * b, d);
                tmem_wait_ld();
#pragma unroll
                for (int h0 = 0; h0 < GT; h0 += 4) {
                    const float4 ci = *reinterpret_cast<const float4 *>(&sm.cin[b][h0]);
                    const float c4[4] = {ci.x, ci.y, ci.z, ci.w};
#pragma unroll
                    for (int e = 0; e < 4; e++)
                        su[h0 + e] = fmaf(bsc_c[b], __uint_as_float(d[h0 + e]) + __uint_as_float(d[GT + h0 + e]) + c4[e],
                                          su[h0 + e]);
                }
            }
            const bool valid = tt * kTM + t < a.kv_len;
            bool up = false;
#pragma unroll
            for (int h = 0; h < GT; h++) {
                su[h] = valid ? su[h] : -INFINITY;
                up |= su[h] > m_run[h];
            }
            // ---- running maximum: rescale only when some score passes it --
            if (named_or(2, 128, up)) {
#pragma unroll
                for (int h = 0; h < GT; h++) {
                    float m = su[h];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                    if (lane == 0) sm.mx[warp][h] = m;
                }
                named_sync(3, 128);
#pragma unroll
                for (int h = 0; h < GT; h++) {
                    const float T = fmaxf(fmaxf(sm.mx[0][h], sm.mx[1][h]), fmaxf(sm.mx[2][h], sm.mx[3][h]));
                    const float m_new = fmaxf(m_run[h], T);
                    const float al = fast_exp2(kc[h] * (m_run[h] - m_new));
                    m_run[h] = m_new;
                    nkm[h] = -kc[h] * m_new;
                    l_sum[h] *= al;
                    if (tid == 0) sm.alpha[par][h] = al;
                }
            } else if (tid == 0) {
#pragma unroll
                for (int h = 0; h < GT; h++) sm.alpha[par][h] = 1.0f;
            }
            // ---- weights -> B_P (MN-major row t), their sums -> sred ------
            float pv[GT];
            uint32_t hw[GT / 2], lw[GT / 2];
#pragma unroll
            for (int h = 0; h < GT; h += 2) {
                float p2[2];
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const float p = fast_exp2(fmaf(kc[h + e], su[h + e], nkm[h + e]));
                    l_sum[h + e] += p;
                    p2[e] = p * vs_c;
                    pv[h + e] = p2[e];
                }
                const __half2 hi2 = __floats2half2_rn(p2[0], p2[1]);
                const float2 back = __half22float2(hi2);
                const __half2 lo2 = __floats2half2_rn(p2[0] - back.x, p2[1] - back.y);
                hw[h / 2] = *reinterpret_cast<const uint32_t *>(&hi2);
                lw[h / 2] = *reinterpret_cast<const uint32_t *>(&lo2);
            }
            unsigned char *prow = sm.bp[par] + (t >> 3) * 256 + (t & 7) * 16;
            if constexpr (GT == 4) {
                *reinterpret_cast<uint4 *>(prow) = make_uint4(hw[0], hw[1], lw[0], lw[1]);
            } else {
                *reinterpret_cast<uint4 *>(prow) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                *reinterpret_cast<uint4 *>(prow + 128) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            }
            const float S = warp_sum_heads<GT>(pv, lane);
            if (head_writer<GT>(lane)) sm.sred[par][warp][head_of_lane<GT>(lane)] = S;
        } else {
            // ---- V row t unpacked into registers while the previous tile's
            // V MMAs run; then that tile's D_O row -> running sums, and the
            // row -> A_V (free once those MMAs are done)
            wait_bar(spb::smem_u32(&sm.bar_ring[st]), (uint32_t)((k / kStages) & 1));
            const unsigned char *stg = sm.ring[st];
            const int odd = t & 1;
            const uint32_t *vr = reinterpret_cast<const uint32_t *>(stg + kKTileB + kVRow * t - 2 * odd);
            uint32_t w[14], nw[13];
#pragma unroll
            for (int i = 0; i < 14; i++) w[i] = vr[i];
            // codes from bit 16 of nw on, whatever the row's alignment
#pragma unroll
            for (int i = 0; i < 13; i++) nw[i] = __funnelshift_r(w[i], w[i + 1], 16 * odd);
            uint32_t v[64];
            static_for<64>([&](auto J) {
                constexpr int j = decltype(J)::value;
                constexpr int W = 16 + 3 * kVPair[j][0] - kVPair[j][2];
                constexpr uint32_t M = (7u << kVPair[j][2]) | (7u << (16 + kVPair[j][3]));
                v[j] = window<W>(nw) & M;
            });
            if (k > seg_first) {
                wait_bar(spb::smem_u32(&sm.bar_o), (uint32_t)((k - 1) & 1));
                tc_fence_after();
                drain(k - 1);
            }
            unsigned char *arow = sm.av + (t >> 3) * 2048 + (t & 7) * 16;
#pragma unroll
            for (int q = 0; q < 16; q++)
                *reinterpret_cast<uint4 *>(arow + q * 128) = make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
        spb::fence_proxy_async();       // B_P / A_V generic stores before the tensor core reads them
        tc_fence_before();
        __syncthreads();
        if (warp >= 4 && warp < 4 + kVIssuers) {
            // V warp 4 + i issues its k-steps into D_O block i
            if (elect_one()) {
                tc_fence_after();
                const int i = warp - 4;
                constexpr int kSteps = 8 / kVIssuers;
                const uint32_t av = spb::smem_u32(sm.av), bp = spb::smem_u32(sm.bp[par]);
#pragma unroll
                for (int s = kSteps * i; s < kSteps * i + kSteps; s++)
                    mma_ss_mn(tmem + kColO + 16u * i, sdesc(av + (uint32_t)s * 4096u, 2048u, 128u),
                              sdesc(bp + (uint32_t)s * 512u, 256u, 128u), (uint32_t)(s > kSteps * i));
                mma_commit(spb::smem_u32(&sm.bar_o));
            }
            __syncwarp();
        }
        if (tid == 0 && k + kStages < n_my) issue(k + kStages);
    }
    if (n_my > 0) finish_unit(cur_u, n_my - 1);

    // After a timed-out wait: let the copies and MMAs in flight land
    // (bounded) before the shared and tensor memory are released.
    __syncthreads();
    if (sm.abort && tid == 0 && n_my > 0) {
        for (int k = n_my - 1; k >= 0 && k >= n_my - kStages; k--)
            spb::wait_stage(spb::smem_u32(&sm.bar_ring[k % kStages]), (uint32_t)((k / kStages) & 1), nullptr);
        spb::wait_stage(spb::smem_u32(&sm.bar_s), (uint32_t)((n_my - 1) & 1), nullptr);
        spb::wait_stage(spb::smem_u32(&sm.bar_o), (uint32_t)((n_my - 1) & 1), nullptr);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

}  // namespace

int sp_attn_tc_supported(const SpAttnArgs &a)
{
    if (sp_attn_mma_supported(a) != SP_OK) return SP_ERR_UNSUPPORTED;
    // Whole 128-position tiles must lie inside each slot.
    const long long tiles = (a.kv_len + kTM - 1) / kTM;
    if (tiles * kKTileB > a.k_slot_stride || tiles * kVTileB > a.v_slot_stride) return SP_ERR_UNSUPPORTED;
    return SP_OK;
}

int sp_attn_tc_launch(const SpAttnArgs &a_in, cudaStream_t s, cudaEvent_t ev_begin, cudaEvent_t ev_end)
{
    SpAttnArgs a = a_in;
    const bool wide = a.group > 4;
    using Kern = void (*)(SpAttnArgs, SpSched);
    static const Kern narrow_k[4] = {k_attn_ship_tc<4, 1>, k_attn_ship_tc<4, 2>, k_attn_ship_tc<4, 3>,
                                     k_attn_ship_tc<4, 4>};
    static const Kern wide_k[4] = {k_attn_ship_tc<8, 1>, k_attn_ship_tc<8, 2>, k_attn_ship_tc<8, 3>,
                                   k_attn_ship_tc<8, 4>};
    const int nbk = a.nb_k < 1 ? 1 : (a.nb_k > 4 ? 4 : a.nb_k);
    Kern kernel = wide ? wide_k[nbk - 1] : narrow_k[nbk - 1];
    const size_t smem = sizeof(TcSmem) + 1024;   // + alignment slack of the dynamic base
    // Per device and per kernel: attribute set and SM count looked up once;
    // atomics, so host threads driving any devices race harmlessly.
    constexpr int kMaxDev = 64;
    static std::atomic<int> ready[kMaxDev][2][4];
    static std::atomic<int> sms_tab[kMaxDev];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDev) return sp_set_error(SP_ERR_CUDA, "tcgen05 attention: device %d", dev);
    if (!ready[dev][wide][nbk - 1].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return sp_check_cuda(cudaGetLastError(), "tcgen05 attention smem attribute");
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        sms_tab[dev].store(sms > 0 ? sms : 148, std::memory_order_relaxed);
        ready[dev][wide][nbk - 1].store(1, std::memory_order_release);
    }
    const int sms = sms_tab[dev].load(std::memory_order_relaxed);
    const int units = a.n_layers * a.n_kv_heads;
    SpSched sc;
    sc.tiles_per_unit = (a.kv_len + kTM - 1) / kTM;
    sc.total_tiles = (long long)units * sc.tiles_per_unit;
    long long n = (long long)sms * 2;            // two CTAs per SM (shared and tensor memory)
    if (n > sc.total_tiles) n = sc.total_tiles;
    if (n > (long long)units * (kAttnMaxSplits - 2)) n = (long long)units * (kAttnMaxSplits - 2);
    sc.n_ctas = (int)n;
    a.n_splits = 0;
    if (ev_begin) cudaEventRecord(ev_begin, s);
    kernel<<<sc.n_ctas, kThreads, smem, s>>>(a, sc);
    if (ev_end) cudaEventRecord(ev_end, s);
    int rc = sp_check_cuda(cudaGetLastError(), "tcgen05 attention launch");
    if (rc) return rc;
    return sp_attn_seg_combine_launch(a, sc, s);
}

// ------------------------------------------- fused-KQ scores op, tcgen05 --
// The scores-only op (sp_cuda_kq_scores[_strided], the GPU body of the
// reference's ggml op llama_sp_kq_compute, llama_sp_fused_kq.cpp:82-165)
// for K rows of the head_dim-128 ship layout and up to 8 query rows: the K
// side of the decode above without the softmax.  A CTA of 4 warps takes
// 128-position tiles of one slot; thread t unpacks row t into tensor memory
// (A operand, codes as fp16 subnormals), band b's warp issues band b's two
// MMAs against the query operand B_q (q' = perm(H q) / sqrt(n) as fp16 hi
// and lo parts), and thread t reads its score row back and writes its
// position's score for every query row (coalesced along positions).
namespace {

constexpr int kKqTcThreads = 128;

__host__ __device__ constexpr bool kq_squarefree(int n)
{
    for (int p = 2; p * p <= n; p++)
        if (n % (p * p) == 0) return false;
    return true;
}
// Squarefree-first order of 0..127 (the order of every ship cache's K rows).
struct KqOrder { int v[kN]; };
__host__ __device__ constexpr KqOrder kq_order()
{
    KqOrder o{};
    int k = 0;
    for (int i = 0; i < kN; i++)
        if (kq_squarefree(i + 1)) o.v[k++] = i;
    for (int i = 0; i < kN; i++)
        if (!kq_squarefree(i + 1)) o.v[k++] = i;
    return o;
}
__constant__ KqOrder c_kq_order = kq_order();

struct alignas(128) KqSmem {
    unsigned char rows[2][kKTileB];          // two tiles of K rows
    unsigned char bq[16 * kN * 2];           // B_q, K-major: (n,k) at n/8*2048 + k/8*128 + n%8*16 + k%8*2
    float qt[8][kN];
    float q[8][kN];
    float qsum[8][4];
    float qmax[8];
    float cin[4][8];
    unsigned long long bar[2], bar_s;
    uint32_t tmem;
    int abort;
};

struct KqTcArgs {
    const uint8_t *packed;
    long long packed_slot;
    const void *q;
    long long q_stride, q_slot;
    float *dst;
    long long dst_stride, dst_slot;
    int n_kv, n_head_q, q_f16;
    float inv_sqrt_n;
};

template <int GT>
__global__ void __launch_bounds__(kKqTcThreads, 3)
k_kq_scores_tc(KqTcArgs a)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    KqSmem &sm = *reinterpret_cast<KqSmem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, t = tid;
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
    const uint8_t *packed = a.packed + (long long)blockIdx.y * a.packed_slot;
    const uint8_t *qb = reinterpret_cast<const uint8_t *>(a.q) + (long long)blockIdx.y * a.q_slot;
    float *dst = reinterpret_cast<float *>(reinterpret_cast<char *>(a.dst) + (long long)blockIdx.y * a.dst_slot);
    const int n_tiles = (a.n_kv + kTM - 1) / kTM;
    constexpr uint32_t kQColS = 0, kQColA = 64, kQCols = 128;

    if (tid == 0) {
        spb::mbar_init(spb::smem_u32(&sm.bar[0]), 1);
        spb::mbar_init(spb::smem_u32(&sm.bar[1]), 1);
        spb::mbar_init(spb::smem_u32(&sm.bar_s), 4);
        spb::mbar_init_fence();
        sm.abort = 0;
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(spb::smem_u32(&sm.tmem)), "r"(kQCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // ---- q' of every query row (warp g: rows g, g + 4) ----
    for (int g = warp; g < GT; g += 4) {
        if (g < a.n_head_q) {
            const uint8_t *qr = qb + (long long)g * a.q_stride;
            float x[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int i = lane * 4 + e;
                x[e] = a.q_f16 ? __half2float(reinterpret_cast<const __half *>(qr)[i])
                               : reinterpret_cast<const float *>(qr)[i];
            }
            sp_warp_wht<4>(x, lane);
#pragma unroll
            for (int e = 0; e < 4; e++) sm.qt[g][lane * 4 + e] = x[e] * a.inv_sqrt_n;
            __syncwarp();
            float mxv = 0.0f, bs = 0.0f;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int i = lane * 4 + e;
                const float v = sm.qt[g][c_kq_order.v[i]];
                sm.q[g][i] = v;
                mxv = fmaxf(mxv, fabsf(v));
                bs += v;
            }
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) bs += __shfl_xor_sync(0xffffffffu, bs, o);
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) mxv = fmaxf(mxv, __shfl_xor_sync(0xffffffffu, mxv, o));
            if ((lane & 7) == 0) sm.qsum[g][lane >> 3] = bs;
            if (lane == 0) sm.qmax[g] = mxv;
        } else {
            for (int i = lane; i < kN; i += 32) sm.q[g][i] = 0.0f;
            if (lane < 4) sm.qsum[g][lane] = 0.0f;
            if (lane == 0) sm.qmax[g] = 0.0f;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem;
    // ---- B_q column k = t; score scales ----
    float kc[GT];
    {
        const int b = t >> 5, r = (t & 31) >> 1, hf = t & 1;
        const int code = c_tabs.k[b][r][hf], d = c_tabs.k[b][r][2 + hf];
        unsigned char *colbase = sm.bq + (t >> 3) * 128 + (t & 7) * 2;
#pragma unroll
        for (int g = 0; g < GT; g++) {
            const float qm = sm.qmax[g];
            const int F = qm > 1e-30f ? 6 - ilogbf(qm) : 0;
            const float v = ldexpf(sm.q[g][32 * b + code], F - d);
            const __half hi = __float2half_rn(v);
            const __half lo = __float2half_rn(v - __half2float(hi));
            const int nh = g, nl = GT + g;
            *reinterpret_cast<__half *>(colbase + (nh >> 3) * 2048 + (nh & 7) * 16) = hi;
            *reinterpret_cast<__half *>(colbase + (nl >> 3) * 2048 + (nl & 7) * 16) = lo;
            kc[g] = ldexpf(1.0f, 24 - F);
            if (t < 4) {
                const float m_b = (float)((1 << (kbits(t) - 1)) - 1);
                sm.cin[t][g] = -ldexpf(m_b * sm.qsum[g][t], F - 24);
            }
        }
        if (GT == 4) {
#pragma unroll
            for (int n = 8; n < 16; n++) *reinterpret_cast<__half *>(colbase + 2048 + (n & 7) * 16) = __float2half_rn(0.0f);
        }
    }
    spb::fence_proxy_async();

    // ---- tiles: full ones by bulk copy (thread 0, one tile ahead), a ragged
    // last one by the threads ----
    uint64_t policy = 0;
    if (tid == 0) policy = spb::evict_first_policy();
    auto full = [&](int tt) { return (tt + 1) * kTM <= a.n_kv; };
    auto issue = [&](int tt, int buf) {
        const uint32_t bar = spb::smem_u32(&sm.bar[buf]);
        spb::fence_proxy_async();
        spb::mbar_expect_tx(bar, kKTileB);
        spb::bulk_g2s(spb::smem_u32(&sm.rows[buf][0]), packed + (long long)tt * kKTileB, kKTileB, bar, policy);
    };
    const int tt0 = blockIdx.x;
    if (tid == 0 && tt0 < n_tiles && full(tt0)) issue(tt0, 0);
    __syncthreads();
    uint32_t phase[2] = {0u, 0u};
    int j = 0;
    for (int tt = tt0; tt < n_tiles; tt += gridDim.x, j++) {
        const int buf = j & 1;
        const int nxt = tt + gridDim.x;
        if (tid == 0 && nxt < n_tiles && full(nxt)) issue(nxt, buf ^ 1);
        const int live = min(kTM, a.n_kv - tt * kTM);
        if (full(tt)) {
            if (!*(volatile int *)&sm.abort &&
                !spb::wait_stage(spb::smem_u32(&sm.bar[buf]), phase[buf], nullptr))
                *(volatile int *)&sm.abort = 1;
            phase[buf] ^= 1u;
        } else {
            const uint16_t *src = reinterpret_cast<const uint16_t *>(packed + (long long)tt * kKTileB);
            uint16_t *d16 = reinterpret_cast<uint16_t *>(&sm.rows[buf][0]);
            for (int i = tid; i < kTM * kKRow / 2; i += kKqTcThreads) d16[i] = i < live * kKRow / 2 ? src[i] : 0;
            __syncthreads();
        }
        const uint32_t *kr = reinterpret_cast<const uint32_t *>(&sm.rows[buf][0] + kKRow * t);
        uint32_t w[19];
#pragma unroll
        for (int i = 0; i < 19; i++) w[i] = kr[i];
        float bsc[4];
        bsc[0] = finite_or_zero_f((unsigned short)(w[0] & 0xffffu));
        bsc[1] = finite_or_zero_f((unsigned short)(w[5] >> 16));
        bsc[2] = finite_or_zero_f((unsigned short)(w[11] & 0xffffu));
        bsc[3] = finite_or_zero_f((unsigned short)(w[15] >> 16));
        static_for<4>([&](auto B) {
            constexpr int b = decltype(B)::value;
            uint32_t v[16];
            static_for<16>([&](auto R) {
                constexpr int r = decltype(R)::value;
                constexpr int bits = kbits(b);
                constexpr int W = kbit(b) + bits * kKPair[b][r][0] - kKPair[b][r][2];
                constexpr uint32_t M = (((1u << bits) - 1u) << kKPair[b][r][2]) |
                                       (((1u << bits) - 1u) << (16 + kKPair[b][r][3]));
                v[r] = window<W>(w) & M;
            });
            tmem_st16(tmem + lane_base + kQColA + 16 * b, v);
        });
        tmem_wait_st();
        tc_fence_before();
        __syncthreads();                 // A rows written; this tile's row buffer read
        if (elect_one()) {
            tc_fence_after();
            const uint32_t bq = spb::smem_u32(sm.bq);
            const int b = warp;
#pragma unroll
            for (int jj = 0; jj < 2; jj++)
                mma_ts(tmem + kQColS + 16u * b, tmem + kQColA + 16u * b + 8u * jj,
                       sdesc(bq + (uint32_t)(4 * b + 2 * jj) * 128u, 128u, 2048u), (uint32_t)jj);
            mma_commit(spb::smem_u32(&sm.bar_s));
        }
        __syncwarp();
        if (!*(volatile int *)&sm.abort && !spb::wait_stage(spb::smem_u32(&sm.bar_s), (uint32_t)(j & 1), nullptr))
            *(volatile int *)&sm.abort = 1;
        tc_fence_after();
        float su[GT];
#pragma unroll
        for (int h = 0; h < GT; h++) su[h] = 0.0f;
#pragma unroll
        for (int b = 0; b < 4; b++) {
            uint32_t d[16];
            if constexpr (GT == 4) tmem_ld8(tmem + lane_base + kQColS + 16 * b, *reinterpret_cast<uint32_t (*)[8]>(&d[0]));
            else tmem_ld16(tmem + lane_base + kQColS + 16 * b, d);
            tmem_wait_ld();
#pragma unroll
            for (int h = 0; h < GT; h++)
                su[h] = fmaf(bsc[b], __uint_as_float(d[h]) + __uint_as_float(d[GT + h]) + sm.cin[b][h], su[h]);
        }
        tc_fence_before();
        if (t < live) {
            const bool bad = *(volatile int *)&sm.abort != 0;
            float *o = dst + (long long)tt * kTM + t;
#pragma unroll
            for (int h = 0; h < GT; h++)
                if (h < a.n_head_q)
                    *reinterpret_cast<float *>(reinterpret_cast<char *>(o) + (long long)h * a.dst_stride) =
                        bad ? __int_as_float(0x7fc00000) : kc[h] * su[h];
        }
    }
    // After a timed-out wait: let the copies and MMAs in flight land
    // (bounded) before the memory is released.
    __syncthreads();
    if (sm.abort && tid == 0) {
        spb::wait_stage(spb::smem_u32(&sm.bar[0]), phase[0], nullptr);
        spb::wait_stage(spb::smem_u32(&sm.bar[1]), phase[1], nullptr);
        if (j > 0) spb::wait_stage(spb::smem_u32(&sm.bar_s), (uint32_t)((j - 1) & 1), nullptr);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kQCols) : "memory");
}

}  // namespace

// The tcgen05 scores op for K rows of the head_dim-128 ship layout with up
// to 8 query rows: 1 and *rc set if it took the call.
int sp_kq_scores_tc_try(const uint8_t *packed, long long packed_slot, int n_slots, int n_kv, const void *q,
                        int q_f16, long long q_stride, long long q_slot, int n_head_q, float *dst,
                        long long dst_stride, long long dst_slot, float inv_sqrt_n, cudaStream_t s, int *rc)
{
    if (n_head_q > 8 || ((uintptr_t)packed & 15) || (packed_slot & 15) || getenv("SHANNON_PRIME_KQ_SIMT"))
        return 0;
    KqTcArgs a{packed, packed_slot, q, q_stride, q_slot, dst, dst_stride, dst_slot, n_kv, n_head_q, q_f16,
               inv_sqrt_n};
    const bool wide = n_head_q > 4;
    auto k = wide ? k_kq_scores_tc<8> : k_kq_scores_tc<4>;
    const size_t smem = sizeof(KqSmem);
    constexpr int kMaxDev = 64;
    static std::atomic<int> ready[kMaxDev][2];
    static std::atomic<int> sms_tab[kMaxDev];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDev) return 0;
    if (!ready[dev][wide].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
            *rc = sp_check_cuda(cudaGetLastError(), "kq_scores tcgen05 smem attribute");
            return 1;
        }
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        sms_tab[dev].store(sms > 0 ? sms : 148, std::memory_order_relaxed);
        ready[dev][wide].store(1, std::memory_order_release);
    }
    const int sms = sms_tab[dev].load(std::memory_order_relaxed);
    const int n_tiles = (n_kv + kTM - 1) / kTM;
    // three resident CTAs per SM in total, each walking its slot's tiles
    // (four measured 1.18 against 1.11 us per slot)
    int gx = (3 * sms + n_slots - 1) / n_slots;
    if (gx > n_tiles) gx = n_tiles;
    if (gx < 1) gx = 1;
    k<<<dim3((unsigned)gx, (unsigned)n_slots), kKqTcThreads, smem, s>>>(a);
    *rc = sp_check_cuda(cudaGetLastError(), "kq_scores tcgen05 launch");
    return 1;
}
