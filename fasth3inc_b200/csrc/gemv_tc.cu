// gemv_tc.cu -- Q4_K GEMV for 1..16 tokens on tcgen05 integer MMAs.
//
// The small-M regime of fh3_matmul (src/core/fh3_ops.c:317-404):
//   y[t][n] = sum_j ( (d*sc_j) * P_tnj - (dmin*m_j) * X_tj ),  P = sum_{k in j} q_nk x_tk,
//   X_tj = sum_{k in j} x_tk over the 32-weight sub-blocks j of each super-block
//   (w = (d*sc)*q - dmin*m as dequant_q4_k, src/core/fh3_quant.c:154-196).
//
// Work unit: a tile of 128 weight rows x one super-block (256 k).  One persistent CTA
// per SM walks a contiguous run of units (stream-K, tile by tile, the super-block
// fastest); a tile split between CTAs is finished by the last CTA to arrive on the tile's
// counter, adding the pieces' partial sums in a fixed order.
//
// * Weights: one TMA box per unit, 144 bytes x 128 rows (the super-block column of the
//   tile), into a ring of stages.  The first stages load before griddepcontrol.wait.
// * 1..5 tokens (kind::i8): warps 0-7 (two per TMEM lane quarter, one weight row per
//   lane) expand the row's 128 nibble bytes into 256 u8 values q in k order (low nibbles
//   of chunk c are k = 64c + i, high nibbles k = 64c + 32 + i) in tensor memory.  B = x of
//   token t and super-block b, rounded to a 23-bit integer under a power of two 2^s
//   (max|x| * 2^s < 2^22), in three balanced signed base-256 digits (row 3t + p holds digit
//   p), built once per CTA for the super-blocks its run touches, K-major in the 128-byte
//   swizzle layout.  One MMA per sub-block (M 128, N 16, K 32) into its own TMEM columns:
//   int32 plane sums, exact; P = P0 + 256 P1 + 65536 P2 (one fp32 rounding), then the
//   scales in fp32 as the reference forms them (d*sc and dmin*m are exact products).
// * 6..16 tokens (kind::f16): warps 0-7 (two per TMEM lane quarter, half a row each)
//   write A = sc * q as f16 (exact) and the eight mins; gemv_xprep_kernel writes B once per call (x as f16 hi + lo pieces
//   and the sub-block sums, in the A operand's k order) and each unit bulk-copies its B
//   block from L2 into a ring; 16 MMAs (K 16) give sum_j sc_j P_tj and one more the min
//   term, each in one accumulator of 2 x tokens columns.
// Roles: the expanders, eight accumulator readers (two per lane quarter; for 6..16 tokens
// the part-0 warp of a quarter reads both accumulators and the part-1 warp has nothing to
// add), one TMA warp and one warp that
// allocates TMEM and issues the MMAs.  A and accumulator buffers let expansion run ahead
// of the MMAs and the accumulator reads trail them.
// Every wait is bounded; on a timeout the kernel records FH3CUDA_E_TIMEOUT, lets its
// copies and MMAs finish and frees tensor memory.
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "common.cuh"

namespace {

constexpr int kGtRows = 128;                               // rows of a tile = TMEM lanes
constexpr int kGtStages = 6;                               // weight stages of 1..5 tokens (6..16: 5)
constexpr int kGtStageBytes = kGtRows * fh3::kQ4KBytes;    // 18432
constexpr int kGtMaxTok = 16;
constexpr int kGtHdrs = 8;                                 // ring of the units' 16-byte row headers
constexpr int kGtPreSegs = 2;                              // other segments of the last tile read ahead
constexpr uint32_t kGtTmemCols = 512;
#ifndef FH3_GT_SPIN
#define FH3_GT_SPIN 0
#endif
constexpr bool kGtSpin = FH3_GT_SPIN != 0;  // spin (no suspend-time hint) in the role warps' waits

constexpr int align16(int v) { return (v + 15) & ~15; }

// Per-token-count configuration: accumulator columns per sub-block, buffer counts,
// B slots and the shared-memory layout.
template <int M>
struct GtCfg {
    // 1..5 tokens: kind::i8 MMAs of the nibbles, one accumulator per sub-block (eight a
    // unit), the B operand of the run's super-blocks resident in shared memory.
    // 6..16 tokens: kind::f16 MMAs of sc * q (the 6-bit scale folded into the A operand,
    // exact in fp16) into one accumulator a unit, and of the mins against the sub-block
    // sums into a second; the B blocks are built once per call by gemv_xprep_kernel and
    // streamed from L2 beside the weights, so the units run tile by tile over the whole K.
    static constexpr bool F16 = M > 5;
    static constexpr int NC = F16 ? (M <= 8 ? 16 : 32) : 16;       // B rows = accumulator columns (a sub-block's / a unit's)
    static constexpr int DB = 2;                                   // accumulator buffers
    static constexpr int ACOLS = F16 ? 144 : 64;                   // TMEM columns of one A buffer (f16: 128 of sc*q, 16 of mins)
    static constexpr int AB = F16 ? 2 : 4;                         // A buffers
    static constexpr int DCOLS = F16 ? 2 * NC : 8 * NC;            // accumulator columns of one unit
    static constexpr uint32_t TM_A = DB * DCOLS;                   // first A column
    static constexpr int STAGES = F16 ? 5 : kGtStages;
    // B of one super-block: K blocks of 128 bytes x NC rows (i8: 2 blocks of 128 k;
    // f16: 4 blocks of 64 k and one holding the 8 sub-block sums)
    static constexpr int SLOT_BYTES = (F16 ? 640 : 256) * NC;
    static constexpr int HALF_BYTES = 128 * NC;                    // one K block
    static constexpr int SLOTS = F16 ? 4 : 20;                     // i8: resident B slots; f16: the B ring's stages
    static constexpr int CHUNK = 0;                                // super-blocks a chunk (0: the whole K)
    // expander warps: two per TMEM lane quarter, half a row each
    static constexpr int EXP = 8;
    static constexpr int WARP_RD = EXP;                            // first of the 8 accumulator readers
    static constexpr int WARP_TMA = EXP + 8, WARP_MMA = EXP + 9;
    static constexpr int THREADS = (EXP + 10) * 32;
    static constexpr int OFF_STAGE = 0;
    static constexpr int OFF_B = OFF_STAGE + STAGES * kGtStageBytes;
    static constexpr int OFF_X = OFF_B + SLOTS * SLOT_BYTES;       // i8: sub-block sums [slot][t][8]
    static constexpr int OFF_FS = OFF_X + (F16 ? 0 : SLOTS * M * 8 * 4);  // i8: 2^-s [slot][t]
    static constexpr int OFF_RED = OFF_FS + (F16 ? 0 : SLOTS * M * 4);    // pair exchange [quarter][lane][t]
    static constexpr int OFF_HDR = align16(OFF_RED + 4 * 32 * M * 4);  // [kGtHdrs][128] x 16 B
    static constexpr int OFF_BAR = OFF_HDR + kGtHdrs * kGtRows * 16;
    static constexpr int NBARS = 2 * STAGES + 2 * AB + 2 * DB + 8 + 2 * kGtHdrs + 2 + (F16 ? 2 * SLOTS : 0);
    static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
    static constexpr int SMEM = OFF_MISC + 16 + 1024;              // + alignment slack
    static_assert(TM_A + ACOLS * AB <= kGtTmemCols, "tensor memory");
    static_assert(OFF_B % 1024 == 0 && SLOT_BYTES % 1024 == 0 && HALF_BYTES % 1024 == 0, "B alignment");
    static_assert((F16 ? 2 : 3) * M <= NC, "B rows");
    static_assert(SLOT_BYTES % 1024 == 0 && OFF_B % 1024 == 0, "B blocks are 1024-byte aligned");
    static_assert(SMEM <= 227 * 1024, "shared memory");
};

struct GtBars {
    uint64_t* full;    // [STAGES] TMA -> expanders
    uint64_t* empty;   // [STAGES] expanders (EXP warps) -> TMA
    uint64_t* afull;   // [AB] A written (EXP warps) -> MMA
    uint64_t* aempty;  // [AB] MMA done -> expanders
    uint64_t* dfull;   // [DB] MMA done -> accumulator readers
    uint64_t* dempty;  // [DB] accumulators read (8 warps) -> MMA
    uint64_t* xfull;   // [4] part-1 warp's sums in shared memory -> part-0 warp
    uint64_t* xempty;  // [4] part-0 warp has read them -> part-1 warp
    uint64_t* hfull;   // [kGtHdrs] headers copied (one warp per lane quarter) -> accumulator readers
    uint64_t* hempty;  // [kGtHdrs] headers read (8 warps) -> expanders
    uint64_t* bfull;   // B operand built (8 warps) -> MMA and accumulator readers
    uint64_t* drain;
    uint64_t* bring;   // f16: [SLOTS] B block landed (TMA) -> MMA
    uint64_t* bfree;   // f16: [SLOTS] MMA done -> TMA
};
template <int M>
__device__ __forceinline__ GtBars gt_bars(uint8_t* smem) {
    using C = GtCfg<M>;
    uint64_t* b = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    GtBars r;
    r.full = b;
    r.empty = r.full + C::STAGES;
    r.afull = r.empty + C::STAGES;
    r.aempty = r.afull + C::AB;
    r.dfull = r.aempty + C::AB;
    r.dempty = r.dfull + C::DB;
    r.xfull = r.dempty + C::DB;
    r.xempty = r.xfull + 4;
    r.hfull = r.xempty + 4;
    r.hempty = r.hfull + kGtHdrs;
    r.bfull = r.hempty + kGtHdrs;
    r.drain = r.bfull + 1;
    r.bring = r.drain + 1;
    r.bfree = r.bring + (C::F16 ? C::SLOTS : 0);
    return r;
}

__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// D[tmem] = A[tmem] * B[smem desc]^T, kind::i8 (A u8, B s8, D s32), one thread.
__device__ __forceinline__ void umma_i8_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// kind::i8 instruction descriptor: A u8, B s8, D s32, both K-major
__host__ __device__ constexpr uint32_t idesc_u8s8_s32(int m, int n) {
    return (2u << 4)                                  // D format: s32
           | (0u << 7)                                // A format: unsigned 8-bit
           | (1u << 10)                               // B format: signed 8-bit
           | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
           | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

// D[tmem] = A[tmem] * B[smem desc]^T, kind::f16 (A and B f16, D f32), one thread.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// kind::f16 instruction descriptor: A and B f16, D f32, both K-major
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n) {
    return (1u << 4)                                  // D format: f32
           | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
           | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}
// a * b + c on f16 pairs, one rounding
__device__ __forceinline__ uint32_t hfma2_bits(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// f16 bits of a small integer |v| <= 2048 * 64 with at most 11 significant bits (exact)
__device__ __forceinline__ uint32_t half_bits_int(int v) {
    return static_cast<uint32_t>(__half_as_ushort(__int2half_rn(v)));
}

// 32 lanes x W consecutive 32-bit columns (one row per thread); W > 16 in loads of 16
template <int W>
__device__ __forceinline__ void tmem_ld_w(uint32_t taddr, uint32_t* r) {
    static_assert(W == 4 || W == 8 || W % 16 == 0, "width");
    if constexpr (W == 4) {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                     : "r"(taddr));
    } else if constexpr (W == 8) {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                       "=r"(r[7])
                     : "r"(taddr));
    } else {
#pragma unroll
        for (int c = 0; c < W / 16; ++c) {
            uint32_t* q = r + 16 * c;
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                "%13, %14, %15}, [%16];"
                : "=r"(q[0]), "=r"(q[1]), "=r"(q[2]), "=r"(q[3]), "=r"(q[4]), "=r"(q[5]), "=r"(q[6]), "=r"(q[7]),
                  "=r"(q[8]), "=r"(q[9]), "=r"(q[10]), "=r"(q[11]), "=r"(q[12]), "=r"(q[13]), "=r"(q[14]),
                  "=r"(q[15])
                : "r"(taddr + 16 * c));
        }
    }
}

__device__ __forceinline__ uint4 lds128(const uint8_t* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(fh3::smem_u32(p)));
    return v;
}

// the CTA whose run [c*U/G, (c+1)*U/G) holds unit u (U * G < 2^32, checked by the host)
__device__ __forceinline__ int gt_cta_of(uint32_t u, uint32_t G, uint32_t units) {
    return static_cast<int>(((u + 1) * G - 1) / units);
}

// Position of a unit in the chunked order: chunk k (super-blocks k*cw .. k*cw + w - 1),
// tile, super-block b.
struct UnitPos {
    int k, tile, b, w;
};
__device__ __forceinline__ UnitPos unit_pos(int64_t u, int ntiles, int nblk, int cw) {
    const int64_t cu = static_cast<int64_t>(ntiles) * cw;  // units of a full chunk
    UnitPos p;
    p.k = static_cast<int>(u / cu);
    const int64_t l = u - p.k * cu;
    p.w = min(cw, nblk - p.k * cw);
    p.tile = static_cast<int>(l / p.w);
    p.b = p.k * cw + static_cast<int>(l - static_cast<int64_t>(p.tile) * p.w);
    return p;
}
__device__ __forceinline__ void unit_next(UnitPos& p, int ntiles, int nblk, int cw) {
    if (++p.b == p.k * cw + p.w) {
        p.b = p.k * cw;
        if (++p.tile == ntiles) {
            p.tile = 0;
            ++p.k;
            p.b = p.k * cw;
            p.w = min(cw, nblk - p.b);
        }
    }
}

// 2^e exactly for -149 <= e <= 127 (subnormal below -126)
__device__ __forceinline__ float pow2_exact(int e) {
    return e >= -126 ? __uint_as_float(static_cast<uint32_t>(e + 127) << 23) : __uint_as_float(1u << (e + 149));
}

// B operand and sub-block sums of one super-block (slot `slot`) for token t from the
// warp's x values (lane l holds elements 8l .. 8l+7, sub-block l/4).
template <int M>
__device__ __forceinline__ void build_b(const float4& v0, const float4& v1, int t, int slot, uint8_t* smem,
                                        int lane) {
    using C = GtCfg<M>;
    const float e[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    float am = 0.0f;
    bool fin = true;  // false for an Inf or NaN element
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        am = fmaxf(am, fabsf(e[i]));
        fin = fin && fabsf(e[i]) <= 3.40282347e38f;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    // a non-finite x has no integer digits: the super-block's factor becomes NaN, so every
    // output of the token is NaN (fh3_matmul gives a non-finite value there too: Inf times
    // a weight, and 0 * Inf for a zero weight)
    const bool all_fin = __all_sync(0xffffffffu, fin);
    // E with am < 2^E from the exponent field (subnormal am scaled up by 2^64 first)
    int E = 0;
    if (am > 0.0f && am <= 3.0e38f)
        E = am >= 1.17549435e-38f ? static_cast<int>(__float_as_uint(am) >> 23) - 126
                                  : static_cast<int>(__float_as_uint(am * 18446744073709551616.0f) >> 23) - 190;
    const int s = min(22 - E, 149);                  // max|x| * 2^s < 2^22
    const int s1 = min(s, 127);
    const float m1 = pow2_exact(s1), m2 = pow2_exact(s - s1);  // x * 2^s exactly, in two steps
    uint32_t pw[3][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        // round to the nearest integer (ties to even) through the bits of 1.5 * 2^23 + v, |v| < 2^22
        const int xi = __float_as_int((e[i] * m1) * m2 + 12582912.0f) - 0x4B400000;
        const int d0 = ((xi + 128) & 255) - 128;
        const int x1 = (xi - d0) >> 8;                   // exact: xi - d0 is a multiple of 256
        const int d1 = ((x1 + 128) & 255) - 128;
        const int d2 = (x1 - d1) >> 8;                   // |d2| <= 64
        const int sh = 8 * (i & 3);
        pw[0][i >> 2] |= static_cast<uint32_t>(d0 & 255) << sh;
        pw[1][i >> 2] |= static_cast<uint32_t>(d1 & 255) << sh;
        pw[2][i >> 2] |= static_cast<uint32_t>(d2 & 255) << sh;
    }
    // element kk = 8l + i: half kk >> 7, 16-byte chunk (kk & 127) >> 4, byte 8(l & 1) + i
    const int h = lane >> 4, c = (lane & 15) >> 1;
    uint8_t* bs = smem + C::OFF_B + slot * C::SLOT_BYTES + h * C::HALF_BYTES;
#pragma unroll
    for (int p = 0; p < 3; ++p) {
        const int n = 3 * t + p;
        uint8_t* dst = bs + (n >> 3) * 1024 + (n & 7) * 128 + ((c ^ (n & 7)) << 4) + 8 * (lane & 1);
        *reinterpret_cast<uint2*>(dst) = make_uint2(pw[p][0], pw[p][1]);
    }
    float sum = ((e[0] + e[1]) + (e[2] + e[3])) + ((e[4] + e[5]) + (e[6] + e[7]));
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    float* sx = reinterpret_cast<float*>(smem + C::OFF_X) + (slot * M + t) * 8;
    if ((lane & 3) == 0) sx[lane >> 2] = sum;
    if (lane == 0)
        reinterpret_cast<float*>(smem + C::OFF_FS)[slot * M + t] = all_fin ? pow2_exact(-s) : __int_as_float(0x7FC00000);
}

// B blocks of 6..16 tokens, once per call: block b (GtCfg<M>::SLOT_BYTES bytes) holds, for
// token t, rows 2t and 2t + 1 (f16, K-major, 128-byte swizzle):
//  * K blocks 0..3: x * 2^s as hi + lo, hi = f16(x 2^s), lo = f16(x 2^s - hi), with one
//    power of two per token and super-block (max|x| * 2^s < 2^15 over the super-block, as
//    the 1..5-token operands; the residual is below 2^-22 of that max), in the A operand's
//    k order: k = 64c + 32hb + 4u + r sits at e = 64c + 8u + 4hb + 2(r & 1) + (r >> 1), so
//    that one 32-bit word of nibbles gives the f16 pairs (k, k + 2) of A with a mask (see
//    the expanders);
//  * K block 4, elements 0..7: the sub-block sums X_j = sum of x over sub-block j (in fp32)
//    times 2^(s-5), as hi + lo; elements 8..15 zero.
// fs[b * M + t] = 2^-s.  Grid (tokens, groups of 4 super-blocks), 1024 threads: thread k of
// super-block q of the group (one element each).
template <int M>
__global__ void __launch_bounds__(1024) gemv_xprep_kernel(const float* __restrict__ x, int nblk,
                                                          uint8_t* __restrict__ bglob, float* __restrict__ fs) {
    using C = GtCfg<M>;
    pdl_launch_dependents();  // the GEMV's weight stream may start now; its B loads wait for this grid
    pdl_wait();               // x, and the B buffer the previous call may still be reading
    __shared__ float red[32];
    const int t = blockIdx.x, tid = threadIdx.x, k = tid & 255, q = tid >> 8, lane = tid & 31, wid = (tid >> 5) & 7;
    const int64_t K = static_cast<int64_t>(nblk) * 256;
    const int b = blockIdx.y * 4 + q;
    const float v = b < nblk ? __ldg(x + t * K + static_cast<int64_t>(b) * 256 + k) : 0.0f;
    float am = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    if (lane == 0) red[tid >> 5] = am;
    __syncthreads();
    am = red[8 * q];
#pragma unroll
    for (int w = 1; w < 8; ++w) am = fmaxf(am, red[8 * q + w]);  // over super-block b
    if (b >= nblk) return;  // uniform over each warp, after the CTA barrier
    int E = 0;  // am < 2^E
    if (am > 0.0f && am <= 3.0e38f)
        E = am >= 1.17549435e-38f ? static_cast<int>(__float_as_uint(am) >> 23) - 126
                                  : static_cast<int>(__float_as_uint(am * 18446744073709551616.0f) >> 23) - 190;
    const int s = min(15 - E, 149);
    const int s1 = min(s, 127), sx = s - 5, sx1 = max(min(sx, 127), -126);
    const float m1 = pow2_exact(s1), m2 = pow2_exact(s - s1);     // x * 2^s exactly, in two steps
    const float n1 = pow2_exact(sx1), n2 = pow2_exact(sx - sx1);   // X * 2^(s-5)
    if (k == 0) fs[static_cast<size_t>(b) * M + t] = pow2_exact(-s);
    // this thread's element and its position in the A operand's k order
    const int c = k >> 6, hb = (k >> 5) & 1, u = (k >> 2) & 7, r = k & 3;
    const int ee = 8 * u + 4 * hb + 2 * (r & 1) + (r >> 1);  // within K block c
    uint8_t* blk = bglob + static_cast<size_t>(b) * C::SLOT_BYTES;
    const float xs = (v * m1) * m2;
    const __half hi = __float2half_rn(xs);
    const __half lo = __float2half_rn(xs - __half2float(hi));  // the difference is exact in fp32
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        const int n = 2 * t + p;
        *reinterpret_cast<__half*>(blk + c * C::HALF_BYTES + (n >> 3) * 1024 + (n & 7) * 128 +
                                   (((ee >> 3) ^ (n & 7)) << 4) + (ee & 7) * 2) = p ? lo : hi;
    }
    // sub-block wid = elements 32 wid .. 32 wid + 31 of this super-block
    float X = v;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) X += __shfl_xor_sync(0xffffffffu, X, o);
    if (lane == 0) {
        const float xs2 = (X * n1) * n2;
        const __half xh = __float2half_rn(xs2);
        const __half xl = __float2half_rn(xs2 - __half2float(xh));
#pragma unroll
        for (int p = 0; p < 2; ++p) {
            const int n = 2 * t + p;
            *reinterpret_cast<__half*>(blk + 4 * C::HALF_BYTES + (n >> 3) * 1024 + (n & 7) * 128 + ((n & 7) << 4) +
                                       wid * 2) = p ? xl : xh;
        }
    }
    if (k < 2) {  // elements 8..15 of K block 4 meet the zero columns of A: keep them finite
        const int n = 2 * t + k;
        *reinterpret_cast<uint4*>(blk + 4 * C::HALF_BYTES + (n >> 3) * 1024 + (n & 7) * 128 + ((1 ^ (n & 7)) << 4)) =
            make_uint4(0u, 0u, 0u, 0u);
    }
}

// exact int -> float for |v| < 2^22 on the FMA pipe: the bits of 1.5 * 2^23 + v
__device__ __forceinline__ float small_i2f(uint32_t v) {
    return __uint_as_float(v + 0x4B400000u) - 12582912.0f;
}

template <int M>
__global__ void __launch_bounds__(GtCfg<M>::THREADS, 1) gemv_tc_kernel(
    const __grid_constant__ CUtensorMap tmW, int nblk, int ntiles, int64_t N, int64_t units, int cw, int split,
    int seg_max, const float* __restrict__ x, const float* __restrict__ bias, float* __restrict__ y, int64_t ldy,
    float* __restrict__ partials, int* __restrict__ counters, const uint8_t* __restrict__ bglob,
    const float* __restrict__ fsg, int* status) {
    using C = GtCfg<M>;
    static_assert(M >= 1 && M <= kGtMaxTok, "1..16 tokens");
    constexpr int W = M == 1 ? 4 : (M == 2 ? 8 : 16 * ((3 * M + 15) / 16));  // accumulator columns read per sub-block
    constexpr int JB = M <= 2 ? 4 : (M <= 5 ? 2 : 1);                         // sub-blocks read per batch
    constexpr bool kOneChunk = C::CHUNK == 0;                                 // cw == nblk
    constexpr uint32_t idesc = idesc_u8s8_s32(128, C::NC);
    constexpr uint32_t idesc16 = idesc_f16_f32(128, C::NC);
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const GtBars B = gt_bars<M>(smem);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int64_t G = gridDim.x;  // <= units: every run is non-empty
    const int64_t u0 = static_cast<int64_t>(blockIdx.x) * units / G;
    const int n = static_cast<int>((static_cast<int64_t>(blockIdx.x) + 1) * units / G - u0);
    const UnitPos p_first = unit_pos(u0, ntiles, nblk, cw);
    const UnitPos p_last = unit_pos(u0 + n - 1, ntiles, nblk, cw);
    // B slots: with one chunk, the run's super-blocks cyclically from its first; with
    // chunks, the super-blocks of the (at most two) chunks the run touches
    const int sbase = kOneChunk ? p_first.b : p_first.k * cw;
    const int nslots = kOneChunk ? min(nblk, n) : min(nblk, (p_last.k + 1) * cw) - sbase;
    auto slot_of = [&](int b) {
        const int d = b - sbase;
        return d < 0 ? d + nblk : d;
    };

    if (threadIdx.x == 0) {
        for (int i = 0; i < C::STAGES; ++i) {
            fh3::mbar_init(&B.full[i], 1);
            fh3::mbar_init(&B.empty[i], C::EXP);
        }
        for (int i = 0; i < C::AB; ++i) {
            fh3::mbar_init(&B.afull[i], C::EXP);
            fh3::mbar_init(&B.aempty[i], 1);
        }
        for (int i = 0; i < C::DB; ++i) {
            fh3::mbar_init(&B.dfull[i], 1);
            fh3::mbar_init(&B.dempty[i], C::F16 ? 4 : 8);  // f16: the part-0 readers alone read them
        }
        for (int i = 0; i < 4; ++i) {
            fh3::mbar_init(&B.xfull[i], 1);
            fh3::mbar_init(&B.xempty[i], 1);
        }
        for (int i = 0; i < kGtHdrs; ++i) {
            fh3::mbar_init(&B.hfull[i], 4);
            fh3::mbar_init(&B.hempty[i], 8);
        }
        fh3::mbar_init(B.bfull, 8);
        fh3::mbar_init(B.drain, 1);
        if constexpr (C::F16)
            for (int i = 0; i < C::SLOTS; ++i) {
                fh3::mbar_init(&B.bring[i], 1);
                fh3::mbar_init(&B.bfree[i], 1);
            }
        *abort_flag = 0;
        fh3::fence_mbar_init();
    }
    if (warp == C::WARP_MMA) {
        fh3::tmem_alloc(tmem_slot, kGtTmemCols);
        fh3::tmem_relinquish();
    }
    fh3::tc_fence_before();
    __syncthreads();
    fh3::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // unit i of this run -> stage i % STAGES; weights do not depend on earlier kernels
    int issued = 0;
    UnitPos lp = p_first;  // the next unit to load
    auto issue = [&](int i) {
        const int st = i % C::STAGES;
        fh3::mbar_arrive_expect_tx(&B.full[st], kGtStageBytes);
        fh3::tma_load_2d(smem + C::OFF_STAGE + st * kGtStageBytes, &tmW, &B.full[st], lp.b * fh3::kQ4KBytes,
                         lp.tile * kGtRows);
        unit_next(lp, ntiles, nblk, cw);
    };
    if (warp == C::WARP_TMA && lane == 0) {
        fh3::tma_prefetch_desc(&tmW);
        for (; issued < min(n, C::STAGES); ++issued) issue(issued);
    }
    pdl_launch_dependents();
    // Only the accumulator readers touch x, y and the scratch (after griddepcontrol.wait);
    // the weight pipeline starts at once.

    // every lane waits (the TMA bytes, shared-memory handoffs and TMEM results become
    // visible to each of them)
    auto wait_all = [&](uint64_t* bar, uint32_t parity) {
        const bool w = fh3::mbar_wait<kGtSpin>(bar, parity, abort_flag, status);
        return __all_sync(0xffffffffu, w);
    };

    if (warp == C::WARP_TMA) {
        // ------------------------------------------------------------ TMA producer
        if (C::F16 && lane == 0) {
            // weights of unit i, then its B block (super-block b of the pre-pass's output;
            // after griddepcontrol.wait), each into its own ring
            pdl_wait();
            UnitPos bp = p_first;
            int bissued = 0;
            bool ok = true;
            for (int i = 0; i < n && ok; ++i) {
                if (i >= issued) {
                    const int st = i % C::STAGES;
                    if (!(ok = fh3::mbar_wait<kGtSpin>(&B.empty[st], ((i / C::STAGES) - 1) & 1, abort_flag, status)))
                        break;
                    issue(i);
                    issued = i + 1;
                }
                const int bs = i % C::SLOTS;
                if (i >= C::SLOTS &&
                    !(ok = fh3::mbar_wait<kGtSpin>(&B.bfree[bs], ((i / C::SLOTS) - 1) & 1, abort_flag, status)))
                    break;
                fh3::mbar_arrive_expect_tx(&B.bring[bs], C::SLOT_BYTES);
                fh3::bulk_load(smem + C::OFF_B + bs * C::SLOT_BYTES, bglob + static_cast<size_t>(bp.b) * C::SLOT_BYTES,
                               C::SLOT_BYTES, &B.bring[bs]);
                bissued = i + 1;
                unit_next(bp, ntiles, nblk, cw);
            }
            // every copy issued lands before the CTA can leave
            volatile int no_abort = 0;
            for (int i = max(0, issued - C::STAGES); i < issued; ++i)
                fh3::mbar_wait<true>(&B.full[i % C::STAGES], (i / C::STAGES) & 1, &no_abort, nullptr);
            for (int i = max(0, bissued - C::SLOTS); i < bissued; ++i)
                fh3::mbar_wait<true>(&B.bring[i % C::SLOTS], (i / C::SLOTS) & 1, &no_abort, nullptr);
        } else if (lane == 0) {
            for (; issued < n; ++issued) {
                const int st = issued % C::STAGES;
                if (!fh3::mbar_wait<kGtSpin>(&B.empty[st], ((issued / C::STAGES) - 1) & 1, abort_flag, status))
                    break;
                issue(issued);
            }
            // every copy issued lands before the CTA can leave
            volatile int no_abort = 0;
            for (int i = max(0, issued - C::STAGES); i < issued; ++i)
                fh3::mbar_wait<true>(&B.full[i % C::STAGES], (i / C::STAGES) & 1, &no_abort, nullptr);
        }
    } else if (warp == C::WARP_MMA) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t bbase = fh3::smem_u32(smem + C::OFF_B);
            const bool bok = fh3::mbar_wait<true>(B.bfull, 0, abort_flag, status);
            UnitPos mp = p_first;
            for (int i = 0; i < n && bok; ++i) {
                const int ab = i % C::AB, d = i % C::DB;
                if (!fh3::mbar_wait<true>(&B.afull[ab], (i / C::AB) & 1, abort_flag, status)) break;
                if (i >= C::DB && !fh3::mbar_wait<true>(&B.dempty[d], ((i / C::DB) - 1) & 1, abort_flag, status))
                    break;
                fh3::tc_fence_after();
                const uint32_t bs = bbase + slot_of(mp.b) * C::SLOT_BYTES;
                if constexpr (C::F16) {
                    // the unit's B block from the ring; 16 steps of K = 16 of sc * q into the
                    // unit's first accumulator, one of the mins against the sub-block sums into
                    // its second
                    const int bsl = i % C::SLOTS;
                    if (!fh3::mbar_wait<true>(&B.bring[bsl], (i / C::SLOTS) & 1, abort_flag, status)) break;
                    fh3::tc_fence_after();
                    const uint32_t bb = bbase + bsl * C::SLOT_BYTES;
#pragma unroll
                    for (int k = 0; k < 16; ++k)
                        umma_f16_ts(tmem + C::DCOLS * d, tmem + C::TM_A + C::ACOLS * ab + 8 * k,
                                    fh3::sdesc_sw128(bb + (k >> 2) * C::HALF_BYTES) + 2 * (k & 3), idesc16,
                                    k != 0 ? 1u : 0u);
                    umma_f16_ts(tmem + C::DCOLS * d + C::NC, tmem + C::TM_A + C::ACOLS * ab + 128,
                                fh3::sdesc_sw128(bb + 4 * C::HALF_BYTES), idesc16, 0u);
                    fh3::umma_commit(&B.bfree[bsl]);
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        umma_i8_ts(tmem + C::DCOLS * d + C::NC * j, tmem + C::TM_A + C::ACOLS * ab + 8 * j,
                                   fh3::sdesc_sw128(bs + (j >> 2) * C::HALF_BYTES) + 2 * (j & 3), idesc, 0u);
                }
                fh3::umma_commit(&B.dfull[d]);
                fh3::umma_commit(&B.aempty[ab]);
                unit_next(mp, ntiles, nblk, cw);
            }
            fh3::umma_commit(B.drain);  // every MMA issued retires before TMEM is freed
            volatile int no_abort = 0;
            fh3::mbar_wait<true>(B.drain, 0, &no_abort, nullptr);
        }
    } else if (warp < C::EXP) {
        // ------------------------------------------------------------ expanders
        // part p of a row: nibble bytes 64p .. 64p+63 (chunks 2p, 2p+1) -> A columns 32p ..;
        // a warp takes PARTS consecutive parts of the rows of its lane quarter
        constexpr int PARTS = 8 / C::EXP;
        const int q = warp & 3, part0 = (warp >> 2) * PARTS;
        const int r = q * 32 + lane;
        const uint32_t ta0 = tmem + (static_cast<uint32_t>(q * 32) << 16) + C::TM_A + 32 * part0;
        for (int i = 0; i < n; ++i) {
            const int st = i % C::STAGES, ab = i % C::AB;
            if (!wait_all(&B.full[st], (i / C::STAGES) & 1)) break;
            const uint8_t* rp = smem + C::OFF_STAGE + st * kGtStageBytes + r * fh3::kQ4KBytes + 16 + 64 * part0;
            uint4 qv[4 * PARTS];
#pragma unroll
            for (int c = 0; c < 4 * PARTS; ++c) qv[c] = lds128(rp + 16 * c);
            uint4 hd = make_uint4(0u, 0u, 0u, 0u);
            if (part0 == 0 || C::F16)  // the row's header: d, dmin, scales, mins
                hd = lds128(smem + C::OFF_STAGE + st * kGtStageBytes + r * fh3::kQ4KBytes);
            // these generic-proxy reads must be performed before the TMA (async proxy)
            // refills the stage: a cross-proxy fence, then the release
            fh3::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) fh3::mbar_arrive(&B.empty[st]);
            if (part0 == 0) {  // header -> ring slot i % kGtHdrs for the accumulator readers
                const int hs = i % kGtHdrs;
                if (i >= kGtHdrs && !wait_all(&B.hempty[hs], ((i / kGtHdrs) - 1) & 1)) break;
                *reinterpret_cast<uint4*>(smem + C::OFF_HDR + (hs * kGtRows + r) * 16) = hd;
                __syncwarp();
                if (lane == 0) fh3::mbar_arrive(&B.hfull[hs]);
            }
            if (i >= C::AB && !wait_all(&B.aempty[ab], ((i / C::AB) - 1) & 1)) break;
            fh3::tc_fence_after();
            if constexpr (C::F16) {
                // column 32c + 4u + {0, 1, 2, 3} of chunk c, word u (bytes b0..b3) holds the f16
                // pairs sc * (lo b0, lo b2), (lo b1, lo b3), (hi b0, hi b2), (hi b1, hi b3):
                // 0x6400 | q is the f16 1024 + q, and (1024 + q) * sc - 1024 sc = sc * q exactly.
                // This warp's half of the row: chunks 2 part0 and 2 part0 + 1.
                const uint32_t taf = tmem + (static_cast<uint32_t>(q * 32) << 16) + C::TM_A + C::ACOLS * ab;
                if (part0 == 0) {
                    // columns 128 .. 143: the mins m_0 .. m_7 as elements 0..7 of one K = 16 step
                    uint32_t mo[16];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        int sc, m;
                        fh3::q4k_scale_min_words(hd.y, hd.z, hd.w, j, sc, m);
                        if (j & 1)
                            mo[j >> 1] |= half_bits_int(m) << 16;
                        else
                            mo[j >> 1] = half_bits_int(m);
                    }
#pragma unroll
                    for (int j = 4; j < 16; ++j) mo[j] = 0u;
                    fh3::tmem_st16(taf + 128, mo);
                }
#pragma unroll
                for (int cl = 0; cl < 2; ++cl) {
                    const int c = 2 * part0 + cl;
                    uint32_t s2[2], n2[2];
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        int sc, m;
                        fh3::q4k_scale_min_words(hd.y, hd.z, hd.w, 2 * c + h, sc, m);
                        const uint32_t hs = half_bits_int(sc), hn = half_bits_int(-1024 * sc);
                        s2[h] = hs | (hs << 16);
                        n2[h] = hn | (hn << 16);
                    }
                    const uint4 a = qv[2 * cl], b2 = qv[2 * cl + 1];
                    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b2.x, b2.y, b2.z, b2.w};
                    uint32_t o[32];
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        o[4 * u + 0] = hfma2_bits((w[u] & 0x000F000Fu) | 0x64006400u, s2[0], n2[0]);
                        o[4 * u + 1] = hfma2_bits(((w[u] >> 8) & 0x000F000Fu) | 0x64006400u, s2[0], n2[0]);
                        o[4 * u + 2] = hfma2_bits(((w[u] >> 4) & 0x000F000Fu) | 0x64006400u, s2[1], n2[1]);
                        o[4 * u + 3] = hfma2_bits(((w[u] >> 12) & 0x000F000Fu) | 0x64006400u, s2[1], n2[1]);
                    }
                    fh3::tmem_st32(taf + 32 * c, o);
                }
            } else {
#pragma unroll
                for (int pp = 0; pp < PARTS; ++pp) {
                    uint32_t o[32];
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc) {
                        const uint4 a = qv[4 * pp + 2 * cc], b2 = qv[4 * pp + 2 * cc + 1];
                        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b2.x, b2.y, b2.z, b2.w};
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            o[16 * cc + k] = w[k] & 0x0F0F0F0Fu;             // k = 64c + 4k .. +3
                            o[16 * cc + 8 + k] = (w[k] >> 4) & 0x0F0F0F0Fu;  // k = 64c + 32 + 4k .. +3
                        }
                    }
                    fh3::tmem_st32(ta0 + C::ACOLS * ab + 32 * pp, o);
                }
            }
            fh3::tmem_st_wait();
            fh3::tc_fence_before();
            __syncwarp();
            if (lane == 0) fh3::mbar_arrive(&B.afull[ab]);
        }
    } else {
        // ------------------------------------------------------------ accumulator readers
        // part p: sub-blocks 4p .. 4p+3 of each unit; the part-1 warp hands its sums to the
        // part-0 warp of its lane quarter at the end of every tile piece
        const int q = warp & 3, part = (warp - C::WARP_RD) >> 2;
        const int r = q * 32 + lane;
        const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16);
        const float* sx = reinterpret_cast<const float*>(smem + C::OFF_X);
        const float* sfs = reinterpret_cast<const float*>(smem + C::OFF_FS);
        float* red = reinterpret_cast<float*>(smem + C::OFF_RED) + (q * 32 + lane) * M;
        const uint32_t uG = static_cast<uint32_t>(G), uU = static_cast<uint32_t>(units);
        const int nch = kOneChunk ? 1 : (nblk + cw - 1) / cw;
        // CTAs of tile `tile`'s piece in chunk kk: the first in cf, the count returned
        auto piece_ctas = [&](int kk, int64_t tile, int& cf) {
            const int w = min(cw, nblk - kk * cw);
            const uint32_t s = static_cast<uint32_t>(static_cast<int64_t>(kk) * ntiles * cw + tile * w);
            cf = gt_cta_of(s, uG, uU);
            return gt_cta_of(s + w - 1, uG, uU) - cf + 1;
        };
        float acc[M];
#pragma unroll
        for (int t = 0; t < M; ++t) acc[t] = 0.0f;
        int fc = 0;  // tile pieces finished
        {
            // B operand of the super-blocks this run touches: (token, slot) items over the
            // eight warps, four items' x loads in flight at a time
            pdl_wait();  // x, y and the scratch are ours from here on
            const int w8 = warp - C::WARP_RD, items = C::F16 ? 0 : M * nslots;  // f16: B comes from the pre-pass
            for (int it0 = w8; it0 < items; it0 += 4 * 8) {
                float4 xv[4][2];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int it = it0 + 8 * k;
                    if (it < items) {
                        const int t = it / nslots, slot = it - t * nslots;
                        const float4* xr = reinterpret_cast<const float4*>(
                                               x + (static_cast<int64_t>(t) * nblk + (sbase + slot) % nblk) * 256) +
                                           2 * lane;
                        xv[k][0] = __ldg(xr);
                        xv[k][1] = __ldg(xr + 1);
                    }
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int it = it0 + 8 * k;
                    if (it < items) {
                        const int t = it / nslots;
                        if constexpr (!C::F16) build_b<M>(xv[k][0], xv[k][1], t, it - t * nslots, smem, lane);
                    }
                }
            }
            fh3::fence_proxy_async_smem();  // B is read by the tensor cores
            __syncwarp();
            if (lane == 0) fh3::mbar_arrive(B.bfull);
        }
        bool ok = wait_all(B.bfull, 0);  // every warp's sub-block sums and scales

        // One chunk only: the run's last tile, when split.  If, two units before the run
        // ends, every other segment has already counted itself, this segment is the last
        // one; the others' partials are read then, off the critical path (no CTA ever waits
        // for another).
        constexpr int kPre = kOneChunk && !C::F16 ? kGtPreSegs : 1;
        const int64_t t_last = p_last.tile;
        int cf_last = 0;
        const int nseg_last = kOneChunk ? piece_ctas(0, t_last, cf_last) : 0;
        const int seg_last = static_cast<int>(blockIdx.x) - cf_last;
        bool pre = false;
        float pv[kPre][M];
        auto try_prefetch = [&]() {
            if (C::F16 || part != 0 || nseg_last < 2 || nseg_last > kGtPreSegs + 1 || nseg_last > seg_max) return;
            int cnt = 0;
            if (lane == 0)
                asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(cnt) : "l"(counters + t_last * 4 + q) : "memory");
            cnt = __shfl_sync(0xffffffffu, cnt, 0);
            if (cnt != nseg_last - 1) return;
            const float* pt = partials + (t_last * seg_max * kGtRows + r) * M;
#pragma unroll
            for (int k = 0; k < kPre; ++k) {
                const int sg = k < seg_last ? k : k + 1;
#pragma unroll
                for (int t = 0; t < M; ++t)
                    pv[k][t] = sg < nseg_last ? __ldcg(pt + static_cast<int64_t>(sg) * kGtRows * M + t) : 0.0f;
            }
            pre = true;
        };
        // end of this run's piece of `tile` in chunk k: the pair's sums, then y or partials + count
        auto finish_piece = [&](int64_t tile, int k) -> bool {
            if (part == 1) {
                if (fc >= 1 && !wait_all(&B.xempty[q], (fc - 1) & 1)) return false;
#pragma unroll
                for (int t = 0; t < M; ++t) red[t] = acc[t];
                __syncwarp();
                if (lane == 0) fh3::mbar_arrive(&B.xfull[q]);
            } else {
                if (!wait_all(&B.xfull[q], fc & 1)) return false;
#pragma unroll
                for (int t = 0; t < M; ++t) acc[t] += red[t];
                __syncwarp();
                if (lane == 0) fh3::mbar_arrive(&B.xempty[q]);
                // the tile's contributions: one piece per chunk, each split between the CTAs
                // its units fall in; contribution (kk, j) has partial slot kk * split + j
                int total = 0;
                for (int kk = 0; kk < nch; ++kk) {
                    int cfk;
                    total += piece_ctas(kk, tile, cfk);
                }
                int cf;
                piece_ctas(k, tile, cf);
                const int idx = k * split + (static_cast<int>(blockIdx.x) - cf);
                const int64_t row = tile * kGtRows + r;
                if (total == 1) {
                    if (row < N) {
                        const float bv = bias ? bias[row] : 0.0f;
#pragma unroll
                        for (int t = 0; t < M; ++t) y[t * ldy + row] = acc[t] + bv;
                    }
                } else if (idx >= seg_max || (kOneChunk && total > seg_max)) {
                    if (lane == 0) fh3::record_status(status, FH3_ERR);  // never write past the slots
                } else if (kOneChunk && pre && tile == t_last) {
                    // every other segment had arrived when checked: this one is the last, and
                    // their partials are already in registers
                    float v[M];
#pragma unroll
                    for (int t = 0; t < M; ++t) v[t] = 0.0f;
#pragma unroll
                    for (int sg = 0; sg < kPre + 1; ++sg) {
                        if (sg >= total) break;
#pragma unroll
                        for (int t = 0; t < M; ++t) {
                            const float lo = pv[sg < kPre ? sg : kPre - 1][t];  // segment sg < idx
                            const float hi = pv[sg > 0 ? sg - 1 : 0][t];        // segment sg > idx
                            v[t] += sg == idx ? acc[t] : (sg < idx ? lo : hi);
                        }
                    }
                    if (row < N) {
                        const float bv = bias ? bias[row] : 0.0f;
#pragma unroll
                        for (int t = 0; t < M; ++t) y[t * ldy + row] = v[t] + bv;
                    }
                    __syncwarp();
                    if (lane == 0) counters[tile * 4 + q] = 0;
                } else {
                    float* pp = partials + ((tile * seg_max + idx) * kGtRows + r) * M;
#pragma unroll
                    for (int t = 0; t < M; ++t) pp[t] = acc[t];
                    // the warp's stores, then lane 0's release/acquire count on the counter of
                    // (tile, quarter): it publishes them at GPU scope and, for the last piece,
                    // acquires the other pieces' stores of these 32 rows
                    __syncwarp();
                    int old = 0;
                    int* ctr = counters + tile * 4 + q;
                    if (lane == 0)
                        asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(old) : "l"(ctr) : "memory");
                    old = __shfl_sync(0xffffffffu, old, 0);
                    if (old == total - 1) {  // last piece: add all in (chunk, CTA) order
                        __syncwarp();
                        const float* pt = partials + (tile * seg_max * kGtRows + r) * M;
                        float v[M];
#pragma unroll
                        for (int t = 0; t < M; ++t) v[t] = 0.0f;
                        for (int kk = 0; kk < nch; ++kk) {
                            int cfk;
                            const int nk = piece_ctas(kk, tile, cfk);
                            for (int j = 0; j < nk; ++j) {
                                const float* ps = pt + static_cast<int64_t>(kk * split + j) * kGtRows * M;
#pragma unroll
                                for (int t = 0; t < M; ++t) v[t] += __ldcg(ps + t);
                            }
                        }
                        if (row < N) {
                            const float bv = bias ? bias[row] : 0.0f;
#pragma unroll
                            for (int t = 0; t < M; ++t) y[t * ldy + row] = v[t] + bv;
                        }
                        if (lane == 0) *ctr = 0;
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < M; ++t) acc[t] = 0.0f;
            ++fc;
            return true;
        };
        UnitPos ep = p_first;  // unit i
        for (int i = 0; i < n && ok; ++i) {
            const int hs = i % kGtHdrs, d = i % C::DB;
            if constexpr (kOneChunk) {
                if (i == max(0, n - 2)) try_prefetch();
            }
            // the row's header: d, dmin, the 6-bit scales and mins
            if (!wait_all(&B.hfull[hs], (i / kGtHdrs) & 1)) break;
            const uint4 hd = lds128(smem + C::OFF_HDR + (hs * kGtRows + r) * 16);
            __syncwarp();
            if (lane == 0) fh3::mbar_arrive(&B.hempty[hs]);
            // 6..16 tokens: 2^-s of the unit's super-block for each token (the pre-pass's), loaded
            // before the accumulator wait; the part-1 warps read no accumulator (and release
            // none), so they do not wait for the MMA either
            float fsr[C::F16 ? M : 1];
            if constexpr (C::F16) {
                if (part == 0) {
#pragma unroll
                    for (int t = 0; t < M; ++t) fsr[t] = __ldg(fsg + static_cast<size_t>(ep.b) * M + t);
                }
            }
            if (!C::F16 || part == 0) {
                if (!wait_all(&B.dfull[d], (i / C::DB) & 1)) break;
                fh3::tc_fence_after();
            }
            const int slot = slot_of(ep.b);
            const float dd = fh3::h2f_bits(hd.x), dmin = fh3::h2f_bits(hd.x >> 16);
            if constexpr (M <= 5) {
                float sum[M], msum[M];
#pragma unroll
                for (int t = 0; t < M; ++t) sum[t] = msum[t] = 0.0f;
#pragma unroll
                for (int j0 = 0; j0 < 4; j0 += JB) {  // JB sub-blocks' accumulators in registers at a time
                    uint32_t v[JB][W];
#pragma unroll
                    for (int jj = 0; jj < JB; ++jj)
                        tmem_ld_w<W>(tl + C::DCOLS * d + C::NC * (4 * part + j0 + jj), v[jj]);
                    fh3::tmem_ld_wait();
#pragma unroll
                    for (int jj = 0; jj < JB; ++jj) fh3::tmem_regs_ready(v[jj]);
                    if (j0 + JB == 4) {  // every column of this buffer is read
                        fh3::tc_fence_before();
                        __syncwarp();
                        if (lane == 0) fh3::mbar_arrive(&B.dempty[d]);
                    }
#pragma unroll
                    for (int jj = 0; jj < JB; ++jj) {
                        const int j = 4 * part + j0 + jj;
                        int sc, m;
                        fh3::q4k_scale_min_words(hd.y, hd.z, hd.w, j, sc, m);
                        const float dsc = dd * small_i2f(static_cast<uint32_t>(sc));
                        const float dm = dmin * small_i2f(static_cast<uint32_t>(m));
#pragma unroll
                        for (int t = 0; t < M; ++t) {
                            const float p = fmaf(65536.0f, small_i2f(v[jj][3 * t + 2]),
                                                 fmaf(256.0f, small_i2f(v[jj][3 * t + 1]), small_i2f(v[jj][3 * t])));
                            sum[t] = fmaf(dsc, p, sum[t]);
                            msum[t] = fmaf(dm, sx[(slot * M + t) * 8 + j], msum[t]);
                        }
                    }
                }
#pragma unroll
                for (int t = 0; t < M; ++t) acc[t] = fmaf(sfs[slot * M + t], sum[t], acc[t]) - msum[t];
            } else {
                // 6..16 tokens: accumulator 1 holds sum_j sc_j P_tj and accumulator 2 sum_j m_j X_tj
                // (x and X scaled by 2^s and 2^(s-5)), each as hi and lo columns 2t, 2t + 1; the
                // part-0 warp reads both, the part-1 warp has nothing to add
                if (part == 0) {
                    // the two accumulators one after the other (fewer live registers)
                    float dp[M];
                    {
                        uint32_t v[C::NC];
                        tmem_ld_w<C::NC>(tl + C::DCOLS * d, v);
                        fh3::tmem_ld_wait();
                        fh3::tmem_regs_ready(v);
#pragma unroll
                        for (int t = 0; t < M; ++t) dp[t] = dd * (__uint_as_float(v[2 * t]) + __uint_as_float(v[2 * t + 1]));
                    }
                    uint32_t v[C::NC];
                    tmem_ld_w<C::NC>(tl + C::DCOLS * d + C::NC, v);
                    fh3::tmem_ld_wait();
                    fh3::tmem_regs_ready(v);
                    fh3::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) fh3::mbar_arrive(&B.dempty[d]);
                    const float dm32 = 32.0f * dmin;
#pragma unroll
                    for (int t = 0; t < M; ++t) {
                        const float q = __uint_as_float(v[2 * t]) + __uint_as_float(v[2 * t + 1]);
                        acc[t] = fmaf(fsr[t], fmaf(-dm32, q, dp[t]), acc[t]);
                    }
                }
            }
            if (ep.b == ep.k * cw + ep.w - 1 || i == n - 1)
                if (!finish_piece(ep.tile, ep.k)) break;
            unit_next(ep, ntiles, nblk, cw);
        }
    }

    fh3::tc_fence_before();
    __syncthreads();
    if (warp == C::WARP_MMA) {
        fh3::tc_fence_after();
        fh3::tmem_dealloc(tmem, kGtTmemCols);
    }
}

cudaLaunchAttribute pdl_attr() {
    cudaLaunchAttribute a;
    a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a.val.programmaticStreamSerializationAllowed = 1;
    return a;
}

struct GtLaunch {
    int nblk, ntiles, cw, split, seg_max, grid;
    int64_t N, units;
};

template <int M>
int launch_tc(const CUtensorMap& tm, const GtLaunch& L, const float* x, const float* bias, float* y,
              float* partials, int* counters, uint8_t* bglob, float* fsg, int* status, cudaStream_t s) {
    constexpr int smem = GtCfg<M>::SMEM;
    if constexpr (GtCfg<M>::F16) {
        // the B blocks first; a programmatic dependent launch too, so its CTAs are placed
        // as the previous kernel's leave (it waits for that kernel before touching memory)
        cudaLaunchConfig_t pc = {};
        pc.gridDim = dim3(M, static_cast<unsigned>((L.nblk + 3) / 4), 1);
        pc.blockDim = dim3(1024, 1, 1);
        pc.stream = s;
        cudaLaunchAttribute pa[1] = {pdl_attr()};
        pc.attrs = pa;
        pc.numAttrs = 1;
        const int rc = fh3host::check_cuda(cudaLaunchKernelEx(&pc, gemv_xprep_kernel<M>, x, L.nblk, bglob, fsg),
                                           "gemv_xprep_kernel launch");
        if (rc) return rc;
    }
    static bool attr = false;
    if (!attr) {
        const int rc = fh3host::check_cuda(
            cudaFuncSetAttribute(gemv_tc_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
            "gemv_tc_kernel smem attribute");
        if (rc) return rc;
        attr = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(L.grid), 1, 1);
    cfg.blockDim = dim3(GtCfg<M>::THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1] = {pdl_attr()};
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return fh3host::check_cuda(cudaLaunchKernelEx(&cfg, gemv_tc_kernel<M>, tm, L.nblk, L.ntiles, L.N, L.units, L.cw,
                                                  L.split, L.seg_max, x, bias, y, L.N, partials, counters,
                                                  static_cast<const uint8_t*>(bglob), static_cast<const float*>(fsg),
                                                  status),
                               "gemv_tc_kernel launch");
}

template <int M>
int dispatch_tc(int n_tok, const CUtensorMap& tm, const GtLaunch& L, const float* x, const float* bias, float* y,
                float* partials, int* counters, uint8_t* bglob, float* fsg, int* status, cudaStream_t s) {
    if constexpr (M > kGtMaxTok) {
        return 1;
    } else {
        if (n_tok == M) return launch_tc<M>(tm, L, x, bias, y, partials, counters, bglob, fsg, status, s);
        return dispatch_tc<M + 1>(n_tok, tm, L, x, bias, y, partials, counters, bglob, fsg, status, s);
    }
}

// super-blocks of a chunk for n_tok tokens (0: one chunk over the whole K), and the B slots
int gt_chunk(int n_tok) {
    return n_tok <= 5 ? GtCfg<5>::CHUNK : (n_tok <= 8 ? GtCfg<8>::CHUNK : GtCfg<16>::CHUNK);
}
int gt_slots(int n_tok) {  // 6..16 tokens stream B: no limit
    return n_tok <= 5 ? GtCfg<5>::SLOTS : (1 << 30);
}
// bytes of one B block of 6..16 tokens
int gt_bblock(int n_tok) { return n_tok <= 8 ? GtCfg<8>::SLOT_BYTES : GtCfg<16>::SLOT_BYTES; }

}  // namespace

namespace fh3host {

// 1..16-token Q4_K GEMV on tcgen05 MMAs; returns 1 (nothing launched) when the
// shape or the pointers do not suit it, so the caller takes the warp-MMA kernels.
int gemv_tc(const Fh3CudaW* w, const float* x, float* y, int n_tok, const float* bias, cudaStream_t s) {
    DevCtx* c = ctx();
    if (!c) return set_error(FH3CUDA_E_NODEV, "gemv_tc: call fh3cuda_init first");
    if (n_tok < 1 || n_tok > kGtMaxTok) return 1;
    if ((reinterpret_cast<uintptr_t>(w->data) & 15) || (reinterpret_cast<uintptr_t>(x) & 15)) return 1;
    GtLaunch L;
    L.N = w->out;
    const int64_t K = w->in;
    L.nblk = static_cast<int>(K / fh3::kQ4KBlock);
    const int64_t ntiles = (L.N + kGtRows - 1) / kGtRows;
    L.ntiles = static_cast<int>(ntiles);
    L.units = ntiles * L.nblk;
    L.grid = static_cast<int>(std::min<int64_t>(ctx_sms(c), L.units));
    if (L.units * L.grid >= (int64_t(1) << 32)) return 1;  // unit -> CTA arithmetic is 32-bit
    const int64_t per = L.units / L.grid;  // >= 1
    const int64_t run_max = (L.units + L.grid - 1) / L.grid;
    const int chunk = gt_chunk(n_tok);
    if (chunk == 0) {
        // one chunk: a run's super-blocks, cyclically, must fit the B slots
        if (std::min<int64_t>(L.nblk, run_max) > gt_slots(n_tok)) return 1;
        L.cw = L.nblk;
        L.split = static_cast<int>(std::min<int64_t>(L.nblk, (L.nblk + per - 1) / per + 1));
        L.seg_max = L.split;
    } else {
        // chunks: a run must touch at most two of them (2 * chunk <= slots)
        L.cw = std::min(L.nblk, chunk);
        if (ntiles * L.cw < run_max) return 1;
        L.split = static_cast<int>(std::min<int64_t>(L.grid, (L.cw + per - 1) / per + 1));
        L.seg_max = (L.nblk + L.cw - 1) / L.cw * L.split;
    }
    float* partials = static_cast<float*>(
        scratch(c, 14, static_cast<size_t>(ntiles) * L.seg_max * kGtRows * n_tok * 4, s));
    int* counters = static_cast<int*>(scratch_zeroed(c, 15, static_cast<size_t>(ntiles) * 4 * 4, s));  // (tile, quarter)
    if (!partials || !counters) return FH3_E_NOMEM;
    uint8_t* bglob = nullptr;  // 6..16 tokens: the pre-pass's B blocks, then 2^-s of each token
    float* fsg = nullptr;
    if (n_tok > 5) {
        const size_t bb = static_cast<size_t>(L.nblk) * gt_bblock(n_tok);
        bglob = static_cast<uint8_t*>(scratch(c, 9, bb + static_cast<size_t>(L.nblk) * n_tok * 4 + 256, s));
        if (!bglob) return FH3_E_NOMEM;
        fsg = reinterpret_cast<float*>(bglob + bb);
    }

    CUtensorMap tm;
    const size_t row_bytes = static_cast<size_t>(L.nblk) * fh3::kQ4KBytes;
    const cuuint64_t gdim[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(L.N)};
    const cuuint64_t gstr[1] = {static_cast<cuuint64_t>(row_bytes)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(fh3::kQ4KBytes), static_cast<cuuint32_t>(kGtRows)};
    const cuuint32_t es[2] = {1, 1};
    if (encode_tiled(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(w->data), gdim, gstr, box, es,
                     CU_TENSOR_MAP_SWIZZLE_NONE) != CUDA_SUCCESS)
        return 1;
    return dispatch_tc<1>(n_tok, tm, L, x, bias, y, partials, counters, bglob, fsg, ctx_status(c), s);
}

}  // namespace fh3host
