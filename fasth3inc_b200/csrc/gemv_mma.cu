// gemv_mma.cu -- Q4_K GEMV (1..16 tokens) on warp-level tensor-core MMAs with
// exact operands.
//
// The small-M regime of fh3_matmul (src/core/fh3_ops.c:317-404) streams 4.5-bit
// weights; at B200's HBM rate that leaves under three warp instructions per 32
// weights, which a float dequantisation plus dot product exceeds.  Here:
//
//   y[t][n] = sum_j ( dl_nj * P_tnj - ml_nj * X_tj ),  P = sum_{k in j} q_nk x_tk,
//   X_tj = sum_{k in j} x_tk  (32-weight sub-blocks j; w = dl*q - ml as in
//   dequant_q4_k, src/core/fh3_quant.c:154-196)
//
// Two families of kernels, both exact in their products:
// * fp16 MMAs (this header's description below): gemv_stream_kernel, and the prep +
//   CTA-per-tile kernels gemv_mma_small_kernel / gemv_mma_kernel;
// * integer MMAs (1..4 tokens, the defaults at 1-2 tokens and at 3-4 when out > in):
//   gemv_i8_kernel and gemv_i8m_kernel, where x enters as base-256 digits and the
//   nibbles as u8 straight from the bytes (see their own descriptions further down).
// gemv_mma() at the end of the file picks the kernel.
//
// * A operand = the nibbles themselves: (word & 0x000F000F) is a pair of fp16
//   subnormals q * 2^-24, exact; high nibbles (word & 0x00F000F0) are 16 q * 2^-24.
//   Eight weights cost one shift and four ANDs.
// * B operand = x split into two fp16 planes x*2^s = h0 + h1 (22 significant bits)
//   under a power of two 2^s per token and super-block that puts the super-block's
//   max|x| just below 2^14.
// * mma.sync.m16n8k16 (fp16 x fp16 -> fp32): a product of a 4-bit integer and an
//   11-bit significand is exact; per sub-block two MMAs (k = 32) into a zeroed
//   accumulator give the plane sums of P in fp32.  acc += dl*(P0 + P1) - ml*X',
//   X' = X * 2^(s-24), each super-block's contribution times 2^(24-s) (+ bias).
//
// Two launches per call:
// * gemv_mma_prep_kernel (grid: 2048-element slices x tokens) writes the planes in
//   the lane order of the mma B fragment, the scaled sub-block sums X' and the
//   exponents.  It triggers the main kernel's launch at once (programmatic
//   dependent launch), so the main kernel's first weight loads overlap it.
// * gemv_mma_kernel: a CTA owns a 16-row tile and a K range; its warps stride over
//   the range's super-blocks with the next super-block's bytes in flight.  After
//   griddepcontrol.wait the CTA copies its range of B fragments and X' into shared
//   memory (cp.async), so a sub-block's B operand is one conflict-free 16-byte
//   shared load.  When the fragments of the whole K would not fit, a cluster of S
//   CTAs splits K and the partial sums meet over distributed shared memory.
//   Every sum runs in a fixed order (deterministic results).
//
// Fragment layout of a sub-block (32 elements i = 8tq + 4st + r): lane tq of a quad
// loads bytes 8tq..8tq+7 of the sub-block pair's 32-byte chunk; word st gives
// a0 = bytes {0,2} (k slots 2tq, 2tq+1) and a2 = bytes {1,3} (k slots 2tq+8,
// 2tq+9).  The B fragment uses the same slots, so the k order inside a sub-block
// is permuted identically on both sides and the dot products are unchanged.
// B fragments are stored compactly: sub-block sb, column col = 2*token + plane,
// lane tq -> frag[sb * 8M + col * 4 + tq] (16 bytes: halves for k-step 0 then 1).
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "common.cuh"

namespace {

#ifndef FH3_GV_MIN_BLOCKS
#define FH3_GV_MIN_BLOCKS 3  // resident CTAs per SM the register budget is sized for
#endif
#ifndef FH3_GV_SMEM_KB
#define FH3_GV_SMEM_KB 64    // shared-memory bytes per CTA above which a cluster splits K
#endif
constexpr int kGvMaxWarps = 8;
constexpr int kPrepSlice = 2048;  // elements of one token per prep CTA
constexpr size_t kGvSmemTarget = FH3_GV_SMEM_KB * 1024;

// half p (0..7) of a lane's 16-byte B fragment holds element 8tq + perm8(p) of the
// sub-block (perm8 is its own inverse: it swaps 1<->2 and 5<->6)
__host__ __device__ constexpr int perm8(int p) { return (p == 1 || p == 2 || p == 5 || p == 6) ? (p ^ 3) : p; }

__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(fh3::smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ uint32_t pack_half2(__half lo, __half hi) {
    return static_cast<uint32_t>(__half_as_ushort(lo)) | (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// grid (ceil(K / 2048), M), 256 threads: thread -> 8 consecutive elements (one lane's
// fragment of one sub-block); 4 consecutive threads cover a sub-block, a warp a
// super-block.
__global__ void __launch_bounds__(256) gemv_mma_prep_kernel(const float* __restrict__ x, int64_t K, int M,
                                                            uint4* __restrict__ frag, uint32_t* __restrict__ mfrag,
                                                            int* __restrict__ expo, float* __restrict__ fsb) {
    pdl_launch_dependents();
    const int t = blockIdx.y;
    const int lane = threadIdx.x & 31;
    const float4* x4 = reinterpret_cast<const float4*>(x + static_cast<int64_t>(t) * K);
    if (blockIdx.x == 0 && threadIdx.x == 0) expo[t] = 0;  // the scales are applied per super-block

    const int64_t k0 = static_cast<int64_t>(blockIdx.x) * kPrepSlice + threadIdx.x * 8;
    if (k0 < K) {  // K % 256 == 0: whole warps (super-blocks) are in or out
        const float4 v0 = __ldg(x4 + k0 / 4), v1 = __ldg(x4 + k0 / 4 + 1);
        const float e[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        // this warp's super-block: its own power of two, max|x| * 2^s < 2^14
        float amax = 0.0f;
#pragma unroll
        for (int u = 0; u < 8; ++u) amax = fmaxf(amax, fabsf(e[u]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        int E = 0;
        if (amax > 0.0f && amax <= 3.0e38f) frexpf(amax, &E);  // amax < 2^E
        const int s = 14 - E;
        if (lane == 0) fsb[(k0 >> 8) * M + t] = ldexpf(1.0f, 24 - s);
        uint32_t pl0[4], pl1[4];
#pragma unroll
        for (int p = 0; p < 8; p += 2) {
            __half h0[2], h1[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const float v = ldexpf(e[perm8(p + u)], s);
                h0[u] = __float2half_rn(v);
                h1[u] = __float2half_rn(v - __half2float(h0[u]));
            }
            pl0[p / 2] = pack_half2(h0[0], h0[1]);
            pl1[p / 2] = pack_half2(h1[0], h1[1]);
        }
        const int64_t sb = k0 >> 5;
        const int tq = lane & 3;
        const int64_t base = sb * 8 * M + 2 * t * 4 + tq;
        frag[base] = make_uint4(pl0[0], pl0[1], pl0[2], pl0[3]);
        frag[base + 4] = make_uint4(pl1[0], pl1[1], pl1[2], pl1[3]);
        // sub-block sums X_j (lanes 4j..4j+3 hold sub-block j of this super-block)
        float sum = ((e[0] + e[1]) + (e[2] + e[3])) + ((e[4] + e[5]) + (e[6] + e[7]));
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        // min-term B fragment: lane q (0..3) of a column holds (X_2q, X_2q+1) * 2^(s-5),
        // split into two fp16 planes like x
        const float xa = __shfl_sync(0xffffffffu, sum, 8 * (lane & 3));
        const float xb = __shfl_sync(0xffffffffu, sum, 8 * (lane & 3) + 4);
        if (lane < 4) {
            const float va = ldexpf(xa, s - 5), vb = ldexpf(xb, s - 5);
            const __half a0 = __float2half_rn(va), b0 = __float2half_rn(vb);
            const __half a1 = __float2half_rn(va - __half2float(a0)), b1 = __float2half_rn(vb - __half2float(b0));
            const int64_t mb = (k0 >> 8) * 8 * M + 2 * t * 4 + lane;
            mfrag[mb] = pack_half2(a0, b0);
            mfrag[mb + 4] = pack_half2(a1, b1);
        }
    }
}

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// the same with a zero accumulator input
__device__ __forceinline__ void mma_16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
    const float z = 0.0f;
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

// Raw bytes of one super-block for this lane: nibble words of rows g and g+8 for the
// four chunks, and the 16-byte headers.
struct SuperBlock {
    uint2 q[2][4];
    uint4 hd[2];
};

__device__ __forceinline__ void load_sb(SuperBlock& sbk, const uint8_t* row0, const uint8_t* row1, int b, int tq) {
    const uint8_t* p0 = row0 + static_cast<size_t>(b) * fh3::kQ4KBytes;
    const uint8_t* p1 = row1 + static_cast<size_t>(b) * fh3::kQ4KBytes;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        sbk.q[0][c] = __ldg(reinterpret_cast<const uint2*>(p0 + 16 + c * 32 + 8 * tq));
        sbk.q[1][c] = __ldg(reinterpret_cast<const uint2*>(p1 + 16 + c * 32 + 8 * tq));
    }
    sbk.hd[0] = __ldg(reinterpret_cast<const uint4*>(p0));
    sbk.hd[1] = __ldg(reinterpret_cast<const uint4*>(p1));
}

// Per-lane constants of the scale decode and the B-fragment slots.
template <int NT>
struct LaneCtx {
    int slot[NT];      // B-fragment slot of this lane in tile nt (clamped into the live range)
    uint32_t sel_sc0;  // byte_perm selectors: scale byte 2(tq&1) / 2(tq&1)+1 -> float 2^23 + byte
    uint32_t sel_sc1;
    uint32_t sel_m;    // min bytes 2(tq&1), 2(tq&1)+1 -> fp16 pair of integers (subnormals m * 2^-24)
    bool lo;           // tq < 2: sub-blocks 0..3 (low scale words), else 4..7
};

template <int NT>
__device__ __forceinline__ LaneCtx<NT> lane_ctx(int lane, int lanes) {
    LaneCtx<NT> lc;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) lc.slot[nt] = min(nt * 32 + lane, lanes - 1);
    const uint32_t k0 = 2u * (lane & 1 ? 1u : 0u);
    lc.sel_sc0 = 0x5440u | k0;
    lc.sel_sc1 = 0x5440u | (k0 + 1);
    lc.sel_m = k0 | 0x40u | ((k0 + 1) << 8) | 0x4000u;
    lc.lo = (lane & 3) < 2;
    return lc;
}

// One super-block of rows g, g+8 against all tokens.  fsb: B fragments of the
// super-block's 8 sub-blocks (stride `lanes` uint4), msb: its min-term B fragments.
// fsc[nt] multiplies this super-block's contribution to token tile nt of this lane
// (2^(24-s), s the super-block's activation exponent of that token).
template <int NT, int LANES = 0>  // LANES: fragment slots per sub-block when known at compile time
__device__ __forceinline__ void compute_sb(const SuperBlock& sbk, int lane, int lanes_rt, const LaneCtx<NT>& lc,
                                           const uint4* __restrict__ fsb, const uint32_t* __restrict__ msb,
                                           float (&acc)[2][NT], const float (&fsc)[NT]) {
    const int lanes = LANES > 0 ? LANES : lanes_rt;
    // lane tq decodes the scales of its sub-blocks 2tq, 2tq+1 (rows g, g+8) and the
    // min-term A fragment; 6-bit fields as in get_scale_min_k4 (src/core/fh3_quant.c)
    float dl[2][2];
    uint32_t am[2];
    float dm32[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint4 h = sbk.hd[i];
        const float d = fh3::h2f_bits(h.x), dmin = fh3::h2f_bits(h.x >> 16);
        const uint32_t scw = lc.lo ? (h.y & 0x3F3F3F3Fu) : ((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u));
        const uint32_t mw = lc.lo ? (h.z & 0x3F3F3F3Fu) : (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u));
        const float sc0 = __uint_as_float(__byte_perm(scw, 0x4B00u, lc.sel_sc0)) - 8388608.0f;  // exact
        const float sc1 = __uint_as_float(__byte_perm(scw, 0x4B00u, lc.sel_sc1)) - 8388608.0f;
        dl[i][0] = d * sc0;                // exact (17 significant bits), the fp32 value fh3 uses
        dl[i][1] = (d * 0.0625f) * sc1;    // high nibbles enter the MMA as 16 q
        am[i] = __byte_perm(mw, 0u, lc.sel_m);
        dm32[i] = dmin * 32.0f;
    }
    // two partial sums per accumulator (low / high nibble sub-blocks) shorten the
    // dependent FMA chains; the min term starts the low one
    float ph[2][NT][2];
    // min term: one k16 MMA over the 8 sub-blocks (k slots 8..15 zero)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        float dm[4];
        mma_16816_z(dm, am[0], am[1], 0u, 0u, msb[lc.slot[nt]], 0u);
        ph[0][nt][0] = -dm32[0] * (dm[0] + dm[1]);
        ph[1][nt][0] = -dm32[1] * (dm[2] + dm[3]);
        ph[0][nt][1] = ph[1][nt][1] = 0.0f;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        // scales of sub-blocks 2c, 2c+1 were decoded by lane tq == c of this row group
        float dlc[2][2];
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) dlc[i][hh] = __shfl_sync(0xffffffffu, dl[i][hh], c, 4);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const uint4* fs = fsb + (2 * c + hh) * lanes;
            const uint32_t mask = hh ? 0x00F000F0u : 0x000F000Fu;
            const uint32_t a00 = sbk.q[0][c].x & mask, a01 = sbk.q[1][c].x & mask;
            const uint32_t a02 = (sbk.q[0][c].x >> 8) & mask, a03 = (sbk.q[1][c].x >> 8) & mask;
            const uint32_t a10 = sbk.q[0][c].y & mask, a11 = sbk.q[1][c].y & mask;
            const uint32_t a12 = (sbk.q[0][c].y >> 8) & mask, a13 = (sbk.q[1][c].y >> 8) & mask;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const uint4 fb = fs[lc.slot[nt]];
                float d4[4];
                mma_16816_z(d4, a00, a01, a02, a03, fb.x, fb.y);
                mma_16816(d4, a10, a11, a12, a13, fb.z, fb.w);
                ph[0][nt][hh] = fmaf(dlc[0][hh], d4[0] + d4[1], ph[0][nt][hh]);
                ph[1][nt][hh] = fmaf(dlc[1][hh], d4[2] + d4[3], ph[1][nt][hh]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[i][nt] = fmaf(fsc[nt], ph[i][nt][0] + ph[i][nt][1], acc[i][nt]);
}

// Warp partials -> CTA partials (fixed order) -> cluster ranks (fixed order) -> y.
// part: [nw][16][TT], cta_part: [16][TT] in shared memory.
template <int NT>
__device__ __forceinline__ void finish_tile(const float (&acc)[2][NT], float* part, float* cta_part, int warp, int nw,
                                            int lane, int S, int rank, int M, int64_t N, const int* __restrict__ expo,
                                            const float* __restrict__ bias, float* __restrict__ y, int64_t ldy) {
    constexpr int TT = 4 * NT;
    const int g = lane >> 2, tq = lane & 3;
    // accumulator (row g or g+8, column 2tq / 2tq+1 of tile nt) -> token nt*4 + tq
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        part[(warp * 16 + g) * TT + nt * 4 + tq] = acc[0][nt];
        part[(warp * 16 + g + 8) * TT + nt * 4 + tq] = acc[1][nt];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 16 * TT; i += blockDim.x) {
        float v = part[i];
        for (int w = 1; w < nw; ++w) v += part[w * 16 * TT + i];
        cta_part[i] = v;
    }
    if (S > 1) fh3::cluster_sync_all();
    else __syncthreads();
    // rank r finishes rows r, r+S, ... of the tile, adding the ranks' partials in order
    for (int i = threadIdx.x; i < 16 * TT; i += blockDim.x) {
        const int r = i / TT, t = i - r * TT;
        if (r % S != rank) continue;
        const int64_t n = static_cast<int64_t>(blockIdx.x) * 16 + r;
        if (t >= M || n >= N) continue;
        float v;
        if (S > 1) {
            v = 0.0f;
            const uint32_t la = fh3::smem_u32(cta_part + i);
            for (int q = 0; q < S; ++q) {
                float pv;
                asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(pv) : "r"(fh3::mapa_shared(la, q)) : "memory");
                v = q == 0 ? pv : v + pv;
            }
        } else {
            v = cta_part[i];
        }
        v = ldexpf(v, expo[t]);
        if (bias) v += bias[n];
        y[t * ldy + n] = v;
    }
    if (S > 1) fh3::cluster_sync_all();  // peers' shared memory stays live until every rank has read it
}

// ---------------------------------------------------------------------------
// 1..4 tokens: a CTA owns a 16-row tile; each warp takes every nw-th super-block and
// stages that super-block's B fragments in its own shared-memory double buffer
// (cp.async, one commit group per super-block), so no CTA-wide barrier precedes
// the first MMA.  Weights of the next super-block load while this one computes.
// Dynamic shared memory: per warp 2 stages x (8 * 8M uint4 + 8M u32); partials.
// ---------------------------------------------------------------------------
template <int LANES>
__device__ __forceinline__ void stage_frag(uint4* st, const uint4* __restrict__ frag, const uint32_t* __restrict__ mfrag,
                                           int b, int lane) {
    const uint4* gf = frag + static_cast<int64_t>(b) * 8 * LANES;
#pragma unroll
    for (int i = 0; i < 8 * LANES / 32; ++i) cp_async16(st + i * 32 + lane, gf + i * 32 + lane);
    const uint4* gm = reinterpret_cast<const uint4*>(mfrag + static_cast<int64_t>(b) * LANES);
    if (lane < LANES / 4) cp_async16(st + 8 * LANES + lane, gm + lane);
    asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int M>
__global__ void __launch_bounds__(kGvMaxWarps * 32, FH3_GV_MIN_BLOCKS) gemv_mma_small_kernel(
    const uint8_t* __restrict__ W, size_t row_bytes, int nblk, int64_t N, const uint4* __restrict__ frag,
    const uint32_t* __restrict__ mfrag, const int* __restrict__ expo, const float* __restrict__ fsb,
    const float* __restrict__ bias, float* __restrict__ y, int64_t ldy) {
    constexpr int LANES = 8 * M;                       // fragment slots per sub-block
    constexpr int STAGE = 8 * LANES + LANES / 4;       // uint4 per stage
    extern __shared__ __align__(128) uint8_t gv_smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
    const int g = lane >> 2, tq = lane & 3;
    uint4* st0 = reinterpret_cast<uint4*>(gv_smem) + static_cast<size_t>(warp) * 2 * STAGE;
    uint4* st1 = st0 + STAGE;
    float* part = reinterpret_cast<float*>(reinterpret_cast<uint4*>(gv_smem) + static_cast<size_t>(nw) * 2 * STAGE);
    float* cta_part = part + nw * 16 * 4;

    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * 16 + g;
    const int64_t r1 = r0 + 8;
    const uint8_t* row0 = W + (r0 < N ? r0 : N - 1) * row_bytes;  // clamp loads; stores are masked
    const uint8_t* row1 = W + (r1 < N ? r1 : N - 1) * row_bytes;
    const LaneCtx<1> lc = lane_ctx<1>(lane, LANES);

    float acc[2][1] = {{0.0f}, {0.0f}};
    const int nbw = warp < nblk ? (nblk - warp + nw - 1) / nw : 0;  // super-blocks of this warp
    if (nbw > 0) {
        // prefetches past the warp's last super-block re-read its last one (cache hits)
        const int blast = warp + (nbw - 1) * nw;
        int b = warp;
        SuperBlock sa, sbuf;
        load_sb(sa, row0, row1, b, tq);  // weights do not depend on the prep kernel
        load_sb(sbuf, row0, row1, min(b + nw, blast), tq);
        pdl_wait();
        // this lane's token (tq; lanes past the last token reuse its factors, their sums
        // are never stored) and the staged super-blocks' factors
        const int tf = min(tq, M - 1);
        stage_frag<LANES>(st0, frag, mfrag, b, lane);
        float f0[1] = {__ldg(fsb + static_cast<int64_t>(b) * M + tf)};
        stage_frag<LANES>(st1, frag, mfrag, min(b + nw, blast), lane);
        float f1[1] = {__ldg(fsb + static_cast<int64_t>(min(b + nw, blast)) * M + tf)};
        for (int it = 0;; it += 2) {
            asm volatile("cp.async.wait_group 1;" ::: "memory");
            __syncwarp();
            compute_sb<1, LANES>(sa, lane, LANES, lc, st0, reinterpret_cast<const uint32_t*>(st0 + 8 * LANES), acc,
                                 f0);
            if (it + 1 >= nbw) break;
            __syncwarp();
            const int b2 = min(b + 2 * nw, blast);
            load_sb(sa, row0, row1, b2, tq);
            stage_frag<LANES>(st0, frag, mfrag, b2, lane);
            f0[0] = __ldg(fsb + static_cast<int64_t>(b2) * M + tf);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
            __syncwarp();
            compute_sb<1, LANES>(sbuf, lane, LANES, lc, st1, reinterpret_cast<const uint32_t*>(st1 + 8 * LANES), acc,
                                 f1);
            if (it + 2 >= nbw) break;
            __syncwarp();
            const int b3 = min(b + 3 * nw, blast);
            load_sb(sbuf, row0, row1, b3, tq);
            stage_frag<LANES>(st1, frag, mfrag, b3, lane);
            f1[0] = __ldg(fsb + static_cast<int64_t>(b3) * M + tf);
            b += 2 * nw;
        }
        asm volatile("cp.async.wait_group 0;" ::: "memory");  // no copy outlives the CTA
    }
    finish_tile<1>(acc, part, cta_part, warp, nw, lane, 1, 0, M, N, expo, bias, y, ldy);
}

// ---------------------------------------------------------------------------
// 1..2 tokens, persistent stream-K, one launch: one CTA per SM.  The ntiles * nblk
// units (16-row tile, super-block) are split into equal contiguous runs, one per
// warp of the grid; a warp streams its run with two units in flight in registers
// (coalesced 8-byte loads: a quad reads a chunk's 32 bytes of a row).  The first two
// units load before griddepcontrol.wait (weights do not depend on the previous
// kernel); then every CTA builds the B fragments of the whole K from x itself (the
// work of gemv_mma_prep_kernel, done once per SM into shared memory), which saves
// the prep launch.  When a run ends inside a tile, the warp stores its partial sums
// and counts itself on the tile's counter; the last of the tile's segments adds the
// partials in segment order (deterministic) and writes y, then zeroes the counter
// for the next call.
// Dynamic shared memory: fragments [nblk*8][8M] uint4 | min-term fragments
// [nblk][8M] u32 | exponents, reduction slots.
// ---------------------------------------------------------------------------
#ifndef FH3_GV_STREAM_WARPS
#define FH3_GV_STREAM_WARPS 16  // warps of the one CTA per SM
#endif
#ifndef FH3_GV_STREAM_MIN_BLOCKS
#define FH3_GV_STREAM_MIN_BLOCKS 1  // CTAs an SM must hold at once (2: consecutive calls overlap)
#endif
constexpr int kStreamWarps = FH3_GV_STREAM_WARPS;

__device__ __forceinline__ int64_t stream_warp_of(int64_t u, int64_t GW, int64_t units) {
    return ((u + 1) * GW - 1) / units;  // the warp whose run [w*U/GW, (w+1)*U/GW) holds unit u
}

// x (M x K fp32) -> this CTA's shared-memory B fragments and min-term fragments in
// one pass over x: a warp takes one super-block (256 elements) of one token at a
// time, its own power of two 2^s (max|x| of the super-block below 2^14) and stores
// fs[t][b] = 2^(24 - s), the factor that brings the super-block's partial sums back
// to x's units (exact; |x| below 2^117).
template <int M>
__device__ __forceinline__ void build_fragments(const float* __restrict__ x, int nblk, uint4* sfrag,
                                                uint32_t* smfrag, float* sfs) {
    constexpr int LANES = 8 * M;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const int k4 = nblk * 64;
    const int items = M * nblk;
    constexpr int kBatch = 4;  // items of a warp whose loads are in flight together
    for (int it0 = warp; it0 < items; it0 += kBatch * nw) {
    float4 xv[kBatch][2];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
        const int it = it0 + u * nw;
        if (it < items) {
            const int t = M == 1 ? 0 : it / nblk;
            const int k0 = (it - t * nblk) * 256 + lane * 8;
            xv[u][0] = __ldg(x4 + t * k4 + k0 / 4);
            xv[u][1] = __ldg(x4 + t * k4 + k0 / 4 + 1);
        }
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
        const int it = it0 + u * nw;
        if (it >= items) break;  // warp-uniform
        const int t = M == 1 ? 0 : it / nblk;
        const int b = it - t * nblk;
        const int k0 = b * 256 + lane * 8;  // this lane: elements k0 .. k0+7 = quad piece of sub-block
        const float4 v0 = xv[u][0], v1 = xv[u][1];
        const float e[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        float am = 0.0f;
#pragma unroll
        for (int u = 0; u < 8; ++u) am = fmaxf(am, fabsf(e[u]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        int E = 0;
        if (am > 0.0f && am <= 3.0e38f) frexpf(am, &E);  // am < 2^E
        const int sx = 14 - E;                            // max|x| * 2^sx < 2^14
        uint32_t pl0[4], pl1[4];
#pragma unroll
        for (int p = 0; p < 8; p += 2) {
            __half h0[2], h1[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const float v = ldexpf(e[perm8(p + u)], sx);
                h0[u] = __float2half_rn(v);
                h1[u] = __float2half_rn(v - __half2float(h0[u]));
            }
            pl0[p / 2] = pack_half2(h0[0], h0[1]);
            pl1[p / 2] = pack_half2(h1[0], h1[1]);
        }
        const int tq = lane & 3;
        uint4* f = sfrag + (k0 >> 5) * LANES + 2 * t * 4 + tq;
        f[0] = make_uint4(pl0[0], pl0[1], pl0[2], pl0[3]);
        f[4] = make_uint4(pl1[0], pl1[1], pl1[2], pl1[3]);
        float sum = ((e[0] + e[1]) + (e[2] + e[3])) + ((e[4] + e[5]) + (e[6] + e[7]));
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        const float xa = __shfl_sync(0xffffffffu, sum, 8 * (lane & 3));
        const float xb = __shfl_sync(0xffffffffu, sum, 8 * (lane & 3) + 4);
        if (lane < 4) {
            const float va = ldexpf(xa, sx - 5), vb = ldexpf(xb, sx - 5);
            const __half a0 = __float2half_rn(va), b0 = __float2half_rn(vb);
            const __half a1 = __float2half_rn(va - __half2float(a0)), b1 = __float2half_rn(vb - __half2float(b0));
            uint32_t* m = smfrag + b * LANES + 2 * t * 4 + lane;
            m[0] = pack_half2(a0, b0);
            m[4] = pack_half2(a1, b1);
        }
        if (lane == 0) sfs[t * nblk + b] = ldexpf(1.0f, 24 - sx);
    }
    }
    __syncthreads();
}

template <int M>
__global__ void __launch_bounds__(kStreamWarps * 32, FH3_GV_STREAM_MIN_BLOCKS) gemv_stream_kernel(
    const uint8_t* __restrict__ W, size_t row_bytes, int nblk, int64_t N, int64_t units, int seg_max,
    const float* __restrict__ x, const float* __restrict__ bias, float* __restrict__ y, int64_t ldy,
    float* __restrict__ partials, int* __restrict__ counters, int* status) {
    constexpr int LANES = 8 * M;
    extern __shared__ __align__(128) uint8_t gv_smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
    const int g = lane >> 2, tq = lane & 3;

    uint4* sfrag = reinterpret_cast<uint4*>(gv_smem);
    uint32_t* smfrag = reinterpret_cast<uint32_t*>(sfrag + static_cast<size_t>(nblk) * 8 * LANES);
    float* sfs = reinterpret_cast<float*>(smfrag + static_cast<size_t>(nblk) * LANES);  // [M][nblk]

    // at most one warp per unit, so every run is non-empty and the runs meeting a
    // tile are consecutive warps (segment index = warp - first warp of the tile)
    const int64_t GW = min(static_cast<int64_t>(gridDim.x) * nw, units);
    const int64_t gw = static_cast<int64_t>(blockIdx.x) * nw + warp;
    const int64_t u0 = gw < GW ? gw * units / GW : units;
    const int64_t u1 = gw < GW ? (gw + 1) * units / GW : units;
    const int n = static_cast<int>(u1 - u0);

    // next unit to load, as (tile, super-block); rows past N are clamped (stores are masked)
    int lt = static_cast<int>(u0 / nblk), lb = static_cast<int>(u0 % nblk);
    auto load_next = [&](SuperBlock& d) {
        const int64_t r0 = static_cast<int64_t>(lt) * 16 + g, r1 = r0 + 8;
        load_sb(d, W + (r0 < N ? r0 : N - 1) * row_bytes, W + (r1 < N ? r1 : N - 1) * row_bytes, lb, tq);
        if (++lb == nblk) {
            lb = 0;
            ++lt;
        }
    };
    SuperBlock sa, sbuf;
    if (n > 0) load_next(sa);
    if (n > 1) load_next(sbuf);
    pdl_launch_dependents();  // the next kernel may start its own weight loads

    pdl_wait();  // x, y and the scratch are ours from here on
    build_fragments<M>(x, nblk, sfrag, smfrag, sfs);
    const float* my_fs = sfs + (tq < M ? tq : M - 1) * nblk;  // this lane's token

    const LaneCtx<1> lc = lane_ctx<1>(lane, LANES);
    float acc[2][1] = {{0.0f}, {0.0f}};
    int t = static_cast<int>(u0 / nblk), b = static_cast<int>(u0 % nblk);  // unit being computed
    // end of this warp's segment of tile t: direct store, or partials + last-arriver sum
    auto finish_segment = [&]() {
        const int64_t wf = stream_warp_of(static_cast<int64_t>(t) * nblk, GW, units);
        const int64_t wl = stream_warp_of(static_cast<int64_t>(t + 1) * nblk - 1, GW, units);
        const int nseg = static_cast<int>(wl - wf + 1);
        const int64_t r0 = static_cast<int64_t>(t) * 16 + g, r1 = r0 + 8;
        if (nseg == 1) {
            if (tq < M) {
                if (r0 < N) y[tq * ldy + r0] = acc[0][0] + (bias ? bias[r0] : 0.0f);
                if (r1 < N) y[tq * ldy + r1] = acc[1][0] + (bias ? bias[r1] : 0.0f);
            }
        } else if (nseg > seg_max) {
            if (lane == 0) fh3::record_status(status, FH3_ERR);  // never write past the slots
        } else {
            const int seg = static_cast<int>(gw - wf);
            float* pp = partials + (static_cast<int64_t>(t) * seg_max + seg) * 16 * M;
            if (tq < M) {
                pp[g * M + tq] = acc[0][0];
                pp[(g + 8) * M + tq] = acc[1][0];
            }
            // the warp's stores, then lane 0's release/acquire count: it publishes them at
            // GPU scope and, for the last segment, acquires the other segments' stores
            __syncwarp();
            int old = 0;
            if (lane == 0)
                asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(old) : "l"(counters + t) : "memory");
            old = __shfl_sync(0xffffffffu, old, 0);
            if (old == nseg - 1) {  // last segment: add all in segment order
                __syncwarp();
                if (tq < M) {
                    const float* pt = partials + static_cast<int64_t>(t) * seg_max * 16 * M;
                    float v0 = 0.0f, v1 = 0.0f;
                    for (int q0 = 0; q0 < nseg; q0 += 4) {  // four segments' loads in flight, added in order
                        float a0[4], a1[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const bool ok = q0 + u < nseg;
                            a0[u] = ok ? __ldcg(pt + ((q0 + u) * 16 + g) * M + tq) : 0.0f;
                            a1[u] = ok ? __ldcg(pt + ((q0 + u) * 16 + g + 8) * M + tq) : 0.0f;
                        }
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            if (q0 + u < nseg) {
                                v0 += a0[u];
                                v1 += a1[u];
                            }
                        }
                    }
                    if (r0 < N) y[tq * ldy + r0] = v0 + (bias ? bias[r0] : 0.0f);
                    if (r1 < N) y[tq * ldy + r1] = v1 + (bias ? bias[r1] : 0.0f);
                }
                if (lane == 0) counters[t] = 0;
            }
        }
        acc[0][0] = acc[1][0] = 0.0f;
    };
    auto step = [&](const SuperBlock& cur, int i) {
        const float f1[1] = {my_fs[b]};
        compute_sb<1, LANES>(cur, lane, LANES, lc, sfrag + b * 8 * LANES, smfrag + b * LANES, acc, f1);
        if (b == nblk - 1 || i == n - 1) finish_segment();
        if (++b == nblk) {
            b = 0;
            ++t;
        }
    };
    for (int i = 0; i < n; i += 2) {
        step(sa, i);
        if (i + 2 < n) load_next(sa);
        if (i + 1 >= n) break;
        step(sbuf, i + 1);
        if (i + 3 < n) load_next(sbuf);
    }
}

// ---------------------------------------------------------------------------
// 1 token on integer MMAs: the persistent stream-K walk of gemv_stream_kernel with the
// dot products on mma.sync.m16n8k32 (u8 nibbles x s8 activation digits -> int32).
//
// * x of each super-block is rounded to an integer under a power of two 2^s
//   (max|x| * 2^s < 2^22) and cut into three balanced signed base-256 digits.
// * The nibbles enter as u8 as they lie in the bytes: low nibbles (w & 0x0F0F0F0F) are
//   q, high nibbles (w & 0xF0F0F0F0) are 16 q; one AND per four weights.
// * One MMA (K 32) takes positions 8tq..8tq+3 (a second one 8tq+4..8tq+7) of both
//   sub-blocks of a 32-byte chunk c: k slots 4tq+r are the low-nibble sub-block 2c, slots
//   16+4tq+r the high-nibble sub-block 2c+1.  B column g holds digit g of sub-block 2c
//   (g < 3) or digit g-3 of sub-block 2c+1 (3 <= g < 6), zero in the other half and in
//   columns 6, 7.  The chunk's accumulator so holds the six digit-plane sums of its two
//   sub-blocks for rows g, g+8, exact; each is multiplied by its sub-block's 6-bit scale
//   and summed over the chunks in int32 (|sum| < 2^28), converted once per super-block
//   and scaled by d * 2^-s in fp32.  A lane's two accumulator columns keep the same digit
//   and nibble half in every chunk, so their weights 256^p (and 1/16 for high nibbles)
//   are applied once, when the tile's segment ends.
// * The min term is one m16n8k16 fp16 MMA of the 6-bit mins (fp16 subnormals m * 2^-24)
//   against the sub-block sums X_j of x * 2^(s-13) in two fp16 planes.
// Shared memory (built by every CTA for the whole K after griddepcontrol.wait):
//   digit fragments [nblk][4 chunks][32 lanes] uint4 | min-term fragments [nblk][32] u32 |
//   factors 2^-s [nblk] (NaN for a super-block holding a non-finite x).
// Limits: |x| < 2^112 (the min term's factor 2^(37-s) stays finite).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_i8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_i8_z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// 2^e as a float for e in [-126, 127] (exact)
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }
// the low bytes of four words -> one word
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    return __byte_perm(__byte_perm(a, b, 0x0040u), __byte_perm(c, d, 0x0040u), 0x5410u);
}

// x (K fp32, one token) -> this CTA's digit fragments, min-term fragments and factors.
// A warp takes one super-block at a time (lane l: elements 8l..8l+7, i.e. sub-block
// l / 4, positions 8(l % 4)..+7), with up to four super-blocks' loads in flight.
// * max|x| from the largest magnitude bit pattern (a NaN or Inf pattern is larger than
//   every finite one, which flags the super-block as non-finite); E with max|x| < 2^E.
// * x * 2^s + 1.5 * 2^23 (one rounding: |x * 2^s| < 2^22 keeps the sum in [2^23, 2^24])
//   holds xi = round-to-nearest-even(x * 2^s) in its low bits: the bit pattern minus
//   0x4B400000.  The balanced digits follow with shifts: r1 = (xi + 128) >> 8 and
//   r2 = (r1 + 128) >> 8 give xi = d0 + 256 d1 + 65536 d2 with d0 = xi - 256 r1,
//   d1 = r1 - 256 r2, d2 = r2, so each digit's byte is the low byte of xi, r1, r2.
// * Scalings by 2^s, 2^(s-13) and 2^-s use two power-of-two factors where one would
//   leave the normal range (s lies in [-106, 170]).
__device__ __forceinline__ void build_i8(const float* __restrict__ x, int nblk, uint4* sB, uint32_t* sM, float* sF) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int tq = lane & 3, j = lane >> 2;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    constexpr int kBatch = 4;
    for (int b0 = warp; b0 < nblk; b0 += kBatch * nw) {
        float4 xv[kBatch][2];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int b = b0 + u * nw;
            if (b < nblk) {
                xv[u][0] = __ldg(x4 + b * 64 + lane * 2);
                xv[u][1] = __ldg(x4 + b * 64 + lane * 2 + 1);
            }
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int b = b0 + u * nw;
            if (b >= nblk) break;  // warp-uniform
            const float e[8] = {xv[u][0].x, xv[u][0].y, xv[u][0].z, xv[u][0].w,
                                xv[u][1].x, xv[u][1].y, xv[u][1].z, xv[u][1].w};
            uint32_t mb = 0u;
#pragma unroll
            for (int v = 0; v < 8; ++v) mb = max(mb, __float_as_uint(e[v]) & 0x7FFFFFFFu);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));
            const bool fin = mb < 0x7F800000u;
            int E = 0;
            if (fin && mb != 0u) E = (mb >> 23) ? static_cast<int>(mb >> 23) - 126 : (32 - __clz(mb)) - 149;
            const int s = 22 - E;  // |x| * 2^s < 2^22
            uint32_t xb[8];
            if (s >= -126 && s <= 127) {
                const float p = pow2f(s);
#pragma unroll
                for (int v = 0; v < 8; ++v) xb[v] = __float_as_uint(fmaf(e[v], p, 12582912.0f));
            } else {
                const int s1 = s >> 1;
                const float p1 = pow2f(s1), p2 = pow2f(s - s1);
#pragma unroll
                for (int v = 0; v < 8; ++v) xb[v] = __float_as_uint(fmaf(e[v] * p1, p2, 12582912.0f));
            }
            uint32_t r1[8], r2[8];
#pragma unroll
            for (int v = 0; v < 8; ++v) {
                const int a = static_cast<int>(xb[v] - 0x4B3FFF80u) >> 8;  // (xi + 128) >> 8
                r1[v] = static_cast<uint32_t>(a);
                r2[v] = static_cast<uint32_t>((a + 128) >> 8);
            }
            const uint32_t D[3][2] = {{pack_low_bytes(xb[0], xb[1], xb[2], xb[3]), pack_low_bytes(xb[4], xb[5], xb[6], xb[7])},
                                      {pack_low_bytes(r1[0], r1[1], r1[2], r1[3]), pack_low_bytes(r1[4], r1[5], r1[6], r1[7])},
                                      {pack_low_bytes(r2[0], r2[1], r2[2], r2[3]), pack_low_bytes(r2[4], r2[5], r2[6], r2[7])}};
            // chunk c = j / 2; low-nibble sub-block (j even) -> columns 0..2, words 0 and 2
            // (k slots of the first and second MMA); high-nibble one -> columns 3..5, words 1, 3
            const int par = j & 1;
            uint4* bc = sB + (static_cast<size_t>(b) * 4 + (j >> 1)) * 32;
#pragma unroll
            for (int p = 0; p < 3; ++p)
                bc[(3 * par + p) * 4 + tq] =
                    par ? make_uint4(0u, D[p][0], 0u, D[p][1]) : make_uint4(D[p][0], 0u, D[p][1], 0u);
            sB[(static_cast<size_t>(b) * 4 + (lane >> 3)) * 32 + 24 + (lane & 7)] = make_uint4(0u, 0u, 0u, 0u);
            // sub-block sums (each quad holds its sub-block's), then lane 4g + tq (g < 2) of the
            // min-term fragment: plane g of (X_2tq, X_2tq+1) * 2^(s-13)  (|X| * 2^(s-13) < 2^14)
            float sum = ((e[0] + e[1]) + (e[2] + e[3])) + ((e[4] + e[5]) + (e[6] + e[7]));
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            const float xa = __shfl_sync(0xffffffffu, sum, 8 * tq);
            const float xc = __shfl_sync(0xffffffffu, sum, 8 * tq + 4);
            uint32_t mw = 0u;
            if (lane < 8) {
                const int t = s - 13, t1 = t >> 1;
                const float pa = pow2f(t1), pb = pow2f(t - t1);
                const float va = (xa * pa) * pb, vc = (xc * pa) * pb;
                const __half ha = __float2half_rn(va), hc = __float2half_rn(vc);
                mw = lane < 4 ? pack_half2(ha, hc)
                              : pack_half2(__float2half_rn(va - __half2float(ha)), __float2half_rn(vc - __half2float(hc)));
            }
            sM[static_cast<size_t>(b) * 32 + lane] = mw;
            if (lane == 0) {
                const int w = -s, w1 = w >> 1;
                sF[b] = fin ? pow2f(w1) * pow2f(w - w1) : __int_as_float(0x7FC00000);
            }
        }
    }
    __syncthreads();
}

// Per-lane constants of the integer unit.
struct I8Lane {
    uint32_t sel_m;       // min bytes 2(tq&1), 2(tq&1)+1 -> fp16 pair of integers
    bool lo;              // tq < 2: mins of sub-blocks 0..3
    uint32_t sel[2][2];   // [chunk parity][column]: scale byte of the column's sub-block
    float cw[2];          // digit weight of the lane's columns 2tq, 2tq+1
};

__device__ __forceinline__ I8Lane i8_lane(int lane) {
    I8Lane L;
    const int tq = lane & 3;
    const uint32_t k0 = 2u * (lane & 1);
    L.sel_m = k0 | 0x40u | ((k0 + 1) << 8) | 0x4000u;
    L.lo = tq < 2;
    // column 2tq + i belongs to the high-nibble sub-block when it is 3..5
    const uint32_t par0 = tq >= 2 ? 1u : 0u, par1 = tq >= 1 ? 1u : 0u;
    L.sel[0][0] = 0x4440u | par0;
    L.sel[0][1] = 0x4440u | par1;
    L.sel[1][0] = 0x4440u | (2u + par0);
    L.sel[1][1] = 0x4440u | (2u + par1);
    // columns 0..2: 256^p; 3..5: 256^p / 16; 6, 7: unused
    L.cw[0] = tq == 0 ? 1.0f : tq == 1 ? 65536.0f : tq == 2 ? 16.0f : 0.0f;
    L.cw[1] = tq == 0 ? 256.0f : tq == 1 ? 0.0625f : tq == 2 ? 4096.0f : 0.0f;
    return L;
}

// One unit: rows g, g+8 of a 16-row tile against one super-block.  bq: the super-block's
// digit fragments ([4][32] uint4), bm: this lane's min-term fragment word, fs = 2^-s.
__device__ __forceinline__ void i8_unit(const SuperBlock& sbk, const uint4* __restrict__ bq, uint32_t bm, float fs,
                                        int lane, const I8Lane& L, float (&accd)[2][2], float (&accm)[2]) {
    uint32_t scl[2], sch[2], am[2];
    float d[2], dmn[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint4 h = sbk.hd[i];
        d[i] = fh3::h2f_bits(h.x);
        dmn[i] = fh3::h2f_bits(h.x >> 16);
        scl[i] = h.y & 0x3F3F3F3Fu;                                       // sc_0..3
        sch[i] = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);        // sc_4..7
        const uint32_t mw = L.lo ? (h.z & 0x3F3F3F3Fu) : (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u));
        am[i] = __byte_perm(mw, 0u, L.sel_m);
    }
    int S[2][2] = {{0, 0}, {0, 0}};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint4 bf = bq[c * 32 + lane];
        const uint2 w0 = sbk.q[0][c], w1 = sbk.q[1][c];
        int C[4];
        mma_i8_z(C, w0.x & 0x0F0F0F0Fu, w1.x & 0x0F0F0F0Fu, w0.x & 0xF0F0F0F0u, w1.x & 0xF0F0F0F0u, bf.x, bf.y);
        mma_i8(C, w0.y & 0x0F0F0F0Fu, w1.y & 0x0F0F0F0Fu, w0.y & 0xF0F0F0F0u, w1.y & 0xF0F0F0F0u, bf.z, bf.w);
        const uint32_t s0 = c < 2 ? scl[0] : sch[0], s1 = c < 2 ? scl[1] : sch[1];
        S[0][0] += static_cast<int>(__byte_perm(s0, 0u, L.sel[c & 1][0])) * C[0];
        S[0][1] += static_cast<int>(__byte_perm(s0, 0u, L.sel[c & 1][1])) * C[1];
        S[1][0] += static_cast<int>(__byte_perm(s1, 0u, L.sel[c & 1][0])) * C[2];
        S[1][1] += static_cast<int>(__byte_perm(s1, 0u, L.sel[c & 1][1])) * C[3];
    }
    float dm4[4];
    mma_16816_z(dm4, am[0], am[1], 0u, 0u, bm, 0u);
    const float f0 = d[0] * fs, f1 = d[1] * fs;
    accd[0][0] = fmaf(__int2float_rn(S[0][0]), f0, accd[0][0]);
    accd[0][1] = fmaf(__int2float_rn(S[0][1]), f0, accd[0][1]);
    accd[1][0] = fmaf(__int2float_rn(S[1][0]), f1, accd[1][0]);
    accd[1][1] = fmaf(__int2float_rn(S[1][1]), f1, accd[1][1]);
    const float fm = fs * 137438953472.0f;  // 2^37: back from the mins' 2^-24 and the planes' 2^(s-13)
    accm[0] = fmaf(dm4[0] + dm4[1], -dmn[0] * fm, accm[0]);
    accm[1] = fmaf(dm4[2] + dm4[3], -dmn[1] * fm, accm[1]);
}

__global__ void __launch_bounds__(kStreamWarps * 32, 1) gemv_i8_kernel(
    const uint8_t* __restrict__ W, size_t row_bytes, int nblk, int64_t N, int64_t units, int seg_max,
    const float* __restrict__ x, const float* __restrict__ bias, float* __restrict__ y,
    float* __restrict__ partials, int* __restrict__ counters, int* status) {
    extern __shared__ __align__(128) uint8_t gv_smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
    const int g = lane >> 2, tq = lane & 3;

    uint4* sB = reinterpret_cast<uint4*>(gv_smem);
    uint32_t* sM = reinterpret_cast<uint32_t*>(sB + static_cast<size_t>(nblk) * 128);
    float* sF = reinterpret_cast<float*>(sM + static_cast<size_t>(nblk) * 32);

    // the run partition of gemv_stream_kernel: equal contiguous runs, at most one warp per
    // unit, so the runs meeting a tile are consecutive warps
    const int64_t GW = min(static_cast<int64_t>(gridDim.x) * nw, units);
    const int64_t gw = static_cast<int64_t>(blockIdx.x) * nw + warp;
    const int64_t u0 = gw < GW ? gw * units / GW : units;
    const int64_t u1 = gw < GW ? (gw + 1) * units / GW : units;
    const int n = static_cast<int>(u1 - u0);

    int lt = static_cast<int>(u0 / nblk), lb = static_cast<int>(u0 % nblk);
    auto load_next = [&](SuperBlock& dst) {
        const int64_t r0 = static_cast<int64_t>(lt) * 16 + g, r1 = r0 + 8;
        load_sb(dst, W + (r0 < N ? r0 : N - 1) * row_bytes, W + (r1 < N ? r1 : N - 1) * row_bytes, lb, tq);
        if (++lb == nblk) {
            lb = 0;
            ++lt;
        }
    };
    SuperBlock sa, sbuf;
    if (n > 0) load_next(sa);
    if (n > 1) load_next(sbuf);
    pdl_launch_dependents();  // the next kernel may start its own weight loads

    pdl_wait();  // x, y and the scratch are ours from here on
    build_i8(x, nblk, sB, sM, sF);

    const I8Lane L = i8_lane(lane);
    float accd[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
    float accm[2] = {0.0f, 0.0f};
    int t = static_cast<int>(u0 / nblk), b = static_cast<int>(u0 % nblk);
    // end of this warp's segment of tile t: direct store, or partials + last-arriver sum
    // (the count sits in the run, where its round trip overlaps the run's loads in flight)
    auto finish_segment = [&]() {
        // the quad's columns -> row sums (fixed order), held by every lane of the quad
        float v0 = fmaf(accd[0][0], L.cw[0], fmaf(accd[0][1], L.cw[1], accm[0]));
        float v1 = fmaf(accd[1][0], L.cw[0], fmaf(accd[1][1], L.cw[1], accm[1]));
        v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
        v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
        v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
        v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
        accd[0][0] = accd[0][1] = accd[1][0] = accd[1][1] = 0.0f;
        accm[0] = accm[1] = 0.0f;
        const int64_t wf = stream_warp_of(static_cast<int64_t>(t) * nblk, GW, units);
        const int64_t wl = stream_warp_of(static_cast<int64_t>(t + 1) * nblk - 1, GW, units);
        const int nseg = static_cast<int>(wl - wf + 1);
        const int64_t r0 = static_cast<int64_t>(t) * 16 + g, r1 = r0 + 8;
        if (nseg == 1) {
            if (tq == 0) {
                if (r0 < N) y[r0] = v0 + (bias ? bias[r0] : 0.0f);
                if (r1 < N) y[r1] = v1 + (bias ? bias[r1] : 0.0f);
            }
            return;
        }
        if (nseg > seg_max) {
            if (lane == 0) fh3::record_status(status, FH3_ERR);  // never write past the slots
            return;
        }
        float* pt = partials + static_cast<int64_t>(t) * seg_max * 16;
        if (tq == 0) {
            pt[(gw - wf) * 16 + g] = v0;
            pt[(gw - wf) * 16 + g + 8] = v1;
        }
        // the warp's stores, then lane 0's release/acquire count: it publishes them at GPU
        // scope and, for the last segment, acquires the other segments' stores
        __syncwarp();
        int old = 0;
        if (lane == 0) asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(old) : "l"(counters + t) : "memory");
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old != nseg - 1) return;
        __syncwarp();
        if (tq == 0) {  // last segment: add all in segment order
            float s0 = 0.0f, s1 = 0.0f;
            for (int q0 = 0; q0 < nseg; q0 += 4) {  // four segments' loads in flight, added in order
                float a0[4], a1[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const bool ok = q0 + u < nseg;
                    a0[u] = ok ? __ldcg(pt + (q0 + u) * 16 + g) : 0.0f;
                    a1[u] = ok ? __ldcg(pt + (q0 + u) * 16 + g + 8) : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    if (q0 + u < nseg) {
                        s0 = q0 + u == 0 ? a0[u] : s0 + a0[u];
                        s1 = q0 + u == 0 ? a1[u] : s1 + a1[u];
                    }
                }
            }
            if (r0 < N) y[r0] = s0 + (bias ? bias[r0] : 0.0f);
            if (r1 < N) y[r1] = s1 + (bias ? bias[r1] : 0.0f);
        }
        if (lane == 0) counters[t] = 0;
    };
    auto step = [&](const SuperBlock& cur, int i) {
        i8_unit(cur, sB + static_cast<size_t>(b) * 128, sM[static_cast<size_t>(b) * 32 + lane], sF[b], lane, L, accd,
                accm);
        if (b == nblk - 1 || i == n - 1) finish_segment();
        if (++b == nblk) {
            b = 0;
            ++t;
        }
    };
    for (int i = 0; i < n; i += 2) {
        step(sa, i);
        if (i + 2 < n) load_next(sa);
        if (i + 1 >= n) break;
        step(sbuf, i + 1);
        if (i + 3 < n) load_next(sbuf);
    }
}

// ---------------------------------------------------------------------------
// 2..4 tokens on integer MMAs: gemv_i8_kernel's walk and activation digits, one MMA per
// nibble half.  With more than one token the two halves' digit columns no longer fit one
// MMA's eight, so each sub-block gets its own MMA (K 32: positions 8tq..8tq+3 in slots
// 4tq+r, 8tq+4..8tq+7 in slots 16+4tq+r) against B columns (token t, digit p) = 3t + p,
// eight per n-group (one n-group for 2 tokens, two for 3 and 4).  A chunk's low- and
// high-nibble accumulators are multiplied by 16 sc_2c and sc_2c+1 (the high nibbles enter as
// 16 q) and summed in int32 (|sum| < 2^29); each token's columns are scaled by d * 2^-s_t
// once per super-block and by 256^p / 16 when the segment ends.
// Shared memory: digit pairs [nblk][8 sub-blocks][3M columns][4 tq] uint2 | min-term
// fragments [nblk][32] u32 (column 2t + plane) | factors 2^-s [nblk][M] (NaN: non-finite x).
// ---------------------------------------------------------------------------
template <int M>
__device__ __forceinline__ void build_i8m(const float* __restrict__ x, int64_t K, int nblk, uint2* sB, uint32_t* sM,
                                          float* sF) {
    // the min-term fragment is one m16n8k16 B operand: eight columns, two per token
    static_assert(M >= 2 && M <= 4, "the integer kernel's min term holds at most 4 tokens");
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int tq = lane & 3, j = lane >> 2;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const int items = M * nblk;
    constexpr int kBatch = 4;
    for (int it0 = warp; it0 < items; it0 += kBatch * nw) {
        float4 xv[kBatch][2];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int it = it0 + u * nw;
            if (it < items) {
                const int t = it / nblk, b = it - t * nblk;
                const float4* xp = x4 + (static_cast<int64_t>(t) * K >> 2) + b * 64 + lane * 2;
                xv[u][0] = __ldg(xp);
                xv[u][1] = __ldg(xp + 1);
            }
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int it = it0 + u * nw;
            if (it >= items) break;  // warp-uniform
            const int t = it / nblk, b = it - t * nblk;
            const float e[8] = {xv[u][0].x, xv[u][0].y, xv[u][0].z, xv[u][0].w,
                                xv[u][1].x, xv[u][1].y, xv[u][1].z, xv[u][1].w};
            uint32_t mb = 0u;
#pragma unroll
            for (int v = 0; v < 8; ++v) mb = max(mb, __float_as_uint(e[v]) & 0x7FFFFFFFu);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));
            const bool fin = mb < 0x7F800000u;
            int E = 0;
            if (fin && mb != 0u) E = (mb >> 23) ? static_cast<int>(mb >> 23) - 126 : (32 - __clz(mb)) - 149;
            const int sx = 22 - E;  // |x| * 2^sx < 2^22
            uint32_t xb[8];
            if (sx >= -126 && sx <= 127) {
                const float pw = pow2f(sx);
#pragma unroll
                for (int v = 0; v < 8; ++v) xb[v] = __float_as_uint(fmaf(e[v], pw, 12582912.0f));
            } else {
                const int s1 = sx >> 1;
                const float p1 = pow2f(s1), p2 = pow2f(sx - s1);
#pragma unroll
                for (int v = 0; v < 8; ++v) xb[v] = __float_as_uint(fmaf(e[v] * p1, p2, 12582912.0f));
            }
            uint32_t r1[8], r2[8];
#pragma unroll
            for (int v = 0; v < 8; ++v) {
                const int a = static_cast<int>(xb[v] - 0x4B3FFF80u) >> 8;  // (xi + 128) >> 8
                r1[v] = static_cast<uint32_t>(a);
                r2[v] = static_cast<uint32_t>((a + 128) >> 8);
            }
            uint2* bc = sB + ((static_cast<size_t>(b) * 8 + j) * (3 * M) + 3 * t) * 4 + tq;
            bc[0] = make_uint2(pack_low_bytes(xb[0], xb[1], xb[2], xb[3]), pack_low_bytes(xb[4], xb[5], xb[6], xb[7]));
            bc[4] = make_uint2(pack_low_bytes(r1[0], r1[1], r1[2], r1[3]), pack_low_bytes(r1[4], r1[5], r1[6], r1[7]));
            bc[8] = make_uint2(pack_low_bytes(r2[0], r2[1], r2[2], r2[3]), pack_low_bytes(r2[4], r2[5], r2[6], r2[7]));
            // sub-block sums, then lanes 8t .. 8t+7 of the min-term fragment: column 2t + plane
            float sum = ((e[0] + e[1]) + (e[2] + e[3])) + ((e[4] + e[5]) + (e[6] + e[7]));
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            const float xa = __shfl_sync(0xffffffffu, sum, 8 * tq);
            const float xc = __shfl_sync(0xffffffffu, sum, 8 * tq + 4);
            if (lane < 8) {
                const int tt = sx - 13, t1 = tt >> 1;
                const float pa = pow2f(t1), pb = pow2f(tt - t1);
                const float va = (xa * pa) * pb, vc = (xc * pa) * pb;
                const __half ha = __float2half_rn(va), hc = __float2half_rn(vc);
                sM[static_cast<size_t>(b) * 32 + 8 * t + lane] =
                    lane < 4 ? pack_half2(ha, hc)
                             : pack_half2(__float2half_rn(va - __half2float(ha)), __float2half_rn(vc - __half2float(hc)));
            }
            if (t == 0 && lane >= 8 * M) sM[static_cast<size_t>(b) * 32 + lane] = 0u;  // columns past 2M
            if (lane == 0) {
                const int w = -sx, w1 = w >> 1;
                sF[static_cast<size_t>(b) * M + t] = fin ? pow2f(w1) * pow2f(w - w1) : __int_as_float(0x7FC00000);
            }
        }
    }
    __syncthreads();
}

template <int M>
__global__ void __launch_bounds__(kStreamWarps * 32, 1) gemv_i8m_kernel(
    const uint8_t* __restrict__ W, size_t row_bytes, int nblk, int64_t K, int64_t N, int64_t units, int seg_max,
    const float* __restrict__ x, const float* __restrict__ bias, float* __restrict__ y, int64_t ldy,
    float* __restrict__ partials, int* __restrict__ counters, int* status) {
    constexpr int NC = 3 * M;         // digit columns
    constexpr int NG = (NC + 7) / 8;  // MMA n-groups of eight
    extern __shared__ __align__(128) uint8_t gv_smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
    const int g = lane >> 2, tq = lane & 3;

    uint2* sB = reinterpret_cast<uint2*>(gv_smem);
    uint32_t* sM = reinterpret_cast<uint32_t*>(sB + static_cast<size_t>(nblk) * 8 * NC * 4);
    float* sF = reinterpret_cast<float*>(sM + static_cast<size_t>(nblk) * 32);

    // the run partition of gemv_stream_kernel
    const int64_t GW = min(static_cast<int64_t>(gridDim.x) * nw, units);
    const int64_t gw = static_cast<int64_t>(blockIdx.x) * nw + warp;
    const int64_t u0 = gw < GW ? gw * units / GW : units;
    const int64_t u1 = gw < GW ? (gw + 1) * units / GW : units;
    const int n = static_cast<int>(u1 - u0);

    int lt = static_cast<int>(u0 / nblk), lb = static_cast<int>(u0 % nblk);
    auto load_next = [&](SuperBlock& dst) {
        const int64_t r0 = static_cast<int64_t>(lt) * 16 + g, r1 = r0 + 8;
        load_sb(dst, W + (r0 < N ? r0 : N - 1) * row_bytes, W + (r1 < N ? r1 : N - 1) * row_bytes, lb, tq);
        if (++lb == nblk) {
            lb = 0;
            ++lt;
        }
    };
    SuperBlock sa, sbuf;
    if (n > 0) load_next(sa);
    if (n > 1) load_next(sbuf);
    pdl_launch_dependents();  // the next kernel may start its own weight loads

    pdl_wait();  // x, y and the scratch are ours from here on
    build_i8m<M>(x, K, nblk, sB, sM, sF);

    // per-lane constants: B column g of each n-group, and the token and digit weight of the
    // accumulator columns 2tq, 2tq+1 of each n-group (token -1: a column past 3M)
    const uint32_t k0 = 2u * (lane & 1);
    const uint32_t sel_m = k0 | 0x40u | ((k0 + 1) << 8) | 0x4000u;
    const bool lo = tq < 2;
    int bcol[NG], tok[NG][2];
    uint32_t bmask[NG];
    float cw[NG][2];
#pragma unroll
    for (int ng = 0; ng < NG; ++ng) {
        const int c = 8 * ng + g;
        bcol[ng] = min(c, NC - 1);
        bmask[ng] = c < NC ? 0xFFFFFFFFu : 0u;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int cc = 8 * ng + 2 * tq + i;
            tok[ng][i] = cc < NC ? cc / 3 : -1;
            const int pd = cc % 3;
            cw[ng][i] = cc < NC ? (pd == 0 ? 0.0625f : pd == 1 ? 16.0f : 4096.0f) : 0.0f;  // 256^p / 16
        }
    }
    float accd[NG][2][2], accm[2] = {0.0f, 0.0f};
#pragma unroll
    for (int ng = 0; ng < NG; ++ng) accd[ng][0][0] = accd[ng][0][1] = accd[ng][1][0] = accd[ng][1][1] = 0.0f;

    int t = static_cast<int>(u0 / nblk), b = static_cast<int>(u0 % nblk);
    auto unit = [&](const SuperBlock& sbk) {
        const uint2* bq = sB + static_cast<size_t>(b) * 8 * NC * 4;
        uint32_t scl[2], sch[2], am[2];
        float d[2], dmn[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const uint4 h = sbk.hd[i];
            d[i] = fh3::h2f_bits(h.x);
            dmn[i] = fh3::h2f_bits(h.x >> 16);
            scl[i] = h.y & 0x3F3F3F3Fu;
            sch[i] = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
            const uint32_t mw = lo ? (h.z & 0x3F3F3F3Fu) : (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u));
            am[i] = __byte_perm(mw, 0u, sel_m);
        }
        int S[NG][2][2];
#pragma unroll
        for (int ng = 0; ng < NG; ++ng) S[ng][0][0] = S[ng][0][1] = S[ng][1][0] = S[ng][1][1] = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint2 w0 = sbk.q[0][c], w1 = sbk.q[1][c];
            const uint32_t s0 = c < 2 ? scl[0] : sch[0], s1 = c < 2 ? scl[1] : sch[1];
            const uint32_t sl = 0x4440u | (2 * (c & 1)), sh = sl + 1;
            const int lo0 = static_cast<int>(__byte_perm(s0, 0u, sl)) << 4, hi0 = static_cast<int>(__byte_perm(s0, 0u, sh));
            const int lo1 = static_cast<int>(__byte_perm(s1, 0u, sl)) << 4, hi1 = static_cast<int>(__byte_perm(s1, 0u, sh));
#pragma unroll
            for (int ng = 0; ng < NG; ++ng) {
                const uint2 bl = bq[((2 * c) * NC + bcol[ng]) * 4 + tq];
                const uint2 bh = bq[((2 * c + 1) * NC + bcol[ng]) * 4 + tq];
                int Cl[4], Ch[4];
                mma_i8_z(Cl, w0.x & 0x0F0F0F0Fu, w1.x & 0x0F0F0F0Fu, w0.y & 0x0F0F0F0Fu, w1.y & 0x0F0F0F0Fu,
                         bl.x & bmask[ng], bl.y & bmask[ng]);
                mma_i8_z(Ch, w0.x & 0xF0F0F0F0u, w1.x & 0xF0F0F0F0u, w0.y & 0xF0F0F0F0u, w1.y & 0xF0F0F0F0u,
                         bh.x & bmask[ng], bh.y & bmask[ng]);
                S[ng][0][0] += lo0 * Cl[0] + hi0 * Ch[0];
                S[ng][0][1] += lo0 * Cl[1] + hi0 * Ch[1];
                S[ng][1][0] += lo1 * Cl[2] + hi1 * Ch[2];
                S[ng][1][1] += lo1 * Cl[3] + hi1 * Ch[3];
            }
        }
        float dm4[4];
        mma_16816_z(dm4, am[0], am[1], 0u, 0u, sM[static_cast<size_t>(b) * 32 + lane], 0u);
        const float* fsb = sF + static_cast<size_t>(b) * M;
        // columns past 3M hold zeros: a zero factor keeps a non-finite token out of them
        const float fm = tq < M ? fsb[tq] * 137438953472.0f : 0.0f;  // 2^37, as gemv_i8_kernel
        accm[0] = fmaf(dm4[0] + dm4[1], -dmn[0] * fm, accm[0]);
        accm[1] = fmaf(dm4[2] + dm4[3], -dmn[1] * fm, accm[1]);
#pragma unroll
        for (int ng = 0; ng < NG; ++ng)
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const float f = tok[ng][i] >= 0 ? fsb[tok[ng][i]] : 0.0f;
                accd[ng][0][i] = fmaf(__int2float_rn(S[ng][0][i]), d[0] * f, accd[ng][0][i]);
                accd[ng][1][i] = fmaf(__int2float_rn(S[ng][1][i]), d[1] * f, accd[ng][1][i]);
            }
    };
    // end of this warp's segment of tile t: direct store, or partials + last-arriver sum
    auto finish_segment = [&]() {
        // each token's columns -> its row sums (fixed order), held by every lane of the quad
        float v[M][2];
#pragma unroll
        for (int tt = 0; tt < M; ++tt)
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                float a = tq == tt ? accm[r] : 0.0f;
#pragma unroll
                for (int ng = 0; ng < NG; ++ng)
#pragma unroll
                    for (int i = 0; i < 2; ++i)
                        if (tok[ng][i] == tt) a = fmaf(accd[ng][r][i], cw[ng][i], a);
                a += __shfl_xor_sync(0xffffffffu, a, 1);
                a += __shfl_xor_sync(0xffffffffu, a, 2);
                v[tt][r] = a;
            }
#pragma unroll
        for (int ng = 0; ng < NG; ++ng) accd[ng][0][0] = accd[ng][0][1] = accd[ng][1][0] = accd[ng][1][1] = 0.0f;
        accm[0] = accm[1] = 0.0f;
        // lane tq keeps token tq's sums
        float v0 = 0.0f, v1 = 0.0f;
#pragma unroll
        for (int tt = 0; tt < M; ++tt)
            if (tq == tt) {
                v0 = v[tt][0];
                v1 = v[tt][1];
            }
        const int64_t wf = stream_warp_of(static_cast<int64_t>(t) * nblk, GW, units);
        const int64_t wl = stream_warp_of(static_cast<int64_t>(t + 1) * nblk - 1, GW, units);
        const int nseg = static_cast<int>(wl - wf + 1);
        const int64_t r0 = static_cast<int64_t>(t) * 16 + g, r1 = r0 + 8;
        if (nseg == 1) {
            if (tq < M) {
                if (r0 < N) y[tq * ldy + r0] = v0 + (bias ? bias[r0] : 0.0f);
                if (r1 < N) y[tq * ldy + r1] = v1 + (bias ? bias[r1] : 0.0f);
            }
            return;
        }
        if (nseg > seg_max) {
            if (lane == 0) fh3::record_status(status, FH3_ERR);  // never write past the slots
            return;
        }
        float* pt = partials + static_cast<int64_t>(t) * seg_max * 16 * M;
        if (tq < M) {
            pt[((gw - wf) * 16 + g) * M + tq] = v0;
            pt[((gw - wf) * 16 + g + 8) * M + tq] = v1;
        }
        // the warp's stores, then lane 0's release/acquire count: it publishes them at GPU
        // scope and, for the last segment, acquires the other segments' stores
        __syncwarp();
        int old = 0;
        if (lane == 0) asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(old) : "l"(counters + t) : "memory");
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old != nseg - 1) return;
        __syncwarp();
        if (tq < M) {  // last segment: add all in segment order
            float s0 = 0.0f, s1 = 0.0f;
            for (int q = 0; q < nseg; ++q) {
                const float a0 = __ldcg(pt + (q * 16 + g) * M + tq), a1 = __ldcg(pt + (q * 16 + g + 8) * M + tq);
                s0 = q == 0 ? a0 : s0 + a0;
                s1 = q == 0 ? a1 : s1 + a1;
            }
            if (r0 < N) y[tq * ldy + r0] = s0 + (bias ? bias[r0] : 0.0f);
            if (r1 < N) y[tq * ldy + r1] = s1 + (bias ? bias[r1] : 0.0f);
        }
        if (lane == 0) counters[t] = 0;
    };
    auto step = [&](const SuperBlock& cur, int i) {
        unit(cur);
        if (b == nblk - 1 || i == n - 1) finish_segment();
        if (++b == nblk) {
            b = 0;
            ++t;
        }
    };
    for (int i = 0; i < n; i += 2) {
        step(sa, i);
        if (i + 2 < n) load_next(sa);
        if (i + 1 >= n) break;
        step(sbuf, i + 1);
        if (i + 3 < n) load_next(sbuf);
    }
}

// ---------------------------------------------------------------------------
// 5..16 tokens: a CTA owns a 16-row tile and a K range; the range's B fragments are
// copied to shared memory once.  When the fragments of the whole K would not fit, a
// cluster of S CTAs splits K and the partial sums meet over distributed shared memory.
// grid (ceil(N / 16), S), cluster (1, S, 1) when S > 1.  Dynamic shared memory:
// B fragments [nsb*8][8M] uint4, min-term B fragments [nsb][8M] u32, partials.
// ---------------------------------------------------------------------------
#ifndef FH3_GV_WIDE_MIN_BLOCKS
#define FH3_GV_WIDE_MIN_BLOCKS 2  // 8..16 tokens: a looser register budget (no spills)
#endif
template <int NT>
__global__ void __launch_bounds__(kGvMaxWarps * 32, NT == 1 ? FH3_GV_MIN_BLOCKS : FH3_GV_WIDE_MIN_BLOCKS)
    gemv_mma_kernel(
    const uint8_t* __restrict__ W, size_t row_bytes, int nblk, int64_t N, const uint4* __restrict__ frag,
    const uint32_t* __restrict__ mfrag, const int* __restrict__ expo, const float* __restrict__ fsb, int M,
    const float* __restrict__ bias, float* __restrict__ y, int64_t ldy, int S, int nsb_max) {
    extern __shared__ __align__(128) uint8_t gv_smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
    const int g = lane >> 2, tq = lane & 3;
    const int rank = S > 1 ? static_cast<int>(fh3::cluster_ctarank()) : 0;
    const int b_lo = static_cast<int>(static_cast<int64_t>(nblk) * rank / S);
    const int b_hi = static_cast<int>(static_cast<int64_t>(nblk) * (rank + 1) / S);
    const int nsb = b_hi - b_lo;
    const int lanes = 8 * M;  // fragment slots per sub-block

    uint4* sfrag = reinterpret_cast<uint4*>(gv_smem);
    uint32_t* smfrag = reinterpret_cast<uint32_t*>(gv_smem + static_cast<size_t>(nsb_max) * 8 * lanes * 16);
    float* part = reinterpret_cast<float*>(smfrag + static_cast<size_t>(nsb_max) * lanes);  // [nw][16][4NT]
    float* cta_part = part + kGvMaxWarps * 16 * 4 * NT;                                      // [16][4NT]

    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * 16 + g;
    const int64_t r1 = r0 + 8;
    const uint8_t* row0 = W + (r0 < N ? r0 : N - 1) * row_bytes;  // clamp loads; stores are masked
    const uint8_t* row1 = W + (r1 < N ? r1 : N - 1) * row_bytes;

    // weights do not depend on the prep kernel: start loading before waiting for it
    SuperBlock sa, sbuf;
    int b = b_lo + warp;
    if (b < b_hi) load_sb(sa, row0, row1, b, tq);
    const LaneCtx<NT> lc = lane_ctx<NT>(lane, lanes);

    pdl_wait();
    {
        const uint4* gf = frag + static_cast<int64_t>(b_lo) * 8 * lanes;
        const int nf = nsb * 8 * lanes;
        for (int i = threadIdx.x; i < nf; i += blockDim.x) cp_async16(sfrag + i, gf + i);
        const uint4* gm = reinterpret_cast<const uint4*>(mfrag + static_cast<int64_t>(b_lo) * lanes);
        const int nm = nsb * lanes / 4;  // 8M words per super-block: whole 16-byte units
        for (int i = threadIdx.x; i < nm; i += blockDim.x) cp_async16(reinterpret_cast<uint4*>(smfrag) + i, gm + i);
        cp_async_wait_all();
        __syncthreads();
    }

    float acc[2][NT];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[i][nt] = 0.0f;

    // the super-block's factor for token nt * 4 + tq of this lane (lanes past the last
    // token reuse its factors; their sums are never stored)
    auto factors = [&](int bb, float (&f)[NT]) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) f[nt] = __ldg(fsb + static_cast<int64_t>(bb) * M + min(nt * 4 + tq, M - 1));
    };
    // two super-blocks in flight: the next one's bytes load while this one computes
    float fa[NT], fb[NT];
    if (b < b_hi) factors(b, fa);
    while (b < b_hi) {
        const int b1 = b + nw;
        if (b1 < b_hi) {
            load_sb(sbuf, row0, row1, b1, tq);
            factors(b1, fb);
        }
        compute_sb<NT>(sa, lane, lanes, lc, sfrag + (b - b_lo) * 8 * lanes, smfrag + (b - b_lo) * lanes, acc, fa);
        if (b1 >= b_hi) break;
        const int b2 = b1 + nw;
        if (b2 < b_hi) {
            load_sb(sa, row0, row1, b2, tq);
            factors(b2, fa);
        }
        compute_sb<NT>(sbuf, lane, lanes, lc, sfrag + (b1 - b_lo) * 8 * lanes, smfrag + (b1 - b_lo) * lanes, acc, fb);
        b = b2;
    }
    finish_tile<NT>(acc, part, cta_part, warp, nw, lane, S, rank, M, N, expo, bias, y, ldy);
}

size_t gv_smem_bytes(int M, int NT, int nsb_max) {
    return static_cast<size_t>(nsb_max) * (8 * 8 * M * 16 + 8 * M * 4) + (kGvMaxWarps + 1) * 16 * 4 * NT * 4;
}

cudaLaunchAttribute pdl_attr() {
    cudaLaunchAttribute a;
    a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a.val.programmaticStreamSerializationAllowed = 1;
    return a;
}

int set_smem(const void* fn, size_t smem, int& cur, const char* what) {
    if (static_cast<int>(smem) <= cur) return 0;
    const int rc = fh3host::check_cuda(
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)), what);
    if (rc == 0) cur = static_cast<int>(smem);
    return rc;
}

template <int M>
int launch_small(const Fh3CudaW* w, const uint4* frag, const uint32_t* mfrag, const int* expo, const float* fsb,
                 float* y, const float* bias, cudaStream_t s) {
    const int64_t N = w->out, K = w->in;
    const int nblk = static_cast<int>(K / fh3::kQ4KBlock);
    // balanced warps: the fewest that keep the per-warp count at ceil(nblk / 8)
    const int per = (nblk + kGvMaxWarps - 1) / kGvMaxWarps;
    const int warps = (nblk + per - 1) / per;
    const int lanes = 8 * M;
    const size_t smem = static_cast<size_t>(warps) * 2 * (8 * lanes + lanes / 4) * 16 + (warps + 1) * 16 * 4 * 4;
    static int smem_set = 0;
    int rc = set_smem(reinterpret_cast<const void*>(gemv_mma_small_kernel<M>), smem, smem_set,
                      "gemv_mma_small_kernel smem attribute");
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((N + 15) / 16), 1, 1);
    cfg.blockDim = dim3(warps * 32, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1] = {pdl_attr()};
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return fh3host::check_cuda(cudaLaunchKernelEx(&cfg, gemv_mma_small_kernel<M>, w->data,
                                                  fh3cuda_row_bytes(FH3CUDA_TYPE_Q4_K, K), nblk, N, frag, mfrag, expo,
                                                  fsb, bias, y, N),
                               "gemv_mma_small_kernel launch");
}

// Launch the stream-K kernel when its shared memory fits; returns 1 (not launched) otherwise.
template <int M>
int launch_stream(const Fh3CudaW* w, const float* x, float* y, const float* bias, cudaStream_t s) {
    using namespace fh3host;
    DevCtx* c = ctx();
    const int64_t N = w->out, K = w->in;
    const int nblk = static_cast<int>(K / fh3::kQ4KBlock);
    constexpr int LANES = 8 * M;
    const size_t smem = static_cast<size_t>(nblk) * (8 * LANES * 16 + LANES * 4 + M * 4);
    if (smem > 227 * 1024) return 1;
    const int sms = ctx_sms(c);
    const int64_t ntiles = (N + 15) / 16;
    const int64_t units = ntiles * nblk;
    const int64_t GW = std::min<int64_t>(static_cast<int64_t>(sms) * kStreamWarps, units);
    const int64_t per = units / GW;  // >= 1: each run spans at least `per` units
    const int seg_max = static_cast<int>(std::min<int64_t>(nblk, (nblk + per - 1) / per + 1));
    float* partials = static_cast<float*>(scratch(c, 6, static_cast<size_t>(ntiles) * seg_max * 16 * M * 4, s));
    int* counters = static_cast<int*>(scratch_zeroed(c, 7, static_cast<size_t>(ntiles) * 4, s));
    if (!partials || !counters) return FH3_E_NOMEM;

    static int smem_set = 0;
    int rc = set_smem(reinterpret_cast<const void*>(gemv_stream_kernel<M>), smem, smem_set,
                      "gemv_stream_kernel smem attribute");
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(sms), 1, 1);
    cfg.blockDim = dim3(kStreamWarps * 32, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1] = {pdl_attr()};
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return check_cuda(cudaLaunchKernelEx(&cfg, gemv_stream_kernel<M>, w->data, fh3cuda_row_bytes(FH3CUDA_TYPE_Q4_K, K),
                                         nblk, N, units, seg_max, x, bias, y, N, partials, counters, ctx_status(c)),
                      "gemv_stream_kernel launch");
}

// Launch the 1-token integer kernel when its shared memory fits; returns 1 (not launched)
// otherwise.  It shares the stream kernel's partial and counter slots (same run partition).
int launch_i8(const Fh3CudaW* w, const float* x, float* y, const float* bias, cudaStream_t s) {
    using namespace fh3host;
    DevCtx* c = ctx();
    const int64_t N = w->out, K = w->in;
    const int nblk = static_cast<int>(K / fh3::kQ4KBlock);
    const size_t smem = static_cast<size_t>(nblk) * (128 * 16 + 32 * 4 + 4);
    if (smem > 227 * 1024) return 1;
    const int sms = ctx_sms(c);
    const int64_t ntiles = (N + 15) / 16;
    const int64_t units = ntiles * nblk;
    const int64_t GW = std::min<int64_t>(static_cast<int64_t>(sms) * kStreamWarps, units);
    const int64_t per = units / GW;  // >= 1: each run spans at least `per` units
    const int seg_max = static_cast<int>(std::min<int64_t>(nblk, (nblk + per - 1) / per + 1));
    float* partials = static_cast<float*>(scratch(c, 6, static_cast<size_t>(ntiles) * seg_max * 16 * 4, s));
    int* counters = static_cast<int*>(scratch_zeroed(c, 7, static_cast<size_t>(ntiles) * 4, s));
    if (!partials || !counters) return FH3_E_NOMEM;

    static int smem_set = 0;
    int rc = set_smem(reinterpret_cast<const void*>(gemv_i8_kernel), smem, smem_set, "gemv_i8_kernel smem attribute");
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(sms), 1, 1);
    cfg.blockDim = dim3(kStreamWarps * 32, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1] = {pdl_attr()};
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return check_cuda(cudaLaunchKernelEx(&cfg, gemv_i8_kernel, w->data, fh3cuda_row_bytes(FH3CUDA_TYPE_Q4_K, K), nblk,
                                         N, units, seg_max, x, bias, y, partials, counters, ctx_status(c)),
                      "gemv_i8_kernel launch");
}

// Launch the 2..4-token integer kernel when its shared memory fits; returns 1 otherwise.
template <int M>
int launch_i8m(const Fh3CudaW* w, const float* x, float* y, const float* bias, cudaStream_t s) {
    using namespace fh3host;
    DevCtx* c = ctx();
    const int64_t N = w->out, K = w->in;
    const int nblk = static_cast<int>(K / fh3::kQ4KBlock);
    const size_t smem = static_cast<size_t>(nblk) * (8 * 3 * M * 4 * 8 + 32 * 4 + M * 4);
    if (smem > 227 * 1024) return 1;
    const int sms = ctx_sms(c);
    const int64_t ntiles = (N + 15) / 16;
    const int64_t units = ntiles * nblk;
    const int64_t GW = std::min<int64_t>(static_cast<int64_t>(sms) * kStreamWarps, units);
    const int64_t per = units / GW;  // >= 1: each run spans at least `per` units
    const int seg_max = static_cast<int>(std::min<int64_t>(nblk, (nblk + per - 1) / per + 1));
    float* partials = static_cast<float*>(scratch(c, 6, static_cast<size_t>(ntiles) * seg_max * 16 * M * 4, s));
    int* counters = static_cast<int*>(scratch_zeroed(c, 7, static_cast<size_t>(ntiles) * 4, s));
    if (!partials || !counters) return FH3_E_NOMEM;

    static int smem_set = 0;
    int rc = set_smem(reinterpret_cast<const void*>(gemv_i8m_kernel<M>), smem, smem_set,
                      "gemv_i8m_kernel smem attribute");
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(sms), 1, 1);
    cfg.blockDim = dim3(kStreamWarps * 32, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1] = {pdl_attr()};
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return check_cuda(cudaLaunchKernelEx(&cfg, gemv_i8m_kernel<M>, static_cast<const uint8_t*>(w->data),
                                         fh3cuda_row_bytes(FH3CUDA_TYPE_Q4_K, K), nblk, K, N, units, seg_max, x, bias,
                                         y, N, partials, counters, ctx_status(c)),
                      "gemv_i8m_kernel launch");
}

template <int NT>
int launch_mma(const Fh3CudaW* w, const uint4* frag, const uint32_t* mfrag, const int* expo, const float* fsb, int M,
               float* y, const float* bias, cudaStream_t s) {
    const int64_t N = w->out, K = w->in;
    const int nblk = static_cast<int>(K / fh3::kQ4KBlock);
    int S = 1;
    while (S < 8 && S < nblk && gv_smem_bytes(M, NT, (nblk + S - 1) / S) > kGvSmemTarget) S *= 2;
    const int nsb_max = (nblk + S - 1) / S;
    const int per = (nsb_max + kGvMaxWarps - 1) / kGvMaxWarps;
    const int warps = (nsb_max + per - 1) / per;
    const size_t smem = gv_smem_bytes(M, NT, nsb_max);
    static int smem_set[5] = {0, 0, 0, 0, 0};  // per instantiation, grows only
    int rc = set_smem(reinterpret_cast<const void*>(gemv_mma_kernel<NT>), smem, smem_set[NT],
                      "gemv_mma_kernel smem attribute");
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((N + 15) / 16), static_cast<unsigned>(S), 1);
    cfg.blockDim = dim3(warps * 32, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na++] = pdl_attr();
    if (S > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = S;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return fh3host::check_cuda(
        cudaLaunchKernelEx(&cfg, gemv_mma_kernel<NT>, w->data, fh3cuda_row_bytes(FH3CUDA_TYPE_Q4_K, K), nblk, N,
                           frag, mfrag, expo, fsb, M, bias, y, N, S, nsb_max),
        "gemv_mma_kernel launch");
}

}  // namespace

namespace fh3host {

// 1..16-token Q4_K GEMV on warp MMAs; scratch slot 5 holds the activation fragments.
int gemv_mma(const Fh3CudaW* w, const float* x, float* y, int n_tok, const float* bias, cudaStream_t s) {
    DevCtx* c = ctx();
    if (!c) return set_error(FH3CUDA_E_NODEV, "gemv_mma: call fh3cuda_init first");
    // Measured on the BASELINE shapes (5120->13824, 13824->5120, 5120->5120):
    // * 1 token: the stream-K kernel on integer MMAs (gemv_i8_kernel), faster on all three;
    // * 2 tokens, and 3..4 tokens when out > in: its 2..4-token form (gemv_i8m_kernel);
    // * the tcgen05 kernel (gemv_tc.cu) at 3..4 tokens when out <= in and from 5 tokens on.
    // FH3CUDA_GEMV_KERNEL=tc forces tcgen05 for every shape; mma-i8 the integer kernels for
    // 1..4 tokens; mma-stream / mma-cta the fp16 warp-MMA kernels (single-launch stream-K for
    // 1..2 tokens, prep + CTA-per-tile otherwise; mma-cta always the latter).
    const char* kname = getenv("FH3CUDA_GEMV_KERNEL");
    const bool cta = kname && strcmp(kname, "mma-cta") == 0;
    const bool warp_mma = kname && (cta || strcmp(kname, "mma-stream") == 0);
    const bool tc_forced = kname && strcmp(kname, "tc") == 0;
    if (n_tok == 1 && !warp_mma && !tc_forced) {
        const int r = launch_i8(w, x, y, bias, s);
        if (r != 1) return r;
    }
    const bool i8_forced = kname && strcmp(kname, "mma-i8") == 0;
    if (n_tok >= 2 && n_tok <= 4 && !warp_mma && !tc_forced && (i8_forced || n_tok == 2 || w->out > w->in)) {
        const int r = n_tok == 2 ? launch_i8m<2>(w, x, y, bias, s)
                    : n_tok == 3 ? launch_i8m<3>(w, x, y, bias, s) : launch_i8m<4>(w, x, y, bias, s);
        if (r != 1) return r;
    }
    if (!warp_mma && (tc_forced || w->out <= w->in || n_tok >= 5)) {
        const int r = gemv_tc(w, x, y, n_tok, bias, s);
        if (r != 1) return r;
    }
    if (!cta && n_tok <= 2) {
        const int r = n_tok == 1 ? launch_stream<1>(w, x, y, bias, s) : launch_stream<2>(w, x, y, bias, s);
        if (r != 1) return r;
    }
    const int NT = (n_tok + 3) / 4;
    const int64_t K = w->in;
    const size_t fbytes = static_cast<size_t>(K) * n_tok * 4;  // (K/32) sub-blocks x 8M slots x 16 B
    const size_t mbytes = static_cast<size_t>(K / 256) * 8 * n_tok * sizeof(uint32_t);
    const size_t sbytes = static_cast<size_t>(K / 256) * n_tok * 4;  // per-super-block factors
    uint8_t* base = static_cast<uint8_t*>(scratch(c, 5, fbytes + mbytes + 256 + sbytes, s));
    if (!base) return FH3_E_NOMEM;
    auto* frag = reinterpret_cast<uint4*>(base);
    auto* mfrag = reinterpret_cast<uint32_t*>(base + fbytes);
    auto* expo = reinterpret_cast<int*>(base + fbytes + mbytes);
    auto* fsb = reinterpret_cast<float*>(base + fbytes + mbytes + 256);
    const dim3 pgrid(static_cast<unsigned>((K + kPrepSlice - 1) / kPrepSlice), static_cast<unsigned>(n_tok));
    gemv_mma_prep_kernel<<<pgrid, 256, 0, s>>>(x, K, n_tok, frag, mfrag, expo, fsb);
    const int rc = check_cuda(cudaGetLastError(), "gemv_mma_prep_kernel launch");
    if (rc) return rc;
    switch (n_tok) {
        case 1: return launch_small<1>(w, frag, mfrag, expo, fsb, y, bias, s);
        case 2: return launch_small<2>(w, frag, mfrag, expo, fsb, y, bias, s);
        case 3: return launch_small<3>(w, frag, mfrag, expo, fsb, y, bias, s);
        case 4: return launch_small<4>(w, frag, mfrag, expo, fsb, y, bias, s);
        default: break;
    }
    switch (NT) {
        case 2: return launch_mma<2>(w, frag, mfrag, expo, fsb, n_tok, y, bias, s);
        case 3: return launch_mma<3>(w, frag, mfrag, expo, fsb, n_tok, y, bias, s);
        default: return launch_mma<4>(w, frag, mfrag, expo, fsb, n_tok, y, bias, s);
    }
}

}  // namespace fh3host
