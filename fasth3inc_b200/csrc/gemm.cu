// gemm.cu -- large-M Q4_K GEMM on the 5th-generation tensor cores (tcgen05).
//
// Replaces fh3_matmul's large-M regime (src/core/fh3_ops.c:317-404: per 64-row
// tile, dequantise to fp32 scratch, then AVX2 dots against every token).
//
//   y[m][n] = epi( sum_k A[m][k] * W[n][k] ),  A = activations (bf16, M x K),
//   W = Q4_K rows (N x K), fp32 accumulation in tensor memory.
//
// Two kernels share the dequantiser and the epilogue:
//
// gemm_q4k_pair_kernel (default for M > 128) -- a 2-CTA cluster on two SMs
//   computes 256 x 256 tiles with tcgen05.mma.cta_group::2 (M = 256): each CTA
//   holds 128 activation rows and dequantises only its 128 weight rows of the
//   tile, so dequantisation and B-operand shared-memory traffic per SM are half
//   of a one-SM 128 x 256 tile with the same tensor work.  The leader CTA (rank
//   0) issues the MMAs; both CTAs' TMA activation loads count their bytes on the
//   leader's barrier; the leader's commits arrive on both CTAs' barriers.
// gemm_q4k_tc_kernel (M <= 128) -- one CTA per SM, 128 x 256 tiles.
//
// Warp roles (both kernels, one persistent CTA per SM, grouped tile raster so
// concurrently running CTAs share weight tiles in L2):
//   warp 0      TMA producer: bf16 activation tiles (128-byte swizzle) and raw
//               Q4_K tiles (weight rows x one 144-byte super-block = K 256).
//   warp 1      TMEM owner; MMA issuer (4 x K-16 MMAs per K-64 stage) into one
//               of two 256-column fp32 accumulators.
//   warps 2-5   epilogue: tcgen05.ld accumulator rows -> bias / bf16 / SwiGLU /
//               gated residual -> global memory.
//   warps 6-13  dequantisers: raw Q4_K in shared memory -> bf16 B operand in the
//               UMMA K-major 128-byte-swizzle layout.  byte_perm builds the fp32
//               pattern 1 + q/128, an exact subtraction gives q/128, and one FMA
//               with the exact scale 128*d*sc and offset -dmin*m gives fh3's fp32
//               weight (dequant_q4_k, src/core/fh3_quant.c:154-196), then one
//               rounding to bf16.
// No TMA multicast anywhere.  Every mbarrier wait is bounded (common.cuh); on a
// timeout the kernel flags FH3CUDA_E_TIMEOUT, drains its own copies/MMAs, frees
// TMEM and returns.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace {

constexpr int BK = 64;                        // K per MMA stage: one 128-byte swizzle row of bf16
constexpr int A_BYTES = 128 * BK * 2;         // 16384: 128 activation rows
constexpr int R_HALF = 128 * fh3::kQ4KBytes;  // 18432: one TMA box (128 weight rows x 144 B)
constexpr int kNumEpiWarps = 4;
constexpr int kNumDqWarps = 8;
constexpr int kEpiWarp0 = 2;
constexpr int kDqWarp0 = kEpiWarp0 + kNumEpiWarps;
constexpr int kThreads = 32 * (kDqWarp0 + kNumDqWarps);  // 448 (one-SM kernel)
constexpr int kRawWarp = kDqWarp0 + kNumDqWarps;         // pair kernel: raw-weight producer
constexpr int kThreadsPair = 32 * (kRawWarp + 1);        // 480
constexpr int kTmemCols = 512;                           // two 256-column accumulators
constexpr int kGroupM = 16;

struct Params {
    int64_t M, N, K;  // N = weight rows; for SwiGLU N = 2F
    int64_t n_out;    // output columns (N, or F for SwiGLU)
    int64_t ldy;
    const float* bias;
    const float* gate;
    void* y;
    int epi;
    int* status;
    // split-K (gemm_q4k_pair_kernel): each tile's super-blocks cut into ksplit ranges, one
    // unit of work each; a unit stores its fp32 accumulator in part[split][M][n_out] (no
    // bias), and splitk_reduce_kernel adds the ranges in order and applies the epilogue
    int ksplit = 1;
    float* part = nullptr;
    // programmatic dependent launch: 0 off; 1 the kernel may start while the previous
    // kernel on its stream runs, and waits for it (griddepcontrol.wait) before its first
    // access to activations, outputs, bias, gate or partials; 2 (gemm_bf16_pair_kernel)
    // the same, except that the weight tiles of the first stages are loaded before that
    // wait (the caller guarantees the weights).  gemm_q4k_pair_kernel with 1 loads and
    // dequantises its Q4_K weights before the wait: no kernel of this library that lets
    // its dependents start early writes Q4_K data (weights arrive by copies, and by
    // kernels that run to completion before any dependent starts)
    int pdl = 0;
};

__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

struct Ring {
    int idx = 0;
    uint32_t phase = 0;
    template <int S>
    __device__ __forceinline__ void next() {
        if (++idx == S) {
            idx = 0;
            phase ^= 1u;
        }
    }
};

__device__ __forceinline__ void tile_coords(int64_t tile, int64_t num_m, int64_t num_n, int64_t& mb,
                                            int64_t& nb) {
    const int64_t per_group = static_cast<int64_t>(kGroupM) * num_n;
    const int64_t group = tile / per_group;
    const int64_t first_m = group * kGroupM;
    const int64_t gsize = (num_m - first_m) < kGroupM ? (num_m - first_m) : kGroupM;
    const int64_t in_group = tile - group * per_group;
    mb = first_m + in_group % gsize;
    nb = in_group / gsize;
}

__device__ __forceinline__ float silu_ref(float g) {
    // fh3_swiglu: g / (1 + expf(-g)), and 0 below -80 (src/core/fh3_ops.c:517-523)
    return g < -80.0f ? 0.0f : g / (1.0f + expf(-g));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}

// Dequantise output chunks [j0, j0 + nj) of one weight row for K-64 stage `sub`
// of a raw super-block into a 128-byte swizzled B row.  Chunk j holds k = 8j..8j+7;
// chunks 0-3 come from the low nibbles (sub-block 2*sub), 4-7 from the high nibbles
// (sub-block 2*sub+1).
template <int J0, int NJ>
__device__ __forceinline__ void dequant_row_stage_q(const uint4& hdr, const uint4& q0, const uint4& q1, int sub,
                                                    uint8_t* brow, uint32_t swz);

template <int J0, int NJ>
__device__ __forceinline__ void dequant_row_stage(const uint8_t* raw, const uint4& hdr, int sub, uint8_t* brow,
                                                  uint32_t swz) {
    const uint4 q0 = *reinterpret_cast<const uint4*>(raw + 16 + sub * 32);
    const uint4 q1 = *reinterpret_cast<const uint4*>(raw + 32 + sub * 32);
    dequant_row_stage_q<J0, NJ>(hdr, q0, q1, sub, brow, swz);
}

// The scale pair of sub-block `sb` of a super-block header: s = 128*(d*sc) (exact scaling
// of fh3's rounded d*sc) and nm = -(dmin*m).
__device__ __forceinline__ void q4k_sub_scales(const uint4& hdr, int sb, float& s, float& nm) {
    const float d = fh3::h2f_bits(hdr.x), dmin = fh3::h2f_bits(hdr.x >> 16);
    int sc, m;
    fh3::q4k_scale_min_words(hdr.y, hdr.z, hdr.w, sb, sc, m);
    s = __fmul_rn(d, static_cast<float>(sc)) * 128.0f;
    nm = -__fmul_rn(dmin, static_cast<float>(m));
}

// Eight consecutive weights of one sub-block as bf16: the low (hh = 0) or high (hh = 1)
// nibbles of the nibble bytes in wa (first four) and wb (next four).  Two weights per
// packed fp32x2 subtract and FMA: (1 + q/128) - 1 = q/128 exact, then one rounding of
// s * q/128 + nm, the same fp32 weight as fh3's (d*sc)*q - dmin*m, then one rounding
// to bf16.  Every Q4_K -> bf16 path of this file goes through here.
__device__ __forceinline__ uint4 q4k_chunk8_bf16(float s, float nm, uint32_t wa, uint32_t wb, int hh) {
    const uint32_t va = ((hh ? (wa >> 4) : wa) & 0x0F0F0F0Fu) | 0x80808080u;
    const uint32_t vb = ((hh ? (wb >> 4) : wb) & 0x0F0F0F0Fu) | 0x80808080u;
    const uint64_t s2 = fh3::f2_pack(s, s), n2 = fh3::f2_pack(nm, nm);
    const uint64_t one2 = fh3::f2_pack(-1.0f, -1.0f);
    auto w2 = [&](uint32_t v, uint32_t sel_a, uint32_t sel_b) {
        const uint64_t nb = fh3::f2_pack(fh3::nib_f(v, sel_a), fh3::nib_f(v, sel_b));
        const float2 w = fh3::f2_unpack(fh3::f2_fma(s2, fh3::f2_add(nb, one2), n2));
        return pack_bf16(w.x, w.y);
    };
    uint4 pk;
    pk.x = w2(va, fh3::kSel0, fh3::kSel1);
    pk.y = w2(va, fh3::kSel2, fh3::kSel3);
    pk.z = w2(vb, fh3::kSel0, fh3::kSel1);
    pk.w = w2(vb, fh3::kSel2, fh3::kSel3);
    return pk;
}

// the same on the stage's 32 nibble bytes already loaded (q0, q1)
template <int J0, int NJ>
__device__ __forceinline__ void dequant_row_stage_q(const uint4& hdr, const uint4& q0, const uint4& q1, int sub,
                                                    uint8_t* brow, uint32_t swz) {
    float s[2], nm[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        if ((hh == 0 && J0 >= 4) || (hh == 1 && J0 + NJ <= 4)) continue;
        q4k_sub_scales(hdr, 2 * sub + hh, s[hh], nm[hh]);
    }
    const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int j = J0; j < J0 + NJ; ++j) {
        const int hh = j >> 2;
        const uint4 pk = q4k_chunk8_bf16(s[hh], nm[hh], qw[2 * (j & 3)], qw[2 * (j & 3) + 1], hh);
        // 16-byte chunk j of this 128-byte row, XOR-swizzled by row % 8
        *reinterpret_cast<uint4*>(brow + ((static_cast<uint32_t>(j) ^ swz) << 4)) = pk;
    }
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* yr, const float* o) {
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
        uint4 pk;
        pk.x = pack_bf16(o[j], o[j + 1]);
        pk.y = pack_bf16(o[j + 2], o[j + 3]);
        pk.z = pack_bf16(o[j + 4], o[j + 5]);
        pk.w = pack_bf16(o[j + 6], o[j + 7]);
        *reinterpret_cast<uint4*>(yr + j) = pk;
    }
}

// The accumulator row of this thread, 32 columns at a time, straight from TMEM.
struct TmemAcc {
    uint32_t tbase;
    __device__ __forceinline__ void load(int col, uint32_t (&v)[32]) const {
        fh3::tmem_ld32(tbase + col, v);
        fh3::tmem_ld_wait();
        fh3::tmem_regs_ready(v);
    }
    __device__ __forceinline__ void load2(int ca, int cb, uint32_t (&a)[32], uint32_t (&b)[32]) const {
        fh3::tmem_ld32(tbase + ca, a);
        fh3::tmem_ld32(tbase + cb, b);
        fh3::tmem_ld_wait();
        fh3::tmem_regs_ready(a);
        fh3::tmem_regs_ready(b);
    }
};

template <class Acc>
__device__ __forceinline__ void epilogue_rows(const Params& p, const Acc& acc, int64_t m, int64_t nb) {
    const bool row_ok = m < p.M;
    if (p.epi == FH3CUDA_EPI_SWIGLU) {
        for (int cc = 0; cc < 4; ++cc) {
            uint32_t v[32], g[32];
            acc.load2(cc * 32, 128 + cc * 32, v, g);
            const int64_t f0 = nb * 128 + cc * 32;
            if (!row_ok || f0 >= p.n_out) continue;
            __nv_bfloat16* yr = static_cast<__nv_bfloat16*>(p.y) + m * p.ldy;
            float o[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                float vv = __uint_as_float(v[j]), gg = __uint_as_float(g[j]);
                if (p.bias) {
                    const int64_t fj = f0 + j < p.n_out ? f0 + j : p.n_out - 1;
                    vv += p.bias[fj];
                    gg += p.bias[p.n_out + fj];
                }
                o[j] = vv * silu_ref(gg);
            }
            if (f0 + 32 <= p.n_out && (reinterpret_cast<uintptr_t>(yr + f0) & 15) == 0) {
                store_bf16x32(yr + f0, o);
            } else {
                for (int j = 0; j < 32; ++j)
                    if (f0 + j < p.n_out) yr[f0 + j] = __float2bfloat16_rn(o[j]);
            }
        }
        return;
    }
    for (int cc = 0; cc < 8; ++cc) {
        uint32_t v[32];
        acc.load(cc * 32, v);
        const int64_t n0 = nb * 256 + cc * 32;
        if (!row_ok || n0 >= p.N) continue;
        float o[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            o[j] = __uint_as_float(v[j]);
            if (p.bias) o[j] += p.bias[n0 + j < p.N ? n0 + j : p.N - 1];
        }
        const bool full = n0 + 32 <= p.N;
        if (p.epi == FH3CUDA_EPI_BF16) {
            __nv_bfloat16* yr = static_cast<__nv_bfloat16*>(p.y) + m * p.ldy + n0;
            if (full && (reinterpret_cast<uintptr_t>(yr) & 15) == 0) {
                store_bf16x32(yr, o);
            } else {
                for (int j = 0; j < 32; ++j)
                    if (n0 + j < p.N) yr[j] = __float2bfloat16_rn(o[j]);
            }
        } else {
            float* yr = static_cast<float*>(p.y) + m * p.ldy + n0;
            if (p.epi == FH3CUDA_EPI_RESID) {
                if (full && ((reinterpret_cast<uintptr_t>(yr) | reinterpret_cast<uintptr_t>(p.gate + n0)) & 15) == 0) {
                    // issue all 16 loads before the first store: y and gate may not
                    // alias in a valid call, and batching them hides the latency
                    const float4* g4 = reinterpret_cast<const float4*>(p.gate + n0);
                    float4* y4 = reinterpret_cast<float4*>(yr);
                    float4 hv[8], gv[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        hv[j] = y4[j];
                        gv[j] = __ldg(g4 + j);
                    }
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        hv[j].x = fmaf(gv[j].x, o[4 * j + 0], hv[j].x);
                        hv[j].y = fmaf(gv[j].y, o[4 * j + 1], hv[j].y);
                        hv[j].z = fmaf(gv[j].z, o[4 * j + 2], hv[j].z);
                        hv[j].w = fmaf(gv[j].w, o[4 * j + 3], hv[j].w);
                    }
#pragma unroll
                    for (int j = 0; j < 8; ++j) y4[j] = hv[j];
                } else {
                    for (int j = 0; j < 32; ++j)
                        if (n0 + j < p.N) yr[j] = fmaf(p.gate[n0 + j], o[j], yr[j]);
                }
            } else if (full && (reinterpret_cast<uintptr_t>(yr) & 15) == 0) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4*>(yr + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
            } else {
                for (int j = 0; j < 32; ++j)
                    if (n0 + j < p.N) yr[j] = o[j];
            }
        }
    }
}

// Drain one 256-column accumulator (this thread's TMEM lane = one output row) and apply
// the epilogue.  `nb` is the tile's column block (256 weight rows, or 128 SwiGLU features).
__device__ __forceinline__ void epilogue_tile(const Params& p, uint32_t tbase, int64_t m, int64_t nb) {
    epilogue_rows(p, TmemAcc{tbase}, m, nb);
}

// =============================================================================
// one-SM kernel: 128 x 256 tiles
// =============================================================================
namespace one {
constexpr int BM = 128, BN = 256;
constexpr int SA = 3, SB = 3, SR = 2;
constexpr int B_BYTES = BN * BK * 2;  // 32768
constexpr int R_BYTES = 2 * R_HALF;   // 36864
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + SA * A_BYTES;
constexpr int OFF_R = OFF_B + SB * B_BYTES;
constexpr int OFF_BAR = OFF_R + SR * R_BYTES;
constexpr int kNumBars = 2 * SA + 2 * SB + 2 * SR + 4 + 1;
constexpr int OFF_MISC = OFF_BAR + kNumBars * 8;
constexpr int SMEM_BYTES = OFF_MISC + 64 + 1024;
static_assert(OFF_B % 1024 == 0 && OFF_R % 1024 == 0, "operand stages must be 1024-byte aligned");
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
}  // namespace one

__global__ void __launch_bounds__(kThreads, 1)
    gemm_q4k_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                       const Params p) {
    using namespace one;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* a_full = bars;
    uint64_t* a_empty = a_full + SA;
    uint64_t* b_full = a_empty + SA;
    uint64_t* b_empty = b_full + SB;
    uint64_t* r_full = b_empty + SB;
    uint64_t* r_empty = r_full + SR;
    uint64_t* acc_full = r_empty + SR;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 8);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const bool swiglu = p.epi == FH3CUDA_EPI_SWIGLU;
    const int64_t num_m = (p.M + BM - 1) / BM;
    const int64_t num_n = swiglu ? (p.n_out + 127) / 128 : (p.N + BN - 1) / BN;
    const int64_t num_tiles = num_m * num_n;
    const int ksteps = static_cast<int>(p.K / BK);

    if (threadIdx.x == 0) {
        for (int i = 0; i < SA; ++i) { fh3::mbar_init(&a_full[i], 1); fh3::mbar_init(&a_empty[i], 1); }
        for (int i = 0; i < SB; ++i) { fh3::mbar_init(&b_full[i], kNumDqWarps); fh3::mbar_init(&b_empty[i], 1); }
        for (int i = 0; i < SR; ++i) { fh3::mbar_init(&r_full[i], 1); fh3::mbar_init(&r_empty[i], kNumDqWarps); }
        for (int i = 0; i < 2; ++i) { fh3::mbar_init(&acc_full[i], 1); fh3::mbar_init(&acc_empty[i], kNumEpiWarps); }
        fh3::mbar_init(drain, 1);
        *abort_flag = 0;
        fh3::fence_mbar_init();
    }
    if (warp == 1) {
        fh3::tmem_alloc(tmem_slot, kTmemCols);
        fh3::tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        fh3::tma_prefetch_desc(&tmA);
        fh3::tma_prefetch_desc(&tmW);
    }
    fh3::tc_fence_before();
    __syncthreads();
    fh3::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            Ring ra, rr;
            uint32_t a_filled = 0, r_filled = 0;  // bit i: stage i has been filled at least once
            uint32_t a_par = 0, r_par = 0;        // parity of the last fill of each stage
            bool ok = true;
            for (int64_t tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                int64_t mb, nb;
                tile_coords(tile, num_m, num_n, mb, nb);
                const int m0 = static_cast<int>(mb * BM);
                int row0, row1;
                if (swiglu) {
                    row0 = static_cast<int>(nb * 128);
                    row1 = static_cast<int>(p.n_out + nb * 128);
                } else {
                    row0 = static_cast<int>(nb * BN);
                    row1 = row0 + 128;
                }
                for (int ks = 0; ks < ksteps && ok; ++ks) {
                    if ((ks & 3) == 0) {
                        if (!(ok = fh3::mbar_wait(&r_empty[rr.idx], rr.phase ^ 1u, abort_flag, p.status))) break;
                        uint8_t* dst = smem + OFF_R + rr.idx * R_BYTES;
                        fh3::mbar_arrive_expect_tx(&r_full[rr.idx], R_BYTES);
                        const int xb = (ks >> 2) * fh3::kQ4KBytes;
                        fh3::tma_load_2d(dst, &tmW, &r_full[rr.idx], xb, row0);
                        fh3::tma_load_2d(dst + R_HALF, &tmW, &r_full[rr.idx], xb, row1);
                        r_filled |= 1u << rr.idx;
                        r_par = (r_par & ~(1u << rr.idx)) | (rr.phase << rr.idx);
                        rr.next<SR>();
                    }
                    if (!(ok = fh3::mbar_wait(&a_empty[ra.idx], ra.phase ^ 1u, abort_flag, p.status))) break;
                    fh3::mbar_arrive_expect_tx(&a_full[ra.idx], A_BYTES);
                    fh3::tma_load_2d(smem + OFF_A + ra.idx * A_BYTES, &tmA, &a_full[ra.idx], ks * BK, m0);
                    a_filled |= 1u << ra.idx;
                    a_par = (a_par & ~(1u << ra.idx)) | (ra.phase << ra.idx);
                    ra.next<SA>();
                }
            }
            if (!ok) {
                // drain: wait (bounded, ignoring the abort flag) for our own copies in flight
                volatile int no_abort = 0;
                for (int i = 0; i < SA; ++i)
                    if (a_filled & (1u << i)) fh3::mbar_wait(&a_full[i], (a_par >> i) & 1u, &no_abort, nullptr);
                for (int i = 0; i < SR; ++i)
                    if (r_filled & (1u << i)) fh3::mbar_wait(&r_full[i], (r_par >> i) & 1u, &no_abort, nullptr);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = fh3::idesc_bf16_f32(BM, BN);
            Ring ra, rb, racc;
            bool ok = true;
            bool issued = false;
            for (int64_t tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                if (!(ok = fh3::mbar_wait(&acc_empty[racc.idx], racc.phase ^ 1u, abort_flag, p.status))) break;
                fh3::tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(racc.idx * BN);
                for (int ks = 0; ks < ksteps && ok; ++ks) {
                    if (!(ok = fh3::mbar_wait(&a_full[ra.idx], ra.phase, abort_flag, p.status))) break;
                    if (!(ok = fh3::mbar_wait(&b_full[rb.idx], rb.phase, abort_flag, p.status))) break;
                    fh3::tc_fence_after();
                    const uint64_t ad = fh3::sdesc_sw128(fh3::smem_u32(smem + OFF_A + ra.idx * A_BYTES));
                    const uint64_t bd = fh3::sdesc_sw128(fh3::smem_u32(smem + OFF_B + rb.idx * B_BYTES));
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        // +32 bytes of K per step inside the 128-byte swizzle row
                        fh3::umma_f16(d_tmem, ad + 2 * kk, bd + 2 * kk, idesc, (ks | kk) != 0 ? 1u : 0u);
                    }
                    issued = true;
                    fh3::umma_commit(&a_empty[ra.idx]);
                    fh3::umma_commit(&b_empty[rb.idx]);
                    ra.next<SA>();
                    rb.next<SB>();
                }
                if (ok) fh3::umma_commit(&acc_full[racc.idx]);
                racc.next<2>();
            }
            if (issued) {
                // all MMAs retired before TMEM is released
                fh3::umma_commit(drain);
                volatile int no_abort = 0;
                fh3::mbar_wait(drain, 0, &no_abort, nullptr);
            }
        }
    } else if (warp < kDqWarp0) {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        Ring racc;
        for (int64_t tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            int64_t mb, nb;
            tile_coords(tile, num_m, num_n, mb, nb);
            int ok = 1;
            if (lane == 0) ok = fh3::mbar_wait(&acc_full[racc.idx], racc.phase, abort_flag, p.status);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            fh3::tc_fence_after();
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(racc.idx * BN);
            epilogue_tile(p, tbase, mb * BM + q * 32 + lane, nb);
            fh3::tc_fence_before();
            __syncwarp();
            if (lane == 0) fh3::mbar_arrive(&acc_empty[racc.idx]);
            racc.next<2>();
        }
    } else {
        // ------------------------------------------------------------ dequantisers
        const int i = threadIdx.x - kDqWarp0 * 32;  // weight row of the tile (0..255)
        const uint32_t swz = static_cast<uint32_t>(i & 7);
        Ring rr, rb;
        bool ok = true;
        for (int64_t tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
            for (int rs = 0; rs < ksteps / 4 && ok; ++rs) {
                int w = 1;
                if (lane == 0) w = fh3::mbar_wait(&r_full[rr.idx], rr.phase, abort_flag, p.status);
                if (!(ok = __shfl_sync(0xffffffffu, w, 0) != 0)) break;
                const uint8_t* raw = smem + OFF_R + rr.idx * R_BYTES + i * fh3::kQ4KBytes;
                const uint4 hdr = *reinterpret_cast<const uint4*>(raw);
                for (int sub = 0; sub < 4 && ok; ++sub) {
                    if (lane == 0) w = fh3::mbar_wait(&b_empty[rb.idx], rb.phase ^ 1u, abort_flag, p.status);
                    if (!(ok = __shfl_sync(0xffffffffu, w, 0) != 0)) break;
                    dequant_row_stage<0, 8>(raw, hdr, sub, smem + OFF_B + rb.idx * B_BYTES + i * 128, swz);
                    fh3::fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) fh3::mbar_arrive(&b_full[rb.idx]);
                    rb.next<SB>();
                }
                __syncwarp();
                if (ok && lane == 0) fh3::mbar_arrive(&r_empty[rr.idx]);
                rr.next<SR>();
            }
        }
    }

    fh3::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        fh3::tc_fence_after();
        fh3::tmem_dealloc(tmem_base, kTmemCols);
    }
}

// =============================================================================
// two-SM kernel: 256 x 256 tiles over a CTA pair (tcgen05 cta_group::2)
// =============================================================================
namespace two {
constexpr int BN = 256;                 // pair tile: 256 weight rows, 128 per CTA
constexpr int SA = 5, SB = 5, SR = 3;
constexpr int B_BYTES = 128 * BK * 2;   // 16384: this CTA's 128 weight rows
constexpr int R_BYTES = R_HALF;         // 18432
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + SA * A_BYTES;
constexpr int OFF_R = OFF_B + SB * B_BYTES;
constexpr int OFF_BAR = OFF_R + SR * R_BYTES;
constexpr int kNumBars = 2 * SA + 2 * SB + 2 * SR + 4 + 1;
constexpr int OFF_MISC = OFF_BAR + kNumBars * 8;
constexpr int SMEM_BYTES = OFF_MISC + 64 + 1024;
static_assert(OFF_B % 1024 == 0 && OFF_R % 1024 == 0, "operand stages must be 1024-byte aligned");
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
}  // namespace two

__global__ void __launch_bounds__(kThreadsPair, 1)
    gemm_q4k_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                         const Params p) {
    using namespace two;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* a_full = bars;             // leader: 1 arrival + both CTAs' A bytes
    uint64_t* a_empty = a_full + SA;     // both: 1 (leader's commit)
    uint64_t* b_full = a_empty + SA;     // leader: kNumDqWarps / 2 from each CTA
    uint64_t* b_empty = b_full + SB;     // both: 1 (leader's commit)
    uint64_t* r_full = b_empty + SB;     // local: 1 arrival + raw bytes
    uint64_t* r_empty = r_full + SR;     // local: kNumDqWarps
    uint64_t* acc_full = r_empty + SR;   // both: 1 (leader's commit)
    uint64_t* acc_empty = acc_full + 2;  // leader: 2 x kNumEpiWarps
    uint64_t* drain = acc_empty + 2;     // both: 1 (leader's commit)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 8);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t cr = fh3::cluster_ctarank();  // 0 = leader
    const bool leader = cr == 0;
    const bool swiglu = p.epi == FH3CUDA_EPI_SWIGLU;
    const int64_t num_m = (p.M + 255) / 256;
    const int64_t num_n = swiglu ? (p.n_out + 127) / 128 : (p.N + BN - 1) / BN;
    const int64_t num_tiles = num_m * num_n;
    const int ksteps = static_cast<int>(p.K / BK);
    const int64_t pair = blockIdx.x >> 1;
    const int64_t npairs = gridDim.x >> 1;
    // units of work: (tile, K range of whole super-blocks); ksplit 1 = whole tiles
    const int ksplit = p.ksplit;
    const int64_t num_units = num_tiles * ksplit;
    const int nsb = ksteps / 4;
    auto unit_of = [&](int64_t u, int64_t& tile, int& split, int& sb0, int& sb1) {
        tile = u / ksplit;
        split = static_cast<int>(u - tile * ksplit);
        sb0 = split * nsb / ksplit;
        sb1 = (split + 1) * nsb / ksplit;
    };
    // the next kernel on this stream (the split-K reduction, the next call's conversion)
    // may be scheduled now; it waits for this whole grid before touching its outputs
    if (p.pdl) griddep_launch_dependents();

    if (threadIdx.x == 0) {
        for (int i = 0; i < SA; ++i) { fh3::mbar_init(&a_full[i], 1); fh3::mbar_init(&a_empty[i], 1); }
        for (int i = 0; i < SB; ++i) {
            fh3::mbar_init(&b_full[i], kNumDqWarps);  // one 4-warp group from each CTA
            fh3::mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < SR; ++i) { fh3::mbar_init(&r_full[i], 1); fh3::mbar_init(&r_empty[i], kNumDqWarps); }
        for (int i = 0; i < 2; ++i) { fh3::mbar_init(&acc_full[i], 1); fh3::mbar_init(&acc_empty[i], 2 * kNumEpiWarps); }
        fh3::mbar_init(drain, 1);
        *abort_flag = 0;
        fh3::fence_mbar_init();
    }
    if (warp == 1) {
        fh3::tmem_alloc_pair(tmem_slot, kTmemCols);
        fh3::tmem_relinquish_pair();
    }
    if (warp == 0 && lane == 0) {
        fh3::tma_prefetch_desc(&tmA);
        fh3::tma_prefetch_desc(&tmW);
    }
    fh3::tc_fence_before();
    fh3::cluster_sync_all();  // both CTAs' barriers initialised before any remote arrival
    fh3::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ activation producer (both CTAs)
        if (lane == 0) {
            Ring ra;
            uint32_t a_filled = 0, a_par = 0;
            bool ok = true;
            if (p.pdl) griddep_wait();  // the activations are the previous kernel's output
            for (int64_t u = pair; u < num_units && ok; u += npairs) {
                int64_t tile, mb, nb;
                int split, sb0, sb1;
                unit_of(u, tile, split, sb0, sb1);
                tile_coords(tile, num_m, num_n, mb, nb);
                const int m0 = static_cast<int>(mb * 256 + cr * 128);
                for (int ks = 4 * sb0; ks < 4 * sb1 && ok; ++ks) {
                    if (!(ok = fh3::mbar_wait(&a_empty[ra.idx], ra.phase ^ 1u, abort_flag, p.status))) break;
                    // both CTAs' activation bytes are counted on the leader's a_full
                    if (leader) fh3::mbar_arrive_expect_tx(&a_full[ra.idx], 2 * A_BYTES);
                    fh3::tma_load_2d_pair(smem + OFF_A + ra.idx * A_BYTES, &tmA,
                                          fh3::mapa_shared(fh3::smem_u32(&a_full[ra.idx]), 0), ks * BK, m0);
                    a_filled |= 1u << ra.idx;
                    a_par = (a_par & ~(1u << ra.idx)) | (ra.phase << ra.idx);
                    ra.next<SA>();
                }
            }
            if (!ok) {
                volatile int no_abort = 0;
                // both CTAs' activation copies count on the leader's a_full: the leader waits
                // for them, and the final cluster barrier keeps the peer resident until then
                if (leader)
                    for (int i = 0; i < SA; ++i)
                        if (a_filled & (1u << i))
                            fh3::mbar_wait_cluster(&a_full[i], (a_par >> i) & 1u, &no_abort, nullptr);
            }
        }
    } else if (warp == kRawWarp) {
        // ------------------------------------------------------------ raw-weight producer (both CTAs)
        // Runs ahead of the activation loads by up to SR super-blocks, so the dequantisers
        // never wait behind a full activation ring.
        if (lane == 0) {
            Ring rr;
            uint32_t r_filled = 0, r_par = 0;
            bool ok = true;
            for (int64_t u = pair; u < num_units && ok; u += npairs) {
                int64_t tile, mb, nb;
                int split, sb0, sb1;
                unit_of(u, tile, split, sb0, sb1);
                tile_coords(tile, num_m, num_n, mb, nb);
                const int wrow = swiglu ? static_cast<int>(cr ? p.n_out + nb * 128 : nb * 128)
                                        : static_cast<int>(nb * BN + cr * 128);
                for (int rs = sb0; rs < sb1 && ok; ++rs) {
                    if (!(ok = fh3::mbar_wait(&r_empty[rr.idx], rr.phase ^ 1u, abort_flag, p.status))) break;
                    fh3::mbar_arrive_expect_tx(&r_full[rr.idx], R_BYTES);
                    fh3::tma_load_2d(smem + OFF_R + rr.idx * R_BYTES, &tmW, &r_full[rr.idx],
                                     rs * fh3::kQ4KBytes, wrow);
                    r_filled |= 1u << rr.idx;
                    r_par = (r_par & ~(1u << rr.idx)) | (rr.phase << rr.idx);
                    rr.next<SR>();
                }
            }
            if (!ok) {
                volatile int no_abort = 0;
                for (int i = 0; i < SR; ++i)
                    if (r_filled & (1u << i)) fh3::mbar_wait(&r_full[i], (r_par >> i) & 1u, &no_abort, nullptr);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (leader)
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = fh3::idesc_bf16_f32(256, BN);
            Ring ra, rb, racc;
            bool ok = true;
            for (int64_t u = pair; u < num_units && ok; u += npairs) {
                int64_t tile;
                int split, sb0, sb1;
                unit_of(u, tile, split, sb0, sb1);
                if (!(ok = fh3::mbar_wait(&acc_empty[racc.idx], racc.phase ^ 1u, abort_flag, p.status))) break;
                fh3::tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(racc.idx * BN);
                for (int ks = 4 * sb0; ks < 4 * sb1 && ok; ++ks) {
                    if (!(ok = fh3::mbar_wait(&a_full[ra.idx], ra.phase, abort_flag, p.status))) break;
                    if (!(ok = fh3::mbar_wait(&b_full[rb.idx], rb.phase, abort_flag, p.status))) break;
                    fh3::tc_fence_after();
                    const uint64_t ad = fh3::sdesc_sw128(fh3::smem_u32(smem + OFF_A + ra.idx * A_BYTES));
                    const uint64_t bd = fh3::sdesc_sw128(fh3::smem_u32(smem + OFF_B + rb.idx * B_BYTES));
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        fh3::umma_f16_pair(d_tmem, ad + 2 * kk, bd + 2 * kk, idesc,
                                           (ks != 4 * sb0 || kk != 0) ? 1u : 0u);
                    fh3::umma_commit_pair(&a_empty[ra.idx], 0x3);
                    fh3::umma_commit_pair(&b_empty[rb.idx], 0x3);
                    ra.next<SA>();
                    rb.next<SB>();
                }
                if (ok) fh3::umma_commit_pair(&acc_full[racc.idx], 0x3);
                racc.next<2>();
            }
            // every MMA of the pair retires before either CTA releases its TMEM
            fh3::umma_commit_pair(drain, 0x3);
        }
        if (lane == 0) {
            volatile int no_abort = 0;
            fh3::mbar_wait_cluster(drain, 0, &no_abort, nullptr);
        }
    } else if (warp < kDqWarp0) {
        // ------------------------------------------------------------ epilogue (both CTAs)
        const int q = warp & 3;
        const uint32_t acc_empty_leader = fh3::mapa_shared(fh3::smem_u32(acc_empty), 0);
        Ring racc;
        if (p.pdl) griddep_wait();  // y, bias, gate and the partials belong to us after it
        for (int64_t u = pair; u < num_units; u += npairs) {
            int64_t tile, mb, nb;
            int split, sb0, sb1;
            unit_of(u, tile, split, sb0, sb1);
            tile_coords(tile, num_m, num_n, mb, nb);
            int ok = 1;
            if (lane == 0) ok = fh3::mbar_wait(&acc_full[racc.idx], racc.phase, abort_flag, p.status);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            fh3::tc_fence_after();
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(racc.idx * BN);
            const int64_t m = mb * 256 + cr * 128 + q * 32 + lane;
            if (ksplit == 1) {
                epilogue_tile(p, tbase, m, nb);
            } else {
                // this K range's fp32 accumulator row, as is
                float* prow = p.part + (static_cast<int64_t>(split) * p.M + m) * p.n_out;
                for (int cc = 0; cc < 8; ++cc) {
                    uint32_t v[32];
                    TmemAcc{tbase}.load(cc * 32, v);
                    const int64_t n0 = nb * 256 + cc * 32;
                    if (m >= p.M || n0 >= p.n_out) continue;
                    if (n0 + 32 <= p.n_out && (reinterpret_cast<uintptr_t>(prow + n0) & 15) == 0) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            __stcg(reinterpret_cast<float4*>(prow + n0 + j),
                                   make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                                               __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3])));
                    } else {
                        for (int j = 0; j < 32; ++j)
                            if (n0 + j < p.n_out) prow[n0 + j] = __uint_as_float(v[j]);
                    }
                }
            }
            fh3::tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (leader) fh3::mbar_arrive(&acc_empty[racc.idx]);
                else fh3::mbar_arrive_remote(acc_empty_leader + 8u * racc.idx);
            }
            racc.next<2>();
        }
    } else {
        // ------------------------------------------------------------ dequantisers (both CTAs)
        // Two groups of 4 warps over this CTA's 128 weight rows, one row per thread: group g
        // dequantises the K-64 stages with index % 2 == g (two stages in flight, a whole
        // 128-byte row of work per thread per stage).
        const int t = threadIdx.x - kDqWarp0 * 32;
        const int grp = t >> 7;
        const int i = t & 127;
        const uint32_t swz = static_cast<uint32_t>(i & 7);
        const uint32_t b_full_leader = fh3::mapa_shared(fh3::smem_u32(b_full), 0);
        Ring rr;
        uint32_t s_base = 0;  // index of the first K-64 stage of the current raw stage
        bool ok = true;
        for (int64_t u = pair; u < num_units && ok; u += npairs) {
            int64_t tile;
            int split, sb0, sb1;
            unit_of(u, tile, split, sb0, sb1);
            for (int rs = sb0; rs < sb1 && ok; ++rs, s_base += 4) {
                int w = 1;
                if (lane == 0) w = fh3::mbar_wait(&r_full[rr.idx], rr.phase, abort_flag, p.status);
                if (!(ok = __shfl_sync(0xffffffffu, w, 0) != 0)) break;
                const uint8_t* raw = smem + OFF_R + rr.idx * R_BYTES + i * fh3::kQ4KBytes;
                const uint4 hdr = *reinterpret_cast<const uint4*>(raw);
                for (int sub = grp; sub < 4 && ok; sub += 2) {
                    const uint32_t s = s_base + static_cast<uint32_t>(sub);
                    const uint32_t bi = s % SB;
                    const uint32_t bph = (s / SB) & 1u;
                    if (lane == 0) w = fh3::mbar_wait(&b_empty[bi], bph ^ 1u, abort_flag, p.status);
                    if (!(ok = __shfl_sync(0xffffffffu, w, 0) != 0)) break;
                    dequant_row_stage<0, 8>(raw, hdr, sub, smem + OFF_B + bi * B_BYTES + i * 128, swz);
                    fh3::fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        if (leader) fh3::mbar_arrive(&b_full[bi]);
                        else fh3::mbar_arrive_remote(b_full_leader + 8u * bi);
                    }
                }
                __syncwarp();
                if (ok && lane == 0) fh3::mbar_arrive(&r_empty[rr.idx]);
                rr.next<SR>();
            }
        }
    }

    fh3::tc_fence_before();
    __syncthreads();
    fh3::cluster_sync_all();  // the peer is done with our barriers and the pair's MMAs have retired
    if (warp == 1) {
        fh3::tc_fence_after();
        fh3::tmem_dealloc_pair(tmem_base, kTmemCols);
    }
}

// =============================================================================
// Two-pass large-M path.  Above kTwoPassRows token rows each weight tile would be
// dequantised once per 256-row M tile by the fused kernels (132 times a call at the
// DiT's 33,784 rows); instead dequant_q4k_bf16_kernel expands the call's weights once
// into a bf16 [N][K] matrix (the same bf16 values the fused dequantisers produce:
// fh3's fp32 weight rounded once), and gemm_bf16_pair_kernel runs the pair tile walk
// with both operands loaded by TMA (128-byte swizzle) -- no dequantiser warps, the
// tensor pipe fed at TMA rate.  MMA shapes and k order equal the fused kernel's, so
// the two paths give the same results.
// =============================================================================
constexpr int64_t kTwoPassRows = 2048;

// Q4_K -> bf16 [N][K], one warp per super-block step: lane l writes output chunk l of
// the super-block (weights 8l..8l+7, 16 bytes), so a warp's store is 512 contiguous
// bytes; every lane reads the 16-byte header (one broadcast request) and the 8 nibble
// bytes its chunk needs (the 32 lanes' reads cover the 128 nibble bytes).  A warp owns a
// contiguous run of super-blocks (row-major over (row, super-block)), walked with an
// incremental (row, super-block) position -- no division per step -- kExpandUnroll at a
// time, all their loads issued before any is converted.  Loads are streaming
// (evict-first): the weights are read once, and L2 is kept for the GEMM's tiles.
constexpr int kExpandUnroll = 4;
constexpr int kExpandThreads = 128;

__global__ void __launch_bounds__(kExpandThreads)
    dequant_q4k_bf16_kernel(const uint8_t* __restrict__ w, size_t rb, int64_t N, int K,
                            __nv_bfloat16* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int nblk = K / fh3::kQ4KBlock;
    const int64_t total = N * nblk;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int64_t begin = warp * total / nwarps, end = (warp + 1) * total / nwarps;
    if (begin >= end) return;
    const int sub = lane >> 3, j = lane & 7, hh = j >> 2;
    const int qoff = 16 + 32 * sub + 8 * (j & 3);  // this lane's 8 nibble bytes
    int64_t n = begin / nblk;
    int b = static_cast<int>(begin - n * nblk);
    const uint8_t* src = w + n * rb + static_cast<size_t>(b) * fh3::kQ4KBytes;
    __nv_bfloat16* dst = out + n * K + static_cast<int64_t>(b) * fh3::kQ4KBlock + lane * 8;
    for (int64_t idx = begin; idx < end; idx += kExpandUnroll) {
        const int cnt = end - idx < kExpandUnroll ? static_cast<int>(end - idx) : kExpandUnroll;
        uint4 hdr[kExpandUnroll];
        uint2 q[kExpandUnroll];
        __nv_bfloat16* d[kExpandUnroll];
#pragma unroll
        for (int u = 0; u < kExpandUnroll; ++u) {
            if (u < cnt) {
                hdr[u] = __ldcs(reinterpret_cast<const uint4*>(src));
                q[u] = __ldcs(reinterpret_cast<const uint2*>(src + qoff));
                d[u] = dst;
                // next super-block of the run (the next row after the last one)
                if (++b == nblk) {
                    b = 0;
                    src += rb - static_cast<size_t>(nblk - 1) * fh3::kQ4KBytes;
                    dst += fh3::kQ4KBlock;
                } else {
                    src += fh3::kQ4KBytes;
                    dst += fh3::kQ4KBlock;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kExpandUnroll; ++u) {
            if (u < cnt) {
                float sc, nm;
                q4k_sub_scales(hdr[u], 2 * sub + hh, sc, nm);
                *reinterpret_cast<uint4*>(d[u]) = q4k_chunk8_bf16(sc, nm, q[u].x, q[u].y, hh);
            }
        }
    }
}

namespace bfp {
constexpr int BN = 256;
constexpr int S = 6;                     // stages of (A, B) halves
constexpr int B_BYTES = 128 * BK * 2;    // this CTA's 128 weight rows
constexpr int STAGE = A_BYTES + B_BYTES; // 32 KB
constexpr int OFF_BAR = S * STAGE;
constexpr int kNumBars = 2 * S + 4 + 1;
constexpr int OFF_MISC = OFF_BAR + kNumBars * 8;
constexpr int SMEM_BYTES = OFF_MISC + 64 + 1024;
constexpr int kThreads = 32 * (kEpiWarp0 + kNumEpiWarps);  // producer, MMA, 4 epilogue warps
static_assert(STAGE % 1024 == 0 && SMEM_BYTES <= 232448, "shared memory layout");
}  // namespace bfp

__global__ void __launch_bounds__(bfp::kThreads, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const Params p) {
    using namespace bfp;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* full = bars;               // leader: 1 arrival + both CTAs' A and B bytes
    uint64_t* empty = full + S;          // both: 1 (leader's commit)
    uint64_t* acc_full = empty + S;      // both: 1 (leader's commit)
    uint64_t* acc_empty = acc_full + 2;  // leader: 2 x kNumEpiWarps
    uint64_t* drain = acc_empty + 2;     // both: 1 (leader's commit)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 8);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t cr = fh3::cluster_ctarank();
    const bool leader = cr == 0;
    const bool swiglu = p.epi == FH3CUDA_EPI_SWIGLU;
    const int64_t num_m = (p.M + 255) / 256;
    const int64_t num_n = swiglu ? (p.n_out + 127) / 128 : (p.N + BN - 1) / BN;
    const int64_t num_tiles = num_m * num_n;
    const int ksteps = static_cast<int>(p.K / BK);
    const int64_t pair = blockIdx.x >> 1;
    const int64_t npairs = gridDim.x >> 1;
    // the next kernel on this stream may be scheduled now: it can only take the SMs this
    // grid leaves as its CTAs finish, and it waits for the whole grid before it reads or
    // writes activations (griddepcontrol.wait)
    if (p.pdl) griddep_launch_dependents();

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            fh3::mbar_init(&full[i], 1);
            fh3::mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            fh3::mbar_init(&acc_full[i], 1);
            fh3::mbar_init(&acc_empty[i], 2 * kNumEpiWarps);
        }
        fh3::mbar_init(drain, 1);
        *abort_flag = 0;
        fh3::fence_mbar_init();
    }
    if (warp == 1) {
        fh3::tmem_alloc_pair(tmem_slot, kTmemCols);
        fh3::tmem_relinquish_pair();
    }
    if (warp == 0 && lane == 0) {
        fh3::tma_prefetch_desc(&tmA);
        fh3::tma_prefetch_desc(&tmB);
    }
    fh3::tc_fence_before();
    fh3::cluster_sync_all();
    fh3::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ A and B producer (both CTAs)
        if (lane == 0) {
            Ring r;
            uint32_t filled = 0, par = 0;
            bool ok = true;
            int ks0 = 0;  // k-steps of the first tile already issued
            if (p.pdl == 2 && pair < num_tiles) {
                // weights of the first stages before the previous kernel has finished; the
                // activations (that kernel's output) only after it
                int64_t mb, nb;
                tile_coords(pair, num_m, num_n, mb, nb);
                const int m0 = static_cast<int>(mb * 256 + cr * 128);
                const int wrow = swiglu ? static_cast<int>(cr ? p.n_out + nb * 128 : nb * 128)
                                        : static_cast<int>(nb * BN + cr * 128);
                ks0 = ksteps < S ? ksteps : S;  // fresh stages: their empty barriers pass at once
                for (int ks = 0; ks < ks0; ++ks) {
                    if (leader) fh3::mbar_arrive_expect_tx(&full[ks], 2 * STAGE);
                    const uint32_t bar = fh3::mapa_shared(fh3::smem_u32(&full[ks]), 0);
                    fh3::tma_load_2d_pair(smem + ks * STAGE + A_BYTES, &tmB, bar, ks * BK, wrow);
                }
                griddep_wait();
                for (int ks = 0; ks < ks0; ++ks) {
                    const uint32_t bar = fh3::mapa_shared(fh3::smem_u32(&full[ks]), 0);
                    fh3::tma_load_2d_pair(smem + ks * STAGE, &tmA, bar, ks * BK, m0);
                    filled |= 1u << r.idx;
                    par = (par & ~(1u << r.idx)) | (r.phase << r.idx);
                    r.next<S>();
                }
            } else if (p.pdl) {
                griddep_wait();
            }
            for (int64_t tile = pair; tile < num_tiles && ok; tile += npairs) {
                int64_t mb, nb;
                tile_coords(tile, num_m, num_n, mb, nb);
                const int m0 = static_cast<int>(mb * 256 + cr * 128);
                const int wrow = swiglu ? static_cast<int>(cr ? p.n_out + nb * 128 : nb * 128)
                                        : static_cast<int>(nb * BN + cr * 128);
                for (int ks = ks0; ks < ksteps && ok; ++ks) {
                    if (!(ok = fh3::mbar_wait(&empty[r.idx], r.phase ^ 1u, abort_flag, p.status))) break;
                    // both CTAs' A and B bytes are counted on the leader's full barrier
                    if (leader) fh3::mbar_arrive_expect_tx(&full[r.idx], 2 * STAGE);
                    const uint32_t bar = fh3::mapa_shared(fh3::smem_u32(&full[r.idx]), 0);
                    uint8_t* st = smem + r.idx * STAGE;
                    fh3::tma_load_2d_pair(st, &tmA, bar, ks * BK, m0);
                    fh3::tma_load_2d_pair(st + A_BYTES, &tmB, bar, ks * BK, wrow);
                    filled |= 1u << r.idx;
                    par = (par & ~(1u << r.idx)) | (r.phase << r.idx);
                    r.next<S>();
                }
                ks0 = 0;
            }
            if (!ok) {
                volatile int no_abort = 0;
                if (leader)
                    for (int i = 0; i < S; ++i)
                        if (filled & (1u << i)) fh3::mbar_wait_cluster(&full[i], (par >> i) & 1u, &no_abort, nullptr);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (leader)
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = fh3::idesc_bf16_f32(256, BN);
            Ring r, racc;
            bool ok = true;
            for (int64_t tile = pair; tile < num_tiles && ok; tile += npairs) {
                if (!(ok = fh3::mbar_wait(&acc_empty[racc.idx], racc.phase ^ 1u, abort_flag, p.status))) break;
                fh3::tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(racc.idx * BN);
                for (int ks = 0; ks < ksteps && ok; ++ks) {
                    if (!(ok = fh3::mbar_wait(&full[r.idx], r.phase, abort_flag, p.status))) break;
                    fh3::tc_fence_after();
                    const uint64_t ad = fh3::sdesc_sw128(fh3::smem_u32(smem + r.idx * STAGE));
                    const uint64_t bd = fh3::sdesc_sw128(fh3::smem_u32(smem + r.idx * STAGE + A_BYTES));
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        fh3::umma_f16_pair(d_tmem, ad + 2 * kk, bd + 2 * kk, idesc, (ks | kk) != 0 ? 1u : 0u);
                    fh3::umma_commit_pair(&empty[r.idx], 0x3);
                    r.next<S>();
                }
                if (ok) fh3::umma_commit_pair(&acc_full[racc.idx], 0x3);
                racc.next<2>();
            }
            fh3::umma_commit_pair(drain, 0x3);
        }
        if (lane == 0) {
            volatile int no_abort = 0;
            fh3::mbar_wait_cluster(drain, 0, &no_abort, nullptr);
        }
    } else {
        // ------------------------------------------------------------ epilogue (both CTAs)
        if (p.pdl) griddep_wait();  // y, bias and gate belong to us only once the previous kernel is done
        const int q = warp & 3;
        const uint32_t acc_empty_leader = fh3::mapa_shared(fh3::smem_u32(acc_empty), 0);
        Ring racc;
        for (int64_t tile = pair; tile < num_tiles; tile += npairs) {
            int64_t mb, nb;
            tile_coords(tile, num_m, num_n, mb, nb);
            int ok = 1;
            if (lane == 0) ok = fh3::mbar_wait(&acc_full[racc.idx], racc.phase, abort_flag, p.status);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            fh3::tc_fence_after();
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(racc.idx * BN);
            epilogue_tile(p, tbase, mb * 256 + cr * 128 + q * 32 + lane, nb);
            fh3::tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (leader) fh3::mbar_arrive(&acc_empty[racc.idx]);
                else fh3::mbar_arrive_remote(acc_empty_leader + 8u * racc.idx);
            }
            racc.next<2>();
        }
    }

    fh3::tc_fence_before();
    __syncthreads();
    fh3::cluster_sync_all();  // the peer is done with our barriers and the pair's MMAs have retired
    if (warp == 1) {
        fh3::tc_fence_after();
        fh3::tmem_dealloc_pair(tmem_base, kTmemCols);
    }
}

// y = epilogue(sum over s of part[s] (+ bias)), the split-K ranges added in order: F32, BF16
// or the gated residual h += gate * (sum + bias).  part is [ksplit][M][N] fp32.  VEC: four
// consecutive elements a thread with 16-byte accesses (N and ldy multiples of 4, y, bias
// and gate aligned), the same additions in the same order as the scalar form.
template <bool VEC>
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int ksplit, int64_t M, int64_t N,
                                     const float* __restrict__ bias, const float* __restrict__ gate, void* y,
                                     int64_t ldy, int epi) {
    // launched as a programmatic dependent of the GEMM: the partials are read after it
    griddep_launch_dependents();
    griddep_wait();
    const int64_t total = M * N;
    if constexpr (VEC) {
        const int64_t t4 = total / 4;
        for (int64_t e4 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e4 < t4;
             e4 += static_cast<int64_t>(gridDim.x) * blockDim.x) {
            const int64_t e = 4 * e4;
            float4 v = __ldcg(reinterpret_cast<const float4*>(part + e));
            for (int sp = 1; sp < ksplit; ++sp) {
                const float4 w = __ldcg(reinterpret_cast<const float4*>(part + sp * total + e));
                v.x += w.x;
                v.y += w.y;
                v.z += w.z;
                v.w += w.w;
            }
            const int64_t m = e / N, n = e - m * N;
            if (bias) {
                const float4 b = *reinterpret_cast<const float4*>(bias + n);
                v.x += b.x;
                v.y += b.y;
                v.z += b.z;
                v.w += b.w;
            }
            if (epi == FH3CUDA_EPI_BF16) {
                const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
                uint2 o;
                o.x = *reinterpret_cast<const uint32_t*>(&lo);
                o.y = *reinterpret_cast<const uint32_t*>(&hi);
                *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(y) + m * ldy + n) = o;
            } else {
                float4* yy = reinterpret_cast<float4*>(static_cast<float*>(y) + m * ldy + n);
                if (epi == FH3CUDA_EPI_RESID) {
                    const float4 g = *reinterpret_cast<const float4*>(gate + n);
                    float4 h = *yy;
                    h.x = fmaf(g.x, v.x, h.x);
                    h.y = fmaf(g.y, v.y, h.y);
                    h.z = fmaf(g.z, v.z, h.z);
                    h.w = fmaf(g.w, v.w, h.w);
                    *yy = h;
                } else {
                    *yy = v;
                }
            }
        }
    } else {
        for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
             e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
            float v = __ldcg(part + e);
            for (int sp = 1; sp < ksplit; ++sp) v += __ldcg(part + sp * total + e);
            const int64_t m = e / N, n = e - m * N;
            if (bias) v += bias[n];
            if (epi == FH3CUDA_EPI_BF16) {
                static_cast<__nv_bfloat16*>(y)[m * ldy + n] = __float2bfloat16_rn(v);
            } else {
                float* yy = static_cast<float*>(y) + m * ldy + n;
                *yy = epi == FH3CUDA_EPI_RESID ? fmaf(gate[n], v, *yy) : v;
            }
        }
    }
}

std::once_flag g_attr_once;
cudaError_t g_attr_err = cudaSuccess;
int g_pair_clusters = 0;  // co-resident CTA pairs on device 0's layout (queried once)
int g_bf_clusters = 0;    // the same for gemm_bf16_pair_kernel

bool use_pair_kernel(int64_t n_tok) {
    const char* e = getenv("FH3CUDA_GEMM_KERNEL");
    if (e && strcmp(e, "1sm") == 0) return false;
    if (e && (strcmp(e, "2sm") == 0 || strcmp(e, "two-pass") == 0)) return true;
    return n_tok > 128;
}

// kernel attributes and the co-resident cluster counts, once per process
int gemm_setup() {
    using namespace fh3host;
    std::call_once(g_attr_once, [] {
        g_attr_err = cudaFuncSetAttribute(gemm_q4k_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          one::SMEM_BYTES);
        if (g_attr_err == cudaSuccess)
            g_attr_err = cudaFuncSetAttribute(gemm_q4k_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              two::SMEM_BYTES);
        if (g_attr_err == cudaSuccess) {
            cudaLaunchConfig_t cfg = {};
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = 2;
            at[0].val.clusterDim.y = 1;
            at[0].val.clusterDim.z = 1;
            cfg.gridDim = dim3(2, 1, 1);
            cfg.blockDim = dim3(kThreadsPair, 1, 1);
            cfg.dynamicSmemBytes = two::SMEM_BYTES;
            cfg.attrs = at;
            cfg.numAttrs = 1;
            g_attr_err = cudaOccupancyMaxActiveClusters(&g_pair_clusters, gemm_q4k_pair_kernel, &cfg);
            if (g_attr_err == cudaSuccess)
                g_attr_err = cudaFuncSetAttribute(gemm_bf16_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  bfp::SMEM_BYTES);
            if (g_attr_err == cudaSuccess) {
                cfg.blockDim = dim3(bfp::kThreads, 1, 1);
                cfg.dynamicSmemBytes = bfp::SMEM_BYTES;
                g_attr_err = cudaOccupancyMaxActiveClusters(&g_bf_clusters, gemm_bf16_pair_kernel, &cfg);
            }
        }
    });
    return g_attr_err == cudaSuccess ? FH3_OK : check_cuda(g_attr_err, "gemm kernel attributes");
}

// checks shared by both GEMM entry points on the activations, output and epilogue
int check_gemm_args(const char* who, const void* x_bf16, int64_t ldx, const void* y, int64_t ldy, int64_t n_tok,
                    int64_t N, int64_t K, const float* gate, int epi) {
    using namespace fh3host;
    if (!x_bf16 || !y || n_tok <= 0 || K <= 0 || N <= 0) return set_error(FH3_E_INVALID, "%s: bad arguments", who);
    if (epi < FH3CUDA_EPI_F32 || epi > FH3CUDA_EPI_RESID)
        return set_error(FH3_E_INVALID, "%s: unknown epilogue %d", who, epi);
    if (epi == FH3CUDA_EPI_RESID && !gate) return set_error(FH3_E_INVALID, "%s: the residual epilogue needs a gate", who);
    if (epi == FH3CUDA_EPI_SWIGLU && (N % 2) != 0)
        return set_error(FH3_E_INVALID, "%s: SwiGLU needs an even number of rows", who);
    if (reinterpret_cast<uintptr_t>(x_bf16) & 15) return set_error(FH3_E_INVALID, "%s: x must be 16-byte aligned", who);
    if (n_tok > 0x7FFFFFFF || N > 0x7FFFFFFF)
        return set_error(FH3_E_INVALID, "%s: dimensions exceed the TMA coordinate range", who);
    const int64_t n_out = epi == FH3CUDA_EPI_SWIGLU ? N / 2 : N;
    if (ldy < n_out) return set_error(FH3_E_INVALID, "%s: ldy < output columns", who);
    if (ldx < K || (ldx % 8) != 0) return set_error(FH3_E_INVALID, "%s: ldx must be >= K and a multiple of 8", who);
    return FH3_OK;
}

// tensor map of the bf16 activations: n_tok rows of K, row stride ldx, 128 x 64 boxes
int map_activations(CUtensorMap* tmA, const void* x_bf16, int64_t ldx, int64_t n_tok, int64_t K) {
    using namespace fh3host;
    const cuuint64_t gdim[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(n_tok)};
    const cuuint64_t gstr[1] = {static_cast<cuuint64_t>(ldx) * 2};
    const cuuint32_t box[2] = {BK, 128};
    const cuuint32_t es[2] = {1, 1};
    CUresult r = encode_tiled(tmA, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x_bf16), gdim, gstr, box,
                              es, CU_TENSOR_MAP_SWIZZLE_128B);
    return r == CUDA_SUCCESS ? FH3_OK : set_error(FH3CUDA_E_CUDA, "cuTensorMapEncodeTiled(A) failed: %d", (int)r);
}

Params make_params(int64_t n_tok, int64_t N, int64_t K, int64_t ldy, const float* bias, const float* gate, void* y,
                   int epi, int* status) {
    Params p;
    p.M = n_tok;
    p.N = N;
    p.K = K;
    p.n_out = epi == FH3CUDA_EPI_SWIGLU ? N / 2 : N;
    p.ldy = ldy;
    p.bias = bias;
    p.gate = gate;
    p.y = y;
    p.epi = epi;
    p.status = status;
    return p;
}

// `at` holds two attributes: the pair cluster, and programmatic stream serialisation
// when `pdl` (the kernel may be scheduled while the previous kernel on s still runs)
cudaLaunchConfig_t pair_config(cudaLaunchAttribute* at, int64_t pairs, int threads, int smem, cudaStream_t s,
                               bool pdl = false) {
    cudaLaunchConfig_t cfg = {};
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 2 : 1;
    return cfg;
}

int64_t gemm_tiles(const Params& p, int64_t rows_per_tile) {
    const int64_t num_n = p.epi == FH3CUDA_EPI_SWIGLU ? (p.n_out + 127) / 128 : (p.N + 255) / 256;
    return ((p.M + rows_per_tile - 1) / rows_per_tile) * num_n;
}

// gemm_bf16_pair_kernel on a bf16 [N][K] weight matrix (K a multiple of 64, 16-byte aligned)
// (ldw: elements between weight rows, >= K; 0 means K)
int launch_bf16_pair(const CUtensorMap& tmA, const __nv_bfloat16* wb, const Params& p, cudaStream_t s,
                     int64_t ldw = 0) {
    using namespace fh3host;
    CUtensorMap tmB;
    const cuuint64_t gdim[2] = {static_cast<cuuint64_t>(p.K), static_cast<cuuint64_t>(p.N)};
    const cuuint64_t gstr[1] = {static_cast<cuuint64_t>(ldw > 0 ? ldw : p.K) * 2};
    const cuuint32_t box[2] = {BK, 128};
    const cuuint32_t es[2] = {1, 1};
    CUresult r = encode_tiled(&tmB, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<__nv_bfloat16*>(wb), gdim, gstr,
                              box, es, CU_TENSOR_MAP_SWIZZLE_128B);
    if (r != CUDA_SUCCESS) return set_error(FH3CUDA_E_CUDA, "cuTensorMapEncodeTiled(B) failed: %d", (int)r);
    const int64_t tiles = gemm_tiles(p, 256);
    const int64_t pairs = tiles < g_bf_clusters ? tiles : g_bf_clusters;
    // FH3CUDA_GEMM_PDL=0 launches without the programmatic dependency (the kernel then waits
    // for the previous kernel before it starts, and its griddepcontrol instructions do nothing)
    const char* pdl_env = getenv("FH3CUDA_GEMM_PDL");
    const bool pdl_on = !(pdl_env && strcmp(pdl_env, "0") == 0);
    cudaLaunchAttribute at[2];
    cudaLaunchConfig_t cfg = pair_config(at, pairs, bfp::kThreads, bfp::SMEM_BYTES, s, pdl_on && p.pdl != 0);
    return check_cuda(cudaLaunchKernelEx(&cfg, gemm_bf16_pair_kernel, tmA, tmB, p), "gemm_bf16_pair_kernel launch");
}

// dequant_q4k_bf16_kernel over the whole weight matrix
int launch_expand(fh3host::DevCtx* c, const Fh3CudaW* w, __nv_bfloat16* wb, cudaStream_t s) {
    using namespace fh3host;
    const int64_t work = w->out * (w->in / fh3::kQ4KBlock);
    const int64_t per_block = (kExpandThreads / 32) * kExpandUnroll;
    const int64_t cap = static_cast<int64_t>(ctx_sms(c)) * (2048 / kExpandThreads);
    const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((work + per_block - 1) / per_block, cap)));
    dequant_q4k_bf16_kernel<<<blocks, kExpandThreads, 0, s>>>(w->data, fh3cuda_row_bytes(FH3CUDA_TYPE_Q4_K, w->in),
                                                              w->out, static_cast<int>(w->in), wb);
    return check_cuda(cudaGetLastError(), "dequant_q4k_bf16_kernel launch");
}

}  // namespace

// kernel launches one fh3cuda_gemm_q4k_dev call of n_tok rows makes (the two-pass path
// adds the dequantisation pass); the same rule as the dispatch below
extern "C" int fh3cuda_gemm_launches(int64_t n_tok) {
    const char* gk = getenv("FH3CUDA_GEMM_KERNEL");
    const bool force_fused = gk && (strcmp(gk, "2sm") == 0 || strcmp(gk, "1sm") == 0);
    const bool force_two = gk && strcmp(gk, "two-pass") == 0;
    const bool two = use_pair_kernel(n_tok) && !force_fused && (force_two || n_tok >= kTwoPassRows);
    return two ? 2 : 1;
}

namespace fh3host {

// The body of fh3cuda_gemm_q4k_dev.  fused_only keeps every row count on the fused
// kernels (no bf16 weight copy, so no scratch) whatever FH3CUDA_GEMM_KERNEL says.
int gemm_q4k(const Fh3CudaW* w, const void* x_bf16, int64_t ldx, void* y, int64_t ldy, int64_t n_tok,
             const float* bias, const float* gate, int epi, void* stream, bool fused_only) {
    const char* who = "fh3cuda_gemm_q4k_dev";
    DevCtx* c = ctx();
    if (!c) return set_error(FH3CUDA_E_NODEV, "%s: call fh3cuda_init first", who);
    if (!w || !w->data) return set_error(FH3_E_INVALID, "%s: bad arguments", who);
    int rc = check_gemm_args(who, x_bf16, ldx, y, ldy, n_tok, w->out, w->in, gate, epi);
    if (rc) return rc;
    if (w->type != FH3CUDA_TYPE_Q4_K || (w->in % fh3::kQ4KBlock) != 0)
        return set_error(FH3_E_INVALID, "%s: Q4_K weights with in %% 256 == 0 required", who);
    if (reinterpret_cast<uintptr_t>(w->data) & 15)
        return set_error(FH3_E_INVALID, "%s: weights and x must be 16-byte aligned", who);
    if ((rc = gemm_setup())) return rc;

    bool pair = use_pair_kernel(n_tok) && g_pair_clusters > 0;
    {
        // up to 128 rows the one-SM kernel takes one CTA per 256 output columns; when that
        // would leave more than half the SMs idle, the pair kernel's split-K spreads the K
        // ranges over them instead (unless FH3CUDA_GEMM_KERNEL forces a kernel)
        const char* gk0 = getenv("FH3CUDA_GEMM_KERNEL");
        const char* sk0 = getenv("FH3CUDA_GEMM_SPLITK");
        const int64_t cols = epi == FH3CUDA_EPI_SWIGLU ? 0 : (w->out + 255) / 256;
        if (!pair && !gk0 && !(sk0 && strcmp(sk0, "0") == 0) && !fused_only && g_pair_clusters > 0 && cols > 0 &&
            ((n_tok + 127) / 128) * cols * 2 <= ctx_sms(c) && (w->in / fh3::kQ4KBlock) >= 4)
            pair = true;
    }
    const size_t rb = fh3cuda_row_bytes(FH3CUDA_TYPE_Q4_K, w->in);
    CUtensorMap tmA, tmW;
    if ((rc = map_activations(&tmA, x_bf16, ldx, n_tok, w->in))) return rc;
    {
        const cuuint64_t gdim[2] = {static_cast<cuuint64_t>(rb), static_cast<cuuint64_t>(w->out)};
        const cuuint64_t gstr[1] = {static_cast<cuuint64_t>(rb)};
        const cuuint32_t box[2] = {static_cast<cuuint32_t>(fh3::kQ4KBytes), 128};
        const cuuint32_t es[2] = {1, 1};
        CUresult r = encode_tiled(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(w->data), gdim,
                                  gstr, box, es, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (r != CUDA_SUCCESS) return set_error(FH3CUDA_E_CUDA, "cuTensorMapEncodeTiled(W) failed: %d", (int)r);
    }
    const Params p = make_params(n_tok, w->out, w->in, ldy, bias, gate, y, epi, ctx_status(c));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // large M: dequantise the weights once to bf16, then the TMA-fed bf16 pair kernel;
    // FH3CUDA_GEMM_KERNEL=2sm / 1sm force the fused kernels, =two-pass this path
    const char* gk = getenv("FH3CUDA_GEMM_KERNEL");
    const bool force_fused = gk && (strcmp(gk, "2sm") == 0 || strcmp(gk, "1sm") == 0);
    const bool force_two = gk && strcmp(gk, "two-pass") == 0;
    const bool two_pass = !fused_only && pair && g_bf_clusters > 0 && !force_fused &&
                          (force_two || n_tok >= kTwoPassRows);
    if (two_pass) {
        auto* wb = static_cast<__nv_bfloat16*>(scratch(c, 11, static_cast<size_t>(w->out) * w->in * 2, s));
        if (!wb) return FH3_E_NOMEM;
        if ((rc = launch_expand(c, w, wb, s))) return rc;
        Params pp = p;
        pp.pdl = 1;  // the GEMM's prologue overlaps the expansion; every load waits for it
        return launch_bf16_pair(tmA, wb, pp, s);
    }
    if (pair) {
        const int64_t tiles = gemm_tiles(p, 256);
        // Split-K when the tiles would keep at most half the CTA pairs busy (small M and N):
        // the tiles' super-blocks are cut into up to four ranges so that more pairs share the
        // dequantisation and the MMAs, and a reduction adds the ranges in order.  Not with
        // the SwiGLU epilogue, and not for fused_only callers (the partials are scratch).
        const char* sk_env = getenv("FH3CUDA_GEMM_SPLITK");
        const int nsb = static_cast<int>(w->in / fh3::kQ4KBlock);
        int ksplit = 1;
        if (!fused_only && epi != FH3CUDA_EPI_SWIGLU && !(sk_env && strcmp(sk_env, "0") == 0) && tiles * 2 <= g_pair_clusters)
            ksplit = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({g_pair_clusters / tiles, nsb / 2, 4})));
        Params pk = p;
        const char* pdl_env = getenv("FH3CUDA_GEMM_PDL");
        pk.pdl = (pdl_env && strcmp(pdl_env, "0") == 0) ? 0 : 1;
        if (ksplit > 1) {
            pk.ksplit = ksplit;
            pk.part = static_cast<float*>(scratch(c, 16, static_cast<size_t>(ksplit) * n_tok * p.n_out * 4, s));
            if (!pk.part) return FH3_E_NOMEM;
        }
        const int64_t units = tiles * pk.ksplit;
        const int64_t pairs = units < g_pair_clusters ? units : g_pair_clusters;
        cudaLaunchAttribute at[2];
        cudaLaunchConfig_t cfg = pair_config(at, pairs, kThreadsPair, two::SMEM_BYTES, s, pk.pdl != 0);
        rc = check_cuda(cudaLaunchKernelEx(&cfg, gemm_q4k_pair_kernel, tmA, tmW, pk), "gemm_q4k_pair_kernel launch");
        if (rc || pk.ksplit == 1) return rc;  // whole tiles: the epilogue wrote y
        const int64_t total = n_tok * p.n_out;
        auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
        const bool vec = p.n_out % 4 == 0 && ldy % 4 == 0 && al16(pk.part) && (!bias || al16(bias)) &&
                         (epi != FH3CUDA_EPI_RESID || al16(gate)) &&
                         (epi == FH3CUDA_EPI_BF16 ? (reinterpret_cast<uintptr_t>(y) & 7) == 0 : al16(y));
        const int64_t work = vec ? total / 4 : total;
        const int blocks = static_cast<int>(std::min<int64_t>((work + 255) / 256, static_cast<int64_t>(ctx_sms(c)) * 8));
        cudaLaunchConfig_t rcfg = {};
        rcfg.gridDim = dim3(static_cast<unsigned>(blocks), 1, 1);
        rcfg.blockDim = dim3(256, 1, 1);
        rcfg.stream = s;
        cudaLaunchAttribute ra[1];
        ra[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        ra[0].val.programmaticStreamSerializationAllowed = 1;
        rcfg.attrs = ra;
        rcfg.numAttrs = pk.pdl ? 1 : 0;
        return check_cuda(cudaLaunchKernelEx(&rcfg, vec ? splitk_reduce_kernel<true> : splitk_reduce_kernel<false>,
                                             static_cast<const float*>(pk.part), ksplit, static_cast<int64_t>(n_tok),
                                             p.n_out, bias, gate, static_cast<void*>(y), ldy, epi),
                          "splitk_reduce_kernel launch");
    }
    const int64_t tiles = gemm_tiles(p, 128);
    const int grid = static_cast<int>(tiles < ctx_sms(c) ? tiles : ctx_sms(c));
    gemm_q4k_tc_kernel<<<grid, kThreads, one::SMEM_BYTES, s>>>(tmA, tmW, p);
    return check_cuda(cudaGetLastError(), "gemm_q4k_tc_kernel launch");
}

}  // namespace fh3host

extern "C" int fh3cuda_gemm_q4k_dev(const Fh3CudaW* w, const void* x_bf16, int64_t ldx, void* y,
                                    int64_t ldy, int64_t n_tok, const float* bias, const float* gate,
                                    int epi, void* stream) {
    return fh3host::gemm_q4k(w, x_bf16, ldx, y, ldy, n_tok, bias, gate, epi, stream, false);
}

extern "C" int fh3cuda_q4k_to_bf16_dev(const Fh3CudaW* w, void* w_bf16, void* stream) {
    using namespace fh3host;
    const char* who = "fh3cuda_q4k_to_bf16_dev";
    DevCtx* c = ctx();
    if (!c) return set_error(FH3CUDA_E_NODEV, "%s: call fh3cuda_init first", who);
    if (!w || !w->data || !w_bf16 || w->in <= 0 || w->out <= 0)
        return set_error(FH3_E_INVALID, "%s: bad arguments", who);
    if (w->type != FH3CUDA_TYPE_Q4_K || (w->in % fh3::kQ4KBlock) != 0)
        return set_error(FH3_E_INVALID, "%s: Q4_K weights with in %% 256 == 0 required", who);
    if ((reinterpret_cast<uintptr_t>(w->data) & 15) || (reinterpret_cast<uintptr_t>(w_bf16) & 15))
        return set_error(FH3_E_INVALID, "%s: weights and output must be 16-byte aligned", who);
    return launch_expand(c, w, static_cast<__nv_bfloat16*>(w_bf16), static_cast<cudaStream_t>(stream));
}

namespace fh3host {

int gemm_bf16w(const void* w_bf16, int64_t ldw, int64_t out, int64_t in, const void* x_bf16, int64_t ldx, void* y,
               int64_t ldy, int64_t n_tok, const float* bias, const float* gate, int epi, int flags, cudaStream_t s) {
    const char* who = "fh3cuda_gemm_bf16w_dev";
    DevCtx* c = ctx();
    if (!c) return set_error(FH3CUDA_E_NODEV, "%s: call fh3cuda_init first", who);
    if (!w_bf16) return set_error(FH3_E_INVALID, "%s: bad arguments", who);
    int rc = check_gemm_args(who, x_bf16, ldx, y, ldy, n_tok, out, in, gate, epi);
    if (rc) return rc;
    if ((in % BK) != 0 || (reinterpret_cast<uintptr_t>(w_bf16) & 15) || ldw < in || (ldw % 8) != 0)
        return set_error(FH3_E_INVALID, "%s: in must be a multiple of 64, the weight rows 16-byte aligned", who);
    if ((rc = gemm_setup())) return rc;
    if (g_bf_clusters <= 0) return set_error(FH3CUDA_E_CUDA, "%s: the pair kernel cannot be resident", who);
    CUtensorMap tmA;
    if ((rc = map_activations(&tmA, x_bf16, ldx, n_tok, in))) return rc;
    Params p = make_params(n_tok, out, in, ldy, bias, gate, y, epi, ctx_status(c));
    p.pdl = (flags & FH3CUDA_GEMM_WEIGHTS_READY) ? 2 : 1;
    return launch_bf16_pair(tmA, static_cast<const __nv_bfloat16*>(w_bf16), p, s, ldw);
}

}  // namespace fh3host

extern "C" int fh3cuda_gemm_bf16w_dev(const void* w_bf16, int64_t out, int64_t in, const void* x_bf16, int64_t ldx,
                                      void* y, int64_t ldy, int64_t n_tok, const float* bias, const float* gate,
                                      int epi, int flags, void* stream) {
    return fh3host::gemm_bf16w(w_bf16, in, out, in, x_bf16, ldx, y, ldy, n_tok, bias, gate, epi, flags,
                               static_cast<cudaStream_t>(stream));
}
