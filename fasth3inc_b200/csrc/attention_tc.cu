// attention_tc.cu -- dense attention (fh3_attention, src/core/fh3_ops.c:587-695) on the
// 5th-generation tensor cores: head_dim 128, bf16 q/k/v, fp32 softmax and accumulation.
//
// A CTA owns 256 query rows of one head as two tiles of 128 (A and B) and walks the keys
// in tiles of 128; for each query tile:
//   S_j = Q K_j^T      tcgen05.mma (M 128, N 128, K 128) into a TMEM score tile
//   P_j = exp2(S_j c - m)   softmax warpgroup: thread i owns query row i (TMEM lane i),
//                      reads its 128 scores with tcgen05.ld and writes P_j back as bf16
//                      pairs into the first 64 columns of its score tile
//   O += P_j V_j       tcgen05.mma (M 128, N 128, K 128) with P taken from tensor memory,
//                      accumulating in a TMEM output tile across the key walk
// P_j is taken against a reference max that is raised only when a tile's row max exceeds
// it by more than 2^8 (then the row of O in TMEM and its sum are rescaled once), so O
// stays in tensor memory.  TMEM: S_A 0, S_B 128, O_A 256, O_B 384.  MMA issue order per
// key tile: PV_A(j), S_A(j+1), PV_B(j), S_B(j+1): the tensor cores run one group's
// products while the other group's softmax runs, and every S commit also covers the PV
// that read the same columns before.
// V is transposed once per call (vt[h][d][key]) so that both products take K-major
// operands, the layout TMA's 128-byte swizzle writes.
//
// Warps: 0 TMA producer (Q once, then K_j and V_j^T tiles, two stages), 1 TMEM owner and
// MMA issuer, 2-5 group A, 6-9 group B.  Every mbarrier wait is bounded (common.cuh); on
// a timeout the roles stop, the MMAs issued so far retire before TMEM is freed, and the
// producer lets its copies in flight land.  No TMA multicast.
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "common.cuh"

namespace {

// max of three floats in one instruction (sm_100)
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

constexpr int kTcHD = 128;              // head_dim
constexpr int kTcRows = 128;            // query rows a tile (two tiles a CTA)
constexpr int kTcKeys = 128;            // keys a tile
constexpr int kBlk = 128 * 64 * 2;      // one [128 rows][64 bf16] 128-byte-swizzle block: 16 KB
constexpr int kTile = 2 * kBlk;         // [128][128] bf16 operand: 32 KB
constexpr uint32_t kTmemCols = 512;    // S_A, S_B, O_A, O_B: 128 columns each

// vt[c][tok] = v[tok][c] (c = h*128 + d) in 64 x 64 tiles of 16-byte accesses (the entry
// point checks that v is 16-byte aligned and ldv a multiple of 8).  grid (ceil(n/64),
// heads*128/64), 256 threads.
__global__ void __launch_bounds__(256) vt_transpose_kernel(const __nv_bfloat16* __restrict__ v, int64_t ldv,
                                                             __nv_bfloat16* __restrict__ vt, int64_t ldt, int n) {
    fh3::transpose64_bf16(v, ldv, [](int p) { return p; }, blockIdx.y * 64, blockIdx.x * 64, n, vt, ldt);
}

constexpr int kPpRows = 256;
constexpr int PP_OFF_QA = 0;
constexpr int PP_OFF_QB = PP_OFF_QA + kTile;
constexpr int PP_OFF_KV = PP_OFF_QB + kTile;           // 2 stages x (K tile, V^T tile)
constexpr int PP_OFF_BAR = PP_OFF_KV + 2 * 2 * kTile;
// q_full, kv_full[2], kv_empty[2], s_full[2 groups], p_full[2 groups], o_full[2 groups], drain
constexpr int kPpBars = 1 + 2 + 2 + 2 + 2 + 2 + 1;
constexpr int PP_OFF_MISC = PP_OFF_BAR + kPpBars * 8;
constexpr int kPpSmem = PP_OFF_MISC + 64 + 1024;
constexpr int kPpThreads = 10 * 32;
static_assert(kPpSmem <= 232448, "shared memory budget");

struct PpBars {
    uint64_t *q_full, *kv_full, *kv_empty, *s_full, *p_full, *o_full, *drain;
};
__device__ __forceinline__ PpBars pp_bars(uint8_t* smem) {
    uint64_t* b = reinterpret_cast<uint64_t*>(smem + PP_OFF_BAR);
    PpBars x;
    x.q_full = b;
    x.kv_full = b + 1;
    x.kv_empty = b + 3;
    x.s_full = b + 5;  // [group]
    x.p_full = b + 7;  // [group]
    x.o_full = b + 9;  // [group]
    x.drain = b + 11;
    return x;
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16 with A in tensor memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

template <bool OUT_BF16>
__global__ void __launch_bounds__(kPpThreads, 1) attention_pp_kernel(
    const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
    const __grid_constant__ CUtensorMap tmVt, void* __restrict__ o, int64_t ldo, int n, float scale_log2,
    int* status) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const PpBars B = pp_bars(smem);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + PP_OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + PP_OFF_MISC + 8);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y;
    const int q0 = blockIdx.x * kPpRows;
    const int T = (n + kTcKeys - 1) / kTcKeys;

    if (threadIdx.x == 0) {
        fh3::mbar_init(B.q_full, 1);
        for (int i = 0; i < 2; ++i) {
            fh3::mbar_init(&B.kv_full[i], 1);
            fh3::mbar_init(&B.kv_empty[i], 1);
            fh3::mbar_init(&B.s_full[i], 1);
            fh3::mbar_init(&B.p_full[i], 4);
            fh3::mbar_init(&B.o_full[i], 1);
        }
        fh3::mbar_init(B.drain, 1);
        *abort_flag = 0;
        fh3::fence_mbar_init();
    }
    if (warp == 1) {
        fh3::tmem_alloc(tmem_slot, kTmemCols);
        fh3::tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        fh3::tma_prefetch_desc(&tmQ);
        fh3::tma_prefetch_desc(&tmK);
        fh3::tma_prefetch_desc(&tmVt);
    }
    fh3::tc_fence_before();
    __syncthreads();
    fh3::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t filled = 0, par = 0;
            fh3::mbar_arrive_expect_tx(B.q_full, 2 * kTile);
            for (int c = 0; c < 2; ++c) {
                fh3::tma_load_2d(smem + PP_OFF_QA + c * kBlk, &tmQ, B.q_full, h * kTcHD + c * 64, q0);
                fh3::tma_load_2d(smem + PP_OFF_QB + c * kBlk, &tmQ, B.q_full, h * kTcHD + c * 64, q0 + kTcRows);
            }
            bool ok = true;
            for (int j = 0; j < T && ok; ++j) {
                const int st = j & 1;
                if (!(ok = fh3::mbar_wait<true>(&B.kv_empty[st], ((j >> 1) & 1) ^ 1u, abort_flag, status))) break;
                uint8_t* kvb = smem + PP_OFF_KV + st * 2 * kTile;
                fh3::mbar_arrive_expect_tx(&B.kv_full[st], 2 * kTile);
                for (int c = 0; c < 2; ++c) {
                    fh3::tma_load_2d(kvb + c * kBlk, &tmK, &B.kv_full[st], h * kTcHD + c * 64, j * kTcKeys);
                    fh3::tma_load_2d(kvb + kTile + c * kBlk, &tmVt, &B.kv_full[st], j * kTcKeys + c * 64, h * kTcHD);
                }
                filled |= 1u << st;
                par = (par & ~(1u << st)) | (static_cast<uint32_t>((j >> 1) & 1) << st);
            }
            volatile int no_abort = 0;
            fh3::mbar_wait<true>(B.q_full, 0, &no_abort, nullptr);  // Q lands before the CTA can leave
            if (!ok)
                for (int i = 0; i < 2; ++i)
                    if (filled & (1u << i)) fh3::mbar_wait<true>(&B.kv_full[i], (par >> i) & 1u, &no_abort, nullptr);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = fh3::idesc_bf16_f32(128, 128);
            bool ok = fh3::mbar_wait<true>(B.q_full, 0, abort_flag, status);
            // S_g(j) = Q_g K_j^T into the group's score tile
            auto qk = [&](int g, int j) {
                const uint32_t qa = fh3::smem_u32(smem + (g ? PP_OFF_QB : PP_OFF_QA));
                const uint32_t ka = fh3::smem_u32(smem + PP_OFF_KV + (j & 1) * 2 * kTile);
#pragma unroll
                for (int c = 0; c < 2; ++c)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        fh3::umma_f16(tmem + 128 * g, fh3::sdesc_sw128(qa + c * kBlk) + 2 * kk,
                                      fh3::sdesc_sw128(ka + c * kBlk) + 2 * kk, idesc, (c | kk) != 0 ? 1u : 0u);
                fh3::umma_commit(&B.s_full[g]);
            };
            // O_g += P_g(j) V_j, P_g in the first 64 columns of the score tile (bf16 pairs)
            auto pv = [&](int g, int j) {
                const uint32_t va = fh3::smem_u32(smem + PP_OFF_KV + (j & 1) * 2 * kTile + kTile);
#pragma unroll
                for (int c = 0; c < 2; ++c)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        umma_f16_ts(tmem + 256 + 128 * g, tmem + 128 * g + 32 * c + 8 * kk,
                                    fh3::sdesc_sw128(va + c * kBlk) + 2 * kk, idesc, (j | c | kk) != 0 ? 1u : 0u);
            };
            if (ok && (ok = fh3::mbar_wait<true>(&B.kv_full[0], 0, abort_flag, status))) {
                fh3::tc_fence_after();
                qk(0, 0);
                qk(1, 0);
            }
            for (int j = 0; j < T && ok; ++j) {
                const bool more = j + 1 < T;
                if (more && !(ok = fh3::mbar_wait<true>(&B.kv_full[(j + 1) & 1], ((j + 1) >> 1) & 1, abort_flag,
                                                        status)))
                    break;
                for (int g = 0; g < 2 && ok; ++g) {
                    if (!(ok = fh3::mbar_wait<true>(&B.p_full[g], j & 1, abort_flag, status))) break;
                    fh3::tc_fence_after();
                    pv(g, j);
                    if (g == 1) fh3::umma_commit(&B.kv_empty[j & 1]);  // K_j and V_j are both consumed
                    if (more) qk(g, j + 1);
                    else fh3::umma_commit(&B.o_full[g]);
                }
            }
            fh3::umma_commit(B.drain);  // every MMA issued retires before TMEM is freed
            volatile int no_abort = 0;
            fh3::mbar_wait<true>(B.drain, 0, &no_abort, nullptr);
        }
    } else {
        // ------------------------------------------------------------ softmax and epilogue
        // group g = (warp - 2) / 4 owns tile g; P_j = 2^(s - m_ref) against a reference max
        // raised only when a tile's max exceeds it by more than 2^8 (then the row of O in
        // TMEM and the row sum are rescaled once).  S_g(j) is committed after PV_g(j-1), so
        // when it is visible the previous P has been consumed and O_g is up to date.
        const int g = (warp - 2) >> 2;
        const int qw = warp & 3;  // TMEM lanes 32*qw .. 32*qw+31 belong to this warp
        const int r = qw * 32 + lane;
        const uint32_t trow = tmem + (static_cast<uint32_t>(qw * 32) << 16);
        const uint32_t ts = trow + 128 * g, to = trow + 256 + 128 * g;
        float m_ref = -INFINITY, l = 0.0f;
        bool ok = true;
        auto wait_warp = [&](uint64_t* bar, uint32_t parity) {
            int w = 1;
            if (lane == 0) w = fh3::mbar_wait<true>(bar, parity, abort_flag, status);
            return __shfl_sync(0xffffffffu, w, 0) != 0;
        };
        for (int j = 0; j < T && ok; ++j) {
            if (!(ok = wait_warp(&B.s_full[g], j & 1))) break;
            fh3::tc_fence_after();
            const int kb = j * kTcKeys;
            const bool tail = kb + kTcKeys > n;  // keys past n only in the last tile
            // pass 1: row max of the raw scores (the scale is positive), 64 columns at a time
            float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                uint32_t v[2][32];
#pragma unroll
                for (int c = 0; c < 2; ++c) fh3::tmem_ld32(ts + 64 * hf + c * 32, v[c]);
                fh3::tmem_ld_wait();
#pragma unroll
                for (int c = 0; c < 2; ++c) fh3::tmem_regs_ready(v[c]);
                if (!tail) {
#pragma unroll
                    for (int c = 0; c < 2; ++c)
#pragma unroll
                        for (int e = 0; e < 32; e += 2)
                            mx4[(e >> 1) & 3] = max3f(mx4[(e >> 1) & 3], __uint_as_float(v[c][e]),
                                                      __uint_as_float(v[c][e + 1]));
                } else {
#pragma unroll
                    for (int c = 0; c < 2; ++c)
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            if (kb + 64 * hf + c * 32 + e < n) mx4[e & 3] = fmaxf(mx4[e & 3], __uint_as_float(v[c][e]));
                }
            }
            const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * scale_log2;
            const bool raise = mx > m_ref + 8.0f;  // always true on the first tile
            if (j > 0 && __any_sync(0xffffffffu, raise)) {
                // PV_g(j-1) has landed (S_g(j) was committed after it)
                const float a = raise ? exp2f(m_ref - mx) : 1.0f;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t ov[32];
                    fh3::tmem_ld32(to + c * 32, ov);
                    fh3::tmem_ld_wait();
                    fh3::tmem_regs_ready(ov);
#pragma unroll
                    for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * a);
                    fh3::tmem_st32(to + c * 32, ov);
                }
                l *= a;
            }
            if (raise) m_ref = mx;
            // pass 2: P as bf16 pairs over the consumed columns (keys 64hf.. -> columns 32hf..);
            // the scale-and-shift and the row sum run on packed fp32 pairs
            uint64_t rs2[2] = {fh3::f2_pack(0.0f, 0.0f), fh3::f2_pack(0.0f, 0.0f)};
            const float nm = -m_ref;
            const uint64_t sc2 = fh3::f2_pack(scale_log2, scale_log2), nm2 = fh3::f2_pack(nm, nm);
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                uint32_t v[2][32];
#pragma unroll
                for (int c = 0; c < 2; ++c) fh3::tmem_ld32(ts + 64 * hf + c * 32, v[c]);
                fh3::tmem_ld_wait();
#pragma unroll
                for (int c = 0; c < 2; ++c) fh3::tmem_regs_ready(v[c]);
                if (tail) {  // keys past n weigh zero
#pragma unroll
                    for (int c = 0; c < 2; ++c)
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            if (kb + 64 * hf + 32 * c + e >= n) v[c][e] = __float_as_uint(-INFINITY);
                }
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t pk[16];  // keys 64hf + 32c .. +31 -> columns 32hf + 16c ..
#pragma unroll
                    for (int u = 0; u < 16; ++u) {
                        const float2 a = fh3::f2_unpack(fh3::f2_fma(
                            fh3::f2_pack(__uint_as_float(v[c][2 * u]), __uint_as_float(v[c][2 * u + 1])), sc2, nm2));
                        const float p0 = fh3::ex2_approx(a.x), p1 = fh3::ex2_approx(a.y);
                        rs2[u & 1] = fh3::f2_add(rs2[u & 1], fh3::f2_pack(p0, p1));
                        const __nv_bfloat162 pp = __floats2bfloat162_rn(p0, p1);
                        pk[u] = *reinterpret_cast<const uint32_t*>(&pp);
                    }
                    fh3::tmem_st16(ts + 32 * hf + 16 * c, pk);
                }
            }
            fh3::tmem_st_wait();
            fh3::tc_fence_before();  // this warp's TMEM reads and writes are complete
            __syncwarp();
            if (lane == 0) fh3::mbar_arrive(&B.p_full[g]);
            const float2 r0 = fh3::f2_unpack(rs2[0]), r1 = fh3::f2_unpack(rs2[1]);
            l += (r0.x + r0.y) + (r1.x + r1.y);
        }
        if (ok) ok = wait_warp(&B.o_full[g], 0);  // the last PV has landed
        if (ok) {
            fh3::tc_fence_after();
            const int row = q0 + kTcRows * g + r;
            uint32_t ov[4][32];
#pragma unroll
            for (int c = 0; c < 4; ++c) fh3::tmem_ld32(to + c * 32, ov[c]);
            fh3::tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < 4; ++c) fh3::tmem_regs_ready(ov[c]);
            if (row < n) {
                const float inv = 1.0f / l;
                const int64_t base = static_cast<int64_t>(row) * ldo + static_cast<int64_t>(h) * kTcHD;
                if (OUT_BF16) {
                    __nv_bfloat16* ob = static_cast<__nv_bfloat16*>(o) + base;
#pragma unroll
                    for (int d = 0; d < kTcHD; d += 8) {
                        uint32_t w[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int e = d + 2 * u;
                            const __nv_bfloat162 pp = __floats2bfloat162_rn(__uint_as_float(ov[e >> 5][e & 31]) * inv,
                                                                            __uint_as_float(ov[(e + 1) >> 5][(e + 1) & 31]) * inv);
                            w[u] = *reinterpret_cast<const uint32_t*>(&pp);
                        }
                        *reinterpret_cast<uint4*>(ob + d) = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                } else {
                    float* of = static_cast<float*>(o) + base;
#pragma unroll
                    for (int d = 0; d < kTcHD; d += 4)
                        *reinterpret_cast<float4*>(of + d) = make_float4(
                            __uint_as_float(ov[d >> 5][d & 31]) * inv, __uint_as_float(ov[d >> 5][(d & 31) + 1]) * inv,
                            __uint_as_float(ov[d >> 5][(d & 31) + 2]) * inv, __uint_as_float(ov[d >> 5][(d & 31) + 3]) * inv);
                }
            }
        }
    }

    fh3::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        fh3::tc_fence_after();
        fh3::tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace

namespace fh3host {

// Dense attention on tcgen05 (head_dim 128); arguments validated by fh3cuda_attention_dev.
int attention_tc(const __nv_bfloat16* q, int64_t ldq, const __nv_bfloat16* k, int64_t ldk, const __nv_bfloat16* v,
                 int64_t ldv, void* o, bool o_bf16, int64_t ldo, int n, int heads, cudaStream_t s) {
    DevCtx* c = ctx();
    const int64_t npad = (static_cast<int64_t>(n) + 7) & ~static_cast<int64_t>(7);
    const int64_t rows = static_cast<int64_t>(heads) * kTcHD;
    auto* vt = static_cast<__nv_bfloat16*>(scratch(c, 12, static_cast<size_t>(rows) * npad * 2, s));
    if (!vt) return FH3_E_NOMEM;
    vt_transpose_kernel<<<dim3(static_cast<unsigned>((n + 63) / 64), static_cast<unsigned>(heads * 2)), 256, 0, s>>>(
        v, ldv, vt, npad, n);
    int rc = check_cuda(cudaGetLastError(), "vt_transpose_kernel launch");
    if (rc) return rc;
    CUtensorMap tq, tk, tvt;
    const cuuint32_t box[2] = {64, 128};
    const cuuint32_t es[2] = {1, 1};
    auto enc = [&](CUtensorMap* m, const void* base, cuuint64_t w, cuuint64_t h, int64_t ld) {
        const cuuint64_t gdim[2] = {w, h};
        const cuuint64_t gstr[1] = {static_cast<cuuint64_t>(ld) * 2};
        return encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), gdim, gstr, box, es,
                            CU_TENSOR_MAP_SWIZZLE_128B);
    };
    if (enc(&tq, q, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(n), ldq) != CUDA_SUCCESS ||
        enc(&tk, k, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(n), ldk) != CUDA_SUCCESS ||
        enc(&tvt, vt, static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(rows), npad) != CUDA_SUCCESS)
        return set_error(FH3CUDA_E_CUDA, "attention: cuTensorMapEncodeTiled failed");
    const float scale_log2 = (1.0f / sqrtf(static_cast<float>(kTcHD))) * 1.4426950408889634f;
    static bool attr = false;
    if (!attr) {
        rc = check_cuda(cudaFuncSetAttribute(attention_pp_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kPpSmem),
                        "attention_pp smem attribute");
        if (!rc) rc = check_cuda(cudaFuncSetAttribute(attention_pp_kernel<true>,
                                                      cudaFuncAttributeMaxDynamicSharedMemorySize, kPpSmem),
                                 "attention_pp smem attribute");
        if (rc) return rc;
        attr = true;
    }
    const dim3 grid(static_cast<unsigned>((n + kPpRows - 1) / kPpRows), static_cast<unsigned>(heads));
    if (o_bf16)
        attention_pp_kernel<true><<<grid, kPpThreads, kPpSmem, s>>>(tq, tk, tvt, o, ldo, n, scale_log2, ctx_status(c));
    else
        attention_pp_kernel<false><<<grid, kPpThreads, kPpSmem, s>>>(tq, tk, tvt, o, ldo, n, scale_log2, ctx_status(c));
    return check_cuda(cudaGetLastError(), "attention_pp_kernel launch");
}

}  // namespace fh3host
