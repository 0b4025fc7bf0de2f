// vsa_tc.cu -- the fine pass of video sparse attention (src/core/fh3_vsa.c:372-432) on
// the 5th-generation tensor cores, for bf16 operands with head_dim 128 and tiles of at
// most 64 tokens (the DiT's configuration).
//
// Kept key tiles are arbitrary token sets, so each call first lays q, k and v out in
// tile order: every tile's tokens become one contiguous run, padded to a multiple of 8
// rows (vsa_padoff_kernel, vsa_pidx_kernel), q and k rows are gathered into Qp / Kp
// (vsa_rows_kernel) and v transposed into VpT[h*128 + d][position] (vsa_vt_kernel).
// Then a kept tile is one TMA box of K rows and one of V^T columns.
//
// vsa_tc64_kernel: a CTA owns one query tile of one head in an M = 64 MMA and walks its
// kept tiles two a step, one softmax warpgroup per tile of the step, each with its own
// running max, sum and TMEM output, merged at the end; coarse * gate is added and rows
// are scattered back to token order.  The roles, barrier protocol and bounded waits
// follow attention_tc.cu.
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

// poff[i] = sum over tiles before i of count rounded up to 8; poff[nt] = the total.
// One CTA of 1024 threads.
__global__ void __launch_bounds__(1024) vsa_padoff_kernel(const int* __restrict__ toff, int nt,
                                                          int* __restrict__ poff) {
    __shared__ int part[1024];
    const int t = threadIdx.x;
    const int per = (nt + 1023) / 1024;
    const int i0 = min(nt, t * per), i1 = min(nt, i0 + per);
    int sum = 0;
    for (int i = i0; i < i1; ++i) sum += (toff[i + 1] - toff[i] + 7) & ~7;
    part[t] = sum;
    __syncthreads();
    if (t == 0) {
        int run = 0;
        for (int u = 0; u < 1024; ++u) {
            const int x = part[u];
            part[u] = run;
            run += x;
        }
        poff[nt] = run;
    }
    __syncthreads();
    int run = part[t];
    for (int i = i0; i < i1; ++i) {
        poff[i] = run;
        run += (toff[i + 1] - toff[i] + 7) & ~7;
    }
}

// pidx[padded position] = token, or -1 in a tile's padding.  grid (tiles), 64 threads.
__global__ void vsa_pidx_kernel(const int* __restrict__ perm, const int* __restrict__ toff,
                                const int* __restrict__ poff, int* __restrict__ pidx) {
    const int i = blockIdx.x;
    const int cnt = toff[i + 1] - toff[i], pcnt = poff[i + 1] - poff[i];
    for (int r = threadIdx.x; r < pcnt; r += blockDim.x) pidx[poff[i] + r] = r < cnt ? perm[toff[i] + r] : -1;
}

// Qp[p] = q[pidx[p]] and Kp[p] = k[pidx[p]] (whole rows of heads*128 bf16), zero in padding
__global__ void vsa_rows_kernel(const __nv_bfloat16* __restrict__ q, int64_t ldq, const __nv_bfloat16* __restrict__ k,
                                int64_t ldk, const int* __restrict__ pidx, int P, int width,
                                __nv_bfloat16* __restrict__ qp, __nv_bfloat16* __restrict__ kp) {
    const int cw = width / 8;  // 16-byte chunks a row
    const int64_t total = static_cast<int64_t>(P) * cw;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t p = e / cw;
        const int c = static_cast<int>(e - p * cw);
        const int t = pidx[p];
        uint4 a = make_uint4(0u, 0u, 0u, 0u), b = a;
        if (t >= 0) {
            a = *reinterpret_cast<const uint4*>(q + static_cast<int64_t>(t) * ldq + c * 8);
            b = *reinterpret_cast<const uint4*>(k + static_cast<int64_t>(t) * ldk + c * 8);
        }
        *reinterpret_cast<uint4*>(qp + p * width + c * 8) = a;
        *reinterpret_cast<uint4*>(kp + p * width + c * 8) = b;
    }
}

// VpT[c][p] = v[pidx[p]][c] (c = h*128 + d), zero in padding, in 64 x 64 tiles of 16-byte
// accesses (the entry point checks that v is 16-byte aligned and ldv a multiple of 8).
// grid (ceil(P/64), width/64), 256 threads.
__global__ void __launch_bounds__(256) vsa_vt_kernel(const __nv_bfloat16* __restrict__ v, int64_t ldv,
                                                       const int* __restrict__ pidx, int P,
                                                       __nv_bfloat16* __restrict__ vpt) {
    fh3::transpose64_bf16(v, ldv, [pidx](int p) { return pidx[p]; }, blockIdx.y * 64, blockIdx.x * 64, P, vpt, P);
}

}  // namespace

namespace {

constexpr int kVB = 128 * 64 * 2;            // [128][64] bf16 128-byte-swizzle block: 16 KB

// The query tile fills an M = 64 MMA once, so no tensor or softmax work goes to
// duplicated rows.  Kept tiles go two a step (chunk c pairs tile a = lst[2c] and tile
// b = lst[2c+1]; an odd last chunk repeats tile a with every key of the copy masked):
//   S_c = Q [K_a; K_b]^T   (M 64, N 128, K 128) into one of two TMEM score tiles
//   P_a, P_b               two softmax warpgroups, A on the keys of tile a, B on those of
//                          tile b, each with its own running max, sum and output
//   O_A += P_a V_a, O_B += P_b V_b   (M 64, N 128, K 64 each) accumulating in TMEM
// and at the end the two partial outputs of each query are merged (shared memory), with
// the lazy reference max of attention_tc.cu (raised only when a tile's row max exceeds it
// by more than 2^8, the row of O and its sum then rescaled once).  Query row m of an
// M = 64 MMA sits in TMEM lane (m % 16) + 32 (m / 16); the 16x32bx2 load shape gives
// lanes l and l + 16 of a warp the same row, 32 keys each.  K and V^T have rings of their own (three 32 KB stages
// each): a K stage is released as soon as its S MMAs complete and a V^T stage when its
// P V MMAs do, and the S and P V MMAs are issued by two threads, so a step's scores never
// wait behind the previous step's P.  Two tiles a step halve the barrier round trips of a
// one-tile step, and two warpgroups give each SM sub-partition two softmax warps.
constexpr int kV6Q = 64 * 64 * 2;            // [64][64] bf16 128-byte-swizzle block: 8 KB
constexpr int kV6S = 3;                      // K stages and V^T stages
constexpr int kV6K = 4 * kV6Q;               // K: 2 d-blocks x [tile a rows; tile b rows]: 32 KB
constexpr int kV6V = 2 * kVB;                // V^T: [128][64 keys of tile a] + [128][64 of tile b]: 32 KB
constexpr int V6_OFF_Q = 0;
constexpr int V6_OFF_K = V6_OFF_Q + 2 * kV6Q;
constexpr int V6_OFF_V = V6_OFF_K + kV6S * kV6K;
constexpr int V6_OFF_P = V6_OFF_V + kV6S * kV6V;  // P_a, P_b: [64][64 keys] each
constexpr int V6_OFF_BAR = V6_OFF_P + 2 * kV6Q;
// q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], s_empty[2], p_full[2],
// pv_done[2], drain_s, drain_o
constexpr int kV6Bars = 1 + 4 * kV6S + 8 + 2;
constexpr int V6_OFF_MISC = V6_OFF_BAR + kV6Bars * 8;
constexpr int kV6Smem = V6_OFF_MISC + 64 + 1024;
constexpr int kV6Threads = 11 * 32;    // TMA, S MMAs, softmax A x 4, softmax B x 4, P V MMAs
constexpr int kV6WarpPV = 10;
constexpr uint32_t kV6TmemCols = 512;  // S0 at 0, S1 at 128, O_A at 256, O_B at 384
constexpr uint32_t kV6TmemO = 256;
static_assert(kV6Smem <= 232448, "shared memory budget");
static_assert(V6_OFF_K % 1024 == 0 && V6_OFF_V % 1024 == 0 && V6_OFF_P % 1024 == 0, "swizzle alignment");
static_assert(64 * 130 * 4 <= kV6S * kV6K, "merge exchange fits the K ring");

// tcgen05.ld / st of shape 16x32bx2, 32 columns: threads 0..15 access lanes 0..15 of the
// warp's lane quarter at columns [c, c + 32), threads 16..31 the same lanes at columns
// [c + OFF, c + OFF + 32) (c = the column of taddr).  With the M = 64 layout (row m in lane
// (m % 16) + 32 (m / 16)) a warp's 32 threads then hold 16 rows, two threads a row.
template <int OFF>
__device__ __forceinline__ void tmem_ld16x2_32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x32bx2.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32], %33;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr), "n"(OFF));
}
template <int OFF>
__device__ __forceinline__ void tmem_st16x2_32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.16x32bx2.x32.b32 [%0], %1, {%2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33};"
        :: "r"(taddr), "n"(OFF), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

template <bool OUT_BF16>
__global__ void __launch_bounds__(kV6Threads, 1) vsa_tc64_kernel(
    const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
    const __grid_constant__ CUtensorMap tmVt, const int* __restrict__ perm, const int* __restrict__ toff,
    const int* __restrict__ poff, const int* __restrict__ sel, const int* __restrict__ selcnt, int nt,
    const __nv_bfloat16* __restrict__ gate, int64_t ldg, const float* __restrict__ outc, int heads,
    void* __restrict__ o, int64_t ldo, float scale_log2, int* status) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + V6_OFF_BAR);
    uint64_t* q_full = bar;
    uint64_t* k_full = bar + 1;
    uint64_t* k_empty = k_full + kV6S;
    uint64_t* v_full = k_empty + kV6S;
    uint64_t* v_empty = v_full + kV6S;
    uint64_t* s_full = v_empty + kV6S;
    uint64_t* s_empty = s_full + 2;
    uint64_t* p_full = s_empty + 2;   // [group]
    uint64_t* pv_done = p_full + 2;   // [group]
    uint64_t* drain_s = pv_done + 2;
    uint64_t* drain_o = drain_s + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + V6_OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + V6_OFF_MISC + 8);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i = blockIdx.x, h = blockIdx.y;
    const size_t rowi = static_cast<size_t>(h) * nt + i;
    const int* lst = sel + rowi * nt;
    const int L = selcnt[rowi];               // >= 1
    const int C = (L + 1) / 2;                // chunks
    const int qrows = toff[i + 1] - toff[i];  // <= 64

    if (threadIdx.x == 0) {
        fh3::mbar_init(q_full, 1);
        for (int s = 0; s < kV6S; ++s) {
            fh3::mbar_init(&k_full[s], 1);
            fh3::mbar_init(&k_empty[s], 1);
            fh3::mbar_init(&v_full[s], 1);
            fh3::mbar_init(&v_empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            fh3::mbar_init(&s_full[s], 1);
            fh3::mbar_init(&s_empty[s], 8);
            fh3::mbar_init(&p_full[s], 4);
            fh3::mbar_init(&pv_done[s], 1);
        }
        fh3::mbar_init(drain_s, 1);
        fh3::mbar_init(drain_o, 1);
        *abort_flag = 0;
        fh3::fence_mbar_init();
    }
    if (warp == 1) {
        fh3::tmem_alloc(tmem_slot, kV6TmemCols);
        fh3::tmem_relinquish();
    }
    fh3::tc_fence_before();
    __syncthreads();
    fh3::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        // K of chunk c goes out before V^T of chunk c - 1: a K stage frees up (S MMAs done)
        // before a V^T stage does (P V MMAs done)
        if (lane == 0) {
            uint32_t kfill = 0, kpar = 0, vfill = 0, vpar = 0;
            fh3::mbar_arrive_expect_tx(q_full, 2 * kV6Q);
            for (int c = 0; c < 2; ++c)
                fh3::tma_load_2d(smem + V6_OFF_Q + c * kV6Q, &tmQ, q_full, h * 128 + c * 64, poff[i]);
            bool ok = true;
            auto load_k = [&](int cc) {
                const int st = cc % kV6S;
                const uint32_t ph = static_cast<uint32_t>((cc / kV6S) & 1);
                if (!(ok = fh3::mbar_wait<true>(&k_empty[st], ph ^ 1u, abort_flag, status))) return;
                const int ya = poff[lst[2 * cc]], yb = poff[lst[min(2 * cc + 1, L - 1)]];
                uint8_t* sb = smem + V6_OFF_K + st * kV6K;
                fh3::mbar_arrive_expect_tx(&k_full[st], kV6K);
                for (int c = 0; c < 2; ++c) {
                    fh3::tma_load_2d(sb + c * 2 * kV6Q, &tmK, &k_full[st], h * 128 + c * 64, ya);
                    fh3::tma_load_2d(sb + c * 2 * kV6Q + kV6Q, &tmK, &k_full[st], h * 128 + c * 64, yb);
                }
                kfill |= 1u << st;
                kpar = (kpar & ~(1u << st)) | (ph << st);
            };
            auto load_v = [&](int cc) {
                const int st = cc % kV6S;
                const uint32_t ph = static_cast<uint32_t>((cc / kV6S) & 1);
                if (!(ok = fh3::mbar_wait<true>(&v_empty[st], ph ^ 1u, abort_flag, status))) return;
                const int ya = poff[lst[2 * cc]], yb = poff[lst[min(2 * cc + 1, L - 1)]];
                uint8_t* sb = smem + V6_OFF_V + st * kV6V;
                fh3::mbar_arrive_expect_tx(&v_full[st], kV6V);
                fh3::tma_load_2d(sb, &tmVt, &v_full[st], ya, h * 128);
                fh3::tma_load_2d(sb + kVB, &tmVt, &v_full[st], yb, h * 128);
                vfill |= 1u << st;
                vpar = (vpar & ~(1u << st)) | (ph << st);
            };
            for (int cc = 0; cc < C && ok; ++cc) {
                load_k(cc);
                if (ok && cc >= 1) load_v(cc - 1);
            }
            if (ok) load_v(C - 1);
            volatile int no_abort = 0;
            fh3::mbar_wait<true>(q_full, 0, &no_abort, nullptr);
            if (!ok)
                for (int s = 0; s < kV6S; ++s) {
                    if (kfill & (1u << s)) fh3::mbar_wait<true>(&k_full[s], (kpar >> s) & 1u, &no_abort, nullptr);
                    if (vfill & (1u << s)) fh3::mbar_wait<true>(&v_full[s], (vpar >> s) & 1u, &no_abort, nullptr);
                }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ S MMAs
        if (lane == 0) {
            constexpr uint32_t idesc = fh3::idesc_bf16_f32(64, 128);
            const uint32_t qa = fh3::smem_u32(smem + V6_OFF_Q);
            bool ok = fh3::mbar_wait<true>(q_full, 0, abort_flag, status);
            for (int cc = 0; cc < C && ok; ++cc) {
                const int b = cc & 1, st = cc % kV6S;
                if (!(ok = fh3::mbar_wait<true>(&k_full[st], (cc / kV6S) & 1, abort_flag, status))) break;
                if (!(ok = fh3::mbar_wait<true>(&s_empty[b], ((cc >> 1) & 1) ^ 1u, abort_flag, status))) break;
                fh3::tc_fence_after();
                const uint32_t ka = fh3::smem_u32(smem + V6_OFF_K + st * kV6K);
#pragma unroll
                for (int c = 0; c < 2; ++c)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        fh3::umma_f16(tmem + b * 128, fh3::sdesc_sw128(qa + c * kV6Q) + 2 * kk,
                                      fh3::sdesc_sw128(ka + c * 2 * kV6Q) + 2 * kk, idesc, (c | kk) != 0 ? 1u : 0u);
                fh3::umma_commit(&s_full[b]);
                fh3::umma_commit(&k_empty[st]);
            }
            fh3::umma_commit(drain_s);
            volatile int no_abort = 0;
            fh3::mbar_wait<true>(drain_s, 0, &no_abort, nullptr);
        }
    } else if (warp == kV6WarpPV) {
        // ------------------------------------------------------------ P V MMAs
        if (lane == 0) {
            constexpr uint32_t idesc = fh3::idesc_bf16_f32(64, 128);
            const uint32_t pa = fh3::smem_u32(smem + V6_OFF_P);
            bool ok = true;
            for (int cc = 0; cc < C && ok; ++cc) {
                const int st = cc % kV6S;
                if (!(ok = fh3::mbar_wait<true>(&v_full[st], (cc / kV6S) & 1, abort_flag, status))) break;
                const uint32_t va = fh3::smem_u32(smem + V6_OFF_V + st * kV6V);
                for (int g = 0; g < 2 && ok; ++g) {
                    if (!(ok = fh3::mbar_wait<true>(&p_full[g], cc & 1, abort_flag, status))) break;
                    fh3::tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        fh3::umma_f16(tmem + kV6TmemO + g * 128, fh3::sdesc_sw128(pa + g * kV6Q) + 2 * kk,
                                      fh3::sdesc_sw128(va + g * kVB) + 2 * kk, idesc, (cc | kk) != 0 ? 1u : 0u);
                    fh3::umma_commit(&pv_done[g]);
                }
                if (ok) fh3::umma_commit(&v_empty[st]);
            }
            fh3::umma_commit(drain_o);
            volatile int no_abort = 0;
            fh3::mbar_wait<true>(drain_o, 0, &no_abort, nullptr);
        }
    } else {
        // ------------------------------------------------------------ softmax, merge and epilogue (warps 2-9)
        // group g (warps 2-5: A, 6-9: B) takes tile g of every chunk; thread lane holds row
        // r = 16 qw + (lane & 15), keys 32 hf .. 32 hf + 31 of the tile and O_g columns
        // 64 hf .. 64 hf + 63; the row's two threads are lanes l and l ^ 16
        const int g = (warp - 2) >> 2;
        const int qw = warp & 3;
        const int hf = lane >> 4;
        const int r = qw * 16 + (lane & 15);
        const uint32_t trow = tmem + (static_cast<uint32_t>(qw * 32) << 16);
        const uint32_t tO = trow + kV6TmemO + g * 128;
        float m_ref = -INFINITY, lsum = 0.0f;  // lsum: this thread's part of the row sum
        bool ok = true;
        auto wait_warp = [&](uint64_t* bw, uint32_t parity) {
            int w = 1;
            if (lane == 0) w = fh3::mbar_wait<true>(bw, parity, abort_flag, status);
            return __shfl_sync(0xffffffffu, w, 0) != 0;
        };
        for (int cc = 0; cc < C && ok; ++cc) {
            const int b = cc & 1;
            const int li = 2 * cc + g;
            const int cnt = (li < L ? toff[lst[li] + 1] - toff[lst[li]] : 0) - 32 * hf;  // valid keys of this half
            if (!(ok = wait_warp(&s_full[b], (cc >> 1) & 1))) break;
            fh3::tc_fence_after();
            uint32_t v[32];
            tmem_ld16x2_32<32>(trow + b * 128 + g * 64, v);
            fh3::tmem_ld_wait();
            fh3::tmem_regs_ready(v);
            // the scores are in registers: the score tile may take chunk cc + 2
            fh3::tc_fence_before();
            __syncwarp();
            if (lane == 0) fh3::mbar_arrive(&s_empty[b]);
            float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            if (cnt >= 32) {  // a full half: no masking
#pragma unroll
                for (int e = 0; e < 32; e += 2)
                    mx4[(e >> 1) & 3] = max3f(mx4[(e >> 1) & 3], __uint_as_float(v[e]), __uint_as_float(v[e + 1]));
            } else {
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    if (e >= cnt) v[e] = __float_as_uint(-INFINITY);  // the next tile's keys, padding
                    mx4[e & 3] = fmaxf(mx4[e & 3], __uint_as_float(v[e]));
                }
            }
            float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16)) * scale_log2;  // the row's max over the tile
            const bool raise = mx > m_ref + 8.0f;  // the same in both threads of a row
            // P_g and O_g are free once the previous chunk's P_g V has completed
            if (cc > 0 && !(ok = wait_warp(&pv_done[g], (cc - 1) & 1))) break;
            if (cc > 0 && __any_sync(0xffffffffu, raise)) {
                fh3::tc_fence_after();
                const float a = raise ? exp2f(m_ref - mx) : 1.0f;  // 0 while this row's O is still empty
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t ov[32];
                    tmem_ld16x2_32<64>(tO + c * 32, ov);
                    fh3::tmem_ld_wait();
                    fh3::tmem_regs_ready(ov);
#pragma unroll
                    for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * a);
                    tmem_st16x2_32<64>(tO + c * 32, ov);
                }
                fh3::tmem_st_wait();
                lsum *= a;
            }
            if (raise) m_ref = mx;
            uint8_t* pb = smem + V6_OFF_P + g * kV6Q;
            // scale-and-shift and the row sum on packed fp32 pairs
            uint64_t rs2[2] = {fh3::f2_pack(0.0f, 0.0f), fh3::f2_pack(0.0f, 0.0f)};
            const float nm = m_ref == -INFINITY ? 0.0f : -m_ref;  // no key seen yet: every p is 0
            const uint64_t sc2 = fh3::f2_pack(scale_log2, scale_log2), nm2 = fh3::f2_pack(nm, nm);
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                uint32_t pk[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int e = 8 * t + 2 * u;
                    const float2 a = fh3::f2_unpack(
                        fh3::f2_fma(fh3::f2_pack(__uint_as_float(v[e]), __uint_as_float(v[e + 1])), sc2, nm2));
                    const float p0 = fh3::ex2_approx(a.x), p1 = fh3::ex2_approx(a.y);
                    rs2[u & 1] = fh3::f2_add(rs2[u & 1], fh3::f2_pack(p0, p1));
                    const __nv_bfloat162 pp = __floats2bfloat162_rn(p0, p1);
                    pk[u] = *reinterpret_cast<const uint32_t*>(&pp);
                }
                const int ch = hf * 4 + t;
                *reinterpret_cast<uint4*>(pb + r * 128 + ((ch ^ (r & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
            const float2 r0 = fh3::f2_unpack(rs2[0]), r1 = fh3::f2_unpack(rs2[1]);
            lsum += (r0.x + r0.y) + (r1.x + r1.y);
            fh3::tc_fence_before();
            fh3::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) fh3::mbar_arrive(&p_full[g]);
        }
        if (ok) ok = wait_warp(&pv_done[g], (C - 1) & 1);  // the last P_g V has landed
        lsum += __shfl_xor_sync(0xffffffffu, lsum, 16);      // the row's sum over group g's keys
        // merge: group B hands (m, l, O_B) to group A through the K ring, free once every
        // S MMA has completed (the last one before the last scores were read)
        float* xch = reinterpret_cast<float*>(smem + V6_OFF_K);  // [64][130]
        if (g == 1 && ok) {
            fh3::tc_fence_after();
            float* d = xch + r * 130;
            if (hf == 0) {
                d[0] = m_ref;
                d[1] = lsum;
            }
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
                uint32_t ov[32];
                tmem_ld16x2_32<64>(tO + c * 32, ov);  // O columns 64 hf + 32 c + e
                fh3::tmem_ld_wait();
                fh3::tmem_regs_ready(ov);
#pragma unroll
                for (int e = 0; e < 32; ++e) d[2 + 64 * hf + 32 * c + e] = __uint_as_float(ov[e]);
            }
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight softmax warps, on every path
        if (g == 0 && ok) {
            fh3::tc_fence_after();
            const float* x = xch + r * 130;
            const float mb = x[0], lb = x[1];
            const float m = fmaxf(m_ref, mb);  // finite: every chunk's first tile holds keys
            const float wa = exp2f(m_ref - m);
            const float wb = mb == -INFINITY ? 0.0f : exp2f(mb - m);
            const float inv = 1.0f / (lsum * wa + lb * wb);
            const bool store = r < qrows;
            const int64_t t = store ? perm[toff[i] + r] : 0;
            const float* cb = gate ? outc + (static_cast<size_t>(i) * heads + h) * 128 : nullptr;
            const int64_t col = static_cast<int64_t>(h) * 128;
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
                uint32_t ov[32];
                tmem_ld16x2_32<64>(tO + c * 32, ov);  // O columns 64 hf + 32 c + e
                fh3::tmem_ld_wait();
                fh3::tmem_regs_ready(ov);
                if (!store) continue;
#pragma unroll
                for (int d8 = 0; d8 < 32; d8 += 8) {
                    const int d = 64 * hf + 32 * c + d8;
                    float w8[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) w8[u] = (__uint_as_float(ov[d8 + u]) * wa + x[2 + d + u] * wb) * inv;
                    if (cb) {
                        const uint4 g4 = *reinterpret_cast<const uint4*>(gate + t * ldg + col + d);
                        const __nv_bfloat16* g8 = reinterpret_cast<const __nv_bfloat16*>(&g4);
#pragma unroll
                        for (int u = 0; u < 8; ++u) w8[u] += cb[d + u] * __bfloat162float(g8[u]);
                    }
                    if (OUT_BF16) {
                        uint32_t w[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const __nv_bfloat162 pp = __floats2bfloat162_rn(w8[2 * u], w8[2 * u + 1]);
                            w[u] = *reinterpret_cast<const uint32_t*>(&pp);
                        }
                        *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(o) + t * ldo + col + d) =
                            make_uint4(w[0], w[1], w[2], w[3]);
                    } else {
                        float* of = static_cast<float*>(o) + t * ldo + col + d;
                        *reinterpret_cast<float4*>(of) = make_float4(w8[0], w8[1], w8[2], w8[3]);
                        *reinterpret_cast<float4*>(of + 4) = make_float4(w8[4], w8[5], w8[6], w8[7]);
                    }
                }
            }
        }
    }

    fh3::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        fh3::tc_fence_after();
        fh3::tmem_dealloc(tmem, kV6TmemCols);
    }
}

}  // namespace

namespace fh3host {

// The fine pass + coarse * gate on tcgen05; tiles of at most 64 tokens, head_dim 128,
// bf16 q / k / v / gate.  The tile-stage arrays come from vsa.cu.
int vsa_fine_tc(const int* perm, const int* toff, const int* sel, const int* selcnt, int nt, int n,
                const __nv_bfloat16* q, int64_t ldq, const __nv_bfloat16* k, int64_t ldk, const __nv_bfloat16* v,
                int64_t ldv, const __nv_bfloat16* gate, int64_t ldg, const float* outc, int heads, void* o, bool o_bf16,
                int64_t ldo, cudaStream_t s) {
    DevCtx* c = ctx();
    const int width = heads * 128;
    const int64_t pmax = ((static_cast<int64_t>(n) + 7 * static_cast<int64_t>(nt)) + 31) & ~static_cast<int64_t>(31);
    auto al = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
    const size_t b_poff = al(static_cast<size_t>(nt + 1) * 4), b_pidx = al(static_cast<size_t>(pmax) * 4);
    const size_t b_act = al(static_cast<size_t>(pmax) * width * 2);
    uint8_t* base = static_cast<uint8_t*>(scratch(c, 13, b_poff + b_pidx + 3 * b_act, s));
    if (!base) return FH3_E_NOMEM;
    int* poff = reinterpret_cast<int*>(base);
    int* pidx = reinterpret_cast<int*>(base + b_poff);
    auto* qp = reinterpret_cast<__nv_bfloat16*>(base + b_poff + b_pidx);
    auto* kp = reinterpret_cast<__nv_bfloat16*>(base + b_poff + b_pidx + b_act);
    auto* vpt = reinterpret_cast<__nv_bfloat16*>(base + b_poff + b_pidx + 2 * b_act);
    int rc = check_cuda(cudaMemsetAsync(pidx, 0xFF, static_cast<size_t>(pmax) * 4, s), "vsa pidx memset");
    if (rc) return rc;
    vsa_padoff_kernel<<<1, 1024, 0, s>>>(toff, nt, poff);
    vsa_pidx_kernel<<<nt, 64, 0, s>>>(perm, toff, poff, pidx);
    const int64_t work = pmax * (width / 8);
    const int blocks = static_cast<int>(std::min<int64_t>((work + 255) / 256, static_cast<int64_t>(ctx_sms(c)) * 16));
    vsa_rows_kernel<<<blocks, 256, 0, s>>>(q, ldq, k, ldk, pidx, static_cast<int>(pmax), width, qp, kp);
    vsa_vt_kernel<<<dim3(static_cast<unsigned>((pmax + 63) / 64), static_cast<unsigned>(width / 64)), 256, 0, s>>>(
        v, ldv, pidx, static_cast<int>(pmax), vpt);
    rc = check_cuda(cudaGetLastError(), "vsa tile-order launches");
    if (rc) return rc;
    CUtensorMap tq, tk, tvt;
    const cuuint32_t es[2] = {1, 1};
    auto enc = [&](CUtensorMap* m, void* ptr, cuuint64_t w, cuuint64_t hgt, int64_t ld, cuuint32_t bw, cuuint32_t bh) {
        const cuuint64_t gdim[2] = {w, hgt};
        const cuuint64_t gstr[1] = {static_cast<cuuint64_t>(ld) * 2};
        const cuuint32_t box[2] = {bw, bh};
        return encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ptr, gdim, gstr, box, es,
                            CU_TENSOR_MAP_SWIZZLE_128B);
    };
    if (enc(&tq, qp, width, static_cast<cuuint64_t>(pmax), width, 64, 64) != CUDA_SUCCESS ||
        enc(&tk, kp, width, static_cast<cuuint64_t>(pmax), width, 64, 64) != CUDA_SUCCESS ||
        enc(&tvt, vpt, static_cast<cuuint64_t>(pmax), width, pmax, 64, 128) != CUDA_SUCCESS)
        return set_error(FH3CUDA_E_CUDA, "vsa: cuTensorMapEncodeTiled failed");
    static bool attr = false;
    if (!attr) {
        rc = check_cuda(cudaFuncSetAttribute(vsa_tc64_kernel<false>,
                                                      cudaFuncAttributeMaxDynamicSharedMemorySize, kV6Smem),
                                 "vsa_tc64 smem attribute");
        if (!rc) rc = check_cuda(cudaFuncSetAttribute(vsa_tc64_kernel<true>,
                                                      cudaFuncAttributeMaxDynamicSharedMemorySize, kV6Smem),
                                 "vsa_tc64 smem attribute");
        if (rc) return rc;
        attr = true;
    }
    const float scale_log2 = (1.0f / sqrtf(128.0f)) * 1.4426950408889634f;
    const dim3 grid(static_cast<unsigned>(nt), static_cast<unsigned>(heads));
    if (o_bf16)
        vsa_tc64_kernel<true><<<grid, kV6Threads, kV6Smem, s>>>(tq, tk, tvt, perm, toff, poff, sel, selcnt, nt, gate, ldg,
                                                               outc, heads, o, ldo, scale_log2, ctx_status(c));
    else
        vsa_tc64_kernel<false><<<grid, kV6Threads, kV6Smem, s>>>(tq, tk, tvt, perm, toff, poff, sel, selcnt, nt, gate,
                                                                ldg, outc, heads, o, ldo, scale_log2, ctx_status(c));
    return check_cuda(cudaGetLastError(), "vsa_tc64_kernel launch");
}

}  // namespace fh3host
