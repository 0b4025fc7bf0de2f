// gemv.cu -- Q4_K GEMV for small token counts (1 <= n_tok <= 16), fp32 on the
// CUDA cores.  Replaces fh3_matmul's small-M regime (src/core/fh3_ops.c:317-404),
// where the reference dequantises a 64-row tile per thread and runs AVX2 dots.
//
// One-shot split-K: a CTA owns R consecutive weight rows; its warps split the
// K range by groups of four super-blocks (warp w takes groups w, w+W, ...).  In a
// warp, lane group g (8 lanes) takes super-block 4*group + g and lane p of it the
// 16-byte nibble piece p (chunk p/2, half p%2): 16 weights of sub-block 2c (low
// nibbles) and 16 of 2c+1 (high nibbles).  Every lane issues the loads of all its
// rows before any arithmetic, so the whole CTA's weights are in flight at once
// (coalesced 16-byte loads; a warp instruction reads four 128-byte nibble runs).
//
// Arithmetic per weight: one byte_perm builds the fp32 pattern of 1 + q/128;
// packed fp32x2 instructions then give q/128 (exact subtraction), w = (128 d sc)
// (q/128) - dmin m (one rounding: the same fp32 value fh3's dequant_q4_k yields,
// since d*sc*q is exact) and the dot-product FMAs, two weights per instruction.
// Lane partial sums are reduced by shuffles, warp partials through shared memory
// in a fixed order, so the result is deterministic.
#include <cstdlib>
#include <cstring>

#include "common.cuh"

namespace {

constexpr int kMaxWarps = 16;

template <int M, int R>
__device__ __forceinline__ void dot_piece(const uint4 (&hdr)[R], const uint4 (&qv)[R], const float* __restrict__ xk,
                                          int64_t K, int c, uint64_t (&acc)[R][M]) {
    const uint64_t minus_one = fh3::f2_pack(-1.0f, -1.0f);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        // exact per-row scale (128*d*sc) and offset (-dmin*m) of sub-block 2c + half
        uint64_t s2[R], nm2[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            int sc, m;
            fh3::q4k_scale_min_words(hdr[r].y, hdr[r].z, hdr[r].w, 2 * c + half, sc, m);
            const float d = fh3::h2f_bits(hdr[r].x), dmin = fh3::h2f_bits(hdr[r].x >> 16);
            const float s = __fmul_rn(d, static_cast<float>(sc)) * 128.0f;
            const float nm = -__fmul_rn(dmin, static_cast<float>(m));
            s2[r] = fh3::f2_pack(s, s);
            nm2[r] = fh3::f2_pack(nm, nm);
        }
        // activations of this half-piece, loaded before the arithmetic (one L1 round trip
        // per half instead of one per 4 weights); M <= 4 keeps them in registers
        constexpr int XP = M <= 4 ? M : 1;
        float4 xpre[XP][4];
        if (M <= 4) {
#pragma unroll
            for (int t = 0; t < XP; ++t)
#pragma unroll
                for (int g = 0; g < 4; ++g)
                    xpre[t][g] = __ldg(reinterpret_cast<const float4*>(xk + half * 32 + t * K + 4 * g));
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            uint64_t w01[R], w23[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const uint32_t word = g == 0 ? qv[r].x : g == 1 ? qv[r].y : g == 2 ? qv[r].z : qv[r].w;
                const uint32_t v = ((half ? (word >> 4) : word) & 0x0F0F0F0Fu) | 0x80808080u;
                const uint64_t f01 = fh3::f2_pack(fh3::nib_f(v, fh3::kSel0), fh3::nib_f(v, fh3::kSel1));
                const uint64_t f23 = fh3::f2_pack(fh3::nib_f(v, fh3::kSel2), fh3::nib_f(v, fh3::kSel3));
                w01[r] = fh3::f2_fma(s2[r], fh3::f2_add(f01, minus_one), nm2[r]);
                w23[r] = fh3::f2_fma(s2[r], fh3::f2_add(f23, minus_one), nm2[r]);
            }
#pragma unroll
            for (int t = 0; t < M; ++t) {
                const float4 xv = M <= 4 ? xpre[M <= 4 ? t : 0][g]
                                         : __ldg(reinterpret_cast<const float4*>(xk + half * 32 + t * K + 4 * g));
                const uint64_t x01 = fh3::f2_pack(xv.x, xv.y);
                const uint64_t x23 = fh3::f2_pack(xv.z, xv.w);
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    acc[r][t] = fh3::f2_fma(x01, w01[r], acc[r][t]);
                    acc[r][t] = fh3::f2_fma(x23, w23[r], acc[r][t]);
                }
            }
        }
    }
}

template <int M, int R>
__global__ void __launch_bounds__(kMaxWarps * 32) gemv_q4k_kernel(
    const uint8_t* __restrict__ W, size_t row_bytes, int nblk, int64_t N, const float* __restrict__ x,
    int64_t K, const float* __restrict__ bias, float* __restrict__ y, int64_t ldy) {
    __shared__ float part[kMaxWarps][R * M];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * R;
    const int grp = lane >> 3;
    const int piece = lane & 7;
    const int c = piece >> 1;
    const int h = piece & 1;
    const int ngroups = (nblk + 3) / 4;

    const uint8_t* rowp[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int64_t n = (n0 + r < N) ? (n0 + r) : (N - 1);  // clamp loads; stores are masked
        rowp[r] = W + n * row_bytes;
    }
    uint64_t acc[R][M];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < M; ++t) acc[r][t] = 0;

    for (int gi = warp; gi < ngroups; gi += nwarps) {
        const int b = gi * 4 + grp;
        if (b < nblk) {
            uint4 hdr[R], qv[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const uint8_t* blk = rowp[r] + static_cast<size_t>(b) * fh3::kQ4KBytes;
                qv[r] = __ldg(reinterpret_cast<const uint4*>(blk + 16 + c * 32 + h * 16));
                hdr[r] = __ldg(reinterpret_cast<const uint4*>(blk));
            }
            dot_piece<M, R>(hdr, qv, x + static_cast<int64_t>(b) * fh3::kQ4KBlock + c * 64 + h * 16, K, c, acc);
        }
    }

    // lanes -> warp partial (shuffles), warps -> result (shared memory, fixed order)
#pragma unroll
    for (int r = 0; r < R; ++r) {
#pragma unroll
        for (int t = 0; t < M; ++t) {
            const float2 pr = fh3::f2_unpack(acc[r][t]);
            float v = pr.x + pr.y;
            v += __shfl_xor_sync(0xffffffffu, v, 16);
            v += __shfl_xor_sync(0xffffffffu, v, 8);
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            if (lane == 0) part[warp][r * M + t] = v;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < R * M; i += blockDim.x) {
        const int r = i / M, t = i - r * M;
        const int64_t n = n0 + r;
        if (n >= N) continue;
        float v = part[0][i];
        for (int w = 1; w < nwarps; ++w) v += part[w][i];
        if (bias) v += bias[n];
        y[t * ldy + n] = v;
    }
}

template <int M, int R>
int launch(const Fh3CudaW* w, const float* x, float* y, const float* bias, cudaStream_t s) {
    const int64_t N = w->out, K = w->in;
    const int nblk = static_cast<int>(K / fh3::kQ4KBlock);
    const int ngroups = (nblk + 3) / 4;
    const int warps = ngroups < kMaxWarps ? ngroups : kMaxWarps;
    const int64_t grid = (N + R - 1) / R;
    gemv_q4k_kernel<M, R><<<static_cast<unsigned>(grid), warps * 32, 0, s>>>(
        w->data, fh3cuda_row_bytes(FH3CUDA_TYPE_Q4_K, K), nblk, N, x, K, bias, y, N);
    return fh3host::check_cuda(cudaGetLastError(), "gemv_q4k_kernel launch");
}

}  // namespace

namespace fh3host {

int gemv_args_ok(const Fh3CudaW* w, const float* x, const float* y, int n_tok, const char* who) {
    if (!ctx()) return set_error(FH3CUDA_E_NODEV, "%s: call fh3cuda_init first", who);
    if (!w || !x || !y || !w->data || n_tok <= 0 || n_tok > 16 || w->in <= 0 || w->out <= 0)
        return set_error(FH3_E_INVALID, "%s: bad arguments (n_tok must be 1..16)", who);
    if (w->type != FH3CUDA_TYPE_Q4_K || (w->in % fh3::kQ4KBlock) != 0)
        return set_error(FH3_E_INVALID, "%s: Q4_K weights with in %% 256 == 0 required", who);
    if ((reinterpret_cast<uintptr_t>(w->data) & 15) || (reinterpret_cast<uintptr_t>(x) & 15))
        return set_error(FH3_E_INVALID, "%s: weights and x must be 16-byte aligned", who);
    return FH3_OK;
}

int gemv_fp32(const Fh3CudaW* w, const float* x, float* y, int n_tok, const float* bias, cudaStream_t s) {
    switch (n_tok) {
        case 1: return launch<1, 4>(w, x, y, bias, s);
        case 2: return launch<2, 4>(w, x, y, bias, s);
        case 3: return launch<3, 4>(w, x, y, bias, s);
        case 4: return launch<4, 4>(w, x, y, bias, s);
        case 5: return launch<5, 2>(w, x, y, bias, s);
        case 6: return launch<6, 2>(w, x, y, bias, s);
        case 7: return launch<7, 2>(w, x, y, bias, s);
        case 8: return launch<8, 2>(w, x, y, bias, s);
        case 9: return launch<9, 1>(w, x, y, bias, s);
        case 10: return launch<10, 1>(w, x, y, bias, s);
        case 11: return launch<11, 1>(w, x, y, bias, s);
        case 12: return launch<12, 1>(w, x, y, bias, s);
        case 13: return launch<13, 1>(w, x, y, bias, s);
        case 14: return launch<14, 1>(w, x, y, bias, s);
        case 15: return launch<15, 1>(w, x, y, bias, s);
        default: return launch<16, 1>(w, x, y, bias, s);
    }
}

}  // namespace fh3host

extern "C" int fh3cuda_gemv_q4k_dev(const Fh3CudaW* w, const float* x, float* y, int n_tok,
                                    const float* bias, void* stream) {
    using namespace fh3host;
    const int rc = gemv_args_ok(w, x, y, n_tok, "fh3cuda_gemv_q4k_dev");
    if (rc != FH3_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // FH3CUDA_GEMV_KERNEL=fp32 selects the CUDA-core kernel; the default is the
    // tensor-core kernel of gemv_mma.cu
    const char* kernel = getenv("FH3CUDA_GEMV_KERNEL");
    if (kernel && strcmp(kernel, "fp32") == 0) return gemv_fp32(w, x, y, n_tok, bias, s);
    return gemv_mma(w, x, y, n_tok, bias, s);
}
