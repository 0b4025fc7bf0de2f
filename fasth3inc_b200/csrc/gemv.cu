// gemv.cu -- Q4_K GEMV for small token counts (1 <= n_tok <= 16), fp32 on the
// CUDA cores.  Replaces fh3_matmul's small-M regime (src/core/fh3_ops.c:317-404),
// where the reference dequantises a 64-row tile per thread and runs AVX2 dots.
//
// Work split: a warp owns R consecutive weight rows and the whole K range.  Its
// 32 lanes form four groups of 8; group g walks super-blocks g, g+4, g+8, ... and
// lane p of a group owns the 16-byte nibble piece p of the block (chunk p/2, half
// p%2): 16 weights of sub-block 2c (low nibbles) and 16 of 2c+1 (high nibbles).
// One warp load instruction therefore reads four whole 128-byte nibble runs
// (coalesced 16-byte vectors) plus the four 16-byte headers.  Each iteration
// covers two super-blocks per lane with all their loads issued first, so a warp
// keeps 2 x R x 1 KiB of weights in flight.
//
// Arithmetic per weight: one byte_perm builds the fp32 pattern of 1 + q/128;
// packed fp32x2 instructions then give q/128 (exact subtraction), w = (128 d sc)
// (q/128) - dmin m (one rounding: the same fp32 value fh3's dequant_q4_k yields,
// since d*sc*q is exact) and the dot-product FMAs, two weights per instruction.
// Each (row, token) keeps an even/odd pair of fp32 accumulators; lanes are
// reduced with shuffles at the end.
#include "common.cuh"

namespace {

constexpr int kWarps = 4;

template <int M, int R>
__global__ void __launch_bounds__(kWarps * 32) gemv_q4k_kernel(
    const uint8_t* __restrict__ W, size_t row_bytes, int nblk, int64_t N, const float* __restrict__ x,
    int64_t K, const float* __restrict__ bias, float* __restrict__ y, int64_t ldy) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
    const int64_t n0 = warp * R;
    if (n0 >= N) return;
    const int grp = lane >> 3;       // which of the 4 super-blocks in flight
    const int piece = lane & 7;      // 16-byte nibble piece inside the block
    const int c = piece >> 1;        // 32-byte chunk: sub-blocks 2c (low) and 2c+1 (high)
    const int h = piece & 1;         // first or second 16 bytes of the chunk

    const uint8_t* rowp[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int64_t n = (n0 + r < N) ? (n0 + r) : (N - 1);  // clamp loads; stores are masked
        rowp[r] = W + n * row_bytes + 16 + c * 32 + h * 16;
    }

    const uint64_t minus_one = fh3::f2_pack(-1.0f, -1.0f);
    uint64_t acc[R][M];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < M; ++t) acc[r][t] = 0;

#pragma unroll 1
    for (int b0 = grp; b0 < nblk; b0 += 8) {
        // issue the loads of both super-blocks of this iteration first
        const bool two = b0 + 4 < nblk;
        uint4 hdr[2][R], qv[2][R];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int b = (u == 0 || two) ? b0 + 4 * u : b0;  // clamp: a duplicate load, never used
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const uint8_t* piecep = rowp[r] + static_cast<size_t>(b) * fh3::kQ4KBytes;
                qv[u][r] = __ldg(reinterpret_cast<const uint4*>(piecep));
                hdr[u][r] = __ldg(reinterpret_cast<const uint4*>(piecep - 16 - c * 32 - h * 16));
            }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            if (u == 1 && !two) break;
            const int b = b0 + 4 * u;
            const float* xk = x + static_cast<int64_t>(b) * fh3::kQ4KBlock + c * 64 + h * 16;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                // exact per-row scale (128*d*sc) and offset (-dmin*m) of sub-block 2c + half
                uint64_t s2[R], nm2[R];
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    int sc, m;
                    fh3::q4k_scale_min_words(hdr[u][r].y, hdr[u][r].z, hdr[u][r].w, 2 * c + half, sc, m);
                    const float d = fh3::h2f_bits(hdr[u][r].x), dmin = fh3::h2f_bits(hdr[u][r].x >> 16);
                    const float s = __fmul_rn(d, static_cast<float>(sc)) * 128.0f;
                    const float nm = -__fmul_rn(dmin, static_cast<float>(m));
                    s2[r] = fh3::f2_pack(s, s);
                    nm2[r] = fh3::f2_pack(nm, nm);
                }
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    uint64_t w01[R], w23[R];
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const uint32_t word = g == 0 ? qv[u][r].x : g == 1 ? qv[u][r].y : g == 2 ? qv[u][r].z : qv[u][r].w;
                        const uint32_t v = ((half ? (word >> 4) : word) & 0x0F0F0F0Fu) | 0x80808080u;
                        const uint64_t f01 = fh3::f2_pack(fh3::nib_f(v, fh3::kSel0), fh3::nib_f(v, fh3::kSel1));
                        const uint64_t f23 = fh3::f2_pack(fh3::nib_f(v, fh3::kSel2), fh3::nib_f(v, fh3::kSel3));
                        w01[r] = fh3::f2_fma(s2[r], fh3::f2_add(f01, minus_one), nm2[r]);
                        w23[r] = fh3::f2_fma(s2[r], fh3::f2_add(f23, minus_one), nm2[r]);
                    }
#pragma unroll
                    for (int t = 0; t < M; ++t) {
                        const float4 xv = __ldg(reinterpret_cast<const float4*>(xk + half * 32 + t * K + 4 * g));
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
    }

    // reduce over the 32 lanes; lane (r*M + t) % 32 stores (r, t)
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
            const int64_t n = n0 + r;
            if (lane == ((r * M + t) & 31) && n < N) {
                if (bias) v += bias[n];
                y[t * ldy + n] = v;
            }
        }
    }
}

template <int M, int R>
int launch(const Fh3CudaW* w, const float* x, float* y, const float* bias, cudaStream_t s) {
    const int64_t N = w->out, K = w->in;
    const int nblk = static_cast<int>(K / fh3::kQ4KBlock);
    const int64_t warps = (N + R - 1) / R;
    const int64_t grid = (warps + kWarps - 1) / kWarps;
    gemv_q4k_kernel<M, R><<<static_cast<unsigned>(grid), kWarps * 32, 0, s>>>(
        w->data, fh3cuda_row_bytes(FH3CUDA_TYPE_Q4_K, K), nblk, N, x, K, bias, y, N);
    return fh3host::check_cuda(cudaGetLastError(), "gemv_q4k_kernel launch");
}

}  // namespace

extern "C" int fh3cuda_gemv_q4k_dev(const Fh3CudaW* w, const float* x, float* y, int n_tok,
                                    const float* bias, void* stream) {
    using namespace fh3host;
    DevCtx* c = ctx();
    if (!c) return set_error(FH3CUDA_E_NODEV, "fh3cuda_gemv_q4k_dev: call fh3cuda_init first");
    if (!w || !x || !y || !w->data || n_tok <= 0 || n_tok > 16 || w->in <= 0 || w->out <= 0)
        return set_error(FH3_E_INVALID, "fh3cuda_gemv_q4k_dev: bad arguments (n_tok must be 1..16)");
    if (w->type != FH3CUDA_TYPE_Q4_K || (w->in % fh3::kQ4KBlock) != 0)
        return set_error(FH3_E_INVALID, "fh3cuda_gemv_q4k_dev: Q4_K weights with in %% 256 == 0 required");
    if ((reinterpret_cast<uintptr_t>(w->data) & 15) || (reinterpret_cast<uintptr_t>(x) & 15))
        return set_error(FH3_E_INVALID, "fh3cuda_gemv_q4k_dev: weights and x must be 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (n_tok) {
        case 1: return launch<1, 2>(w, x, y, bias, s);
        case 2: return launch<2, 2>(w, x, y, bias, s);
        case 3: return launch<3, 2>(w, x, y, bias, s);
        case 4: return launch<4, 2>(w, x, y, bias, s);
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
