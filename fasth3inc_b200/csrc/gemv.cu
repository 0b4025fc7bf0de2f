// gemv.cu -- Q4_K GEMV for small token counts (1 <= n_tok <= 16), fp32 on the
// CUDA cores.  Replaces fh3_matmul's small-M regime (src/core/fh3_ops.c:317-404),
// where the reference dequantises a 64-row tile per thread and runs AVX2 dots.
//
// Work split: a warp owns R consecutive weight rows and the whole K range.  Its
// 32 lanes form four groups of 8; group g walks super-blocks g, g+4, g+8, ...
// and lane p of a group owns the 16-byte nibble piece p of the block (chunk
// p/2, half p%2), i.e. 16 weights of sub-block 2c (low nibbles) and 16 of
// 2c+1 (high nibbles).  So one warp load instruction reads four whole 128-byte
// nibble runs (coalesced 16-byte vectors) plus the four 16-byte headers.
//
// Per weight: one byte_perm builds the fp32 pattern of 1 + q/128, one exact
// subtraction gives q/128, and one FMA with the exact scale 128*d*sc and the
// exact offset -dmin*m yields w = dl*q - ml with a single rounding -- the same
// fp32 value fh3's dequant_q4_k produces (dl*q is exact there, too).  The dot
// products then run as plain fp32 FMAs against x, one accumulator per
// (row, token); lanes are reduced with shuffles at the end.
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
        rowp[r] = W + n * row_bytes;
    }

    float acc[R][M];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < M; ++t) acc[r][t] = 0.0f;

#pragma unroll 1
    for (int b = grp; b < nblk; b += 4) {
        uint4 hdr[R], qv[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const uint8_t* blk = rowp[r] + static_cast<size_t>(b) * fh3::kQ4KBytes;
            hdr[r] = __ldg(reinterpret_cast<const uint4*>(blk));
            qv[r] = __ldg(reinterpret_cast<const uint4*>(blk + 16 + c * 32 + h * 16));
        }
        const int64_t kb = static_cast<int64_t>(b) * fh3::kQ4KBlock + c * 64 + h * 16;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            // exact per-row scale (128*d*sc) and offset (-dmin*m) of this sub-block
            float s[R], nm[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                int sc, m;
                fh3::q4k_scale_min_words(hdr[r].y, hdr[r].z, hdr[r].w, 2 * c + half, sc, m);
                const float d = fh3::h2f_bits(hdr[r].x), dmin = fh3::h2f_bits(hdr[r].x >> 16);
                s[r] = __fmul_rn(d, static_cast<float>(sc)) * 128.0f;
                nm[r] = -__fmul_rn(dmin, static_cast<float>(m));
            }
            const float* xk = x + kb + half * 32;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                float w[R][4];
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const uint32_t word = g == 0 ? qv[r].x : g == 1 ? qv[r].y : g == 2 ? qv[r].z : qv[r].w;
                    const uint32_t v = ((half ? (word >> 4) : word) & 0x0F0F0F0Fu) | 0x80808080u;
                    w[r][0] = fmaf(s[r], fh3::nib_f(v, fh3::kSel0) - 1.0f, nm[r]);
                    w[r][1] = fmaf(s[r], fh3::nib_f(v, fh3::kSel1) - 1.0f, nm[r]);
                    w[r][2] = fmaf(s[r], fh3::nib_f(v, fh3::kSel2) - 1.0f, nm[r]);
                    w[r][3] = fmaf(s[r], fh3::nib_f(v, fh3::kSel3) - 1.0f, nm[r]);
                }
#pragma unroll
                for (int t = 0; t < M; ++t) {
                    const float4 xv = __ldg(reinterpret_cast<const float4*>(xk + t * K + 4 * g));
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        float a = acc[r][t];
                        a = fmaf(xv.x, w[r][0], a);
                        a = fmaf(xv.y, w[r][1], a);
                        a = fmaf(xv.z, w[r][2], a);
                        a = fmaf(xv.w, w[r][3], a);
                        acc[r][t] = a;
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
            float v = acc[r][t];
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
int launch(const Fh3CudaW* w, const float* x, float* y, const float* bias, cudaStream_t s, int sms) {
    (void)sms;
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
    const int sms = ctx_sms(c);
    switch (n_tok) {
        case 1: return launch<1, 2>(w, x, y, bias, s, sms);
        case 2: return launch<2, 2>(w, x, y, bias, s, sms);
        case 3: return launch<3, 4>(w, x, y, bias, s, sms);
        case 4: return launch<4, 4>(w, x, y, bias, s, sms);
        case 5: return launch<5, 4>(w, x, y, bias, s, sms);
        case 6: return launch<6, 4>(w, x, y, bias, s, sms);
        case 7: return launch<7, 4>(w, x, y, bias, s, sms);
        case 8: return launch<8, 4>(w, x, y, bias, s, sms);
        case 9: return launch<9, 2>(w, x, y, bias, s, sms);
        case 10: return launch<10, 2>(w, x, y, bias, s, sms);
        case 11: return launch<11, 2>(w, x, y, bias, s, sms);
        case 12: return launch<12, 2>(w, x, y, bias, s, sms);
        case 13: return launch<13, 2>(w, x, y, bias, s, sms);
        case 14: return launch<14, 2>(w, x, y, bias, s, sms);
        case 15: return launch<15, 2>(w, x, y, bias, s, sms);
        default: return launch<16, 2>(w, x, y, bias, s, sms);
    }
}
