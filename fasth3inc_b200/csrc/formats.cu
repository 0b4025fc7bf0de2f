// formats.cu -- fh3_matmul (src/core/fh3_ops.c:317-404) for the weight formats other
// than Q4_K: the text encoder's Q5_K / Q6_K (src/model/fh3_te.c:455-487), the F16 / F32
// globals, and every other format fh3_dequant expands (Q8_0, Q2_K, Q3_K, BF16).  Each
// weight is first formed exactly as fh3_dequant forms it in fp32 (formats.cuh), then:
//
// 1..16 tokens -- gemv_fmt_kernel: one warp per output row on the CUDA cores; a lane
//   decodes 16-weight groups and accumulates them against every token in fp32 (fmaf),
//   the warp reduces with shuffles.  The weights are read once.
// more tokens -- the fp32 contraction on the tcgen05 tensor cores as four bf16
//   products: w = wh + wl and x = xh + xl, each part a bf16 rounding (wh = bf16(w),
//   wl = bf16(w - wh); w - wh is exact in fp32, so w - wh - wl is below 2^-17 |w|), and
//   y = xh.wh + xh.wl + xl.wh + xl.wl accumulated in fp32.  K (padded to a multiple of
//   16 with zeros) is cut into slices of kSliceK; for each slice split_weights_kernel
//   writes W'_s = [wh | wl | wh | wl] and split_rows_kernel A'_s = [xh | xh | xl | xl]
//   side by side in one row, and gemm_bf16_pair_kernel (gemm.cu) runs A'_s . W'_s^T per
//   slice.  The tensor cores' fp32 accumulation is not rounded to nearest: over tens of
//   thousands of products its error drifts past 1e-5, so each slice (4 x 1024 products
//   a term at most) has its own accumulation and the slices are added in fp32 rounded to
//   nearest (the first slice's epilogue writes y = acc + bias, the others add acc with the
//   gated-residual epilogue under a gate of ones).  Weight rows and activation rows are
//   processed in chunks of at most 256 MB of expanded bf16 each.
#include <algorithm>

#include "common.cuh"
#include "formats.cuh"

namespace {

using namespace fh3fmt;

// F32 / F16 / BF16 rows are element arrays; the block formats are decoded per group.
template <int TYPE>
struct FmtBlock {
    static constexpr int ELEMS = TYPE == FH3CUDA_TYPE_Q8_0 ? 32 : 256;
    static constexpr int BYTES = TYPE == FH3CUDA_TYPE_Q8_0 ? 34 : TYPE == FH3CUDA_TYPE_Q2_K ? 84
                                 : TYPE == FH3CUDA_TYPE_Q3_K ? 110 : TYPE == FH3CUDA_TYPE_Q5_K ? 176 : 210;
};

// weights k = 16g .. 16g+15 of a row (k >= K read as 0), exactly fh3_dequant's fp32 values
template <int TYPE>
__device__ __forceinline__ void decode_group(const uint8_t* __restrict__ row, int64_t g, int64_t K, float (&o)[16]) {
    const int64_t k0 = g * 16;
    if (TYPE == FH3CUDA_TYPE_F32 || TYPE == FH3CUDA_TYPE_F16 || TYPE == FH3CUDA_TYPE_BF16) {
#pragma unroll
        for (int l = 0; l < 16; ++l) {
            const int64_t k = k0 + l;
            float v = 0.0f;
            if (k < K) {
                if (TYPE == FH3CUDA_TYPE_F32) {
                    v = __ldg(reinterpret_cast<const float*>(row) + k);
                } else {
                    const uint8_t* p = row + 2 * k;
                    const uint32_t h = static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8);
                    v = TYPE == FH3CUDA_TYPE_BF16 ? __uint_as_float(h << 16) : fh3::h2f_bits(h);
                }
            }
            o[l] = v;
        }
        return;
    }
    using B = FmtBlock<TYPE>;
    constexpr int gpb = B::ELEMS / 16;
    const uint8_t* blk = row + (g / gpb) * B::BYTES;
    const int gi = static_cast<int>(g % gpb);
    if (TYPE == FH3CUDA_TYPE_Q8_0) grp_q8_0(blk, gi, o);
    else if (TYPE == FH3CUDA_TYPE_Q2_K) grp_q2_k(blk, gi, o);
    else if (TYPE == FH3CUDA_TYPE_Q3_K) grp_q3_k(blk, gi, o);
    else if (TYPE == FH3CUDA_TYPE_Q5_K) grp_q5_k(blk, gi, o);
    else grp_q6_k(blk, gi, o);
}

// y[t][n] = sum_k x[t][k] w[n][k] (+ bias[n]) for n_tok <= 16; one warp per row n.
template <int TYPE>
__global__ void __launch_bounds__(256) gemv_fmt_kernel(const uint8_t* __restrict__ w, size_t rb, int64_t N, int64_t K,
                                                       const float* __restrict__ x, float* __restrict__ y, int n_tok,
                                                       const float* __restrict__ bias) {
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int64_t G = (K + 15) / 16;
    for (int64_t n = warp0; n < N; n += nwarps) {
        const uint8_t* row = w + n * rb;
        float acc[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) acc[t] = 0.0f;
        for (int64_t g = lane; g < G; g += 32) {
            float o[16];
            decode_group<TYPE>(row, g, K, o);
            const int64_t k0 = g * 16;
            const int kn = K - k0 < 16 ? static_cast<int>(K - k0) : 16;
#pragma unroll
            for (int t = 0; t < 16; ++t) {
                if (t >= n_tok) break;
                const float* xt = x + t * K + k0;
                float a = acc[t];
                if (kn == 16 && ((reinterpret_cast<uintptr_t>(xt) & 15) == 0)) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 xv = __ldg(reinterpret_cast<const float4*>(xt) + q);
                        a = fmaf(o[4 * q], xv.x, a);
                        a = fmaf(o[4 * q + 1], xv.y, a);
                        a = fmaf(o[4 * q + 2], xv.z, a);
                        a = fmaf(o[4 * q + 3], xv.w, a);
                    }
                } else {
                    for (int l = 0; l < kn; ++l) a = fmaf(o[l], __ldg(xt + l), a);
                }
                acc[t] = a;
            }
        }
#pragma unroll
        for (int t = 0; t < 16; ++t) {
            if (t >= n_tok) break;
            float a = acc[t];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
            if (lane == 0) y[t * N + n] = bias ? __fadd_rn(a, bias[n]) : a;
        }
    }
}

__device__ __forceinline__ void split_bf16(float v, __nv_bfloat16& hi, __nv_bfloat16& lo) {
    hi = __float2bfloat16_rn(v);
    lo = __float2bfloat16_rn(__fsub_rn(v, __bfloat162float(hi)));
}

constexpr int64_t kSliceK = 1024;  // weights a slice; each slice accumulates 4 x kSliceK products

// Where the 16 values of group g go in an expanded row of 4 Kp: slice s = 16g / kSliceK
// starts at 4 kSliceK s and holds its four parts of width ws (kSliceK, or what is left of Kp).
__device__ __forceinline__ void slice_pos(int64_t g, int64_t Kp, int64_t& base, int64_t& ws) {
    const int64_t k0 = g * 16, s = k0 / kSliceK;
    ws = Kp - s * kSliceK < kSliceK ? Kp - s * kSliceK : kSliceK;
    base = 4 * kSliceK * s + (k0 - s * kSliceK);
}

__device__ __forceinline__ void store_parts(__nv_bfloat16* row, int64_t base, int64_t ws, const uint4 (&a)[2],
                                            const uint4 (&b)[2], const uint4 (&c)[2], const uint4 (&d)[2]) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        reinterpret_cast<uint4*>(row + base)[q] = a[q];
        reinterpret_cast<uint4*>(row + base + ws)[q] = b[q];
        reinterpret_cast<uint4*>(row + base + 2 * ws)[q] = c[q];
        reinterpret_cast<uint4*>(row + base + 3 * ws)[q] = d[q];
    }
}

// W' rows: per slice [wh | wl | wh | wl] (Kp a multiple of 16; zeros past K)
template <int TYPE>
__global__ void __launch_bounds__(256) split_weights_kernel(const uint8_t* __restrict__ w, size_t rb, int64_t rows,
                                                            int64_t K, int64_t Kp, __nv_bfloat16* __restrict__ out) {
    const int64_t G = Kp / 16;
    const int64_t total = rows * G;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / G, g = i - r * G;
        float o[16];
        decode_group<TYPE>(w + r * rb, g, K, o);
        __align__(16) __nv_bfloat16 hi[16], lo[16];
#pragma unroll
        for (int l = 0; l < 16; ++l) split_bf16(o[l], hi[l], lo[l]);
        const uint4 h4[2] = {reinterpret_cast<const uint4*>(hi)[0], reinterpret_cast<const uint4*>(hi)[1]};
        const uint4 l4[2] = {reinterpret_cast<const uint4*>(lo)[0], reinterpret_cast<const uint4*>(lo)[1]};
        int64_t base, ws;
        slice_pos(g, Kp, base, ws);
        store_parts(out + r * 4 * Kp, base, ws, h4, l4, h4, l4);
    }
}

// A' rows of x rows [0, rows): per slice [xh | xh | xl | xl] (zeros past K)
__global__ void __launch_bounds__(256) split_rows_kernel(const float* __restrict__ x, int64_t rows, int64_t K,
                                                         int64_t Kp, __nv_bfloat16* __restrict__ out) {
    const int64_t G = Kp / 16;
    const int64_t total = rows * G;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / G, g = i - r * G;
        __align__(16) __nv_bfloat16 hi[16], lo[16];
#pragma unroll
        for (int l = 0; l < 16; ++l) {
            const int64_t k = g * 16 + l;
            split_bf16(k < K ? x[r * K + k] : 0.0f, hi[l], lo[l]);
        }
        const uint4 h4[2] = {reinterpret_cast<const uint4*>(hi)[0], reinterpret_cast<const uint4*>(hi)[1]};
        const uint4 l4[2] = {reinterpret_cast<const uint4*>(lo)[0], reinterpret_cast<const uint4*>(lo)[1]};
        int64_t base, ws;
        slice_pos(g, Kp, base, ws);
        store_parts(out + r * 4 * Kp, base, ws, h4, h4, l4, l4);
    }
}

__global__ void fill_kernel(float* __restrict__ p, int64_t n, float v) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        p[i] = v;
}

unsigned grid_of(fh3host::DevCtx* c, int64_t threads) {
    const int64_t cap = static_cast<int64_t>(fh3host::ctx_sms(c)) * 16;
    const int64_t g = (threads + 255) / 256;
    return static_cast<unsigned>(std::max<int64_t>(1, std::min(g, cap)));
}

template <int TYPE>
int launch_gemv(fh3host::DevCtx* c, const Fh3CudaW* w, size_t rb, const float* x, float* y, int n_tok,
                const float* bias, cudaStream_t s) {
    gemv_fmt_kernel<TYPE><<<grid_of(c, w->out * 32), 256, 0, s>>>(w->data, rb, w->out, w->in, x, y, n_tok, bias);
    return fh3host::check_cuda(cudaGetLastError(), "gemv_fmt_kernel launch");
}

template <int TYPE>
int launch_split_weights(fh3host::DevCtx* c, const uint8_t* rows_ptr, size_t rb, int64_t rows, int64_t K, int64_t Kp,
                         __nv_bfloat16* out, cudaStream_t s) {
    split_weights_kernel<TYPE><<<grid_of(c, rows * (Kp / 16)), 256, 0, s>>>(rows_ptr, rb, rows, K, Kp, out);
    return fh3host::check_cuda(cudaGetLastError(), "split_weights_kernel launch");
}

constexpr size_t kChunkBytes = size_t(256) << 20;

}  // namespace

namespace fh3host {

int matmul_formats(DevCtx* c, const Fh3CudaW* w, const float* x, float* y, int n_tok, const float* bias,
                   cudaStream_t s) {
    const int64_t K = w->in, N = w->out;
    int be = 1;
    switch (w->type) {
        case FH3CUDA_TYPE_F32: case FH3CUDA_TYPE_F16: case FH3CUDA_TYPE_BF16: be = 1; break;
        case FH3CUDA_TYPE_Q8_0: be = 32; break;
        case FH3CUDA_TYPE_Q2_K: case FH3CUDA_TYPE_Q3_K: case FH3CUDA_TYPE_Q5_K: case FH3CUDA_TYPE_Q6_K: be = 256; break;
        default:
            return set_error(FH3_E_INVALID, "fh3cuda_matmul_dev: weight type %d is not a format fh3_dequant expands",
                             w->type);
    }
    if (K % be)
        return set_error(FH3_E_INVALID, "fh3cuda_matmul_dev: in = %lld is not a multiple of the %d-weight block",
                         static_cast<long long>(K), be);
    if (w->type == FH3CUDA_TYPE_F32 && (reinterpret_cast<uintptr_t>(w->data) & 3))
        return set_error(FH3_E_INVALID, "fh3cuda_matmul_dev: F32 weights must be 4-byte aligned");
    const size_t rb = fh3cuda_row_bytes(w->type, K);
    if (n_tok <= 16) {
        switch (w->type) {
            case FH3CUDA_TYPE_F32: return launch_gemv<FH3CUDA_TYPE_F32>(c, w, rb, x, y, n_tok, bias, s);
            case FH3CUDA_TYPE_F16: return launch_gemv<FH3CUDA_TYPE_F16>(c, w, rb, x, y, n_tok, bias, s);
            case FH3CUDA_TYPE_BF16: return launch_gemv<FH3CUDA_TYPE_BF16>(c, w, rb, x, y, n_tok, bias, s);
            case FH3CUDA_TYPE_Q8_0: return launch_gemv<FH3CUDA_TYPE_Q8_0>(c, w, rb, x, y, n_tok, bias, s);
            case FH3CUDA_TYPE_Q2_K: return launch_gemv<FH3CUDA_TYPE_Q2_K>(c, w, rb, x, y, n_tok, bias, s);
            case FH3CUDA_TYPE_Q3_K: return launch_gemv<FH3CUDA_TYPE_Q3_K>(c, w, rb, x, y, n_tok, bias, s);
            case FH3CUDA_TYPE_Q5_K: return launch_gemv<FH3CUDA_TYPE_Q5_K>(c, w, rb, x, y, n_tok, bias, s);
            default: return launch_gemv<FH3CUDA_TYPE_Q6_K>(c, w, rb, x, y, n_tok, bias, s);
        }
    }
    // split-bf16 contraction on the tensor cores, in chunks of weight rows and of tokens
    const int64_t Kp = (K + 15) / 16 * 16;
    const size_t row4 = static_cast<size_t>(4 * Kp) * 2;  // bytes of one expanded row
    // chunk boundaries on whole 256-row tiles, so every chunk's output columns start aligned
    const int64_t fit = std::max<int64_t>(256, static_cast<int64_t>(kChunkBytes / row4) / 256 * 256);
    const int64_t wrows = std::min<int64_t>(N, fit);
    const int64_t xrows = std::min<int64_t>(n_tok, fit);
    auto* wsplit = static_cast<__nv_bfloat16*>(scratch(c, 8, static_cast<size_t>(wrows) * row4, s));
    auto* xsplit = static_cast<__nv_bfloat16*>(scratch(c, 0, static_cast<size_t>(xrows) * row4, s));
    const int64_t nslices = (Kp + kSliceK - 1) / kSliceK;
    float* ones = nullptr;
    if (nslices > 1) {
        ones = static_cast<float*>(scratch(c, 17, static_cast<size_t>(wrows) * 4, s));
        if (ones) {
            fill_kernel<<<grid_of(c, wrows), 256, 0, s>>>(ones, wrows, 1.0f);
            if (int rc = check_cuda(cudaGetLastError(), "fill_kernel launch")) return rc;
        }
    }
    if (!wsplit || !xsplit || (nslices > 1 && !ones)) return FH3_E_NOMEM;
    for (int64_t t0 = 0; t0 < n_tok; t0 += xrows) {
        const int64_t tn = std::min<int64_t>(xrows, n_tok - t0);
        split_rows_kernel<<<grid_of(c, tn * (Kp / 16)), 256, 0, s>>>(x + t0 * K, tn, K, Kp, xsplit);
        int rc = check_cuda(cudaGetLastError(), "split_rows_kernel launch");
        if (rc) return rc;
        for (int64_t o0 = 0; o0 < N; o0 += wrows) {
            const int64_t rows = std::min<int64_t>(wrows, N - o0);
            const uint8_t* src = w->data + o0 * rb;
            switch (w->type) {
                case FH3CUDA_TYPE_F32: rc = launch_split_weights<FH3CUDA_TYPE_F32>(c, src, rb, rows, K, Kp, wsplit, s); break;
                case FH3CUDA_TYPE_F16: rc = launch_split_weights<FH3CUDA_TYPE_F16>(c, src, rb, rows, K, Kp, wsplit, s); break;
                case FH3CUDA_TYPE_BF16: rc = launch_split_weights<FH3CUDA_TYPE_BF16>(c, src, rb, rows, K, Kp, wsplit, s); break;
                case FH3CUDA_TYPE_Q8_0: rc = launch_split_weights<FH3CUDA_TYPE_Q8_0>(c, src, rb, rows, K, Kp, wsplit, s); break;
                case FH3CUDA_TYPE_Q2_K: rc = launch_split_weights<FH3CUDA_TYPE_Q2_K>(c, src, rb, rows, K, Kp, wsplit, s); break;
                case FH3CUDA_TYPE_Q3_K: rc = launch_split_weights<FH3CUDA_TYPE_Q3_K>(c, src, rb, rows, K, Kp, wsplit, s); break;
                case FH3CUDA_TYPE_Q5_K: rc = launch_split_weights<FH3CUDA_TYPE_Q5_K>(c, src, rb, rows, K, Kp, wsplit, s); break;
                default: rc = launch_split_weights<FH3CUDA_TYPE_Q6_K>(c, src, rb, rows, K, Kp, wsplit, s); break;
            }
            if (rc) return rc;
            for (int64_t sl = 0; sl < nslices; ++sl) {
                const int64_t ws = std::min(kSliceK, Kp - sl * kSliceK);
                const int64_t off = 4 * kSliceK * sl;
                rc = gemm_bf16w(wsplit + off, 4 * Kp, rows, 4 * ws, xsplit + off, 4 * Kp, y + t0 * N + o0, N, tn,
                                sl == 0 && bias ? bias + o0 : nullptr, sl == 0 ? nullptr : ones,
                                sl == 0 ? FH3CUDA_EPI_F32 : FH3CUDA_EPI_RESID, 0, s);
                if (rc) return rc;
            }
        }
    }
    return FH3_OK;
}

}  // namespace fh3host
