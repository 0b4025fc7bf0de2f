// dequant.cu -- fh3_dequant on the GPU: Q4_K (the trunk's format) and every other
// format the reference expands, bit-exact with its fp32 arithmetic
// (src/core/fh3_quant.c:36-318).
//
// One warp per 256-weight super-block: lane l writes weights 8l..8l+7 (sub-block
// l/4), so a warp reads its 144-byte block once (8-byte nibble loads plus the
// 16-byte header, broadcast) and writes 1 KiB contiguous.  The reference's
// arithmetic is reproduced with explicit IEEE roundings: dl = d*sc and
// ml = dmin*m, then dl*q and a separate subtraction (no FMA contraction,
// matching its -ffp-contract=off build).  HBM-bound: 144 B read + 1024 B
// written per block.
#include "common.cuh"
#include "formats.cuh"

namespace {

__global__ void __launch_bounds__(256) dequant_q4k_kernel(const uint8_t* __restrict__ src,
                                                          float* __restrict__ dst, int64_t rows,
                                                          int64_t blocks_per_row, int64_t n,
                                                          size_t row_bytes) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int64_t total = rows * blocks_per_row;
    const int j = lane >> 2;          // sub-block
    const int part = lane & 3;        // which 8 of its 32 weights
    for (int64_t g = warp; g < total; g += nwarps) {
        const int64_t r = g / blocks_per_row;
        const int64_t b = g - r * blocks_per_row;
        const uint8_t* blk = src + r * row_bytes + b * fh3::kQ4KBytes;
        // header: d, dmin, 12 scale bytes (16-byte aligned since 144 = 9*16 and rows are whole blocks)
        const uint4 hdr = __ldg(reinterpret_cast<const uint4*>(blk));
        const float d = fh3::h2f_bits(hdr.x), dmin = fh3::h2f_bits(hdr.x >> 16);
        int sc, m;
        fh3::q4k_scale_min_words(hdr.y, hdr.z, hdr.w, j, sc, m);
        const float dl = __fmul_rn(d, static_cast<float>(sc));
        const float ml = __fmul_rn(dmin, static_cast<float>(m));
        // 8 nibble bytes: chunk j/2, bytes part*8 .. part*8+7
        const uint2 qv = __ldg(reinterpret_cast<const uint2*>(blk + 16 + (j >> 1) * 32 + part * 8));
        const int shift = (j & 1) ? 4 : 0;
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const uint32_t word = e < 4 ? qv.x : qv.y;
            const int q = (word >> (8 * (e & 3) + shift)) & 0xF;
            o[e] = __fsub_rn(__fmul_rn(dl, static_cast<float>(q)), ml);
        }
        float* out = dst + r * n + b * fh3::kQ4KBlock + lane * 8;
        if ((n & 3) == 0) {
            reinterpret_cast<float4*>(out)[0] = make_float4(o[0], o[1], o[2], o[3]);
            reinterpret_cast<float4*>(out)[1] = make_float4(o[4], o[5], o[6], o[7]);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) out[e] = o[e];
        }
    }
}

// The other formats' 16-weight group decoders live in formats.cuh (shared with the
// matmul of those formats, formats.cu).
using namespace fh3fmt;

// rows x (whole blocks of) n weights of format TYPE; thread per 16-output group
template <int TYPE>
__global__ void __launch_bounds__(256) dequant_blocks_kernel(const uint8_t* __restrict__ src, float* __restrict__ dst,
                                                             int64_t rows, int64_t n, size_t row_bytes, int blk_elems,
                                                             int blk_bytes) {
    const int gpb = blk_elems / 16;                 // groups per block
    const int64_t gpr = (n / blk_elems) * gpb;      // groups per row (whole blocks only)
    const int64_t total = rows * gpr;
    for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
         g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = g / gpr;
        const int64_t gr = g - r * gpr;
        const int64_t b = gr / gpb;
        const int gi = static_cast<int>(gr - b * gpb);
        const uint8_t* blk = src + r * row_bytes + b * blk_bytes;
        float o[16];
        if (TYPE == 8) grp_q8_0(blk, gi, o);
        else if (TYPE == 10) grp_q2_k(blk, gi, o);
        else if (TYPE == 11) grp_q3_k(blk, gi, o);
        else if (TYPE == 13) grp_q5_k(blk, gi, o);
        else grp_q6_k(blk, gi, o);
        float* out = dst + r * n + b * blk_elems + gi * 16;
#pragma unroll
        for (int l = 0; l < 16; ++l) out[l] = o[l];
    }
}

// F16 (exact) and BF16 (bits << 16) element-wise
template <bool BF16>
__global__ void __launch_bounds__(256) dequant_half_kernel(const uint8_t* __restrict__ src, float* __restrict__ dst,
                                                           int64_t rows, int64_t n, size_t row_bytes) {
    const int64_t total = rows * n;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / n, e = i - r * n;
        const uint8_t* p = src + r * row_bytes + 2 * e;
        const uint32_t h = static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8);
        dst[i] = BF16 ? __uint_as_float(h << 16) : fh3::h2f_bits(h);
    }
}

}  // namespace

extern "C" int fh3cuda_dequant_dev(int type, const void* src, float* dst, int64_t rows, int64_t n,
                                   void* stream) {
    using namespace fh3host;
    DevCtx* c = ctx();
    if (!c) return set_error(FH3CUDA_E_NODEV, "fh3cuda_dequant_dev: call fh3cuda_init first");
    if (!src || !dst || rows <= 0 || n <= 0)
        return set_error(FH3_E_INVALID, "fh3cuda_dequant_dev: bad arguments");
    if (type != FH3CUDA_TYPE_Q4_K) {
        const size_t rb = fh3cuda_row_bytes(type, n);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        const auto* sp = static_cast<const uint8_t*>(src);
        const int64_t cap = static_cast<int64_t>(ctx_sms(c)) * 16;
        auto grid_for = [&](int64_t threads) {
            const int64_t g = (threads + 255) / 256;
            return static_cast<unsigned>(g < 1 ? 1 : (g > cap ? cap : g));
        };
        switch (type) {
            case FH3CUDA_TYPE_F32:
                return check_cuda(cudaMemcpy2DAsync(dst, static_cast<size_t>(n) * 4, src, rb, static_cast<size_t>(n) * 4,
                                                    static_cast<size_t>(rows), cudaMemcpyDeviceToDevice, s),
                                  "fh3cuda_dequant_dev: F32 copy");
            case FH3CUDA_TYPE_F16:
                dequant_half_kernel<false><<<grid_for(rows * n), 256, 0, s>>>(sp, dst, rows, n, rb);
                return check_cuda(cudaGetLastError(), "dequant_half_kernel launch");
            case FH3CUDA_TYPE_BF16:
                dequant_half_kernel<true><<<grid_for(rows * n), 256, 0, s>>>(sp, dst, rows, n, rb);
                return check_cuda(cudaGetLastError(), "dequant_half_kernel launch");
            default: break;
        }
        int be = 256, bb = 0;
        switch (type) {
            case FH3CUDA_TYPE_Q8_0: be = 32; bb = 34; break;
            case FH3CUDA_TYPE_Q2_K: bb = 84; break;
            case FH3CUDA_TYPE_Q3_K: bb = 110; break;
            case FH3CUDA_TYPE_Q5_K: bb = 176; break;
            case FH3CUDA_TYPE_Q6_K: bb = 210; break;
            default: return set_error(FH3_E_INVALID, "fh3cuda_dequant_dev: unsupported type %d", type);
        }
        if (n / be == 0) return FH3_OK;  // no whole block: nothing written, as in the reference
        const unsigned grid = grid_for(rows * (n / be) * (be / 16));
#define FH3_DQ(T) dequant_blocks_kernel<T><<<grid, 256, 0, s>>>(sp, dst, rows, n, rb, be, bb)
        switch (type) {
            case FH3CUDA_TYPE_Q8_0: FH3_DQ(8); break;
            case FH3CUDA_TYPE_Q2_K: FH3_DQ(10); break;
            case FH3CUDA_TYPE_Q3_K: FH3_DQ(11); break;
            case FH3CUDA_TYPE_Q5_K: FH3_DQ(13); break;
            default: FH3_DQ(14); break;
        }
#undef FH3_DQ
        return check_cuda(cudaGetLastError(), "dequant_blocks_kernel launch");
    }
    if ((reinterpret_cast<uintptr_t>(src) & 15) != 0)
        return set_error(FH3_E_INVALID, "fh3cuda_dequant_dev: src must be 16-byte aligned");
    const int64_t bpr = n / fh3::kQ4KBlock;
    if (bpr == 0) return FH3_OK;  // no whole block: nothing written, as in the reference
    const size_t rb = fh3cuda_row_bytes(type, n);
    const int64_t total = rows * bpr;
    int64_t grid = (total + 7) / 8;
    const int64_t cap = static_cast<int64_t>(ctx_sms(c)) * 16;
    if (grid > cap) grid = cap;
    dequant_q4k_kernel<<<static_cast<unsigned>(grid), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(src), dst, rows, bpr, n, rb);
    return check_cuda(cudaGetLastError(), "dequant_q4k_kernel launch");
}
