// dequant.cu -- Q4_K -> fp32, bit-exact with fh3's dequant_q4_k
// (src/core/fh3_quant.c:154-196).
//
// One warp per 256-weight super-block: lane l writes weights 8l..8l+7 (sub-block
// l/4), so a warp reads its 144-byte block once (8-byte nibble loads plus the
// 16-byte header, broadcast) and writes 1 KiB contiguous.  The reference's
// arithmetic is reproduced with explicit IEEE roundings: dl = d*sc and
// ml = dmin*m, then dl*q and a separate subtraction (no FMA contraction,
// matching its -ffp-contract=off build).  HBM-bound: 144 B read + 1024 B
// written per block.
#include "common.cuh"

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

}  // namespace

extern "C" int fh3cuda_dequant_dev(int type, const void* src, float* dst, int64_t rows, int64_t n,
                                   void* stream) {
    using namespace fh3host;
    DevCtx* c = ctx();
    if (!c) return set_error(FH3CUDA_E_NODEV, "fh3cuda_dequant_dev: call fh3cuda_init first");
    if (type != FH3CUDA_TYPE_Q4_K)
        return set_error(FH3_E_INVALID, "fh3cuda_dequant_dev: unsupported type %d", type);
    if (!src || !dst || rows <= 0 || n <= 0)
        return set_error(FH3_E_INVALID, "fh3cuda_dequant_dev: bad arguments");
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
