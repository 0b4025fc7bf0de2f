// gen.cu -- seeded synthetic Q4_K weights generated on the device.
//
// Benchmark input generator: producing 11.9 GB of Q4_K trunk weights on the
// host would take minutes, so the trunk is generated in HBM instead.  One warp
// per 256-weight super-block; lane l draws weights 8l..8l+7 (sub-block l/4)
// from Philox4x32-10 (counter = element/4, stream; key = seed) and a
// single-precision Box-Muller transform, then the block is quantised with the
// same rule as the project's CPU quantiser (oracle/fh3_oracle.c):
//   lo_j = min(0, min x), hi_j = max x, scale_j = (hi-lo)/15, mn_j = -lo,
//   d = fp16(max scale / 63), dmin = fp16(max mn / 63),
//   sc_j = rint(scale_j/d), m_j = rint(mn_j/dmin) in [0,63],
//   q = rint((x + dmin*m_j) / (d*sc_j)) in [0,15].
// The normals are not bit-identical to the CPU generator (float vs double
// Box-Muller); parity tests therefore use host-generated weights.
#include "common.cuh"

namespace {

__device__ __forceinline__ void philox10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t hi0 = __umulhi(0xD2511F53u, c[0]), lo0 = 0xD2511F53u * c[0];
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c[2]), lo1 = 0xCD9E8D57u * c[2];
        const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
        c[0] = n0;
        c[1] = lo1;
        c[2] = n2;
        c[3] = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
}

__global__ void make_q4k_kernel(uint64_t seed, uint64_t stream_id, float scale, int64_t nblocks,
                                int64_t blocks_per_row, uint8_t* __restrict__ dst) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
    for (int64_t blk = warp; blk < nblocks; blk += nwarps) {
        // element index of this lane's first weight; 8 weights = two Philox outputs
        const uint64_t e0 = static_cast<uint64_t>(blk) * 256 + lane * 8;
        float x[8];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint64_t ctr = e0 / 4 + h;
            uint32_t c[4] = {static_cast<uint32_t>(ctr), static_cast<uint32_t>(ctr >> 32),
                             static_cast<uint32_t>(stream_id), static_cast<uint32_t>(stream_id >> 32)};
            philox10(c, k0, k1);
#pragma unroll
            for (int pr = 0; pr < 2; ++pr) {
                const float u0 = (static_cast<float>(c[2 * pr]) + 1.0f) * 2.3283064e-10f;
                const float u1 = (static_cast<float>(c[2 * pr + 1]) + 1.0f) * 2.3283064e-10f;
                const float r = sqrtf(-2.0f * logf(fminf(u0, 1.0f)));
                float sn, cs;
                sincosf(6.2831853f * u1, &sn, &cs);
                x[4 * h + 2 * pr] = r * cs * scale;
                x[4 * h + 2 * pr + 1] = r * sn * scale;
            }
        }
        // sub-block j = lane/4: min/max over its 4 lanes
        float lo = 0.0f, hi = -INFINITY;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            lo = fminf(lo, x[e]);
            hi = fmaxf(hi, x[e]);
        }
#pragma unroll
        for (int o = 1; o < 4; o <<= 1) {
            lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
            hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
        }
        if (hi < lo) hi = lo;
        const float sj = __fdiv_rn(hi - lo, 15.0f);
        const float mj = -lo;
        float smax = sj, mmax = mj;
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, o));
            mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffffu, mmax, o));
        }
        const __half dh = __float2half_rn(__fdiv_rn(smax, 63.0f));
        const __half mh = __float2half_rn(__fdiv_rn(mmax, 63.0f));
        const float d = __half2float(dh), dmin = __half2float(mh);
        int sc = d > 0.0f ? static_cast<int>(rintf(__fdiv_rn(sj, d))) : 0;
        int m = dmin > 0.0f ? static_cast<int>(rintf(__fdiv_rn(mj, dmin))) : 0;
        sc = min(max(sc, 0), 63);
        m = min(max(m, 0), 63);
        const float dl = d * static_cast<float>(sc), ml = dmin * static_cast<float>(m);
        uint32_t qlo = 0, qhi = 0;  // 8 nibbles of this lane, one byte each
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            int q = 0;
            if (dl > 0.0f) q = min(max(static_cast<int>(rintf(__fdiv_rn(x[e] + ml, dl))), 0), 15);
            if (e < 4) qlo |= static_cast<uint32_t>(q) << (8 * e);
            else qhi |= static_cast<uint32_t>(q) << (8 * (e - 4));
        }
        uint8_t* b = dst + blk * fh3::kQ4KBytes;
        // nibble bytes: lanes of even sub-blocks combine with the lane 4 above (odd sub-block)
        const uint32_t olo = __shfl_down_sync(0xffffffffu, qlo, 4);
        const uint32_t ohi = __shfl_down_sync(0xffffffffu, qhi, 4);
        const int j = lane >> 2;
        if ((j & 1) == 0) {
            uint2 pk;
            pk.x = qlo | (olo << 4);
            pk.y = qhi | (ohi << 4);
            *reinterpret_cast<uint2*>(b + 16 + (j >> 1) * 32 + (lane & 3) * 8) = pk;
        }
        // header: gather the eight (sc, m) pairs from lanes 0,4,...,28
        int scs[8], ms[8];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
            scs[jj] = __shfl_sync(0xffffffffu, sc, jj * 4);
            ms[jj] = __shfl_sync(0xffffffffu, m, jj * 4);
        }
        if (lane == 0) {
            uint8_t hb[16];
            const unsigned short dbits = __half_as_ushort(dh), mbits = __half_as_ushort(mh);
            hb[0] = dbits & 0xFF;
            hb[1] = dbits >> 8;
            hb[2] = mbits & 0xFF;
            hb[3] = mbits >> 8;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                hb[4 + jj] = static_cast<uint8_t>((scs[jj] & 63) | ((scs[jj + 4] >> 4) << 6));
                hb[8 + jj] = static_cast<uint8_t>((ms[jj] & 63) | ((ms[jj + 4] >> 4) << 6));
                hb[12 + jj] = static_cast<uint8_t>((scs[jj + 4] & 15) | ((ms[jj + 4] & 15) << 4));
            }
            uint4 h4;
            memcpy(&h4, hb, 16);
            *reinterpret_cast<uint4*>(b) = h4;
        }
        (void)blocks_per_row;
    }
}

}  // namespace

extern "C" int fh3cuda_make_q4k_weights_dev(uint64_t seed, uint64_t stream_id, float scale, int64_t rows,
                                            int64_t n, void* dst, void* stream) {
    using namespace fh3host;
    DevCtx* c = ctx();
    if (!c) return set_error(FH3CUDA_E_NODEV, "fh3cuda_make_q4k_weights_dev: call fh3cuda_init first");
    if (!dst || rows <= 0 || n <= 0 || (n % fh3::kQ4KBlock) != 0 || (reinterpret_cast<uintptr_t>(dst) & 15))
        return set_error(FH3_E_INVALID, "fh3cuda_make_q4k_weights_dev: bad arguments");
    const int64_t bpr = n / fh3::kQ4KBlock;
    const int64_t nblocks = rows * bpr;
    int64_t grid = (nblocks + 7) / 8;
    const int64_t cap = static_cast<int64_t>(ctx_sms(c)) * 32;
    if (grid > cap) grid = cap;
    make_q4k_kernel<<<static_cast<unsigned>(grid), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        seed, stream_id, scale, nblocks, bpr, static_cast<uint8_t*>(dst));
    return check_cuda(cudaGetLastError(), "make_q4k_kernel launch");
}
