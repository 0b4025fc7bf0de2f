// flash.cuh -- the per-warp core of the flash-attention kernels (dense attention,
// attention.cu; the fine pass of video sparse attention, vsa.cu): bf16 operands on
// mma.sync.m16n8k16, fp32 online softmax in the exp2 domain.
//
// Tiles in shared memory are [rows][HD] bf16, each 16-byte chunk c of row r stored
// at chunk (c ^ (r & 7)) of the row (a 128-byte XOR swizzle), so ldmatrix reads
// them without bank conflicts.  A warp owns 16 query rows: their A fragments stay in
// registers for the whole key walk, and so does the 16 x HD output accumulator.
// Per 64-key tile: S = Q K^T (HD/16 k-steps x 8 key groups), scores of keys at or
// past `nvalid` become -inf, the running row max m rescales the accumulator and the
// row sums, P = exp2(S*c - m) is packed to bf16 straight from the S accumulators into
// the A fragments of O += P V (V fragments from ldmatrix.trans).
#pragma once

#include "common.cuh"

namespace fh3flash {

constexpr int kKeys = 64;  // keys per tile

// byte offset of 16-byte chunk c of row r in a swizzled [rows][HD] bf16 tile
template <int HD>
__device__ __forceinline__ uint32_t swz(int r, int c) {
    return static_cast<uint32_t>(r * (HD * 2) + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// One warp's 16 query rows through a walk over 64-key tiles.  Lane (g, tq) holds
// rows g and g+8 of the accumulator, columns 8j + 2tq, +1 of n8 tile j.
template <int HD>
struct WarpFlash {
    static_assert(HD % 16 == 0 && HD >= 32 && HD <= 128, "head_dim");
    uint32_t qf[HD / 16][4];  // A fragments of the rows, k16 steps over head_dim
    float o[HD / 8][4];       // output accumulator, n8 tiles over head_dim
    float m0, m1;             // running max of rows g and g+8 (exp2 domain)
    float l0, l1;             // this lane's part of the row sums

    __device__ __forceinline__ void init() {
#pragma unroll
        for (int j = 0; j < HD / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
        m0 = m1 = -INFINITY;
        l0 = l1 = 0.0f;
    }

    // A fragments of rows row0 .. row0+15 of a swizzled Q tile
    __device__ __forceinline__ void load_q(uint32_t sQ, int row0, int lane) {
        const int mi = lane >> 3;
        const int row = row0 + (lane & 7) + (mi & 1) * 8;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
            ldsm_x4(sQ + swz<HD>(row, 2 * kk + (mi >> 1)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
    }

    // one tile of 64 keys (rows of sK / sV); keys >= nvalid (nvalid >= 1) take no weight
    __device__ __forceinline__ void step(uint32_t sK, uint32_t sV, int nvalid, float scale_log2, int lane) {
        const int tq = lane & 3;
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int krow = j * 8 + (lane & 7);
#pragma unroll
            for (int kk = 0; kk < HD / 16; kk += 2) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4(sK + swz<HD>(krow, 2 * kk + (lane >> 3)), b0, b1, b2, b3);
                mma_bf16(s[j], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
                mma_bf16(s[j], qf[kk + 1][0], qf[kk + 1][1], qf[kk + 1][2], qf[kk + 1][3], b2, b3);
            }
        }
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const bool ok = j * 8 + 2 * tq + e < nvalid;
                s[j][e] = ok ? s[j][e] * scale_log2 : -INFINITY;
                s[j][2 + e] = ok ? s[j][2 + e] * scale_log2 : -INFINITY;
                mx0 = fmaxf(mx0, s[j][e]);
                mx1 = fmaxf(mx1, s[j][2 + e]);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);  // finite: every tile has a valid key
        const float a0 = exp2f(m0 - mn0), a1 = exp2f(m1 - mn1);
        m0 = mn0;
        m1 = mn1;
        l0 *= a0;
        l1 *= a1;
#pragma unroll
        for (int j = 0; j < HD / 8; ++j) {
            o[j][0] *= a0;
            o[j][1] *= a0;
            o[j][2] *= a1;
            o[j][3] *= a1;
        }
        uint32_t pf[4][4];  // P as A fragments, k16 steps over the tile's keys
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float p0 = exp2f(s[j][0] - mn0), p1 = exp2f(s[j][1] - mn0);
            const float p2 = exp2f(s[j][2] - mn1), p3 = exp2f(s[j][3] - mn1);
            l0 += p0 + p1;
            l1 += p2 + p3;
            pf[j >> 1][(j & 1) * 2 + 0] = pack_bf16(p0, p1);  // rows g:   keys 8j + 2tq, +1
            pf[j >> 1][(j & 1) * 2 + 1] = pack_bf16(p2, p3);  // rows g+8
        }
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            const int mi = lane >> 3;
            const int vrow = ks * 16 + (lane & 7) + (mi & 1) * 8;
#pragma unroll
            for (int jd = 0; jd < HD / 8; jd += 2) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(sV + swz<HD>(vrow, jd + (mi >> 1)), b0, b1, b2, b3);
                mma_bf16(o[jd], pf[ks][0], pf[ks][1], pf[ks][2], pf[ks][3], b0, b1);
                mma_bf16(o[jd + 1], pf[ks][0], pf[ks][1], pf[ks][2], pf[ks][3], b2, b3);
            }
        }
    }

    // 1 / row sum of rows g and g+8 (0 for a row that saw no key)
    __device__ __forceinline__ void inv_sums(float& i0, float& i1) {
        float s0 = l0, s1 = l1;
        s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
        s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
        s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
        s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
        i0 = s0 > 0.0f ? 1.0f / s0 : 0.0f;
        i1 = s1 > 0.0f ? 1.0f / s1 : 0.0f;
    }
};

}  // namespace fh3flash
