// formats.cuh -- 16-weight group decoders of the formats fh3_dequant expands besides
// Q4_K (src/core/fh3_quant.c:36-318), bit-exact with its fp32 arithmetic: explicit IEEE
// roundings, no contraction (the reference builds with -ffp-contract=off).  Shared by
// fh3cuda_dequant_dev (dequant.cu) and the matmul of these formats (formats.cu).
#pragma once

#include "common.cuh"

namespace fh3fmt {

// ---------------------------------------------------------------------------
// The other formats of fh3_dequant (src/core/fh3_quant.c:36-318), bit-exact with
// its fp32 arithmetic (explicit roundings, no contraction).  A thread writes 16
// consecutive outputs (a "group"): K-quant blocks hold 16 groups, Q8_0 blocks 2;
// F16 / BF16 are converted 16 elements per thread.  Block sizes (34, 84, 110, 176,
// 210 bytes) are not 16-byte multiples, so the bytes are read one by one (these
// formats are the text encoder's and the globals', not the DiT trunk's).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float f16_at(const uint8_t* p) {
    return fh3::h2f_bits(static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8));
}

// 16 outputs of group gi (0..15) of a Q2_K block (fh3_quant.c:73-108): group
// (c*4 + shift)*2 + half reads bytes 16 + 32c + 16half .. +15 at bit 2*shift.
__device__ __forceinline__ void grp_q2_k(const uint8_t* blk, int gi, float (&o)[16]) {
    const float d = f16_at(blk + 80), dmin = f16_at(blk + 82);
    const float dl = __fmul_rn(d, static_cast<float>(blk[gi] & 0x0F));
    const float ml = __fmul_rn(dmin, static_cast<float>(blk[gi] >> 4));
    const int c = gi >> 3, sh = (gi >> 1) & 3, half = gi & 1;
    const uint8_t* q = blk + 16 + c * 32 + half * 16;
#pragma unroll
    for (int l = 0; l < 16; ++l) o[l] = __fsub_rn(__fmul_rn(dl, static_cast<float>((q[l] >> (2 * sh)) & 3)), ml);
}

// Q3_K (fh3_quant.c:110-152): scale (low nibble | 2 high bits << 4) - 32, quant
// 2 low bits minus 4 when the hmask bit is clear.
__device__ __forceinline__ void grp_q3_k(const uint8_t* blk, int g, float (&o)[16]) {
    const uint8_t* hm = blk;
    const uint8_t* qs = blk + 32;
    const uint8_t* sr = blk + 96;
    const float d = f16_at(blk + 108);
    const int lo = g < 8 ? (sr[g] & 0x0F) : ((sr[g - 8] >> 4) & 0x0F);
    const int hi = (sr[8 + (g & 3)] >> ((g >> 2) * 2)) & 3;
    const float dl = __fmul_rn(d, static_cast<float>((lo | (hi << 4)) - 32));
    const int c = g >> 3, rem = g & 7;
    const int shl = (rem >> 1) * 2, offl = c * 32 + (rem & 1) * 16;
    const int shh = g >> 1, offh = (g & 1) * 16;
#pragma unroll
    for (int l = 0; l < 16; ++l) {
        const int q = ((qs[offl + l] >> shl) & 3) - ((((hm[offh + l] >> shh) & 1) ^ 1) << 2);
        o[l] = __fmul_rn(dl, static_cast<float>(q));
    }
}

// Q5_K (fh3_quant.c:198-240): Q4_K's scales, fifth bit of weight l of sub-block j
// in bit j of qh[l]; group gi = half gi%2 of sub-block gi/2.
__device__ __forceinline__ void grp_q5_k(const uint8_t* blk, int gi, float (&o)[16]) {
    const float d = f16_at(blk), dmin = f16_at(blk + 2);
    const int j = gi >> 1, l0 = (gi & 1) * 16;
    const uint8_t* s = blk + 4;
    int sc, m;
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
    const float dl = __fmul_rn(d, static_cast<float>(sc)), ml = __fmul_rn(dmin, static_cast<float>(m));
    const uint8_t* qh = blk + 16;
    const uint8_t* qs = blk + 48 + (j >> 1) * 32;
    const int shq = (j & 1) * 4;
#pragma unroll
    for (int l = 0; l < 16; ++l) {
        const int q = ((qs[l0 + l] >> shq) & 0x0F) | (((qh[l0 + l] >> j) & 1) << 4);
        o[l] = __fsub_rn(__fmul_rn(dl, static_cast<float>(q)), ml);
    }
}

// Q6_K (fh3_quant.c:242-282): 4 low bits from ql, 2 high bits from qh, minus 32,
// times d * int8 scale of the 16-weight group.
__device__ __forceinline__ void grp_q6_k(const uint8_t* blk, int g, float (&o)[16]) {
    const uint8_t* ql = blk;
    const uint8_t* qh = blk + 128;
    const float d = f16_at(blk + 208);
    const float dl = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(blk[192 + g])));
    const int c = g >> 3, rem = g & 7;
    const int shl = (rem >> 2) * 4, offl = c * 64 + (rem & 3) * 16;
    const int shh = (rem >> 1) * 2, offh = c * 32 + (rem & 1) * 16;
#pragma unroll
    for (int l = 0; l < 16; ++l) {
        const int q = (((ql[offl + l] >> shl) & 0x0F) | (((qh[offh + l] >> shh) & 3) << 4)) - 32;
        o[l] = __fmul_rn(dl, static_cast<float>(q));
    }
}

// Q8_0 (fh3_quant.c:58-71): group gi (0, 1) of a 32-weight block, (float)q * d.
__device__ __forceinline__ void grp_q8_0(const uint8_t* blk, int gi, float (&o)[16]) {
    const float d = f16_at(blk);
#pragma unroll
    for (int l = 0; l < 16; ++l)
        o[l] = __fmul_rn(static_cast<float>(static_cast<int8_t>(blk[2 + gi * 16 + l])), d);
}

}  // namespace fh3fmt
