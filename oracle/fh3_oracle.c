/*
 * fh3_oracle.c -- CPU restatement of fh3's Q4_K dequantise-and-multiply path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle for libfh3cuda: the
 * pytest suite, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load
 * it, as the checker.  The product path (libfh3cuda, fasth3inc_b200) never links,
 * loads or calls it, and there is no CPU fallback to it.
 *
 * Each function restates one reference function in plain C99 and names the
 * reference file:line it follows (paths are relative to the fh3 project root).
 * Parity is pinned two ways (tests/test_oracle.py):
 *   - against the reference's own golden vectors (tests/fixtures/quant/Q4_K.bin,
 *     tests/fixtures/quant/matmul_ref.bin, copied into tests/golden/), and
 *   - bit-for-bit against the reference functions themselves, compiled from the
 *     reference sources into oracle/_ref/ by oracle/Makefile (when present).
 *
 * The Q4_K quantiser at the bottom has no counterpart in fh3 (fh3 only
 * dequantises; gguf-py 0.19.0 raises NotImplementedError for Q4_K quantise).
 * It is this project's input generator, pinned by round-trip bounds only.
 *
 * Build flags must keep -ffp-contract=off so that a*b-c stays two roundings,
 * as in the reference build (CMakeLists.txt:15-26).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define Q4K_TYPE 12
#define Q4K_BLOCK 256
#define Q4K_BYTES 144

/* fp16 -> fp32, exact.  Restates fh3_f16_to_f32 (src/core/fh3_quant.h:20-41)
 * from the IEEE-754 binary16 definition (normal, subnormal, inf/nan). */
static float h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t expo = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    uint32_t bits;
    if (expo == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            /* subnormal: value = mant * 2^-24; normalise */
            int e = -1;
            do { mant <<= 1; e++; } while ((mant & 0x400u) == 0);
            mant &= 0x3FFu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
        }
    } else if (expo == 31) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((expo + 112u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

float oracle_f16_to_f32(uint16_t h) { return h2f(h); }

/* fp32 -> fp16, round to nearest even (for the quantiser's d/dmin fields). */
static uint16_t f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    int32_t expo = (int32_t)((x >> 23) & 0xFF) - 127 + 15;
    uint32_t mant = x & 0x7FFFFFu;
    if (((x >> 23) & 0xFF) == 0xFF) return (uint16_t)(sign | 0x7C00u | (mant ? 0x200u : 0));
    if (expo >= 31) return (uint16_t)(sign | 0x7C00u);
    if (expo <= 0) {
        if (expo < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        uint32_t shift = (uint32_t)(14 - expo);
        uint32_t half = 1u << (shift - 1);
        uint32_t rem = mant & ((1u << shift) - 1);
        uint32_t r = mant >> shift;
        if (rem > half || (rem == half && (r & 1u))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t r = mant >> 13;
    uint32_t rem = mant & 0x1FFFu;
    uint32_t out = ((uint32_t)expo << 10) | r;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) out++;
    return (uint16_t)(sign | out);
}

/* Restates fh3_row_bytes (src/core/fh3_quant.c:14-34) for the types fh3_dequant
 * can expand (:284-318): F32, F16, BF16, Q8_0 and the K-quants Q2_K..Q6_K. */
size_t oracle_row_bytes(int type, int64_t n) {
    if (n <= 0) return 0;
    switch (type) {
        case 0: return (size_t)n * 4;                      /* F32  */
        case 1: case 30: return (size_t)n * 2;             /* F16, BF16 */
        case 8: return (size_t)((n + 31) / 32) * 34;       /* Q8_0 */
        case 10: return (size_t)((n + 255) / 256) * 84;    /* Q2_K */
        case 11: return (size_t)((n + 255) / 256) * 110;   /* Q3_K */
        case Q4K_TYPE: return (size_t)((n + 255) / 256) * Q4K_BYTES;
        case 13: return (size_t)((n + 255) / 256) * 176;   /* Q5_K */
        case 14: return (size_t)((n + 255) / 256) * 210;   /* Q6_K */
        default: return 0;
    }
}

/* Unpack the 6-bit scale and min of sub-block j (0..7) from the 12 packed
 * bytes at block offset 4.  Layout per src/core/fh3_quant.c:167-177. */
static void q4k_scale_min(const uint8_t *s, int j, int *sc, int *m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* Restates dequant_q4_k (src/core/fh3_quant.c:154-196): per 256-weight
 * super-block, dl = d*sc and ml = dmin*m in fp32, then w = dl*q - ml as a
 * multiply and a separate subtract.  Only whole blocks are written (n/256,
 * :155): a partial trailing block is ignored, as in the reference. */
void oracle_dequant_q4k(const uint8_t *src, float *dst, int64_t n) {
    if (!src || !dst || n <= 0) return;
    int64_t nb = n / Q4K_BLOCK;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t *blk = src + b * Q4K_BYTES;
        uint16_t dh, mh;
        memcpy(&dh, blk, 2);
        memcpy(&mh, blk + 2, 2);
        float d = h2f(dh), dmin = h2f(mh);
        const uint8_t *qs = blk + 16;
        float *out = dst + b * Q4K_BLOCK;
        for (int j = 0; j < 8; j++) {
            int sc, m;
            q4k_scale_min(blk + 4, j, &sc, &m);
            float dl = d * (float)sc;
            float ml = dmin * (float)m;
            const uint8_t *chunk = qs + (j >> 1) * 32;
            for (int l = 0; l < 32; l++) {
                int q = (j & 1) ? (chunk[l] >> 4) : (chunk[l] & 0x0F);
                float prod = dl * (float)q;
                out[j * 32 + l] = prod - ml;
            }
        }
    }
}

/* Restates dequant_q8_0 (src/core/fh3_quant.c:58-71): blocks of 32 int8 with one
 * fp16 scale, w = (float)q * d. */
static void dq_q8_0(const uint8_t *src, float *dst, int64_t n) {
    for (int64_t b = 0; b < n / 32; b++) {
        const uint8_t *blk = src + b * 34;
        uint16_t dh;
        memcpy(&dh, blk, 2);
        const float d = h2f(dh);
        for (int i = 0; i < 32; i++) dst[b * 32 + i] = (float)(int8_t)blk[2 + i] * d;
    }
}

/* Restates dequant_q2_k (src/core/fh3_quant.c:73-108): 84-byte blocks, 16 bytes of
 * 4-bit scale|min pairs, 64 bytes of 2-bit quants, fp16 d and dmin at 80/82; for
 * chunk c (2) and shift s (4) the two 16-weight groups g0 = 2(4c+s), g0+1 read
 * bytes 0..15 / 16..31 of the chunk: w = (d*sc)*q - dmin*m. */
static void dq_q2_k(const uint8_t *src, float *dst, int64_t n) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t *blk = src + b * 84;
        uint16_t dh, mh;
        memcpy(&dh, blk + 80, 2);
        memcpy(&mh, blk + 82, 2);
        const float d = h2f(dh), dmin = h2f(mh);
        float *out = dst + b * 256;
        for (int c = 0; c < 2; c++) {
            for (int sh = 0; sh < 4; sh++) {
                for (int half = 0; half < 2; half++) {
                    const int grp = (c * 4 + sh) * 2 + half;
                    const float dl = d * (float)(blk[grp] & 0x0F);
                    const float ml = dmin * (float)(blk[grp] >> 4);
                    for (int l = 0; l < 16; l++) {
                        const int q = (blk[16 + c * 32 + half * 16 + l] >> (2 * sh)) & 3;
                        const float prod = dl * (float)q;
                        *out++ = prod - ml;
                    }
                }
            }
        }
    }
}

/* Restates dequant_q3_k (src/core/fh3_quant.c:110-152): 110-byte blocks: hmask[32],
 * qs[64], 12 scale bytes (8 low nibbles + 4 bytes of 2-bit highs), fp16 d at 108;
 * 16 groups of 16: scale = (low | high<<4) - 32, q = low2 - (hbit ? 0 : 4),
 * w = (d*scale) * q. */
static void dq_q3_k(const uint8_t *src, float *dst, int64_t n) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t *blk = src + b * 110;
        const uint8_t *hm = blk, *qs = blk + 32, *sr = blk + 96;
        uint16_t dh;
        memcpy(&dh, blk + 108, 2);
        const float d = h2f(dh);
        float *out = dst + b * 256;
        for (int g = 0; g < 16; g++) {
            const int lo = (g < 8) ? (sr[g] & 0x0F) : ((sr[g - 8] >> 4) & 0x0F);
            const int hi = (sr[8 + (g % 4)] >> ((g / 4) * 2)) & 3;
            const float dl = d * (float)((lo | (hi << 4)) - 32);
            const int c = g / 8, rem = g % 8;
            const int shl = (rem / 2) * 2, offl = c * 32 + (rem % 2) * 16;
            const int shh = g / 2, offh = (g % 2) * 16;
            for (int l = 0; l < 16; l++) {
                const int q = ((qs[offl + l] >> shl) & 3) - ((((hm[offh + l] >> shh) & 1) ^ 1) << 2);
                *out++ = dl * (float)q;
            }
        }
    }
}

/* Restates dequant_q5_k (src/core/fh3_quant.c:198-240): Q4_K's layout plus 32 bytes
 * of fifth bits (qh) before the nibbles: q = nibble | ((qh[l] >> g) & 1) << 4,
 * w = (d*sc)*q - dmin*m. */
static void dq_q5_k(const uint8_t *src, float *dst, int64_t n) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t *blk = src + b * 176;
        uint16_t dh, mh;
        memcpy(&dh, blk, 2);
        memcpy(&mh, blk + 2, 2);
        const float d = h2f(dh), dmin = h2f(mh);
        const uint8_t *qh = blk + 16, *qs = blk + 48;
        float *out = dst + b * 256;
        for (int g = 0; g < 8; g++) {
            int sc, m;
            q4k_scale_min(blk + 4, g, &sc, &m);
            const float dl = d * (float)sc, ml = dmin * (float)m;
            for (int l = 0; l < 32; l++) {
                const int q = ((qs[(g / 2) * 32 + l] >> ((g % 2) * 4)) & 0x0F) | (((qh[l] >> g) & 1) << 4);
                const float prod = dl * (float)q;
                out[g * 32 + l] = prod - ml;
            }
        }
    }
}

/* Restates dequant_q6_k (src/core/fh3_quant.c:242-282): 210-byte blocks: ql[128]
 * (4 low bits), qh[64] (2 high bits), 16 int8 scales, fp16 d at 208; 16 groups of
 * 16: q = (low | high<<4) - 32, w = (d*scale) * q. */
static void dq_q6_k(const uint8_t *src, float *dst, int64_t n) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t *blk = src + b * 210;
        const uint8_t *ql = blk, *qh = blk + 128;
        const int8_t *sc = (const int8_t *)(blk + 192);
        uint16_t dh;
        memcpy(&dh, blk + 208, 2);
        const float d = h2f(dh);
        float *out = dst + b * 256;
        for (int g = 0; g < 16; g++) {
            const float dl = d * (float)sc[g];
            const int c = g / 8, rem = g % 8;
            const int shl = (rem / 4) * 4, offl = c * 64 + (rem % 4) * 16;
            const int shh = (rem / 2) * 2, offh = c * 32 + (rem % 2) * 16;
            for (int l = 0; l < 16; l++) {
                const int q = (((ql[offl + l] >> shl) & 0x0F) | (((qh[offh + l] >> shh) & 3) << 4)) - 32;
                out[g * 16 + l] = dl * (float)q;
            }
        }
    }
}

/* Restates fh3_dequant (src/core/fh3_quant.c:284-318): one row of n weights of any
 * type above into fp32 (exact for F32/F16/BF16).  Returns -8 for other types. */
int oracle_dequant(int type, const uint8_t *src, float *dst, int64_t n) {
    if (!src || !dst || n <= 0) return -8;
    switch (type) {
        case 0: memcpy(dst, src, (size_t)n * 4); return 0;
        case 1:
            for (int64_t i = 0; i < n; i++) {
                uint16_t h;
                memcpy(&h, src + 2 * i, 2);
                dst[i] = h2f(h);
            }
            return 0;
        case 30:
            for (int64_t i = 0; i < n; i++) {
                uint16_t h;
                memcpy(&h, src + 2 * i, 2);
                const uint32_t u = (uint32_t)h << 16;
                memcpy(dst + i, &u, 4);
            }
            return 0;
        case 8: dq_q8_0(src, dst, n); return 0;
        case 10: dq_q2_k(src, dst, n); return 0;
        case 11: dq_q3_k(src, dst, n); return 0;
        case Q4K_TYPE: oracle_dequant_q4k(src, dst, n); return 0;
        case 13: dq_q5_k(src, dst, n); return 0;
        case 14: dq_q6_k(src, dst, n); return 0;
        default: return -8;
    }
}

/* fixed 8-lane tree of src/core/fh3_ops.c:19-27 */
static float tree8(const float a[8]) {
    float s01 = a[0] + a[1], s23 = a[2] + a[3];
    float s45 = a[4] + a[5], s67 = a[6] + a[7];
    return (s01 + s23) + (s45 + s67);
}

/* Dot product with the reference's summation order: 8 strided fp32 FMA lanes
 * over k, the fixed tree, then an fmaf tail (src/core/fh3_ops.c:29-47; the
 * AVX2 kernels :50-207 use the same lanes and tree, which is why the reference
 * asserts scalar == AVX2 == OpenMP bitwise, tests/unit/test_matmul.c:107-139). */
static float dot_ref_order(const float *x, const float *w, int64_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int64_t n8 = n - (n % 8);
    for (int64_t k = 0; k < n8; k += 8)
        for (int l = 0; l < 8; l++) acc[l] = fmaf(x[k + l], w[k + l], acc[l]);
    float dot = tree8(acc);
    for (int64_t k = n8; k < n; k++) dot = fmaf(x[k], w[k], dot);
    return dot;
}

/* Restates fh3_matmul (src/core/fh3_ops.c:317-404) for Q4_K and F32 weights:
 * y[t][o] = dot(x[t], dequant(W[o])) (+ bias[o]); y is overwritten.  Returns 0,
 * or -8 (FH3_E_INVALID) where the reference returns silently (:318-321). */
int oracle_matmul(int type, const uint8_t *wdata, int64_t in, int64_t out,
                  const float *x, float *y, int n_tok, const float *bias) {
    if (!wdata || !x || !y || n_tok <= 0 || in <= 0 || out <= 0) return -8;
    size_t rb = oracle_row_bytes(type, in);
    if (rb == 0) return -8;
    int64_t o;
#pragma omp parallel for schedule(dynamic, 16)
    for (o = 0; o < out; o++) {
        float *wrow = (float *)malloc((size_t)in * sizeof(float));
        if (!wrow) continue;
        memset(wrow, 0, (size_t)in * sizeof(float));
        oracle_dequant(type, wdata + (size_t)o * rb, wrow, in);
        for (int t = 0; t < n_tok; t++) {
            float d = dot_ref_order(x + (size_t)t * in, wrow, in);
            if (bias) d += bias[o];
            y[(size_t)t * out + o] = d;
        }
        free(wrow);
    }
    return 0;
}

/* Restates fh3_swiglu (src/core/fh3_ops.c:507-527): value-first halves,
 * out = val * g / (1 + expf(-g)), and 0 for g < -80. */
void oracle_swiglu(const float *in, float *out, int n, int F) {
    int i;
#pragma omp parallel for schedule(static)
    for (i = 0; i < n; i++) {
        const float *val = in + (size_t)i * 2 * F;
        const float *gate = val + F;
        for (int j = 0; j < F; j++) {
            float g = gate[j];
            float s = (g < -80.0f) ? 0.0f : g / (1.0f + expf(-g));
            out[(size_t)i * F + j] = val[j] * s;
        }
    }
}

/* Restates fh3_rmsnorm (src/core/fh3_ops.c:410-456): 8-lane FMA sum of
 * squares + tree, variance = sum/dim, inv = 1/sqrtf(var+eps), row*inv*w. */
void oracle_rmsnorm(float *x, const float *w, int n, int dim, float eps) {
    int i;
#pragma omp parallel for schedule(static)
    for (i = 0; i < n; i++) {
        float *row = x + (size_t)i * dim;
        float sum = dot_ref_order(row, row, dim);
        float var = sum / (float)dim;
        float inv = 1.0f / sqrtf(var + eps);
        for (int d = 0; d < dim; d++) {
            float t = row[d] * inv;
            row[d] = t * w[d];
        }
    }
}

/* Restates fh3_rope3 (src/core/fh3_ops.c:458-505): for token i and head h the
 * first rot_dim channels rotate in halves, v0 = x[j], v1 = x[rot/2 + j]:
 * x[j] = v0*cos[j] - v1*sin[j], x[rot/2+j] = v1*cos[rot/2+j] + v0*sin[rot/2+j]
 * (two products rounded, then one add/sub: -ffp-contract=off, as the
 * reference's mul/sub intrinsics); cos/sin are [n][rot_dim]; channels
 * rot_dim..head_dim-1 are untouched.  Invalid arguments leave x unchanged. */
void oracle_rope3(float *x, const float *cos_t, const float *sin_t, int n, int heads, int head_dim, int rot_dim) {
    if (!x || !cos_t || !sin_t || n <= 0 || heads <= 0 || head_dim <= 0 || rot_dim <= 0 || rot_dim > head_dim ||
        (rot_dim % 2) != 0)
        return;
    const int half = rot_dim / 2;
    for (int i = 0; i < n; i++) {
        const float *c = cos_t + (size_t)i * rot_dim;
        const float *s = sin_t + (size_t)i * rot_dim;
        for (int h = 0; h < heads; h++) {
            float *v = x + ((size_t)i * heads + h) * head_dim;
            for (int j = 0; j < half; j++) {
                const float v0 = v[j], v1 = v[half + j];
                const float a = v0 * c[j], b = v1 * s[j];
                const float e = v1 * c[half + j], f = v0 * s[half + j];
                v[j] = a - b;
                v[half + j] = e + f;
            }
        }
    }
}

/* Restates fh3_attention (src/core/fh3_ops.c:587-695): dense, non-causal
 * softmax attention over q/k/v laid out [n][heads][hd]; scale = 1/sqrtf(hd);
 * keys in tiles of 64 with the reference's online softmax: scores = dot*scale
 * (8-lane dot order), m_new = max(m, tile max), alpha = expf(m - m_new),
 * l *= alpha, acc *= alpha, then per key p = expf(s - m_new), l += p,
 * acc = fmaf(p, v, acc); o = acc * (l > 0 ? 1/l : 0). */
void oracle_attention(const float *q, const float *k, const float *v, float *o, int n, int heads, int hd) {
    if (!q || !k || !v || !o || n <= 0 || heads <= 0 || hd <= 0) return;
    const float scale = 1.0f / sqrtf((float)hd);
    int hi;
#pragma omp parallel for schedule(static)
    for (hi = 0; hi < heads * n; hi++) {
        const int h = hi / n, i = hi % n;
        float *acc = (float *)calloc((size_t)hd, sizeof(float));
        float scores[64];
        if (!acc) continue;
        const float *qi = q + ((size_t)i * heads + h) * hd;
        float *oi = o + ((size_t)i * heads + h) * hd;
        float m = -1e30f, l = 0.0f;
        for (int j0 = 0; j0 < n; j0 += 64) {
            const int B = (j0 + 64 <= n) ? 64 : (n - j0);
            for (int t = 0; t < B; t++) {
                const float *kj = k + ((size_t)(j0 + t) * heads + h) * hd;
                scores[t] = dot_ref_order(qi, kj, hd) * scale;
            }
            float mt = scores[0];
            for (int t = 1; t < B; t++)
                if (scores[t] > mt) mt = scores[t];
            const float mn = (m > mt) ? m : mt;
            const float alpha = expf(m - mn);
            l *= alpha;
            for (int d = 0; d < hd; d++) acc[d] *= alpha;
            for (int t = 0; t < B; t++) {
                const float *vj = v + ((size_t)(j0 + t) * heads + h) * hd;
                const float p = expf(scores[t] - mn);
                l += p;
                for (int d = 0; d < hd; d++) acc[d] = fmaf(p, vj[d], acc[d]);
            }
            m = mn;
        }
        const float inv = (l > 0.0f) ? (1.0f / l) : 0.0f;
        for (int d = 0; d < hd; d++) oi[d] = acc[d] * inv;
        free(acc);
    }
}

/* Restates fh3_modulate (src/core/fh3_ops.c:529-557): x = fma(x, 1+scale,
 * shift) on whole 8-wide vectors of each 1024-element chunk, and the unfused
 * x*(1+scale)+shift on a chunk's tail. shift/scale span the whole n*dim
 * array, as in the reference. */
void oracle_modulate(float *x, const float *shift, const float *scale, int n, int dim) {
    int64_t total = (int64_t)n * dim;
    for (int64_t k0 = 0; k0 < total; k0 += 1024) {
        int64_t k1 = (k0 + 1024 <= total) ? k0 + 1024 : total;
        int64_t k = k0;
        for (; k + 8 <= k1; k += 8)
            for (int l = 0; l < 8; l++) x[k + l] = fmaf(x[k + l], 1.0f + scale[k + l], shift[k + l]);
        for (; k < k1; k++) {
            float t = x[k] * (1.0f + scale[k]);
            x[k] = t + shift[k];
        }
    }
}

/* Restates fh3_gate_residual (src/core/fh3_ops.c:559-585): h = fma(g, y, h). */
void oracle_gate_residual(float *h, const float *gate, const float *y, int n, int dim) {
    int64_t total = (int64_t)n * dim;
    for (int64_t k = 0; k < total; k++) h[k] = fmaf(gate[k], y[k], h[k]);
}

/* Philox4x32-10 (Salmon et al., SC'11, "Parallel random numbers: as easy as
 * 1, 2, 3") followed by Box-Muller in double, as fh3_rng_normal
 * (src/model/fh3_sched.c:84-159) uses it: counter = {block lo, block hi,
 * stream lo, stream hi}, key = {seed lo, seed hi}; each 128-bit output gives
 * four normals, u = (c + 1) / (2^32 + 2). */
static void philox10(uint32_t c[4], uint32_t k0, uint32_t k1) {
    for (int r = 0; r < 10; r++) {
        uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
        uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
        uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0;
        uint32_t n1 = (uint32_t)p1;
        uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
        uint32_t n3 = (uint32_t)p0;
        c[0] = n0; c[1] = n1; c[2] = n2; c[3] = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
}

void oracle_rng_normal(uint64_t seed, uint64_t stream, float *out, size_t n) {
    if (!out || n == 0) return;
    size_t nb = (n + 3) / 4;
    long long b;
#pragma omp parallel for schedule(static)
    for (b = 0; b < (long long)nb; b++) {
        uint32_t c[4] = {(uint32_t)((uint64_t)b & 0xFFFFFFFFu), (uint32_t)((uint64_t)b >> 32),
                         (uint32_t)(stream & 0xFFFFFFFFu), (uint32_t)(stream >> 32)};
        philox10(c, (uint32_t)(seed & 0xFFFFFFFFu), (uint32_t)(seed >> 32));
        float z[4];
        for (int p = 0; p < 2; p++) {
            double u0 = ((double)c[2 * p] + 1.0) / 4294967298.0;
            double u1 = ((double)c[2 * p + 1] + 1.0) / 4294967298.0;
            double r = sqrt(-2.0 * log(u0));
            double th = 6.28318530717958647692 * u1;
            z[2 * p] = (float)(r * cos(th));
            z[2 * p + 1] = (float)(r * sin(th));
        }
        size_t base = (size_t)b * 4;
        for (int i = 0; i < 4; i++)
            if (base + i < n) out[base + i] = z[i];
    }
}

/* ------------------------------------------------------------------------
 * Q4_K quantiser (this project's input generator; no fh3 counterpart).
 *
 * Per 32-weight sub-block j: lo_j = min(0, min x), hi_j = max x; the sub-block
 * is represented as w = (d*sc_j)*q - (dmin*m_j) with q in [0,15].  d and dmin
 * are the fp16-rounded maxima of (hi-lo)/15 and -lo over the eight sub-blocks,
 * divided by 63; sc_j = round(((hi-lo)/15)/d) and m_j = round(-lo/dmin) in
 * [0,63]; q = round((x + dmin*m_j)/(d*sc_j)) clamped to [0,15].  The packing
 * is the exact inverse of dequant_q4_k's unpacking (src/core/fh3_quant.c:167-193).
 * ------------------------------------------------------------------------ */
static void quantize_block(const float *x, uint8_t *blk) {
    float scale[8], mn[8];
    float max_scale = 0.0f, max_mn = 0.0f;
    for (int j = 0; j < 8; j++) {
        float lo = 0.0f, hi = -INFINITY;
        for (int l = 0; l < 32; l++) {
            float v = x[j * 32 + l];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        if (hi < lo) hi = lo;
        scale[j] = (hi - lo) / 15.0f;
        mn[j] = -lo;
        if (scale[j] > max_scale) max_scale = scale[j];
        if (mn[j] > max_mn) max_mn = mn[j];
    }
    uint16_t dh = f2h(max_scale / 63.0f);
    uint16_t mh = f2h(max_mn / 63.0f);
    float d = h2f(dh), dmin = h2f(mh);
    int sc[8], m[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = d > 0.0f ? (int)lrintf(scale[j] / d) : 0;
        m[j] = dmin > 0.0f ? (int)lrintf(mn[j] / dmin) : 0;
        if (sc[j] < 0) sc[j] = 0;
        if (sc[j] > 63) sc[j] = 63;
        if (m[j] < 0) m[j] = 0;
        if (m[j] > 63) m[j] = 63;
    }
    memset(blk, 0, Q4K_BYTES);
    memcpy(blk, &dh, 2);
    memcpy(blk + 2, &mh, 2);
    uint8_t *s = blk + 4;
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((m[j + 4] & 15) << 4));
    }
    uint8_t *qs = blk + 16;
    for (int j = 0; j < 8; j++) {
        float dl = d * (float)sc[j];
        float ml = dmin * (float)m[j];
        for (int l = 0; l < 32; l++) {
            int q = 0;
            if (dl > 0.0f) {
                q = (int)lrintf((x[j * 32 + l] + ml) / dl);
                if (q < 0) q = 0;
                if (q > 15) q = 15;
            }
            uint8_t *byte = qs + (j >> 1) * 32 + l;
            if (j & 1) *byte = (uint8_t)((*byte & 0x0F) | (q << 4));
            else *byte = (uint8_t)((*byte & 0xF0) | q);
        }
    }
}

/* Quantise rows x [rows][n] (n a multiple of 256) to Q4_K rows. */
int oracle_quantize_q4k(const float *x, uint8_t *dst, int64_t rows, int64_t n) {
    if (!x || !dst || rows <= 0 || n <= 0 || (n % Q4K_BLOCK) != 0) return -8;
    int64_t nb = rows * (n / Q4K_BLOCK);
    int64_t b;
#pragma omp parallel for schedule(static)
    for (b = 0; b < nb; b++) quantize_block(x + b * Q4K_BLOCK, dst + b * Q4K_BYTES);
    return 0;
}

/* Seeded Q4_K weight generator: W = scale * N(0,1) from oracle_rng_normal
 * (seed, stream), quantised row by row.  Streams the normals through a
 * bounded buffer so that multi-GB weights need no multi-GB fp32 copy. */
int oracle_make_q4k_weights(uint64_t seed, uint64_t stream, float scale,
                            int64_t rows, int64_t n, uint8_t *dst) {
    if (!dst || rows <= 0 || n <= 0 || (n % Q4K_BLOCK) != 0) return -8;
    const int64_t chunk_rows = (int64_t)((64ll << 20) / (n * 4)) > 0 ? (int64_t)((64ll << 20) / (n * 4)) : 1;
    float *buf = (float *)malloc((size_t)chunk_rows * n * sizeof(float));
    if (!buf) return -7;
    size_t rb = oracle_row_bytes(Q4K_TYPE, n);
    for (int64_t r0 = 0; r0 < rows; r0 += chunk_rows) {
        int64_t nr = rows - r0 < chunk_rows ? rows - r0 : chunk_rows;
        /* element index e = r*n + k of the whole matrix maps to normal number e */
        size_t first = (size_t)(r0 * n);
        size_t cnt = (size_t)(nr * n);
        /* generate normals [first, first+cnt): first is a multiple of 4 since n%256==0 */
        size_t nb = cnt / 4;
        long long b;
#pragma omp parallel for schedule(static)
        for (b = 0; b < (long long)nb; b++) {
            uint64_t gb = (uint64_t)(first / 4) + (uint64_t)b;
            uint32_t c[4] = {(uint32_t)(gb & 0xFFFFFFFFu), (uint32_t)(gb >> 32),
                             (uint32_t)(stream & 0xFFFFFFFFu), (uint32_t)(stream >> 32)};
            philox10(c, (uint32_t)(seed & 0xFFFFFFFFu), (uint32_t)(seed >> 32));
            for (int p = 0; p < 2; p++) {
                double u0 = ((double)c[2 * p] + 1.0) / 4294967298.0;
                double u1 = ((double)c[2 * p + 1] + 1.0) / 4294967298.0;
                double r = sqrt(-2.0 * log(u0));
                double th = 6.28318530717958647692 * u1;
                buf[b * 4 + 2 * p] = (float)(r * cos(th)) * scale;
                buf[b * 4 + 2 * p + 1] = (float)(r * sin(th)) * scale;
            }
        }
        int rc = oracle_quantize_q4k(buf, dst + (size_t)r0 * rb, nr, n);
        if (rc) { free(buf); return rc; }
    }
    free(buf);
    return 0;
}

/* ---- video sparse attention (fh3_vsa_attention, src/core/fh3_vsa.c:186-507) ----
 *
 * Tile geometry (build_vsa_geometry, src/core/fh3_vsa.c:32-161), restated in
 * closed form: text tokens [0, T) and audio tokens [T, T+A) are cut into runs of
 * `tile` tokens ("prefix" tiles); video tokens [T+A, N) on the grid (gt, gh, gw)
 * are cut into 4x4x4 cells, visited t-major then h then w, the tokens of a cell in
 * row-major (t, h, w) order.  A sequence whose modality counts do not add up to N
 * is all video; a grid whose product is not V is (1, 1, V). */
typedef struct {
    int n, T, A, V, tile, nT, nA, npre, gt, gh, gw, ct, ch, cw, nvid, ntiles;
} VsaGeo;

static int vsa_geo(VsaGeo *g, int n, int T, int A, int V, int gt, int gh, int gw, int tile) {
    memset(g, 0, sizeof(*g));
    if (n <= 0) return -1;
    if (tile <= 0) tile = 64;
    if (T < 0) T = 0;
    if (A < 0) A = 0;
    if (V < 0) V = 0;
    if (T + A + V != n) { T = 0; A = 0; V = n; }
    if (gt <= 0 || gh <= 0 || gw <= 0 || (int64_t)gt * gh * gw != V) { gt = 1; gh = 1; gw = V; }
    g->n = n; g->T = T; g->A = A; g->V = V; g->tile = tile;
    g->nT = (T + tile - 1) / tile;
    g->nA = (A + tile - 1) / tile;
    g->npre = g->nT + g->nA;
    g->gt = gt; g->gh = gh; g->gw = gw;
    g->ct = (gt + 3) / 4; g->ch = (gh + 3) / 4; g->cw = (gw + 3) / 4;
    g->nvid = V > 0 ? g->ct * g->ch * g->cw : 0;
    g->ntiles = g->npre + g->nvid;
    return g->ntiles > 0 ? 0 : -1;
}

/* tokens of tile i: count, offset in tile order, and token of its r-th member */
static int vsa_tile_count(const VsaGeo *g, int i) {
    if (i < g->nT) return (i + 1) * g->tile <= g->T ? g->tile : g->T - i * g->tile;
    if (i < g->npre) { int a = i - g->nT; return (a + 1) * g->tile <= g->A ? g->tile : g->A - a * g->tile; }
    int v = i - g->npre, tt = v / (g->ch * g->cw), hh = (v / g->cw) % g->ch, ww = v % g->cw;
    int et = g->gt - 4 * tt < 4 ? g->gt - 4 * tt : 4;
    int eh = g->gh - 4 * hh < 4 ? g->gh - 4 * hh : 4;
    int ew = g->gw - 4 * ww < 4 ? g->gw - 4 * ww : 4;
    return et * eh * ew;
}

static int vsa_tile_token(const VsaGeo *g, int i, int r) {
    if (i < g->nT) return i * g->tile + r;
    if (i < g->npre) return g->T + (i - g->nT) * g->tile + r;
    int v = i - g->npre, tt = v / (g->ch * g->cw), hh = (v / g->cw) % g->ch, ww = v % g->cw;
    int eh = g->gh - 4 * hh < 4 ? g->gh - 4 * hh : 4;
    int ew = g->gw - 4 * ww < 4 ? g->gw - 4 * ww : 4;
    int dt = r / (eh * ew), dh = (r / ew) % eh, dw = r % ew;
    return g->T + g->A + ((4 * tt + dt) * g->gh + 4 * hh + dh) * g->gw + 4 * ww + dw;
}

/* number of tiles (and the prefix / video split) of a sequence */
int oracle_vsa_tiles(int n, int T, int A, int V, int gt, int gh, int gw, int tile, int *out3) {
    VsaGeo g;
    if (vsa_geo(&g, n, T, A, V, gt, gh, gw, tile)) return -1;
    out3[0] = g.ntiles;
    out3[1] = g.npre;
    out3[2] = g.nvid;
    return 0;
}

/* compute_topk (src/core/fh3_vsa.c:163-169), float arithmetic as there */
static int vsa_topk(float sparsity, int nblocks) {
    if (nblocks <= 0) return 0;
    int k = (int)ceilf((1.0f - sparsity) * (float)nblocks);
    return k < 1 ? 1 : (k > nblocks ? nblocks : k);
}

/* Restates fh3_vsa_attention (src/core/fh3_vsa.c:186-507).  q/k/v/gate/o are
 * [n][heads][hd] fp32; gate may be NULL (no coarse branch).  Operation order
 * follows the reference where it fixes the rounding: tile means accumulate
 * q * (1/count) over the tile's tokens in tile order (:230-256); a tile score is
 * a sequential dot product times 1/sqrt(hd) (:268-281); a video query tile keeps
 * the prefix key tiles and the top-k video key tiles by (score desc, index asc)
 * (:295-356), all key tiles when sparsity <= 0 or k covers them all; prefix query
 * tiles keep all key tiles.  Fine attention: max, expf, sequential sum, and
 * o += (p * (1/sum)) * v over the kept keys in tile order (:372-432).  Coarse:
 * the same softmax over every tile score of the row, against the tile means of v
 * (:442-473); o = fine + coarse * gate (:476-487).
 * Optional outputs: scores [heads][ntiles][ntiles] and mask (same shape, 0/1).
 * Returns 0, or -8 where the reference returns silently. */
int oracle_vsa(int tile, float sparsity, const float *q, const float *k, const float *v, const float *gate,
               float *o, int n, int T, int A, int V, int gt, int gh, int gw, int heads, int hd,
               float *scores_out, uint8_t *mask_out) {
    if (!q || !k || !v || !o || n <= 0 || heads <= 0 || hd <= 0) return -8;
    VsaGeo g;
    if (vsa_geo(&g, n, T, A, V, gt, gh, gw, tile)) return -8;
    const int nt = g.ntiles;
    const float scale = 1.0f / sqrtf((float)hd);
    const size_t pool_sz = (size_t)heads * nt * hd;
    float *qp = (float *)calloc(pool_sz, sizeof(float));
    float *kp = (float *)calloc(pool_sz, sizeof(float));
    float *vp = gate ? (float *)calloc(pool_sz, sizeof(float)) : NULL;
    float *S = (float *)malloc((size_t)heads * nt * nt * sizeof(float));
    uint8_t *M = (uint8_t *)calloc((size_t)heads * nt * nt, 1);
    int *off = (int *)malloc((size_t)(nt + 1) * sizeof(int));
    int *tok = (int *)malloc((size_t)n * sizeof(int));
    float *fine = (float *)calloc((size_t)n * heads * hd, sizeof(float));
    if (!qp || !kp || (gate && !vp) || !S || !M || !off || !tok || !fine) {
        free(qp); free(kp); free(vp); free(S); free(M); free(off); free(tok); free(fine);
        return -8;
    }
    off[0] = 0;
    for (int i = 0; i < nt; i++) {
        int c = vsa_tile_count(&g, i);
        for (int r = 0; r < c; r++) tok[off[i] + r] = vsa_tile_token(&g, i, r);
        off[i + 1] = off[i] + c;
    }
    /* tile means */
    for (int i = 0; i < nt; i++) {
        const int c = off[i + 1] - off[i];
        const float inv = 1.0f / (float)c;
        for (int r = 0; r < c; r++) {
            const int t = tok[off[i] + r];
            for (int h = 0; h < heads; h++) {
                const size_t src = ((size_t)t * heads + h) * hd, dst = ((size_t)h * nt + i) * hd;
                for (int d = 0; d < hd; d++) {
                    qp[dst + d] += q[src + d] * inv;
                    kp[dst + d] += k[src + d] * inv;
                    if (vp) vp[dst + d] += v[src + d] * inv;
                }
            }
        }
    }
    /* tile scores */
    int hi;
#pragma omp parallel for schedule(static)
    for (hi = 0; hi < heads * nt; hi++) {
        const int h = hi / nt, i = hi % nt;
        const float *a = qp + ((size_t)h * nt + i) * hd;
        for (int j = 0; j < nt; j++) {
            const float *b = kp + ((size_t)h * nt + j) * hd;
            float dot = 0.0f;
            for (int d = 0; d < hd; d++) dot += a[d] * b[d];
            S[((size_t)h * nt + i) * nt + j] = dot * scale;
        }
    }
    /* tile mask: a video key tile j is kept for row (h, i) when fewer than k video
     * key tiles precede it in (score desc, index asc) order */
    const int kv = vsa_topk(sparsity, g.nvid);
    const int dense = sparsity <= 0.0f || kv == g.nvid;
#pragma omp parallel for schedule(static)
    for (hi = 0; hi < heads * nt; hi++) {
        const int i = hi % nt;
        const float *s = S + (size_t)hi * nt;
        uint8_t *m = M + (size_t)hi * nt;
        if (i < g.npre || dense) {
            memset(m, 1, (size_t)nt);
            continue;
        }
        memset(m, 1, (size_t)g.npre);
        for (int j = g.npre; j < nt; j++) {
            int before = 0;
            for (int j2 = g.npre; j2 < nt && before < kv; j2++)
                if (s[j2] > s[j] || (s[j2] == s[j] && j2 < j)) before++;
            m[j] = before < kv;
        }
    }
    /* fine attention per (head, query tile) */
#pragma omp parallel for schedule(dynamic)
    for (hi = 0; hi < heads * nt; hi++) {
        const int h = hi / nt, i = hi % nt;
        const uint8_t *m = M + (size_t)hi * nt;
        int nk = 0;
        for (int j = 0; j < nt; j++)
            if (m[j]) nk += off[j + 1] - off[j];
        int *keys = (int *)malloc((size_t)nk * sizeof(int));
        float *p = (float *)malloc((size_t)nk * sizeof(float));
        if (!keys || !p) { free(keys); free(p); continue; }
        nk = 0;
        for (int j = 0; j < nt; j++)
            if (m[j])
                for (int r = off[j]; r < off[j + 1]; r++) keys[nk++] = tok[r];
        for (int r = off[i]; r < off[i + 1]; r++) {
            const float *qi = q + ((size_t)tok[r] * heads + h) * hd;
            float mx = -1e30f;
            for (int e = 0; e < nk; e++) {
                const float *kj = k + ((size_t)keys[e] * heads + h) * hd;
                float dot = 0.0f;
                for (int d = 0; d < hd; d++) dot += qi[d] * kj[d];
                p[e] = dot * scale;
                if (p[e] > mx) mx = p[e];
            }
            float sum = 0.0f;
            for (int e = 0; e < nk; e++) {
                p[e] = expf(p[e] - mx);
                sum += p[e];
            }
            const float inv = 1.0f / sum;
            float *oi = fine + ((size_t)tok[r] * heads + h) * hd;
            for (int e = 0; e < nk; e++) {
                const float *vj = v + ((size_t)keys[e] * heads + h) * hd;
                const float w = p[e] * inv;
                for (int d = 0; d < hd; d++) oi[d] += w * vj[d];
            }
        }
        free(keys);
        free(p);
    }
    /* coarse branch and combination */
    if (gate) {
        float *w = (float *)malloc((size_t)nt * sizeof(float));
        float *c = (float *)malloc((size_t)hd * sizeof(float));
        for (int i = 0; i < nt && w && c; i++) {
            for (int h = 0; h < heads; h++) {
                const float *s = S + ((size_t)h * nt + i) * nt;
                float mx = -1e30f, sum = 0.0f;
                for (int j = 0; j < nt; j++) if (s[j] > mx) mx = s[j];
                for (int j = 0; j < nt; j++) sum += expf(s[j] - mx);
                const float inv = 1.0f / sum;
                for (int d = 0; d < hd; d++) c[d] = 0.0f;
                for (int j = 0; j < nt; j++) {
                    const float wj = expf(s[j] - mx) * inv;
                    const float *vj = vp + ((size_t)h * nt + j) * hd;
                    for (int d = 0; d < hd; d++) c[d] += wj * vj[d];
                }
                for (int r = off[i]; r < off[i + 1]; r++) {
                    const size_t e = ((size_t)tok[r] * heads + h) * hd;
                    for (int d = 0; d < hd; d++) o[e + d] = fine[e + d] + c[d] * gate[e + d];
                }
            }
        }
        if (!w || !c) memcpy(o, fine, (size_t)n * heads * hd * sizeof(float));
        free(w);
        free(c);
    } else {
        memcpy(o, fine, (size_t)n * heads * hd * sizeof(float));
    }
    if (scores_out) memcpy(scores_out, S, (size_t)heads * nt * nt * sizeof(float));
    if (mask_out) memcpy(mask_out, M, (size_t)heads * nt * nt);
    free(qp); free(kp); free(vp); free(S); free(M); free(off); free(tok); free(fine);
    return 0;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
