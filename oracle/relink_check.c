/* relink_check.c -- TEST INFRASTRUCTURE: the drop-in proven from C99.
 *
 * fh3 code calls fh3_matmul (include/fh3/fh3.h:107).  Linked with
 * -Wl,--wrap=fh3_matmul against libfh3cuda.so, those calls land in the library's
 * __wrap_fh3_matmul (GPU), while __real_fh3_matmul stays the reference's own CPU
 * function compiled from src/core/fh3_ops.c into the same program.  This program is
 * such an fh3 caller: it runs both on the reference's golden matmul file
 * (tests/fixtures/quant/matmul_ref.bin, copied to tests/golden/) and on seeded Q4_K
 * matrices at GEMV and GEMM token counts, and compares them.
 *
 *   relink_check <matmul_ref.bin>      exit 0 and "relink ok" when every case passes
 *
 * Tolerances (relative Frobenius error): 1e-5 up to 16 tokens (fp32 GEMV path),
 * 5e-3 above (bf16 tensor-core GEMM path).  Built by `make -C oracle relink`. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "fh3/fh3.h"

void __real_fh3_matmul(const Fh3W *w, const float *x, float *y, int n_tok, const float *bias_or_null);
/* from libfh3cuda (include/fh3cuda.h): the drop-in's sticky status */
int fh3cuda_take_status(void);

static double rel_fro(const float *a, const float *b, size_t n) {
    double num = 0.0, den = 0.0;
    for (size_t i = 0; i < n; ++i) {
        const double d = (double)a[i] - (double)b[i];
        num += d * d;
        den += (double)b[i] * (double)b[i];
    }
    return den > 0.0 ? sqrt(num / den) : sqrt(num);
}

static uint64_t g_lcg = 0x9E3779B97F4A7C15ull;
static uint32_t next_u32(void) {
    g_lcg = g_lcg * 6364136223846793005ull + 1442695040888963407ull;
    return (uint32_t)(g_lcg >> 33);
}

/* Q4_K rows with finite fp16 scales: d and dmin in [2^-8, 2^-7), random 6-bit scales
 * and mins, random nibbles (the byte layout of src/core/fh3_quant.c:154-196). */
static void fill_q4k(uint8_t *w, size_t blocks) {
    for (size_t b = 0; b < blocks; ++b) {
        uint8_t *blk = w + b * 144;
        const uint16_t d = (uint16_t)(0x1C00u | (next_u32() & 0x3FFu));
        const uint16_t dmin = (uint16_t)(0x1C00u | (next_u32() & 0x3FFu));
        memcpy(blk, &d, 2);
        memcpy(blk + 2, &dmin, 2);
        for (int i = 4; i < 144; ++i) blk[i] = (uint8_t)next_u32();
    }
}

static int compare(const char *what, const Fh3W *w, const float *x, int n_tok, const float *bias,
                   const float *expect_or_null) {
    const size_t ny = (size_t)n_tok * (size_t)w->out;
    float *gpu = malloc(ny * sizeof(float));
    float *cpu = malloc(ny * sizeof(float));
    if (!gpu || !cpu) {
        fprintf(stderr, "%s: out of host memory\n", what);
        return 1;
    }
    for (size_t i = 0; i < ny; ++i) gpu[i] = NAN;
    fh3_matmul(w, x, gpu, n_tok, bias);           /* wrapped: libfh3cuda on the GPU */
    const int st = fh3cuda_take_status();
    __real_fh3_matmul(w, x, cpu, n_tok, bias);     /* the reference's CPU function */
    const double tol = n_tok <= 16 ? 1e-5 : 5e-3;
    const double e_cpu = rel_fro(gpu, cpu, ny);
    const double e_ref = expect_or_null ? rel_fro(gpu, expect_or_null, ny) : 0.0;
    const int ok = st == 0 && e_cpu <= tol && e_ref <= tol;
    printf("%-28s n_tok %4d  status %d  vs __real_fh3_matmul %.3e  vs golden %.3e  (tol %.0e) %s\n", what, n_tok,
           st, e_cpu, e_ref, tol, ok ? "ok" : "FAIL");
    free(gpu);
    free(cpu);
    return ok ? 0 : 1;
}

int main(int argc, char **argv) {
    if (argc < 2) {
        fprintf(stderr, "usage: %s <matmul_ref.bin>\n", argv[0]);
        return 2;
    }
    int bad = 0;
    /* the reference's golden file: <IIIII> type, K, N, M, wbytes; W; x[M][K]; bias[N]; y[M][N] */
    FILE *f = fopen(argv[1], "rb");
    if (!f) {
        fprintf(stderr, "cannot open %s\n", argv[1]);
        return 2;
    }
    uint32_t hdr[5];
    if (fread(hdr, 4, 5, f) != 5) return 2;
    const uint32_t K = hdr[1], N = hdr[2], M = hdr[3], wb = hdr[4];
    uint8_t *gw = malloc(wb);
    float *gx = malloc((size_t)M * K * 4), *gb = malloc((size_t)N * 4), *gy = malloc((size_t)M * N * 4);
    if (!gw || !gx || !gb || !gy) return 2;
    if (fread(gw, 1, wb, f) != wb || fread(gx, 4, (size_t)M * K, f) != (size_t)M * K ||
        fread(gb, 4, N, f) != N || fread(gy, 4, (size_t)M * N, f) != (size_t)M * N)
        return 2;
    fclose(f);
    Fh3W w = {(int)hdr[0], K, N, gw};
    bad |= compare("golden matmul_ref.bin", &w, gx, (int)M, gb, gy);
    bad |= compare("golden, first 16 tokens", &w, gx, 16, gb, gy);
    free(gw);
    free(gx);
    free(gb);
    free(gy);

    /* seeded matrices at the DiT's widths: GEMV (1, 4, 16 tokens) and GEMM (300) */
    const int64_t shapes[2][2] = {{5120, 1024}, {13824, 512}};
    const int toks[4] = {1, 4, 16, 300};
    for (int s = 0; s < 2; ++s) {
        const int64_t in = shapes[s][0], out = shapes[s][1];
        const size_t rb = fh3_row_bytes(FH3_QUANT_Q4_K, in);
        uint8_t *qw = malloc(rb * (size_t)out);
        float *x = malloc((size_t)300 * in * 4), *bias = malloc((size_t)out * 4);
        if (!qw || !x || !bias) return 2;
        fill_q4k(qw, rb * (size_t)out / 144);
        for (size_t i = 0; i < (size_t)300 * in; ++i) x[i] = (float)((int)(next_u32() % 2001u) - 1000) * 1e-3f;
        for (int64_t i = 0; i < out; ++i) bias[i] = (float)((int)(next_u32() % 201u) - 100) * 1e-3f;
        Fh3W q = {FH3_QUANT_Q4_K, in, out, qw};
        for (int t = 0; t < 4; ++t) {
            char name[64];
            snprintf(name, sizeof(name), "seeded Q4_K %lldx%lld", (long long)in, (long long)out);
            bad |= compare(name, &q, x, toks[t], t & 1 ? NULL : bias, NULL);
        }
        free(qw);
        free(x);
        free(bias);
    }
    if (bad) {
        printf("relink FAILED\n");
        return 1;
    }
    printf("relink ok\n");
    return 0;
}
