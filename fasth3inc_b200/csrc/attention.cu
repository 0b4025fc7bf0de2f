// attention.cu -- dense, non-causal softmax attention (fh3_attention,
// src/core/fh3_ops.c:587-695) for head_dim 128 on bf16 q/k/v, fp32 softmax and
// accumulation, flash-attention style (the score matrix never leaves the SM).
//
// A CTA owns 128 query rows of one head (8 warps x 16 rows); it walks the keys in
// tiles of 64 with the online softmax: per tile S = Q K^T (warp: 16 x 64, 64 MMAs),
// running row max m and exp2-domain rescale of the output accumulator, P = exp2(S*c
// - m) packed to bf16 straight from the S accumulators into the A fragments of
// O += P V (64 MMAs).  Q stays in registers (32 per lane) for the whole walk; K and
// V tiles are double-buffered in shared memory with cp.async (rows past n are
// zero-filled without being read), stored 128-byte XOR-swizzled so ldmatrix reads
// them without bank conflicts; V fragments come from ldmatrix.trans.  Keys past n
// get score -inf.  Row sums stay per lane until the end (one quad reduction).
//
// Operands: element (token i, head h, channel d) of q / k / v at
// base + i*ld + h*128 + d (bf16), o at o + i*ldo + h*128 + d (fp32 or bf16).
#include "common.cuh"

namespace {

constexpr int kHD = 128;       // head_dim
constexpr int kBM = 128;       // query rows per CTA
constexpr int kBN = 64;        // keys per tile
constexpr int kAttnWarps = kBM / 16;
constexpr int kRowBytes = kHD * 2;                 // 256 B per row of a tile
constexpr int kQBytes = kBM * kRowBytes;           // 32 KB
constexpr int kKVBytes = kBN * kRowBytes;          // 16 KB
constexpr int kAttnSmem = kQBytes + 4 * kKVBytes;  // Q + 2 x (K, V) = 96 KB

// byte offset of 16-byte chunk c (0..15) of row r in a swizzled [rows][128 bf16] tile
__device__ __forceinline__ uint32_t swz(int r, int c) {
    return static_cast<uint32_t>(r * kRowBytes + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}

// rows [row0, row0 + rows) of head h into a swizzled tile; rows >= n are zero-filled
__device__ __forceinline__ void load_tile(uint32_t tile, const __nv_bfloat16* __restrict__ base, int64_t ld,
                                          int h, int row0, int rows, int n) {
    for (int idx = threadIdx.x; idx < rows * 16; idx += blockDim.x) {
        const int r = idx >> 4, c = idx & 15;
        const int row = row0 + r;
        const bool ok = row < n;
        const __nv_bfloat16* src = base + static_cast<int64_t>(ok ? row : 0) * ld + h * kHD + c * 8;
        cp_async16_zfill(tile + swz(r, c), src, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
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

template <bool OUT_BF16>
__global__ void __launch_bounds__(kAttnWarps * 32, 1) attention_kernel(
    const __nv_bfloat16* __restrict__ q, int64_t ldq, const __nv_bfloat16* __restrict__ k, int64_t ldk,
    const __nv_bfloat16* __restrict__ v, int64_t ldv, void* __restrict__ o, int64_t ldo, int n, float scale_log2) {
    extern __shared__ __align__(128) uint8_t attn_smem[];
    const uint32_t sbase = fh3::smem_u32(attn_smem);
    const uint32_t sQ = sbase;
    const uint32_t sK[2] = {sbase + kQBytes, sbase + kQBytes + kKVBytes};
    const uint32_t sV[2] = {sbase + kQBytes + 2 * kKVBytes, sbase + kQBytes + 3 * kKVBytes};
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, tq = lane & 3;
    const int h = blockIdx.y;
    const int q0 = blockIdx.x * kBM;
    const int ntiles = (n + kBN - 1) / kBN;

    load_tile(sQ, q, ldq, h, q0, kBM, n);
    load_tile(sK[0], k, ldk, h, 0, kBN, n);
    load_tile(sV[0], v, ldv, h, 0, kBN, n);

    uint32_t qf[8][4];  // A fragments of the warp's 16 query rows, k16 steps over head_dim
    float oacc[16][4];  // 16 rows x 128 channels: n8 tiles over head_dim
#pragma unroll
    for (int j = 0; j < 16; ++j) oacc[j][0] = oacc[j][1] = oacc[j][2] = oacc[j][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY;  // running max of rows g and g+8 (exp2 domain)
    float l0 = 0.0f, l1 = 0.0f;            // this lane's part of the row sums

    for (int t = 0; t < ntiles; ++t) {
        const int st = t & 1;
        if (t + 1 < ntiles) {
            load_tile(sK[st ^ 1], k, ldk, h, (t + 1) * kBN, kBN, n);
            load_tile(sV[st ^ 1], v, ldv, h, (t + 1) * kBN, kBN, n);
            asm volatile("cp.async.wait_group 2;" ::: "memory");  // all but the two newest groups
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        if (t == 0) {
            const int mi = lane >> 3;
            const int row = warp * 16 + (lane & 7) + (mi & 1) * 8;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
                ldsm_x4(sQ + swz(row, 2 * kk + (mi >> 1)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
        }
        // S = Q K^T for this warp's rows and the tile's 64 keys
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int krow = j * 8 + (lane & 7);
#pragma unroll
            for (int kk = 0; kk < 8; kk += 2) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4(sK[st] + swz(krow, 2 * kk + (lane >> 3)), b0, b1, b2, b3);
                mma_bf16(s[j], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
                mma_bf16(s[j], qf[kk + 1][0], qf[kk + 1][1], qf[kk + 1][2], qf[kk + 1][3], b2, b3);
            }
        }
        // online softmax (exp2 domain); keys past n score -inf
        const int kbase = t * kBN;
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const bool ok = kbase + j * 8 + 2 * tq + e < n;
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
        for (int j = 0; j < 16; ++j) {
            oacc[j][0] *= a0;
            oacc[j][1] *= a0;
            oacc[j][2] *= a1;
            oacc[j][3] *= a1;
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
        // O += P V
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            const int mi = lane >> 3;
            const int vrow = ks * 16 + (lane & 7) + (mi & 1) * 8;
#pragma unroll
            for (int jd = 0; jd < 16; jd += 2) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(sV[st] + swz(vrow, jd + (mi >> 1)), b0, b1, b2, b3);
                mma_bf16(oacc[jd], pf[ks][0], pf[ks][1], pf[ks][2], pf[ks][3], b0, b1);
                mma_bf16(oacc[jd + 1], pf[ks][0], pf[ks][1], pf[ks][2], pf[ks][3], b2, b3);
            }
        }
        __syncthreads();  // the next iteration's prefetch overwrites this stage
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const float i0 = l0 > 0.0f ? 1.0f / l0 : 0.0f, i1 = l1 > 0.0f ? 1.0f / l1 : 0.0f;
    const int r0 = q0 + warp * 16 + g, r1 = r0 + 8;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int d = h * kHD + j * 8 + 2 * tq;
        if (OUT_BF16) {
            __nv_bfloat16* ob = static_cast<__nv_bfloat16*>(o);
            if (r0 < n) *reinterpret_cast<uint32_t*>(ob + static_cast<int64_t>(r0) * ldo + d) =
                pack_bf16(oacc[j][0] * i0, oacc[j][1] * i0);
            if (r1 < n) *reinterpret_cast<uint32_t*>(ob + static_cast<int64_t>(r1) * ldo + d) =
                pack_bf16(oacc[j][2] * i1, oacc[j][3] * i1);
        } else {
            float* of = static_cast<float*>(o);
            if (r0 < n) *reinterpret_cast<float2*>(of + static_cast<int64_t>(r0) * ldo + d) =
                make_float2(oacc[j][0] * i0, oacc[j][1] * i0);
            if (r1 < n) *reinterpret_cast<float2*>(of + static_cast<int64_t>(r1) * ldo + d) =
                make_float2(oacc[j][2] * i1, oacc[j][3] * i1);
        }
    }
}

}  // namespace

extern "C" int fh3cuda_attention_dev(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                                     int64_t ldv, void* o, int o_bf16, int64_t ldo, int n, int heads, int head_dim,
                                     void* stream) {
    using namespace fh3host;
    const char* who = "fh3cuda_attention_dev";
    if (!ctx()) return set_error(FH3CUDA_E_NODEV, "%s: call fh3cuda_init first", who);
    if (!q || !k || !v || !o || n <= 0 || heads <= 0) return set_error(FH3_E_INVALID, "%s: bad arguments", who);
    if (head_dim != kHD) return set_error(FH3_E_INVALID, "%s: head_dim must be 128 (got %d)", who, head_dim);
    const int64_t row = static_cast<int64_t>(heads) * kHD;
    const bool aligned = !((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                            reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(o)) & 15);
    if (ldq < row || ldk < row || ldv < row || ldo < row || (ldq % 8) || (ldk % 8) || (ldv % 8) || (ldo % 8) ||
        !aligned)
        return set_error(FH3_E_INVALID, "%s: rows must hold heads*128 elements, strides a multiple of 8, "
                         "pointers 16-byte aligned", who);
    if (heads > 65535) return set_error(FH3_E_INVALID, "%s: at most 65535 heads", who);
    const float scale_log2 = (1.0f / sqrtf(static_cast<float>(kHD))) * 1.4426950408889634f;
    const dim3 grid(static_cast<unsigned>((n + kBM - 1) / kBM), static_cast<unsigned>(heads));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    static bool attr_set = false;
    if (!attr_set) {
        int rc = check_cuda(cudaFuncSetAttribute(attention_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 kAttnSmem), "attention smem attribute");
        if (!rc) rc = check_cuda(cudaFuncSetAttribute(attention_kernel<true>,
                                                      cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem),
                                 "attention smem attribute");
        if (rc) return rc;
        attr_set = true;
    }
    const auto* qb = static_cast<const __nv_bfloat16*>(q);
    const auto* kb = static_cast<const __nv_bfloat16*>(k);
    const auto* vb = static_cast<const __nv_bfloat16*>(v);
    if (o_bf16)
        attention_kernel<true><<<grid, kAttnWarps * 32, kAttnSmem, s>>>(qb, ldq, kb, ldk, vb, ldv, o, ldo, n,
                                                                         scale_log2);
    else
        attention_kernel<false><<<grid, kAttnWarps * 32, kAttnSmem, s>>>(qb, ldq, kb, ldk, vb, ldv, o, ldo, n,
                                                                          scale_log2);
    return check_cuda(cudaGetLastError(), "attention launch");
}
