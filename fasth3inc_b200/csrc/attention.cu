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
// get score -inf.  Row sums stay per lane until the end (one quad reduction).  The
// per-warp tile step is fh3flash::WarpFlash (flash.cuh), shared with vsa.cu.
//
// Operands: element (token i, head h, channel d) of q / k / v at
// base + i*ld + h*128 + d (bf16), o at o + i*ldo + h*128 + d (fp32 or bf16).
#include <cstdlib>
#include <cstring>

#include "flash.cuh"

namespace {

using namespace fh3flash;

constexpr int kHD = 128;       // head_dim
constexpr int kBM = 128;       // query rows per CTA
constexpr int kBN = kKeys;     // keys per tile
constexpr int kAttnWarps = kBM / 16;
constexpr int kRowBytes = kHD * 2;                 // 256 B per row of a tile
constexpr int kQBytes = kBM * kRowBytes;           // 32 KB
constexpr int kKVBytes = kBN * kRowBytes;          // 16 KB
constexpr int kAttnSmem = kQBytes + 4 * kKVBytes;  // Q + 2 x (K, V) = 96 KB

// rows [row0, row0 + rows) of head h into a swizzled tile; rows >= n are zero-filled
__device__ __forceinline__ void load_tile(uint32_t tile, const __nv_bfloat16* __restrict__ base, int64_t ld,
                                          int h, int row0, int rows, int n) {
    for (int idx = threadIdx.x; idx < rows * 16; idx += blockDim.x) {
        const int r = idx >> 4, c = idx & 15;
        const int row = row0 + r;
        const bool ok = row < n;
        const __nv_bfloat16* src = base + static_cast<int64_t>(ok ? row : 0) * ld + h * kHD + c * 8;
        cp_async16_zfill(tile + swz<kHD>(r, c), src, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
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

    WarpFlash<kHD> wf;
    wf.init();
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
        if (t == 0) wf.load_q(sQ, warp * 16, lane);
        wf.step(sK[st], sV[st], min(kBN, n - t * kBN), scale_log2, lane);  // keys past n score -inf
        __syncthreads();  // the next iteration's prefetch overwrites this stage
    }
    float i0, i1;
    wf.inv_sums(i0, i1);
    const int r0 = q0 + warp * 16 + g, r1 = r0 + 8;
#pragma unroll
    for (int j = 0; j < kHD / 8; ++j) {
        const int d = h * kHD + j * 8 + 2 * tq;
        if (OUT_BF16) {
            __nv_bfloat16* ob = static_cast<__nv_bfloat16*>(o);
            if (r0 < n) *reinterpret_cast<uint32_t*>(ob + static_cast<int64_t>(r0) * ldo + d) =
                pack_bf16(wf.o[j][0] * i0, wf.o[j][1] * i0);
            if (r1 < n) *reinterpret_cast<uint32_t*>(ob + static_cast<int64_t>(r1) * ldo + d) =
                pack_bf16(wf.o[j][2] * i1, wf.o[j][3] * i1);
        } else {
            float* of = static_cast<float*>(o);
            if (r0 < n) *reinterpret_cast<float2*>(of + static_cast<int64_t>(r0) * ldo + d) =
                make_float2(wf.o[j][0] * i0, wf.o[j][1] * i0);
            if (r1 < n) *reinterpret_cast<float2*>(of + static_cast<int64_t>(r1) * ldo + d) =
                make_float2(wf.o[j][2] * i1, wf.o[j][3] * i1);
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
    // tcgen05 kernel (attention_tc.cu) by default; FH3CUDA_ATTN_KERNEL=mma selects the mma.sync one
    const char* ak = getenv("FH3CUDA_ATTN_KERNEL");
    if (!(ak && strcmp(ak, "mma") == 0)) return attention_tc(qb, ldq, kb, ldk, vb, ldv, o, o_bf16 != 0, ldo, n, heads, s);
    if (o_bf16)
        attention_kernel<true><<<grid, kAttnWarps * 32, kAttnSmem, s>>>(qb, ldq, kb, ldk, vb, ldv, o, ldo, n,
                                                                         scale_log2);
    else
        attention_kernel<false><<<grid, kAttnWarps * 32, kAttnSmem, s>>>(qb, ldq, kb, ldk, vb, ldv, o, ldo, n,
                                                                          scale_log2);
    return check_cuda(cudaGetLastError(), "attention launch");
}
