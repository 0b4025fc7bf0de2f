// attention_f32.cu -- softmax attention on fp32 operands with fp32 arithmetic:
// fh3_attention (src/core/fh3_ops.c:587-695) and the fine pass of
// fh3_vsa_attention (src/core/fh3_vsa.c:372-432) at the reference's precision.
//
// The bf16 tensor-core kernels (attention.cu, vsa.cu) carry the production shapes;
// this one serves fp32 callers that need the CPU path's accuracy (the DiT forward's
// parity mode, tiny models, fp32 VSA inputs).  A warp owns one query row: each lane
// holds head_dim/32 channels of q and of the output accumulator, a key's score is a
// warp all-reduce of the lanes' partial dot products, and the softmax runs online
// (running max, rescaled sum and accumulator) in fp32 with expf.
#include "common.cuh"

namespace {

constexpr int kF32Warps = 4;

template <int C>  // channels per lane: head_dim = 32 * C
struct RowAttn {
    float q[C], acc[C];
    float m, l;

    __device__ __forceinline__ void init(const float* __restrict__ qrow, int lane) {
#pragma unroll
        for (int c = 0; c < C; ++c) {
            q[c] = qrow[lane + 32 * c];
            acc[c] = 0.0f;
        }
        m = -INFINITY;
        l = 0.0f;
    }

    __device__ __forceinline__ void key(const float* __restrict__ krow, const float* __restrict__ vrow, float scale,
                                        int lane) {
        float part = 0.0f;
#pragma unroll
        for (int c = 0; c < C; ++c) part = fmaf(q[c], krow[lane + 32 * c], part);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        const float s = part * scale;
        const float mn = fmaxf(m, s);
        const float a = expf(m - mn), p = expf(s - mn);
        m = mn;
        l = l * a + p;
#pragma unroll
        for (int c = 0; c < C; ++c) acc[c] = fmaf(p, vrow[lane + 32 * c], acc[c] * a);
    }
};

// Dense: grid (ceil(n / 4), heads); warp w of CTA b owns query row 4b + w.
// VSA (sel != nullptr): grid (tiles, heads); the warps take the rows of query tile b
// in turn and walk the kept key tiles sel[h][b][0 .. selcnt) in tile order; with a
// gate, o = fine + outc[b][h] * gate.
template <int C>
__global__ void __launch_bounds__(kF32Warps * 32) attn_f32_kernel(
    const float* __restrict__ q, int64_t ldq, const float* __restrict__ k, int64_t ldk, const float* __restrict__ v,
    int64_t ldv, float* __restrict__ o, int64_t ldo, int n, float scale, const int* __restrict__ perm,
    const int* __restrict__ toff, const int* __restrict__ sel, const int* __restrict__ selcnt, int nt,
    const float* __restrict__ gate, int64_t ldg, const float* __restrict__ outc, int heads) {
    constexpr int HD = 32 * C;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int h = blockIdx.y;
    const int64_t col = static_cast<int64_t>(h) * HD;
    if (!sel) {
        const int row = blockIdx.x * kF32Warps + warp;
        if (row >= n) return;
        RowAttn<C> ra;
        ra.init(q + row * ldq + col, lane);
        for (int e = 0; e < n; ++e) ra.key(k + e * ldk + col, v + e * ldv + col, scale, lane);
        const float inv = 1.0f / ra.l;
#pragma unroll
        for (int c = 0; c < C; ++c) o[row * ldo + col + lane + 32 * c] = ra.acc[c] * inv;
        return;
    }
    const int i = blockIdx.x;
    const size_t rowi = static_cast<size_t>(h) * nt + i;
    const int* lst = sel + rowi * nt;
    const int L = selcnt[rowi];
    const int q0 = toff[i], qn = toff[i + 1] - q0;
    const float* cb = gate ? outc + (static_cast<size_t>(i) * heads + h) * HD : nullptr;
    for (int r = warp; r < qn; r += kF32Warps) {
        const int64_t t = perm[q0 + r];
        RowAttn<C> ra;
        ra.init(q + t * ldq + col, lane);
        for (int li = 0; li < L; ++li) {
            const int j = lst[li];
            for (int e = toff[j]; e < toff[j + 1]; ++e) {
                const int64_t kt = perm[e];
                ra.key(k + kt * ldk + col, v + kt * ldv + col, scale, lane);
            }
        }
        const float inv = 1.0f / ra.l;
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const int d = lane + 32 * c;
            float val = ra.acc[c] * inv;
            if (cb) val += cb[d] * gate[t * ldg + col + d];
            o[t * ldo + col + d] = val;
        }
    }
}

}  // namespace

namespace fh3host {

// fp32 attention launch shared by the dense entry point below and the VSA fp32 path
// (vsa.cu).  head_dim a multiple of 32 up to 256.
int attention_f32_launch(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv,
                         float* o, int64_t ldo, int n, int heads, int head_dim, const int* perm, const int* toff,
                         const int* sel, const int* selcnt, int nt, const float* gate, int64_t ldg,
                         const float* outc, cudaStream_t s) {
    const float scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    const dim3 grid(sel ? static_cast<unsigned>(nt) : static_cast<unsigned>((n + kF32Warps - 1) / kF32Warps),
                    static_cast<unsigned>(heads));
#define FH3_F32_ATTN(CC)                                                                                       \
    attn_f32_kernel<CC><<<grid, kF32Warps * 32, 0, s>>>(q, ldq, k, ldk, v, ldv, o, ldo, n, scale, perm, toff, \
                                                        sel, selcnt, nt, gate, ldg, outc, heads)
    switch (head_dim / 32) {
        case 1: FH3_F32_ATTN(1); break;
        case 2: FH3_F32_ATTN(2); break;
        case 3: FH3_F32_ATTN(3); break;
        case 4: FH3_F32_ATTN(4); break;
        case 5: FH3_F32_ATTN(5); break;
        case 6: FH3_F32_ATTN(6); break;
        case 7: FH3_F32_ATTN(7); break;
        case 8: FH3_F32_ATTN(8); break;
        default: return set_error(FH3_E_INVALID, "attention_f32: head_dim must be a multiple of 32 up to 256");
    }
#undef FH3_F32_ATTN
    return check_cuda(cudaGetLastError(), "attention_f32 launch");
}

}  // namespace fh3host

extern "C" int fh3cuda_attention_f32_dev(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v,
                                         int64_t ldv, float* o, int64_t ldo, int n, int heads, int head_dim,
                                         void* stream) {
    using namespace fh3host;
    const char* who = "fh3cuda_attention_f32_dev";
    if (!ctx()) return set_error(FH3CUDA_E_NODEV, "%s: call fh3cuda_init first", who);
    if (!q || !k || !v || !o || n <= 0 || heads <= 0 || heads > 65535)
        return set_error(FH3_E_INVALID, "%s: bad arguments", who);
    if (head_dim <= 0 || head_dim % 32 || head_dim > 256)
        return set_error(FH3_E_INVALID, "%s: head_dim must be a multiple of 32 up to 256 (got %d)", who, head_dim);
    const int64_t row = static_cast<int64_t>(heads) * head_dim;
    if (ldq < row || ldk < row || ldv < row || ldo < row)
        return set_error(FH3_E_INVALID, "%s: rows must hold heads*head_dim elements", who);
    return attention_f32_launch(q, ldq, k, ldk, v, ldv, o, ldo, n, heads, head_dim, nullptr, nullptr, nullptr,
                                nullptr, 0, nullptr, 0, nullptr, static_cast<cudaStream_t>(stream));
}
