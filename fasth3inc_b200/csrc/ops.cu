// ops.cu -- the elementwise work around the GEMMs of a DiT block.
//
//   fh3cuda_f32_to_bf16_dev       activations fp32 -> bf16 (GEMM A operand)
//   fh3cuda_rmsnorm_modulate_dev  GEMM prologue: rmsnorm (src/core/fh3_ops.c:410-456)
//                                 then modulate (:529-557), written as bf16
//   fh3cuda_swiglu_dev            fh3_swiglu (:507-527) on fp32 (the unfused form;
//                                 the GEMM has it as an epilogue)
//   fh3cuda_qk_norm_rope_dev      per-head rmsnorm (:410-456) then fh3_rope3 (:458-505)
//                                 of q or k straight from the QKV output, bit-exact
// All HBM-bound streaming kernels with 16-byte accesses.
#include <type_traits>

#include "common.cuh"

namespace {

__global__ void f32_to_bf16_kernel(const float4* __restrict__ x, uint2* __restrict__ y, int64_t n4) {
    // a GEMM launched next as a programmatic dependent may start its prologue and weight
    // loads now; it waits for this grid before it reads the converted activations
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float4 v = x[i];
        __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
        __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
        uint2 o;
        o.x = *reinterpret_cast<uint32_t*>(&a);
        o.y = *reinterpret_cast<uint32_t*>(&b);
        y[i] = o;
    }
}

__global__ void f32_to_bf16_tail_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                        int64_t start, int64_t n) {
    const int64_t i = start + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __float2bfloat16_rn(x[i]);
}

// One CTA per row.  Sum of squares in fp32 (fixed per-thread order + tree),
// inv = 1/sqrtf(mean + eps), v = x*inv*w, out = v*(1+scale) + shift -> bf16.
constexpr int kNormThreads = 256;

// The norms run between the trunk's GEMMs as programmatic dependents: the next GEMM may be
// scheduled (and load its weights) at once, and this kernel reads x only after the previous
// kernel has finished.  Writing y then is safe too: the kernel that last read y (the GEMM
// before the previous one) finished before the previous kernel did.
__device__ __forceinline__ void norm_griddep() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__global__ void __launch_bounds__(kNormThreads) rmsnorm_modulate_kernel(
    const float* __restrict__ x, const float* __restrict__ nw, const float* __restrict__ shift,
    const float* __restrict__ scale, __nv_bfloat16* __restrict__ y, int dim, float eps) {
    __shared__ float red[kNormThreads / 32];
    norm_griddep();
    const float* row = x + static_cast<int64_t>(blockIdx.x) * dim;
    __nv_bfloat16* out = y + static_cast<int64_t>(blockIdx.x) * dim;
    float ss = 0.0f;
    for (int k = threadIdx.x; k < dim; k += kNormThreads) ss = fmaf(row[k], row[k], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; ++w) tot += red[w];
    const float inv = 1.0f / sqrtf(tot / static_cast<float>(dim) + eps);
    for (int k = threadIdx.x; k < dim; k += kNormThreads) {
        float v = row[k] * inv;
        if (nw) v = v * nw[k];
        v = fmaf(v, 1.0f + scale[k], shift[k]);
        out[k] = __float2bfloat16_rn(v);
    }
}

// The same for rows of 4*kNormThreads*V' elements at most (dim a multiple of 4, 16-byte
// aligned rows): each thread keeps its V float4 of the row in registers, so the row is
// read from HBM once, and every access is 16 bytes (8 bytes for the bf16 output).  The
// sum of squares runs in a fixed order (per thread, then the same shuffle tree and warp
// sums as above), so a row's output does not depend on the others.
template <int V>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_modulate_vec_kernel(
    const float4* __restrict__ x, const float4* __restrict__ nw, const float4* __restrict__ shift,
    const float4* __restrict__ scale, uint2* __restrict__ y, int dim4, float inv_dim, float eps) {
    __shared__ float red[kNormThreads / 32];
    norm_griddep();
    const float4* row = x + static_cast<int64_t>(blockIdx.x) * dim4;
    uint2* out = y + static_cast<int64_t>(blockIdx.x) * dim4;
    float4 v[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int k = threadIdx.x + i * kNormThreads;
        v[i] = k < dim4 ? row[k] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        ss = fmaf(v[i].x, v[i].x, ss);
        ss = fmaf(v[i].y, v[i].y, ss);
        ss = fmaf(v[i].z, v[i].z, ss);
        ss = fmaf(v[i].w, v[i].w, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; ++w) tot += red[w];
    const float inv = 1.0f / sqrtf(tot * inv_dim + eps);
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int k = threadIdx.x + i * kNormThreads;
        if (k >= dim4) break;
        float4 a = make_float4(v[i].x * inv, v[i].y * inv, v[i].z * inv, v[i].w * inv);
        if (nw) {
            const float4 w = __ldg(nw + k);
            a = make_float4(a.x * w.x, a.y * w.y, a.z * w.z, a.w * w.w);
        }
        const float4 sc = __ldg(scale + k), sh = __ldg(shift + k);
        __nv_bfloat162 lo = __floats2bfloat162_rn(fmaf(a.x, 1.0f + sc.x, sh.x), fmaf(a.y, 1.0f + sc.y, sh.y));
        __nv_bfloat162 hi = __floats2bfloat162_rn(fmaf(a.z, 1.0f + sc.z, sh.z), fmaf(a.w, 1.0f + sc.w, sh.w));
        uint2 o;
        o.x = *reinterpret_cast<uint32_t*>(&lo);
        o.y = *reinterpret_cast<uint32_t*>(&hi);
        out[k] = o;
    }
}

__global__ void swiglu_kernel(const float* __restrict__ in, float* __restrict__ out, int64_t n, int F) {
    const int64_t total = n * F;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / F;
        const int64_t j = i - r * F;
        const float v = in[r * 2 * F + j];
        const float g = in[r * 2 * F + F + j];
        const float s = g < -80.0f ? 0.0f : g / (1.0f + expf(-g));
        out[i] = v * s;
    }
}

int grid_for(int64_t work, int threads) {
    using namespace fh3host;
    int64_t g = (work + threads - 1) / threads;
    const int64_t cap = static_cast<int64_t>(ctx_sms(ctx())) * 8;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return static_cast<int>(g);
}

// ---------------------------------------------------------------------------
// q / k after the QKV projection (fh3_dit.c:397-401): for token i and head h the
// head_dim-vector is rms-normalised with the shared weights w[head_dim], then its
// first rot_dim channels are rotated by cos/sin row i.  An 8-lane group owns one
// vector, staged in shared memory (16-byte global accesses).  Bit-exact with fh3:
// lane j sums x[j + 8m]^2 with fmaf in increasing m (the reference's eight AVX2
// lanes), the lanes meet in its fixed tree ((0+1)+(2+3))+((4+5)+(6+7)), then
// var = sum / dim, inv = 1 / sqrt(var + eps) correctly rounded, y = (x*inv)*w and
// the rotation with its products rounded before the add/sub.
// ---------------------------------------------------------------------------
constexpr int kQkThreads = 256;  // 32 vectors per CTA

template <bool SRC_BF16, bool DST_BF16>
__global__ void __launch_bounds__(kQkThreads) qk_norm_rope_kernel(
    const void* __restrict__ src, int64_t ld_src, void* __restrict__ dst, int64_t ld_dst, const float* __restrict__ w,
    const float* __restrict__ cs, const float* __restrict__ sn, int64_t nvec, int heads, int hd, int rot, float eps) {
    extern __shared__ __align__(16) float qk_smem[];
    const int l8 = threadIdx.x & 7;
    const int grp = threadIdx.x >> 3;
    const int64_t v = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 3) + grp;
    if (v >= nvec) return;  // whole 8-lane groups leave together
    const unsigned gmask = 0xFFu << (threadIdx.x & 24);
    const int64_t i = v / heads;
    const int h = static_cast<int>(v - i * heads);
    float* vec = qk_smem + grp * (hd + 8);  // padded: the four groups of a warp use different banks

    // load: lane l8 takes elements 4*l8 .. 4*l8+3 of every 32
    if (SRC_BF16) {
        const __nv_bfloat16* s = static_cast<const __nv_bfloat16*>(src) + i * ld_src + static_cast<int64_t>(h) * hd;
        for (int d = 4 * l8; d < hd; d += 32) {
            const uint2 u = *reinterpret_cast<const uint2*>(s + d);
            const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
            const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
            *reinterpret_cast<float4*>(vec + d) = make_float4(a.x, a.y, b.x, b.y);
        }
    } else {
        const float* s = static_cast<const float*>(src) + i * ld_src + static_cast<int64_t>(h) * hd;
        for (int d = 4 * l8; d < hd; d += 32)
            *reinterpret_cast<float4*>(vec + d) = *reinterpret_cast<const float4*>(s + d);
    }
    __syncwarp(gmask);
    float ss = 0.0f;
    for (int d = l8; d < hd; d += 8) ss = fmaf(vec[d], vec[d], ss);
    ss = __fadd_rn(ss, __shfl_xor_sync(gmask, ss, 1, 8));
    ss = __fadd_rn(ss, __shfl_xor_sync(gmask, ss, 2, 8));
    ss = __fadd_rn(ss, __shfl_xor_sync(gmask, ss, 4, 8));
    const float var = __fdiv_rn(ss, static_cast<float>(hd));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    for (int d = l8; d < hd; d += 8) vec[d] = __fmul_rn(__fmul_rn(vec[d], inv), w[d]);
    __syncwarp(gmask);
    if (rot > 0) {
        const int half = rot / 2;
        const float* c = cs + i * rot;
        const float* sg = sn + i * rot;
        for (int j = l8; j < half; j += 8) {
            const float v0 = vec[j], v1 = vec[half + j];
            vec[j] = __fsub_rn(__fmul_rn(v0, c[j]), __fmul_rn(v1, sg[j]));
            vec[half + j] = __fadd_rn(__fmul_rn(v1, c[half + j]), __fmul_rn(v0, sg[half + j]));
        }
        __syncwarp(gmask);
    }
    if (DST_BF16) {
        __nv_bfloat16* o = static_cast<__nv_bfloat16*>(dst) + i * ld_dst + static_cast<int64_t>(h) * hd;
        for (int d = 4 * l8; d < hd; d += 32) {
            const float4 f = *reinterpret_cast<const float4*>(vec + d);
            const __nv_bfloat162 a = __floats2bfloat162_rn(f.x, f.y), b = __floats2bfloat162_rn(f.z, f.w);
            uint2 u;
            u.x = *reinterpret_cast<const uint32_t*>(&a);
            u.y = *reinterpret_cast<const uint32_t*>(&b);
            *reinterpret_cast<uint2*>(o + d) = u;
        }
    } else {
        float* o = static_cast<float*>(dst) + i * ld_dst + static_cast<int64_t>(h) * hd;
        for (int d = 4 * l8; d < hd; d += 32)
            *reinterpret_cast<float4*>(o + d) = *reinterpret_cast<const float4*>(vec + d);
    }
}

// The same for a compile-time head_dim HD and half rotation HALF (a multiple of 8,
// or 0).  An 8-lane group takes kQkHeadsPerGroup heads of one token: the norm
// weights and the token's cos/sin live in registers for all of them, the next
// kQkAhead heads' rows are in flight while the current one is computed, and each lane keeps its
// HD/8 strided values in registers after one staging pass; both halves of every
// rotation pair (channels j and j + HALF) are in the same lane.
constexpr int kQkHeadsPerGroup = 8;
#ifndef FH3_QK_AHEAD
#define FH3_QK_AHEAD 2
#endif
constexpr int kQkAhead = FH3_QK_AHEAD;  // heads of a group in flight

template <bool SRC_BF16, int HD>
struct QkRaw {
    using T = typename std::conditional<SRC_BF16, uint2, float4>::type;  // 4 elements per lane and step
    T r[HD / 32];
};

template <bool SRC_BF16, int HD>
__device__ __forceinline__ void qk_load(QkRaw<SRC_BF16, HD>& raw, const void* src, int64_t off, int l8) {
#pragma unroll
    for (int k = 0; k < HD / 32; ++k) {
        if (SRC_BF16)
            raw.r[k] = *reinterpret_cast<const typename QkRaw<SRC_BF16, HD>::T*>(
                static_cast<const __nv_bfloat16*>(src) + off + 4 * l8 + 32 * k);
        else
            raw.r[k] = *reinterpret_cast<const typename QkRaw<SRC_BF16, HD>::T*>(
                static_cast<const float*>(src) + off + 4 * l8 + 32 * k);
    }
}

template <bool SRC_BF16, bool DST_BF16, int HD, int HALF>
__global__ void __launch_bounds__(kQkThreads) qk_norm_rope_reg_kernel(
    const void* __restrict__ src, int64_t ld_src, void* __restrict__ dst, int64_t ld_dst, const float* __restrict__ w,
    const float* __restrict__ cs, const float* __restrict__ sn, int64_t nunits, int heads, float eps) {
    static_assert(HD % 32 == 0 && HALF % 8 == 0 && 2 * HALF <= HD, "register path shape");
    constexpr int NV = HD / 8;
    constexpr int NR = HALF / 8 > 0 ? HALF / 8 : 1;
    constexpr int ROT = 2 * HALF;
    __shared__ __align__(16) float qk_stage[kQkThreads / 8][HD + 8];
    const int l8 = threadIdx.x & 7;
    const int grp = threadIdx.x >> 3;
    const int64_t u = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 3) + grp;
    if (u >= nunits) return;  // whole 8-lane groups leave together
    const unsigned gmask = 0xFFu << (threadIdx.x & 24);
    const int chunks = (heads + kQkHeadsPerGroup - 1) / kQkHeadsPerGroup;
    const int64_t i = u / chunks;
    const int h0 = static_cast<int>(u - i * chunks) * kQkHeadsPerGroup;
    const int h1 = min(heads, h0 + kQkHeadsPerGroup);
    float* vec = qk_stage[grp];

    float wr[NV];
#pragma unroll
    for (int m = 0; m < NV; ++m) wr[m] = __ldg(w + l8 + 8 * m);
    float c0[NR], s0[NR], c1[NR], s1[NR];
    if (HALF > 0) {
#pragma unroll
        for (int m = 0; m < NR; ++m) {
            const int j = l8 + 8 * m;
            c0[m] = __ldg(cs + i * ROT + j);
            s0[m] = __ldg(sn + i * ROT + j);
            c1[m] = __ldg(cs + i * ROT + HALF + j);
            s1[m] = __ldg(sn + i * ROT + HALF + j);
        }
    }
    // a ring of kQkAhead heads in flight: a slot is refilled as soon as its head is staged
    QkRaw<SRC_BF16, HD> buf[kQkAhead];
#pragma unroll
    for (int k = 0; k < kQkAhead; ++k)
        if (h0 + k < h1) qk_load<SRC_BF16, HD>(buf[k], src, i * ld_src + static_cast<int64_t>(h0 + k) * HD, l8);
#pragma unroll
    for (int jj = 0; jj < kQkHeadsPerGroup; ++jj) {
        const int h = h0 + jj;
        if (h >= h1) break;
        QkRaw<SRC_BF16, HD>& cur = buf[jj % kQkAhead];
#pragma unroll
        for (int k = 0; k < HD / 32; ++k) {
            float4 f;
            if (SRC_BF16) {
                const uint2 q = *reinterpret_cast<const uint2*>(&cur.r[k]);
                const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.x));
                const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.y));
                f = make_float4(a.x, a.y, b.x, b.y);
            } else {
                f = *reinterpret_cast<const float4*>(&cur.r[k]);
            }
            *reinterpret_cast<float4*>(vec + 4 * l8 + 32 * k) = f;
        }
        if (h + kQkAhead < h1)
            qk_load<SRC_BF16, HD>(cur, src, i * ld_src + static_cast<int64_t>(h + kQkAhead) * HD, l8);
        __syncwarp(gmask);
        float val[NV];
        float ss = 0.0f;
#pragma unroll
        for (int m = 0; m < NV; ++m) {
            val[m] = vec[l8 + 8 * m];
            ss = fmaf(val[m], val[m], ss);
        }
        ss = __fadd_rn(ss, __shfl_xor_sync(gmask, ss, 1, 8));
        ss = __fadd_rn(ss, __shfl_xor_sync(gmask, ss, 2, 8));
        ss = __fadd_rn(ss, __shfl_xor_sync(gmask, ss, 4, 8));
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(HD)), eps)));
#pragma unroll
        for (int m = 0; m < NV; ++m) val[m] = __fmul_rn(__fmul_rn(val[m], inv), wr[m]);
        if (HALF > 0) {
#pragma unroll
            for (int m = 0; m < HALF / 8; ++m) {
                const float v0 = val[m], v1 = val[m + HALF / 8];
                val[m] = __fsub_rn(__fmul_rn(v0, c0[m]), __fmul_rn(v1, s0[m]));
                val[m + HALF / 8] = __fadd_rn(__fmul_rn(v1, c1[m]), __fmul_rn(v0, s1[m]));
            }
        }
        __syncwarp(gmask);  // every lane has read the staged input
#pragma unroll
        for (int m = 0; m < NV; ++m) vec[l8 + 8 * m] = val[m];
        __syncwarp(gmask);
        const int64_t oo = i * ld_dst + static_cast<int64_t>(h) * HD;
#pragma unroll
        for (int k = 0; k < HD / 32; ++k) {
            const int d = 4 * l8 + 32 * k;
            const float4 f = *reinterpret_cast<const float4*>(vec + d);
            if (DST_BF16) {
                const __nv_bfloat162 a = __floats2bfloat162_rn(f.x, f.y), b = __floats2bfloat162_rn(f.z, f.w);
                uint2 q;
                q.x = *reinterpret_cast<const uint32_t*>(&a);
                q.y = *reinterpret_cast<const uint32_t*>(&b);
                *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(dst) + oo + d) = q;
            } else {
                *reinterpret_cast<float4*>(static_cast<float*>(dst) + oo + d) = f;
            }
        }
        __syncwarp(gmask);  // the stage is rewritten by the next head
    }
}

}  // namespace

extern "C" int fh3cuda_qk_norm_rope_dev(const void* src, int src_bf16, int64_t ld_src, void* dst, int dst_bf16,
                                        int64_t ld_dst, const float* norm_w, const float* cos_t, const float* sin_t,
                                        int n, int heads, int head_dim, int rot_dim, float eps, void* stream) {
    using namespace fh3host;
    const char* who = "fh3cuda_qk_norm_rope_dev";
    if (!ctx()) return set_error(FH3CUDA_E_NODEV, "%s: call fh3cuda_init first", who);
    if (!src || !dst || !norm_w || n <= 0 || heads <= 0)
        return set_error(FH3_E_INVALID, "%s: bad arguments", who);
    if (head_dim < 32 || head_dim > 256 || (head_dim % 32) != 0)
        return set_error(FH3_E_INVALID, "%s: head_dim must be a multiple of 32 in [32, 256] (got %d)", who, head_dim);
    if (rot_dim < 0 || rot_dim > head_dim || (rot_dim % 2) != 0 || (rot_dim > 0 && (!cos_t || !sin_t)))
        return set_error(FH3_E_INVALID, "%s: rot_dim must be even in [0, head_dim] with cos/sin given", who);
    const int64_t row = static_cast<int64_t>(heads) * head_dim;
    if (ld_src < row || ld_dst < row || (ld_src % 8) != 0 || (ld_dst % 8) != 0 ||
        (reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 15))
        return set_error(FH3_E_INVALID, "%s: rows must hold heads*head_dim elements, strides a multiple of 8, "
                         "pointers 16-byte aligned", who);
    if (src == dst && (src_bf16 != dst_bf16 || ld_src != ld_dst))
        return set_error(FH3_E_INVALID, "%s: in place needs the same element type and stride", who);
    const int64_t nvec = static_cast<int64_t>(n) * heads;
    const int groups = kQkThreads / 8;
    const unsigned grid = static_cast<unsigned>((nvec + groups - 1) / groups);
    const size_t smem = static_cast<size_t>(groups) * (head_dim + 8) * sizeof(float);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // head_dim 128 with rot_dim 0 / 96 / 128 (the DiT's q and k): the register path
    if (head_dim == 128 && (rot_dim == 0 || rot_dim == 96 || rot_dim == 128)) {
        const int64_t nunits = static_cast<int64_t>(n) * ((heads + kQkHeadsPerGroup - 1) / kQkHeadsPerGroup);
        const unsigned rgrid = static_cast<unsigned>((nunits + groups - 1) / groups);
#define FH3_QK_REG(SB, DB, HALF)                                                                     \
    qk_norm_rope_reg_kernel<SB, DB, 128, HALF><<<rgrid, kQkThreads, 0, s>>>(src, ld_src, dst, ld_dst, norm_w, \
                                                                           cos_t, sin_t, nunits, heads, eps)
#define FH3_QK_REG_ROT(SB, DB)                                  \
    do {                                                         \
        if (rot_dim == 0) FH3_QK_REG(SB, DB, 0);                 \
        else if (rot_dim == 96) FH3_QK_REG(SB, DB, 48);          \
        else FH3_QK_REG(SB, DB, 64);                             \
    } while (0)
        if (src_bf16) {
            if (dst_bf16) FH3_QK_REG_ROT(true, true);
            else FH3_QK_REG_ROT(true, false);
        } else {
            if (dst_bf16) FH3_QK_REG_ROT(false, true);
            else FH3_QK_REG_ROT(false, false);
        }
#undef FH3_QK_REG_ROT
#undef FH3_QK_REG
        return check_cuda(cudaGetLastError(), "qk_norm_rope launch");
    }
#define FH3_QK_LAUNCH(SB, DB)                                                                              \
    qk_norm_rope_kernel<SB, DB><<<grid, kQkThreads, smem, s>>>(src, ld_src, dst, ld_dst, norm_w, cos_t, sin_t, \
                                                               nvec, heads, head_dim, rot_dim, eps)
    if (src_bf16) {
        if (dst_bf16) FH3_QK_LAUNCH(true, true);
        else FH3_QK_LAUNCH(true, false);
    } else {
        if (dst_bf16) FH3_QK_LAUNCH(false, true);
        else FH3_QK_LAUNCH(false, false);
    }
#undef FH3_QK_LAUNCH
    return check_cuda(cudaGetLastError(), "qk_norm_rope launch");
}

extern "C" int fh3cuda_f32_to_bf16_dev(const float* x, void* y, int64_t n, void* stream) {
    using namespace fh3host;
    if (!ctx()) return set_error(FH3CUDA_E_NODEV, "fh3cuda_f32_to_bf16_dev: call fh3cuda_init first");
    if (!x || !y || n < 0) return set_error(FH3_E_INVALID, "fh3cuda_f32_to_bf16_dev: bad arguments");
    if (n == 0) return FH3_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int64_t n4 = 0;
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 7) == 0) {
        n4 = n / 4;
        if (n4 > 0)
            f32_to_bf16_kernel<<<grid_for(n4, 256), 256, 0, s>>>(reinterpret_cast<const float4*>(x),
                                                                  static_cast<uint2*>(y), n4);
    }
    const int64_t start = n4 * 4;
    if (start < n)
        f32_to_bf16_tail_kernel<<<static_cast<unsigned>((n - start + 255) / 256), 256, 0, s>>>(
            x, static_cast<__nv_bfloat16*>(y), start, n);
    return check_cuda(cudaGetLastError(), "f32_to_bf16 launch");
}

extern "C" int fh3cuda_rmsnorm_modulate_dev(const float* x, const float* norm_w, const float* shift,
                                            const float* scale, void* y_bf16, int n, int dim, float eps,
                                            void* stream) {
    using namespace fh3host;
    if (!ctx()) return set_error(FH3CUDA_E_NODEV, "fh3cuda_rmsnorm_modulate_dev: call fh3cuda_init first");
    if (!x || !shift || !scale || !y_bf16 || n <= 0 || dim <= 0)
        return set_error(FH3_E_INVALID, "fh3cuda_rmsnorm_modulate_dev: bad arguments");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const bool vec = (dim % 4) == 0 && al16(x) && al16(shift) && al16(scale) && (!norm_w || al16(norm_w)) &&
                     (reinterpret_cast<uintptr_t>(y_bf16) & 7) == 0;
    const int dim4 = dim / 4;
    const float inv_dim = 1.0f / static_cast<float>(dim);
    // a programmatic dependent of the previous kernel (the kernels wait before reading x)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(n), 1, 1);
    cfg.blockDim = dim3(kNormThreads, 1, 1);
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    const auto* x4 = reinterpret_cast<const float4*>(x);
    const auto* w4 = reinterpret_cast<const float4*>(norm_w);
    const auto* sh4 = reinterpret_cast<const float4*>(shift);
    const auto* sc4 = reinterpret_cast<const float4*>(scale);
    auto* y2 = static_cast<uint2*>(y_bf16);
    cudaError_t e;
    if (vec && dim4 <= 2 * kNormThreads)
        e = cudaLaunchKernelEx(&cfg, rmsnorm_modulate_vec_kernel<2>, x4, w4, sh4, sc4, y2, dim4, inv_dim, eps);
    else if (vec && dim4 <= 5 * kNormThreads)
        e = cudaLaunchKernelEx(&cfg, rmsnorm_modulate_vec_kernel<5>, x4, w4, sh4, sc4, y2, dim4, inv_dim, eps);
    else if (vec && dim4 <= 8 * kNormThreads)
        e = cudaLaunchKernelEx(&cfg, rmsnorm_modulate_vec_kernel<8>, x4, w4, sh4, sc4, y2, dim4, inv_dim, eps);
    else
        e = cudaLaunchKernelEx(&cfg, rmsnorm_modulate_kernel, x, norm_w, shift, scale,
                               static_cast<__nv_bfloat16*>(y_bf16), dim, eps);
    return check_cuda(e, "rmsnorm_modulate launch");
}

extern "C" int fh3cuda_swiglu_dev(const float* in, float* out, int n, int F, void* stream) {
    using namespace fh3host;
    if (!ctx()) return set_error(FH3CUDA_E_NODEV, "fh3cuda_swiglu_dev: call fh3cuda_init first");
    if (!in || !out || n <= 0 || F <= 0) return set_error(FH3_E_INVALID, "fh3cuda_swiglu_dev: bad arguments");
    const int64_t total = static_cast<int64_t>(n) * F;
    swiglu_kernel<<<grid_for(total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(in, out, n, F);
    return check_cuda(cudaGetLastError(), "swiglu launch");
}
