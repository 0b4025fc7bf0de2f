// ops.cu -- the elementwise work around the GEMMs of a DiT block.
//
//   fh3cuda_f32_to_bf16_dev       activations fp32 -> bf16 (GEMM A operand)
//   fh3cuda_rmsnorm_modulate_dev  GEMM prologue: rmsnorm (src/core/fh3_ops.c:410-456)
//                                 then modulate (:529-557), written as bf16
//   fh3cuda_swiglu_dev            fh3_swiglu (:507-527) on fp32 (the unfused form;
//                                 the GEMM has it as an epilogue)
// All HBM-bound streaming kernels with 16-byte accesses.
#include "common.cuh"

namespace {

__global__ void f32_to_bf16_kernel(const float4* __restrict__ x, uint2* __restrict__ y, int64_t n4) {
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

__global__ void __launch_bounds__(kNormThreads) rmsnorm_modulate_kernel(
    const float* __restrict__ x, const float* __restrict__ nw, const float* __restrict__ shift,
    const float* __restrict__ scale, __nv_bfloat16* __restrict__ y, int dim, float eps) {
    __shared__ float red[kNormThreads / 32];
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

}  // namespace

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
    rmsnorm_modulate_kernel<<<n, kNormThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        x, norm_w, shift, scale, static_cast<__nv_bfloat16*>(y_bf16), dim, eps);
    return check_cuda(cudaGetLastError(), "rmsnorm_modulate launch");
}

extern "C" int fh3cuda_swiglu_dev(const float* in, float* out, int n, int F, void* stream) {
    using namespace fh3host;
    if (!ctx()) return set_error(FH3CUDA_E_NODEV, "fh3cuda_swiglu_dev: call fh3cuda_init first");
    if (!in || !out || n <= 0 || F <= 0) return set_error(FH3_E_INVALID, "fh3cuda_swiglu_dev: bad arguments");
    const int64_t total = static_cast<int64_t>(n) * F;
    swiglu_kernel<<<grid_for(total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(in, out, n, F);
    return check_cuda(cudaGetLastError(), "swiglu launch");
}
