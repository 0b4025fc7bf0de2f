// attention.cu -- the dense-attention entry point (fh3_attention, src/core/fh3_ops.c:587-695):
// non-causal softmax attention for head_dim 128 on bf16 q/k/v with fp32 softmax and
// accumulation.  It checks the arguments and runs the tcgen05 kernel (attention_tc.cu).
//
// Operands: element (token i, head h, channel d) of q / k / v at
// base + i*ld + h*128 + d (bf16), o at o + i*ldo + h*128 + d (fp32 or bf16).
#include "common.cuh"

namespace {
constexpr int kHD = 128;  // head_dim
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
    return attention_tc(static_cast<const __nv_bfloat16*>(q), ldq, static_cast<const __nv_bfloat16*>(k), ldk,
                        static_cast<const __nv_bfloat16*>(v), ldv, o, o_bf16 != 0, ldo, n, heads,
                        static_cast<cudaStream_t>(stream));
}
