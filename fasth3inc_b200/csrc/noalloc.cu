// noalloc.cu -- fh3cuda_matmul_noalloc_dev: the device-pointer matmul without any
// device allocation on the call path.
//
// Who needs it: callers that cannot let a library call cudaMalloc while they run.
//   * An fh3 host that budgets device memory once, up front, the way fh3 budgets host
//     memory with its plan preflight (src/io/fh3_trunk.c:101-129): scratch that grows
//     behind its back breaks that budget, and an allocation failure mid-step has no
//     recovery.
//   * A process whose device memory belongs to another allocator (a caching allocator
//     that has already reserved the free memory): cudaMalloc would fail although the
//     caller's pool has room.
//   * Latency-critical loops: cudaMalloc/cudaFree may synchronise the device and stall
//     every stream, which is what fh3cuda_matmul_dev's scratch growth does.
//
// How: the bf16 copy of the activations (the GEMM's A operand) lives in a file-scope
// static __device__ array of kNoAllocMaxElems elements (8 MiB).  Every GPU that loads
// this library holds that array until the process exits.  Host code must not use the
// array's name as a device address (in host code it names a host-side stand-in); the
// address is fetched once per device with cudaGetSymbolAddress, on the first call of
// the entry point on that device (set-up: do that first call before any stream capture).
// fh3cuda_init(device) must have been called before (it is the library's set-up).
//
// Every call shares the array, which keeps the last call's contents.  Nothing needs
// clearing: a call overwrites elements [0, n_tok*in) before the GEMM reads them, and the
// GEMM's TMA never reads beyond n_tok rows (rows past the end are zero-filled by TMA, not
// read from the array).  Calls that overlap on the GPU (two streams, or two host threads
// on one device) race on the array: serialise them.
//
// The GEMM runs on the fused kernels at every row count (dequantisation in shared
// memory), never on the two-pass path that the allocating entry point takes from 2048
// rows: that path expands the weights into a bf16 copy in allocated scratch.  So
// FH3CUDA_GEMM_KERNEL=two-pass has no effect here, and large row counts trade the
// two-pass path's speed for the absence of scratch.  The cached symbol address is only
// valid for the CUDA context it was taken in; like the rest of the library's per-device
// state it does not survive cudaDeviceReset.
#include <mutex>

#include "common.cuh"

namespace {

constexpr int64_t kNoAllocMaxElems = int64_t(4) << 20;  // 4 Mi bf16 = 8 MiB

static __device__ __align__(256) __nv_bfloat16 g_noalloc_act[kNoAllocMaxElems];

constexpr int kMaxDev = 64;
void* g_act_addr[kMaxDev] = {};
std::mutex g_mu;

// Device address of g_noalloc_act on the current device (set-up on first use).
int act_scratch(void** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fh3host::check_cuda(e, "fh3cuda_matmul_noalloc_dev: cudaGetDevice");
    if (dev < 0 || dev >= kMaxDev) return fh3host::set_error(FH3_E_INVALID, "fh3cuda_matmul_noalloc_dev: device %d", dev);
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_act_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_act);
        if (e != cudaSuccess || !p)
            return fh3host::check_cuda(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                                       "fh3cuda_matmul_noalloc_dev: cudaGetSymbolAddress");
        g_act_addr[dev] = p;
    }
    *out = g_act_addr[dev];
    return FH3_OK;
}

}  // namespace

extern "C" int fh3cuda_matmul_noalloc_dev(const Fh3CudaW* w, const float* x, float* y, int n_tok,
                                          const float* bias, void* stream) {
    using namespace fh3host;
    if (!ctx()) return set_error(FH3CUDA_E_NODEV, "fh3cuda_matmul_noalloc_dev: call fh3cuda_init first");
    if (!w || !x || !y || !w->data || n_tok <= 0 || w->in <= 0 || w->out <= 0)
        return set_error(FH3_E_INVALID, "fh3cuda_matmul_noalloc_dev: bad arguments");
    if (w->type != FH3CUDA_TYPE_Q4_K || (w->in % fh3::kQ4KBlock) != 0)
        return set_error(FH3_E_INVALID, "fh3cuda_matmul_noalloc_dev: Q4_K weights with in %% 256 == 0 required");
    if (n_tok <= 16) {
        // the CUDA-core GEMV reads x and the weights and writes y, nothing else (the
        // default tensor-core GEMV stages activation fragments in allocated scratch)
        const int rc = gemv_args_ok(w, x, y, n_tok, "fh3cuda_matmul_noalloc_dev");
        if (rc != FH3_OK) return rc;
        return gemv_fp32(w, x, y, n_tok, bias, static_cast<cudaStream_t>(stream));
    }
    const int64_t elems = static_cast<int64_t>(n_tok) * w->in;
    if (elems > kNoAllocMaxElems)
        return set_error(FH3_E_INVALID,
                         "fh3cuda_matmul_noalloc_dev: n_tok * in = %lld exceeds the fixed scratch of %lld "
                         "elements (8 MiB of bf16); split the rows or use fh3cuda_matmul_dev",
                         static_cast<long long>(elems), static_cast<long long>(kNoAllocMaxElems));
    void* act = nullptr;
    int rc = act_scratch(&act);
    if (rc != FH3_OK) return rc;
    rc = fh3cuda_f32_to_bf16_dev(x, act, elems, stream);
    if (rc != FH3_OK) return rc;
    return gemm_q4k(w, act, w->in, y, w->out, n_tok, bias, nullptr, FH3CUDA_EPI_F32, stream, /*fused_only=*/true);
}
