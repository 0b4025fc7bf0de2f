// api.cu -- libfh3cuda's host side: per-device contexts, error reporting,
// the weight registry, the device-pointer dispatcher and the host-pointer
// drop-in for fh3_matmul (include/fh3/fh3.h:107, src/core/fh3_ops.c:317-404).
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace fh3host {

// scratch slots: 0 bf16 activations of the GEMM, 1 staged weights, 2-4 the host
// drop-in's x / y / bias, 5 GEMV fragments, 6 split-tile partials, 7 tile counters,
// 8 split-bf16 weight rows of the non-Q4_K formats, 9 video sparse attention's tile data,
// 10 the DiT forward's activations, 11 bf16 weights of the two-pass large-M GEMM,
// 12 the transposed V of the tensor-core attention, 13 video sparse attention's tile-order
// copies of q, k and v, 14 / 15 the tcgen05 GEMV's split-tile partials and counters,
// 16 the fused GEMM's split-K partials, 17 the unit gate that adds the K slices of the
// non-Q4_K formats' GEMM
constexpr int kScratchSlots = 18;

struct DevCtx {
    int device = -1;
    int sms = 0;
    int* d_status = nullptr;      // written by bounded device-side waits
    cudaStream_t stream = nullptr; // the drop-in's stream
    void* scratch_ptr[kScratchSlots] = {};
    size_t scratch_size[kScratchSlots] = {};
};

namespace {
constexpr int kMaxDev = 64;
DevCtx* g_ctx[kMaxDev] = {};
std::mutex g_mu;
thread_local char g_msg[512] = "";
thread_local int g_sticky = FH3_OK;

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn g_encode = nullptr;

struct Region {
    const uint8_t* host;
    size_t bytes;
    const uint8_t* dev;
    bool owned;
};
std::vector<Region> g_regions;
}  // namespace

DevCtx* ctx() {
    int d = -1;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDev) return nullptr;
    return g_ctx[d];
}
int* ctx_status(DevCtx* c) { return c ? c->d_status : nullptr; }
int ctx_sms(DevCtx* c) { return c ? c->sms : 0; }
int ctx_device(DevCtx* c) { return c ? c->device : -1; }

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    return code;
}

int check_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return FH3_OK;
    return set_error(FH3CUDA_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

CUresult encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, cuuint32_t rank, void* gaddr,
                      const cuuint64_t* gdim, const cuuint64_t* gstride, const cuuint32_t* box,
                      const cuuint32_t* estride, CUtensorMapSwizzle swz) {
    if (!g_encode) return CUDA_ERROR_NOT_INITIALIZED;
    return g_encode(map, dtype, rank, gaddr, gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

namespace {
std::atomic<uint64_t> g_alloc_calls{0};      // cudaMalloc calls made by the library
std::atomic<uint64_t> g_scratch_held{0};     // bytes of scratch held, all devices
std::atomic<uint64_t> g_scratch_limit{0};    // 0 = unlimited
}  // namespace

int dev_alloc(void** p, size_t bytes, bool limited, const char* who) {
    *p = nullptr;
    if (limited) {
        const uint64_t lim = g_scratch_limit.load();
        const uint64_t held = g_scratch_held.load();
        if (lim != 0 && held + bytes > lim)
            return set_error(FH3_E_NOMEM, "%s: %zu bytes of scratch would exceed the limit of %llu (%llu held)", who,
                             bytes, static_cast<unsigned long long>(lim), static_cast<unsigned long long>(held));
    }
    g_alloc_calls.fetch_add(1);
    if (cudaMalloc(p, bytes) != cudaSuccess) {
        cudaGetLastError();  // a failed cudaMalloc leaves no sticky error; clear the last-error slot
        *p = nullptr;
        return set_error(FH3_E_NOMEM, "%s: cudaMalloc(%zu) failed", who, bytes);
    }
    if (limited) g_scratch_held.fetch_add(bytes);
    return FH3_OK;
}

void dev_free(void* p, size_t bytes, bool limited) {
    if (!p) return;
    cudaFree(p);
    if (limited) g_scratch_held.fetch_sub(bytes);
}

void* scratch(DevCtx* c, int slot, size_t bytes, cudaStream_t s) {
    if (!c || slot < 0 || slot >= kScratchSlots) return nullptr;
    if (c->scratch_size[slot] >= bytes && c->scratch_ptr[slot]) return c->scratch_ptr[slot];
    // grow: earlier work on this stream may still read the old buffer
    if (c->scratch_ptr[slot]) {
        cudaStreamSynchronize(s);
        dev_free(c->scratch_ptr[slot], c->scratch_size[slot], true);
        c->scratch_ptr[slot] = nullptr;
        c->scratch_size[slot] = 0;
    }
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    void* p = nullptr;
    if (dev_alloc(&p, want, true, "scratch") != FH3_OK) return nullptr;
    c->scratch_ptr[slot] = p;
    c->scratch_size[slot] = want;
    return p;
}

void* scratch_zeroed(DevCtx* c, int slot, size_t bytes, cudaStream_t s) {
    if (!c || slot < 0 || slot >= kScratchSlots) return nullptr;
    const void* before = c->scratch_ptr[slot];
    const size_t size_before = c->scratch_size[slot];
    void* p = scratch(c, slot, bytes, s);
    if (p && (p != before || c->scratch_size[slot] != size_before)) {
        if (check_cuda(cudaMemsetAsync(p, 0, c->scratch_size[slot], s), "scratch_zeroed: memset")) return nullptr;
    }
    return p;
}

}  // namespace fh3host

using namespace fh3host;

extern "C" int fh3cuda_init(int device) {
    std::lock_guard<std::mutex> lk(g_mu);
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0)
        return set_error(FH3CUDA_E_NODEV, "fh3cuda_init: no CUDA device");
    if (device < 0 || device >= n || device >= kMaxDev)
        return set_error(FH3_E_INVALID, "fh3cuda_init: device %d out of range (%d devices)", device, n);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return check_cuda(e, "cudaSetDevice");
    if (g_ctx[device]) return FH3_OK;
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return check_cuda(e, "cudaGetDeviceProperties");
    if (prop.major != 10)
        return set_error(FH3CUDA_E_NODEV, "fh3cuda_init: device %d is sm_%d%d; this library is built for sm_100a",
                         device, prop.major, prop.minor);
    if (!g_encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
            return set_error(FH3CUDA_E_CUDA, "fh3cuda_init: cuTensorMapEncodeTiled unavailable");
        g_encode = reinterpret_cast<EncodeFn>(fn);
    }
    DevCtx* c = new DevCtx();
    c->device = device;
    c->sms = prop.multiProcessorCount;
    void* st = nullptr;
    if (dev_alloc(&st, sizeof(int) * 4, false, "fh3cuda_init") != FH3_OK) {
        delete c;
        return FH3_E_NOMEM;
    }
    c->d_status = static_cast<int*>(st);
    e = cudaMemset(c->d_status, 0, sizeof(int) * 4);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete c;
        return check_cuda(e, "fh3cuda_init");
    }
    g_ctx[device] = c;
    return FH3_OK;
}

extern "C" const char* fh3cuda_last_error(void) { return g_msg; }

extern "C" int fh3cuda_take_status(void) {
    const int s = g_sticky;
    g_sticky = FH3_OK;
    return s;
}

extern "C" int fh3cuda_sm_count(void) { return ctx_sms(ctx()); }

extern "C" void fh3cuda_set_scratch_limit(uint64_t bytes) { g_scratch_limit.store(bytes); }

namespace fh3selftest {
// One CTA of one thread: an mbarrier that expects one arrival nobody makes, waited on
// with the library's bounded wait (the routine every kernel's waits use) under
// `limit_ns`.  Nothing else is in flight, so the kernel simply returns when the wait
// gives up; the status word then holds FH3CUDA_E_TIMEOUT.
__global__ void wait_selftest_kernel(uint64_t limit_ns, int* status, int* gave_up) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    fh3::mbar_init(&bar, 1);
    abort_flag = 0;
    fh3::fence_mbar_init();
    const bool ok = fh3::mbar_wait_for(&bar, 0u, &abort_flag, status, limit_ns);
    *gave_up = ok ? 0 : 1;
}
}  // namespace fh3selftest

extern "C" int fh3cuda_wait_selftest_dev(uint64_t limit_ns, void* stream) {
    DevCtx* c = ctx();
    if (!c) return set_error(FH3CUDA_E_NODEV, "fh3cuda_wait_selftest_dev: call fh3cuda_init first");
    if (limit_ns == 0 || limit_ns > 2000000000ull)
        return set_error(FH3_E_INVALID, "fh3cuda_wait_selftest_dev: limit must be in (0, 2 s]");
    // the flag lives in the status block's second word (allocated at set-up)
    fh3selftest::wait_selftest_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, c->d_status, c->d_status + 1);
    return check_cuda(cudaGetLastError(), "wait_selftest_kernel launch");
}

extern "C" void fh3cuda_alloc_stats(uint64_t* alloc_calls, uint64_t* scratch_bytes) {
    if (alloc_calls) *alloc_calls = g_alloc_calls.load();
    if (scratch_bytes) *scratch_bytes = g_scratch_held.load();
}

extern "C" int fh3cuda_device_status(void* stream) {
    DevCtx* c = ctx();
    if (!c) return set_error(FH3CUDA_E_NODEV, "fh3cuda_device_status: call fh3cuda_init first");
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return check_cuda(e, "fh3cuda_device_status: stream");
    int v = 0;
    e = cudaMemcpy(&v, c->d_status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return check_cuda(e, "fh3cuda_device_status: read");
    if (v != 0) {
        cudaMemset(c->d_status, 0, sizeof(int));
        return set_error(v, "device-side wait gave up (status %d)", v);
    }
    return FH3_OK;
}

extern "C" size_t fh3cuda_row_bytes(int type, int64_t n) {
    // fh3_row_bytes (src/core/fh3_quant.c:14-34) for the formats fh3_dequant expands
    if (n <= 0) return 0;
    switch (type) {
        case FH3CUDA_TYPE_F32: return static_cast<size_t>(n) * 4;
        case FH3CUDA_TYPE_F16:
        case FH3CUDA_TYPE_BF16: return static_cast<size_t>(n) * 2;
        case FH3CUDA_TYPE_Q8_0: return static_cast<size_t>((n + 31) / 32) * 34;
        case FH3CUDA_TYPE_Q2_K: return static_cast<size_t>((n + 255) / 256) * 84;
        case FH3CUDA_TYPE_Q3_K: return static_cast<size_t>((n + 255) / 256) * 110;
        case FH3CUDA_TYPE_Q4_K: return static_cast<size_t>((n + 255) / 256) * fh3::kQ4KBytes;
        case FH3CUDA_TYPE_Q5_K: return static_cast<size_t>((n + 255) / 256) * 176;
        case FH3CUDA_TYPE_Q6_K: return static_cast<size_t>((n + 255) / 256) * 210;
        default: return 0;
    }
}


extern "C" int fh3cuda_matmul_dev(const Fh3CudaW* w, const float* x, float* y, int n_tok,
                                  const float* bias, void* stream) {
    DevCtx* c = ctx();
    if (!c) return set_error(FH3CUDA_E_NODEV, "fh3cuda_matmul_dev: call fh3cuda_init first");
    if (!w || !x || !y || !w->data || n_tok <= 0 || w->in <= 0 || w->out <= 0)
        return set_error(FH3_E_INVALID, "fh3cuda_matmul_dev: bad arguments");
    if (w->type != FH3CUDA_TYPE_Q4_K)
        return matmul_formats(c, w, x, y, n_tok, bias, static_cast<cudaStream_t>(stream));
    if ((w->in % fh3::kQ4KBlock) != 0)
        return set_error(FH3_E_INVALID, "fh3cuda_matmul_dev: Q4_K weights need in %% 256 == 0");
    if (n_tok <= 16) return fh3cuda_gemv_q4k_dev(w, x, y, n_tok, bias, stream);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t abytes = static_cast<size_t>(n_tok) * static_cast<size_t>(w->in) * 2;
    void* xa = scratch(c, 0, abytes, s);
    if (!xa) return FH3_E_NOMEM;
    int rc = fh3cuda_f32_to_bf16_dev(x, xa, static_cast<int64_t>(n_tok) * w->in, stream);
    if (rc != FH3_OK) return rc;
    return fh3cuda_gemm_q4k_dev(w, xa, w->in, y, w->out, n_tok, bias, nullptr, FH3CUDA_EPI_F32, stream);
}

extern "C" int fh3cuda_register_weights(const void* host, size_t bytes, const void* dev) {
    if (!host || !dev || bytes == 0) return set_error(FH3_E_INVALID, "fh3cuda_register_weights: bad arguments");
    std::lock_guard<std::mutex> lk(g_mu);
    const uint8_t* h = static_cast<const uint8_t*>(host);
    for (const Region& r : g_regions)
        if (h < r.host + r.bytes && r.host < h + bytes)
            return set_error(FH3_E_INVALID, "fh3cuda_register_weights: range overlaps a registered range");
    g_regions.push_back({h, bytes, static_cast<const uint8_t*>(dev), false});
    return FH3_OK;
}

extern "C" int fh3cuda_unregister_weights(const void* host) {
    std::lock_guard<std::mutex> lk(g_mu);
    for (size_t i = 0; i < g_regions.size(); ++i)
        if (g_regions[i].host == host && !g_regions[i].owned) {
            g_regions.erase(g_regions.begin() + static_cast<long>(i));
            return FH3_OK;
        }
    return set_error(FH3_E_INVALID, "fh3cuda_unregister_weights: not a registered (borrowed) range");
}

extern "C" int fh3cuda_upload_weights(const void* host, size_t bytes, void** dev_out) {
    if (!host || bytes == 0 || !dev_out) return set_error(FH3_E_INVALID, "fh3cuda_upload_weights: bad arguments");
    if (!ctx()) return set_error(FH3CUDA_E_NODEV, "fh3cuda_upload_weights: call fh3cuda_init first");
    void* d = nullptr;
    if (dev_alloc(&d, bytes, false, "fh3cuda_upload_weights") != FH3_OK) return FH3_E_NOMEM;
    cudaError_t e = cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(d);
        return check_cuda(e, "fh3cuda_upload_weights: copy");
    }
    int rc = fh3cuda_register_weights(host, bytes, d);
    if (rc != FH3_OK) {
        cudaFree(d);
        return rc;
    }
    {
        std::lock_guard<std::mutex> lk(g_mu);
        g_regions.back().owned = true;
    }
    *dev_out = d;
    return FH3_OK;
}

extern "C" int fh3cuda_release_weights(const void* host) {
    std::lock_guard<std::mutex> lk(g_mu);
    for (size_t i = 0; i < g_regions.size(); ++i)
        if (g_regions[i].host == host && g_regions[i].owned) {
            cudaFree(const_cast<uint8_t*>(g_regions[i].dev));
            g_regions.erase(g_regions.begin() + static_cast<long>(i));
            return FH3_OK;
        }
    return set_error(FH3_E_INVALID, "fh3cuda_release_weights: not an uploaded range");
}

namespace {

const uint8_t* lookup_weights(const uint8_t* host, size_t bytes) {
    std::lock_guard<std::mutex> lk(g_mu);
    for (const Region& r : g_regions)
        if (host >= r.host && host + bytes <= r.host + r.bytes) return r.dev + (host - r.host);
    return nullptr;
}

int matmul_host(const Fh3CudaW* w, const float* x, float* y, int n_tok, const float* bias) {
    DevCtx* c = ctx();
    if (!c) {
        // an unmodified fh3 caller relinked onto the drop-in never calls fh3cuda_init: set up
        // the calling thread's current device (device 0 unless the caller chose another)
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
        const int rc = fh3cuda_init(dev);
        if (rc != FH3_OK) return rc;
        c = ctx();
        if (!c) return set_error(FH3CUDA_E_NODEV, "fh3_matmul drop-in: no device context");
    }
    // fh3_matmul returns silently on these (src/core/fh3_ops.c:318-321); report them instead
    if (!w || !x || !y || !w->data || n_tok <= 0 || w->in <= 0 || w->out <= 0)
        return set_error(FH3_E_INVALID, "fh3_matmul drop-in: bad arguments");
    if (fh3cuda_row_bytes(w->type, w->in) == 0)
        return set_error(FH3_E_INVALID, "fh3_matmul drop-in: weight type %d is not a format fh3_dequant expands",
                         w->type);
    cudaStream_t s = c->stream;
    const size_t wbytes = static_cast<size_t>(w->out) * fh3cuda_row_bytes(w->type, w->in);
    const size_t xbytes = static_cast<size_t>(n_tok) * static_cast<size_t>(w->in) * 4;
    const size_t ybytes = static_cast<size_t>(n_tok) * static_cast<size_t>(w->out) * 4;
    const uint8_t* dw = lookup_weights(w->data, wbytes);
    if (!dw) {
        void* stage = scratch(c, 1, wbytes, s);
        if (!stage) return FH3_E_NOMEM;
        int rc = check_cuda(cudaMemcpyAsync(stage, w->data, wbytes, cudaMemcpyHostToDevice, s), "stage weights");
        if (rc) return rc;
        dw = static_cast<const uint8_t*>(stage);
    }
    void* dx = scratch(c, 2, xbytes, s);
    void* dy = scratch(c, 3, ybytes, s);
    void* db = bias ? scratch(c, 4, static_cast<size_t>(w->out) * 4, s) : nullptr;
    if (!dx || !dy || (bias && !db)) return FH3_E_NOMEM;
    int rc = check_cuda(cudaMemcpyAsync(dx, x, xbytes, cudaMemcpyHostToDevice, s), "copy x");
    if (!rc && bias) rc = check_cuda(cudaMemcpyAsync(db, bias, static_cast<size_t>(w->out) * 4,
                                                     cudaMemcpyHostToDevice, s), "copy bias");
    if (rc) return rc;
    Fh3CudaW dwd = *w;
    dwd.data = dw;
    rc = fh3cuda_matmul_dev(&dwd, static_cast<const float*>(dx), static_cast<float*>(dy), n_tok,
                            static_cast<const float*>(db), s);
    if (rc) return rc;
    rc = check_cuda(cudaMemcpyAsync(y, dy, ybytes, cudaMemcpyDeviceToHost, s), "copy y");
    if (rc) return rc;
    return fh3cuda_device_status(s);
}

}  // namespace

extern "C" void fh3cuda_matmul(const Fh3CudaW* w, const float* x, float* y, int n_tok, const float* bias) {
    const int rc = matmul_host(w, x, y, n_tok, bias);
    if (rc != FH3_OK) {
        if (g_sticky == FH3_OK) {
            g_sticky = rc;
            fprintf(stderr, "fh3cuda_matmul: %s (status %d)\n", g_msg, rc);
        }
    }
}

extern "C" void __wrap_fh3_matmul(const Fh3CudaW* w, const float* x, float* y, int n_tok, const float* bias) {
    fh3cuda_matmul(w, x, y, n_tok, bias);
}
