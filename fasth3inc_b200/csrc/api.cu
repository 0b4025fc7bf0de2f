// api.cu -- libfh3cuda's host side: per-device contexts, error reporting,
// the weight registry, the device-pointer dispatcher and the host-pointer
// drop-in for fh3_matmul (include/fh3/fh3.h:107, src/core/fh3_ops.c:317-404).
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace fh3host {

struct DevCtx {
    int device = -1;
    int sms = 0;
    int* d_status = nullptr;      // written by bounded device-side waits
    cudaStream_t stream = nullptr; // the drop-in's stream
    void* scratch_ptr[8] = {};
    size_t scratch_size[8] = {};
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

void* scratch(DevCtx* c, int slot, size_t bytes, cudaStream_t s) {
    if (!c || slot < 0 || slot >= 8) return nullptr;
    if (c->scratch_size[slot] >= bytes && c->scratch_ptr[slot]) return c->scratch_ptr[slot];
    // grow: earlier work on this stream may still read the old buffer
    if (c->scratch_ptr[slot]) {
        cudaStreamSynchronize(s);
        cudaFree(c->scratch_ptr[slot]);
        c->scratch_ptr[slot] = nullptr;
        c->scratch_size[slot] = 0;
    }
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    void* p = nullptr;
    if (cudaMalloc(&p, want) != cudaSuccess) {
        set_error(FH3_E_NOMEM, "scratch: cudaMalloc(%zu) failed", want);
        return nullptr;
    }
    c->scratch_ptr[slot] = p;
    c->scratch_size[slot] = want;
    return p;
}

void* scratch_zeroed(DevCtx* c, int slot, size_t bytes, cudaStream_t s) {
    if (!c || slot < 0 || slot >= 8) return nullptr;
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
    e = cudaMalloc(&c->d_status, sizeof(int) * 4);
    if (e == cudaSuccess) e = cudaMemset(c->d_status, 0, sizeof(int) * 4);
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
    // fh3_row_bytes (src/core/fh3_quant.c:14-34) for F32 (:17) and Q4_K (:27)
    if (n <= 0) return 0;
    if (type == FH3CUDA_TYPE_F32) return static_cast<size_t>(n) * 4;
    if (type == FH3CUDA_TYPE_Q4_K) return static_cast<size_t>((n + 255) / 256) * fh3::kQ4KBytes;
    return 0;
}

extern "C" int fh3cuda_matmul_dev(const Fh3CudaW* w, const float* x, float* y, int n_tok,
                                  const float* bias, void* stream) {
    DevCtx* c = ctx();
    if (!c) return set_error(FH3CUDA_E_NODEV, "fh3cuda_matmul_dev: call fh3cuda_init first");
    if (!w || !x || !y || !w->data || n_tok <= 0 || w->in <= 0 || w->out <= 0)
        return set_error(FH3_E_INVALID, "fh3cuda_matmul_dev: bad arguments");
    if (w->type != FH3CUDA_TYPE_Q4_K || (w->in % fh3::kQ4KBlock) != 0)
        return set_error(FH3_E_INVALID, "fh3cuda_matmul_dev: Q4_K weights with in %% 256 == 0 required (type %d)",
                         w->type);
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
    if (cudaMalloc(&d, bytes) != cudaSuccess) return set_error(FH3_E_NOMEM, "fh3cuda_upload_weights: cudaMalloc(%zu)", bytes);
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
    if (!c) return set_error(FH3CUDA_E_NODEV, "fh3_matmul drop-in: call fh3cuda_init first");
    // fh3_matmul returns silently on these (src/core/fh3_ops.c:318-321); report them instead
    if (!w || !x || !y || !w->data || n_tok <= 0 || w->in <= 0 || w->out <= 0)
        return set_error(FH3_E_INVALID, "fh3_matmul drop-in: bad arguments");
    if (w->type != FH3CUDA_TYPE_Q4_K || (w->in % fh3::kQ4KBlock) != 0)
        return set_error(FH3_E_INVALID, "fh3_matmul drop-in: only Q4_K weights with in %% 256 == 0 (type %d)",
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
