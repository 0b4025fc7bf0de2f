// trunk_io.cu -- the packed DiT trunk (FH3P) and the folded AdaLN table (FH3A),
// read once and kept resident in HBM.
//
// fh3 streams trunk layers from NVMe through a ring of pinned slots
// (src/io/fh3_trunk.c:135-501, fh3_pack_open src/io/fh3_pack.c:23-106).  On a B200
// the whole trunk (11.9 GB for the 50-block model) fits next to the activations, so
// fh3cuda_pack_open reads the file once -- header, layer index, then each 4096-byte
// aligned layer run through two pinned bounce buffers, disk reads overlapping the
// host->device copies -- into one device allocation, and layer views are device
// pointers into it.  The AdaLN table (fh3_adaln_open, src/io/fh3_pack.c:188-290) is
// uploaded the same way and rows are addressed as fh3_adaln_row does (:311-355).
//
// On-disk layouts (little-endian, packed), as src/io/fh3_pack.h:29-88 defines them:
//   FH3P header (128 B): magic 'FH3P', version 1, num_layers, layer_alignment 4096,
//     index_offset, index_bytes, data_offset, total_bytes (u64), 80 reserved bytes.
//   layer descriptor (index_bytes / num_layers bytes each): file_offset, size_bytes
//     (u64), n_tensors, reserved (u32), then n_tensors tensor descriptors of 168 B:
//     name[64], type, n_dims (u32), shape[4] (i64), offset_in_layer, size_bytes
//     (u64), in_dim, out_dim (i64), 32 reserved bytes.  Tensor order in a layer:
//     qkv, gate_compress, out, fc1, fc2, norm1, norm2, q_norm, k_norm.
//   FH3A header (128 B): magic 'FH3A', version 1, n_steps, n_blocks, pairs_per_step,
//     hidden_size (u32), schedule_hash, trunk_offset, trunk_bytes, final_offset,
//     final_bytes (u64), 64 reserved bytes.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <memory>
#include <vector>

#include "common.cuh"

namespace {

constexpr uint32_t kPackMagic = 0x50334846u;   // 'FH3P'
constexpr uint32_t kAdalnMagic = 0x41334846u;  // 'FH3A'
constexpr uint32_t kFormatVersion = 1u;
constexpr uint32_t kPackAlignment = 4096u;
constexpr int kLayerTensors = 9;
constexpr int kMaxLayerTensors = 16;
constexpr size_t kHeaderBytes = 128;
constexpr size_t kLayerDescBytes = 24;
constexpr size_t kTensorDescBytes = 168;
constexpr size_t kBounceBytes = 64u << 20;  // one pinned bounce buffer

template <typename T>
T rd(const uint8_t* p) {
    T v;
    std::memcpy(&v, p, sizeof(T));
    return v;
}

// a file opened for pread; closes itself
struct File {
    int fd = -1;
    uint64_t size = 0;
    ~File() {
        if (fd >= 0) close(fd);
    }
    int open_read(const char* path) {
        fd = ::open(path, O_RDONLY);
        if (fd < 0) return FH3_E_IO;
        struct stat st;
        if (fstat(fd, &st) != 0) return FH3_E_IO;
        size = static_cast<uint64_t>(st.st_size);
        return FH3_OK;
    }
    // reads exactly n bytes at off
    bool read_at(void* dst, size_t n, uint64_t off) const {
        uint8_t* d = static_cast<uint8_t*>(dst);
        while (n > 0) {
            const ssize_t r = pread(fd, d, n, static_cast<off_t>(off));
            if (r <= 0) return false;
            d += r;
            n -= static_cast<size_t>(r);
            off += static_cast<uint64_t>(r);
        }
        return true;
    }
};

// Copies file bytes [off, off + n) to device memory through two pinned bounce
// buffers: the read of chunk c+1 overlaps the copy of chunk c.
int upload_range(const File& f, uint64_t off, uint64_t n, uint8_t* dev, uint8_t* const bounce[2],
                 cudaEvent_t const done[2], cudaStream_t s) {
    using namespace fh3host;
    int b = 0;
    for (uint64_t pos = 0; pos < n; pos += kBounceBytes, b ^= 1) {
        const size_t len = static_cast<size_t>(n - pos < kBounceBytes ? n - pos : kBounceBytes);
        int rc = check_cuda(cudaEventSynchronize(done[b]), "upload: bounce buffer wait");
        if (rc) return rc;
        if (!f.read_at(bounce[b], len, off + pos)) return set_error(FH3_E_IO, "upload: read failed");
        rc = check_cuda(cudaMemcpyAsync(dev + pos, bounce[b], len, cudaMemcpyHostToDevice, s), "upload: copy");
        if (!rc) rc = check_cuda(cudaEventRecord(done[b], s), "upload: event");
        if (rc) return rc;
    }
    return FH3_OK;
}

// two pinned bounce buffers and their events for one upload
struct Bounce {
    uint8_t* buf[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    int init() {
        using namespace fh3host;
        for (int i = 0; i < 2; ++i) {
            if (cudaMallocHost(&buf[i], kBounceBytes) != cudaSuccess)
                return set_error(FH3_E_NOMEM, "upload: pinned bounce buffer");
            int rc = check_cuda(cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming), "upload: event");
            if (!rc) rc = check_cuda(cudaEventRecord(ev[i], nullptr), "upload: event");
            if (rc) return rc;
        }
        return FH3_OK;
    }
    ~Bounce() {
        for (int i = 0; i < 2; ++i) {
            if (ev[i]) {
                cudaEventSynchronize(ev[i]);
                cudaEventDestroy(ev[i]);
            }
            if (buf[i]) cudaFreeHost(buf[i]);
        }
    }
};

}  // namespace

struct Fh3CudaPack {
    struct Tensor {
        uint32_t type;
        int64_t in_dim, out_dim;
        uint64_t offset, size;  // within the layer run
    };
    struct Layer {
        uint64_t file_off, dev_off, size;
        Tensor t[kLayerTensors];
    };
    int device = -1;
    uint8_t* dev = nullptr;  // every layer run, back to back (4096-byte aligned)
    uint64_t bytes = 0;
    std::vector<Layer> layers;
    ~Fh3CudaPack() {
        if (dev) {
            int cur = -1;
            cudaGetDevice(&cur);
            if (device >= 0 && cur != device) cudaSetDevice(device);
            cudaFree(dev);
            if (device >= 0 && cur >= 0 && cur != device) cudaSetDevice(cur);
        }
    }
};

extern "C" int fh3cuda_pack_open(const char* path, Fh3CudaPack** out) {
    using namespace fh3host;
    const char* who = "fh3cuda_pack_open";
    if (!path || !out) return set_error(FH3_ERR, "%s: bad arguments", who);
    *out = nullptr;
    File f;
    if (f.open_read(path)) return set_error(FH3_E_IO, "%s: cannot open %s", who, path);
    if (f.size < kHeaderBytes) return set_error(FH3_E_TRUNCATED, "%s: %s shorter than its header", who, path);
    uint8_t hdr[kHeaderBytes];
    if (!f.read_at(hdr, kHeaderBytes, 0)) return set_error(FH3_E_IO, "%s: header read failed", who);
    if (rd<uint32_t>(hdr) != kPackMagic) return set_error(FH3_E_BAD_MAGIC, "%s: not an FH3P file", who);
    if (rd<uint32_t>(hdr + 4) != kFormatVersion) return set_error(FH3_E_BAD_VERSION, "%s: FH3P version", who);
    const uint32_t nl = rd<uint32_t>(hdr + 8);
    if (rd<uint32_t>(hdr + 12) != kPackAlignment || nl == 0)
        return set_error(FH3_E_INVALID, "%s: layer alignment must be 4096 and layers > 0", who);
    const uint64_t index_offset = rd<uint64_t>(hdr + 16), index_bytes = rd<uint64_t>(hdr + 24);
    const uint64_t desc_bytes = index_bytes / nl;
    if (desc_bytes < kLayerDescBytes || index_offset + index_bytes > f.size)
        return set_error(FH3_E_TRUNCATED, "%s: layer index outside the file", who);

    auto p = std::make_unique<Fh3CudaPack>();
    p->layers.resize(nl);
    std::vector<uint8_t> desc(kLayerDescBytes + kMaxLayerTensors * kTensorDescBytes);
    const size_t want = static_cast<size_t>(desc_bytes < desc.size() ? desc_bytes : desc.size());
    uint64_t dev_off = 0;
    for (uint32_t L = 0; L < nl; ++L) {
        if (!f.read_at(desc.data(), want, index_offset + L * desc_bytes))
            return set_error(FH3_E_IO, "%s: layer %u descriptor read failed", who, L);
        Fh3CudaPack::Layer& ly = p->layers[L];
        ly.file_off = rd<uint64_t>(desc.data());
        ly.size = rd<uint64_t>(desc.data() + 8);
        const uint32_t nt = rd<uint32_t>(desc.data() + 16);
        const size_t avail = (want - kLayerDescBytes) / kTensorDescBytes;
        if (nt < kLayerTensors || avail < kLayerTensors)
            return set_error(FH3_E_INVALID, "%s: layer %u holds %u tensors, 9 needed", who, L, nt);
        if (ly.file_off + ly.size > f.size) return set_error(FH3_E_TRUNCATED, "%s: layer %u past the file end", who, L);
        for (int t = 0; t < kLayerTensors; ++t) {
            const uint8_t* td = desc.data() + kLayerDescBytes + t * kTensorDescBytes;
            Fh3CudaPack::Tensor& x = ly.t[t];
            x.type = rd<uint32_t>(td + 64);
            x.offset = rd<uint64_t>(td + 104);
            x.size = rd<uint64_t>(td + 112);
            x.in_dim = rd<int64_t>(td + 120);
            x.out_dim = rd<int64_t>(td + 128);
            if (x.offset + x.size > ly.size)
                return set_error(FH3_E_INVALID, "%s: layer %u tensor %d outside its run", who, L, t);
        }
        ly.dev_off = dev_off;
        dev_off += (ly.size + kPackAlignment - 1) / kPackAlignment * kPackAlignment;
    }
    p->bytes = dev_off;
    if (!ctx()) return set_error(FH3CUDA_E_NODEV, "%s: call fh3cuda_init first", who);  // the file checks out
    p->device = ctx_device(ctx());
    {
        void* d = nullptr;
        if (dev_alloc(&d, p->bytes, false, who) != FH3_OK) return FH3_E_NOMEM;
        p->dev = static_cast<uint8_t*>(d);
    }
    Bounce bb;
    int rc = bb.init();
    for (uint32_t L = 0; L < nl && !rc; ++L)
        rc = upload_range(f, p->layers[L].file_off, p->layers[L].size, p->dev + p->layers[L].dev_off, bb.buf, bb.ev,
                          nullptr);
    if (!rc) rc = check_cuda(cudaStreamSynchronize(nullptr), "fh3cuda_pack_open: upload");
    if (rc) return rc;
    *out = p.release();
    return FH3_OK;
}

extern "C" int fh3cuda_pack_num_layers(const Fh3CudaPack* p) { return p ? static_cast<int>(p->layers.size()) : 0; }

extern "C" uint64_t fh3cuda_pack_device_bytes(const Fh3CudaPack* p) { return p ? p->bytes : 0; }

extern "C" int fh3cuda_pack_layer(const Fh3CudaPack* p, int L, Fh3CudaLayerView* out) {
    using namespace fh3host;
    if (!p || !out || L < 0 || L >= static_cast<int>(p->layers.size()))
        return set_error(FH3_E_INVALID, "fh3cuda_pack_layer: bad arguments");
    const Fh3CudaPack::Layer& ly = p->layers[L];
    Fh3CudaW* w[kLayerTensors] = {&out->qkv, &out->gate_compress, &out->out, &out->fc1, &out->fc2,
                                  &out->norm1, &out->norm2, &out->q_norm, &out->k_norm};
    for (int t = 0; t < kLayerTensors; ++t) {
        w[t]->type = static_cast<int>(ly.t[t].type);
        w[t]->in = ly.t[t].in_dim;
        w[t]->out = ly.t[t].out_dim;
        w[t]->data = p->dev + ly.dev_off + ly.t[t].offset;
    }
    return FH3_OK;
}

extern "C" void fh3cuda_pack_close(Fh3CudaPack* p) { delete p; }

struct Fh3CudaAdaln {
    int device = -1;
    float* dev = nullptr;  // trunk table then final-layer table
    int n_steps = 0, n_blocks = 0, pairs = 0, hidden = 0;
    uint64_t hash = 0;
    const float* trunk = nullptr;  // [n_steps][n_blocks][pairs][6][hidden]
    const float* fin = nullptr;    // [n_steps][pairs][2][hidden] (null when absent)
    ~Fh3CudaAdaln() {
        if (dev) {
            int cur = -1;
            cudaGetDevice(&cur);
            if (device >= 0 && cur != device) cudaSetDevice(device);
            cudaFree(dev);
            if (device >= 0 && cur >= 0 && cur != device) cudaSetDevice(cur);
        }
    }
};

extern "C" int fh3cuda_adaln_open(const char* path, uint64_t expect_hash, Fh3CudaAdaln** out) {
    using namespace fh3host;
    const char* who = "fh3cuda_adaln_open";
    if (!path || !out) return set_error(FH3_ERR, "%s: bad arguments", who);
    *out = nullptr;
    File f;
    if (f.open_read(path)) return set_error(FH3_E_IO, "%s: cannot open %s", who, path);
    if (f.size < kHeaderBytes) return set_error(FH3_E_TRUNCATED, "%s: %s shorter than its header", who, path);
    uint8_t hdr[kHeaderBytes];
    if (!f.read_at(hdr, kHeaderBytes, 0)) return set_error(FH3_E_IO, "%s: header read failed", who);
    if (rd<uint32_t>(hdr) != kAdalnMagic) return set_error(FH3_E_BAD_MAGIC, "%s: not an FH3A file", who);
    if (rd<uint32_t>(hdr + 4) != kFormatVersion) return set_error(FH3_E_BAD_VERSION, "%s: FH3A version", who);
    auto a = std::make_unique<Fh3CudaAdaln>();
    a->n_steps = static_cast<int>(rd<uint32_t>(hdr + 8));
    a->n_blocks = static_cast<int>(rd<uint32_t>(hdr + 12));
    a->pairs = static_cast<int>(rd<uint32_t>(hdr + 16));
    a->hidden = static_cast<int>(rd<uint32_t>(hdr + 20));
    a->hash = rd<uint64_t>(hdr + 24);
    if (expect_hash != 0 && a->hash != expect_hash)
        return set_error(FH3_E_INVALID, "%s: schedule hash does not match", who);
    const uint64_t trunk_off = rd<uint64_t>(hdr + 32), trunk_bytes = rd<uint64_t>(hdr + 40);
    const uint64_t final_off = rd<uint64_t>(hdr + 48), final_bytes = rd<uint64_t>(hdr + 56);
    if (trunk_off + trunk_bytes > f.size || final_off + final_bytes > f.size)
        return set_error(FH3_E_TRUNCATED, "%s: tables past the file end", who);
    const uint64_t trunk_need = static_cast<uint64_t>(a->n_steps) * a->n_blocks * a->pairs * 6 * a->hidden * 4;
    const uint64_t final_need = static_cast<uint64_t>(a->n_steps) * a->pairs * 2 * a->hidden * 4;
    if (trunk_bytes < trunk_need || (final_bytes > 0 && final_bytes < final_need))
        return set_error(FH3_E_TRUNCATED, "%s: tables smaller than their dimensions", who);
    if (!ctx()) return set_error(FH3CUDA_E_NODEV, "%s: call fh3cuda_init first", who);  // the file checks out
    a->device = ctx_device(ctx());
    const uint64_t trunk_alloc = (trunk_bytes + 255) & ~static_cast<uint64_t>(255);
    {
        void* d = nullptr;
        if (dev_alloc(&d, trunk_alloc + final_bytes + 4, false, who) != FH3_OK) return FH3_E_NOMEM;
        a->dev = static_cast<float*>(d);
    }
    Bounce bb;
    int rc = bb.init();
    uint8_t* base = reinterpret_cast<uint8_t*>(a->dev);
    if (!rc) rc = upload_range(f, trunk_off, trunk_bytes, base, bb.buf, bb.ev, nullptr);
    if (!rc && final_bytes > 0) rc = upload_range(f, final_off, final_bytes, base + trunk_alloc, bb.buf, bb.ev, nullptr);
    if (!rc) rc = check_cuda(cudaStreamSynchronize(nullptr), "fh3cuda_adaln_open: upload");
    if (rc) return rc;
    a->trunk = a->dev;
    a->fin = final_bytes > 0 ? reinterpret_cast<const float*>(base + trunk_alloc) : nullptr;
    *out = a.release();
    return FH3_OK;
}

extern "C" int fh3cuda_adaln_dims(const Fh3CudaAdaln* a, int* n_steps, int* n_blocks, int* pairs, int* hidden) {
    if (!a) return fh3host::set_error(FH3_E_INVALID, "fh3cuda_adaln_dims: null table");
    if (n_steps) *n_steps = a->n_steps;
    if (n_blocks) *n_blocks = a->n_blocks;
    if (pairs) *pairs = a->pairs;
    if (hidden) *hidden = a->hidden;
    return FH3_OK;
}

// fh3_adaln_row (src/io/fh3_pack.c:311-355): chunk 0..5 of a trunk block, or 0..1 of
// the final layer (block == n_blocks or -1); NULL outside the table
extern "C" const float* fh3cuda_adaln_row(const Fh3CudaAdaln* a, int step, int block, int pair, int chunk) {
    if (!a || step < 0 || step >= a->n_steps || pair < 0 || pair >= a->pairs) return nullptr;
    const size_t hid = static_cast<size_t>(a->hidden);
    if (block >= 0 && block < a->n_blocks) {
        if (chunk < 0 || chunk >= 6) return nullptr;
        return a->trunk + (((static_cast<size_t>(step) * a->n_blocks + block) * a->pairs + pair) * 6 + chunk) * hid;
    }
    if (block == a->n_blocks || block == -1) {
        if (chunk < 0 || chunk >= 2 || !a->fin) return nullptr;
        return a->fin + ((static_cast<size_t>(step) * a->pairs + pair) * 2 + chunk) * hid;
    }
    return nullptr;
}

extern "C" void fh3cuda_adaln_close(Fh3CudaAdaln* a) { delete a; }
