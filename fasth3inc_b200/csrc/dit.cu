// dit.cu -- the DiT forward of fh3 on the device: fh3_dit_prepare_text and
// fh3_dit_forward (src/model/fh3_dit.c:221-467) chained from this library's entry
// points, with the trunk and the AdaLN table resident in HBM (trunk_io.cu).
//
// Per block, as the reference:  h -> rmsnorm(norm1) -> modulate(shift, scale of the
// row's modality pair) -> QKV -> per-head rmsnorm of q, k + rope3 (96 channels) ->
// attention (dense, or video sparse with the gate_compress projection) -> out proj ->
// h += gate * y; then rmsnorm(norm2) -> modulate -> fc1 -> swiglu -> fc2 -> h += gate * y.
// Final layer: rmsnorm(final_norm) -> modulate (final AdaLN rows) -> video / audio
// heads.  The text refiner has plain residuals and no modulation or rope.
//
// Activations are fp32 [rows][width] in one scratch slot.  A trunk block whose projections
// are all Q4_K, with bf16 tensor-core attention (cfg.attn_bf16 = 1), runs on bf16 operands
// with the GEMMs' fused prologue and epilogues (fused_block_run, the bench trunk's
// launches).  Otherwise projections go through fh3cuda_matmul_dev, so every weight format
// fh3 packs is served (F32 and the other formats on their paths), and attention runs in
// fp32 (cfg.attn_bf16 = 0: the CPU path's accuracy) or on bf16 tensor cores.
// Rows are ordered text | audio | video; AdaLN pair of a row: text 1, audio 2,
// video 0 (fh3_seq_build, src/model/fh3_seq.c:56-72).
#include <algorithm>

#include "common.cuh"

namespace {

constexpr int kDitThreads = 256;

// shift / scale (or gate) vectors of the three modality pairs, and the row bounds
struct PairRows {
    const float* a[3];  // indexed by pair: 0 video, 1 text, 2 audio
    const float* b[3];
    int T, A;           // rows [0, T) text, [T, T+A) audio, the rest video
};

__device__ __forceinline__ int row_pair(const PairRows& p, int row) {
    return row < p.T ? 1 : (row < p.T + p.A ? 2 : 0);
}

// One CTA per row: y = rmsnorm(x) * w (fh3_rmsnorm, src/core/fh3_ops.c:410-456), then,
// when pr.a[0] is set, y = y * (1 + scale) + shift of the row's pair (fh3_modulate,
// :529-557, fused multiply-add as its vector body).  w may be null (all ones).
__global__ void __launch_bounds__(kDitThreads) dit_norm_kernel(const float* __restrict__ x,
                                                               const float* __restrict__ w, float* __restrict__ y,
                                                               int dim, float eps, PairRows pr) {
    __shared__ float red[kDitThreads / 32];
    const int r = blockIdx.x;
    const float* row = x + static_cast<int64_t>(r) * dim;
    float* out = y + static_cast<int64_t>(r) * dim;
    float ss = 0.0f;
    for (int k = threadIdx.x; k < dim; k += kDitThreads) ss = fmaf(row[k], row[k], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < kDitThreads / 32; ++i) tot += red[i];
    const float inv = 1.0f / sqrtf(tot / static_cast<float>(dim) + eps);
    const int p = row_pair(pr, r);
    const float* shift = pr.a[0] ? pr.a[p] : nullptr;
    const float* scale = pr.a[0] ? pr.b[p] : nullptr;
    for (int k = threadIdx.x; k < dim; k += kDitThreads) {
        float v = row[k] * inv;
        if (w) v = v * w[k];
        if (shift) v = fmaf(v, 1.0f + scale[k], shift[k]);
        out[k] = v;
    }
}

// h = gate * y + h with the gate of the row's pair (fh3_gate_residual,
// src/core/fh3_ops.c:559-585); gate null: h = h + y (the refiner's residual).
__global__ void dit_residual_kernel(float* __restrict__ h, const float* __restrict__ y, int64_t n, int dim,
                                    PairRows pr) {
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < n * dim;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(e / dim), k = static_cast<int>(e - static_cast<int64_t>(r) * dim);
        h[e] = pr.a[0] ? fmaf(pr.a[row_pair(pr, r)][k], y[e], h[e]) : h[e] + y[e];
    }
}

// fp32 -> bf16 of a [rows][width] block with row strides (attention operands)
__global__ void dit_to_bf16_kernel(const float* __restrict__ x, int64_t ldx, __nv_bfloat16* __restrict__ y,
                                   int64_t ldy, int64_t rows, int width) {
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < rows * width;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = e / width, c = e - r * width;
        y[r * ldy + c] = __float2bfloat16_rn(x[r * ldx + c]);
    }
}

int grid_1d(int64_t work) {
    using namespace fh3host;
    const int64_t cap = static_cast<int64_t>(std::max(1, ctx_sms(ctx()))) * 8;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(cap, (work + 255) / 256)));
}

}  // namespace

namespace {

constexpr int kDitSlot = 10;

// activations of one call, [rows][width] fp32 (bf16 copies for tensor-core attention,
// and the bf16 operands of the fused Q4_K block)
struct DitBufs {
    float *h, *normed, *qkv, *attn, *proj, *fc1, *sw, *gatec;
    __nv_bfloat16 *qkvb, *gateb, *ab, *attnb, *gb;
};

size_t dit_layout(int64_t rows, const Fh3CudaDitCfg& c, uint8_t* base, DitBufs* b) {
    const int64_t hid = c.hidden_size, inner = static_cast<int64_t>(c.num_heads) * c.head_dim, F = c.ffn_dim;
    size_t off = 0;
    auto take = [&](int64_t elems, int bytes) {
        uint8_t* p = base ? base + off : nullptr;
        off += (static_cast<size_t>(rows * elems * bytes) + 255) & ~static_cast<size_t>(255);
        return p;
    };
    DitBufs x{};
    x.h = reinterpret_cast<float*>(take(hid, 4));
    x.normed = reinterpret_cast<float*>(take(hid, 4));
    x.qkv = reinterpret_cast<float*>(take(3 * inner, 4));
    x.attn = reinterpret_cast<float*>(take(inner, 4));
    x.proj = reinterpret_cast<float*>(take(hid, 4));
    x.fc1 = reinterpret_cast<float*>(take(2 * F, 4));
    x.sw = reinterpret_cast<float*>(take(F, 4));
    x.gatec = reinterpret_cast<float*>(take(inner, 4));
    if (c.attn_bf16) {
        x.qkvb = reinterpret_cast<__nv_bfloat16*>(take(3 * inner, 2));
        x.gateb = reinterpret_cast<__nv_bfloat16*>(take(inner, 2));
        x.ab = reinterpret_cast<__nv_bfloat16*>(take(hid, 2));
        x.attnb = reinterpret_cast<__nv_bfloat16*>(take(inner, 2));
        x.gb = reinterpret_cast<__nv_bfloat16*>(take(F, 2));
    }
    if (b) *b = x;
    return off;
}

int dit_bufs(const char* who, int64_t rows, const Fh3CudaDitCfg& c, cudaStream_t s, DitBufs& b) {
    using namespace fh3host;
    const size_t bytes = dit_layout(rows, c, nullptr, nullptr);
    uint8_t* base = static_cast<uint8_t*>(scratch(ctx(), kDitSlot, bytes, s));
    if (!base) return set_error(FH3_E_NOMEM, "%s: activation scratch", who);
    dit_layout(rows, c, base, &b);
    return FH3_OK;
}

int cfg_ok(const char* who, const Fh3CudaDitCfg* c) {
    using namespace fh3host;
    if (!c || c->hidden_size <= 0 || c->num_heads <= 0 || c->head_dim <= 0 || c->ffn_dim <= 0 ||
        c->num_layers < 0 || c->num_refiner_layers < 0 || c->num_refiner_layers > 4)
        return set_error(FH3_E_INVALID, "%s: bad configuration", who);
    if (c->head_dim % 32 || c->head_dim > 256 || (c->attn_bf16 && c->head_dim != 128) ||
        (c->attn == 1 && c->head_dim != 64 && c->head_dim != 128))
        return set_error(FH3_E_INVALID, "%s: head_dim %d not served by the chosen attention", who, c->head_dim);
    return FH3_OK;
}

int mm(const Fh3CudaW& w, const float* x, float* y, int64_t n, const float* bias, cudaStream_t s) {
    if (n <= 0) return FH3_OK;
    return fh3cuda_matmul_dev(&w, x, y, static_cast<int>(n), bias, s);
}

int norm(const float* x, const float* w, float* y, int64_t rows, int dim, float eps, const PairRows& pr,
         cudaStream_t s) {
    if (rows <= 0) return FH3_OK;
    dit_norm_kernel<<<static_cast<unsigned>(rows), kDitThreads, 0, s>>>(x, w, y, dim, eps, pr);
    return fh3host::check_cuda(cudaGetLastError(), "dit norm launch");
}

int residual(float* h, const float* y, int64_t rows, int dim, const PairRows& pr, cudaStream_t s) {
    dit_residual_kernel<<<grid_1d(rows * dim), 256, 0, s>>>(h, y, rows, dim, pr);
    return fh3host::check_cuda(cudaGetLastError(), "dit residual launch");
}

// attention of one block on b.qkv ([rows][q | k | v]) into b.attn; seq null: dense
int dit_attention(const Fh3CudaDitCfg& c, const DitBufs& b, int64_t rows, const Fh3CudaSeq* seq,
                  const float* gate, cudaStream_t s) {
    using namespace fh3host;
    const int heads = c.num_heads, hd = c.head_dim;
    const int64_t inner = static_cast<int64_t>(heads) * hd, ld = 3 * inner;
    const int n = static_cast<int>(rows);
    if (c.attn_bf16) {
        dit_to_bf16_kernel<<<grid_1d(rows * ld), 256, 0, s>>>(b.qkv, ld, b.qkvb, ld, rows, static_cast<int>(ld));
        if (gate)
            dit_to_bf16_kernel<<<grid_1d(rows * inner), 256, 0, s>>>(gate, inner, b.gateb, inner, rows,
                                                                     static_cast<int>(inner));
        const __nv_bfloat16* q = b.qkvb;
        if (seq)
            return fh3cuda_vsa_attention_dev(c.vsa_tile, c.vsa_sparsity, seq, q, ld, q + inner, ld, q + 2 * inner, ld,
                                             1, gate ? b.gateb : nullptr, inner, b.attn, 0, inner, heads, hd, s);
        return fh3cuda_attention_dev(q, ld, q + inner, ld, q + 2 * inner, ld, b.attn, 0, inner, n, heads, hd, s);
    }
    const float* q = b.qkv;
    if (seq)
        return fh3cuda_vsa_attention_dev(c.vsa_tile, c.vsa_sparsity, seq, q, ld, q + inner, ld, q + 2 * inner, ld, 0,
                                         gate, inner, b.attn, 0, inner, heads, hd, s);
    return attention_f32_launch(q, ld, q + inner, ld, q + 2 * inner, ld, b.attn, inner, n, heads, hd, nullptr,
                                nullptr, nullptr, nullptr, 0, nullptr, 0, nullptr, s);
}

const PairRows kNoPairs = {{nullptr, nullptr, nullptr}, {nullptr, nullptr, nullptr}, 0, 0};

// A block whose projections are all Q4_K runs on bf16 operands end to end (with bf16
// tensor-core attention): the rmsnorm+modulate prologue writes bf16, the QKV and
// gate_compress GEMMs write bf16, q and k are normalised and rotated in bf16, attention
// writes bf16, the O and fc2 GEMMs add gate * y into h in their epilogue, and fc1 applies
// SwiGLU in its epilogue -- the launches the bench's trunk makes.  Otherwise (F32 or other
// formats, or fp32 attention) the block takes the fp32 chain below.
bool fused_block(const Fh3CudaDitCfg& c, const Fh3CudaLayerView& v) {
    auto q4k = [](const Fh3CudaW& w) { return w.type == FH3CUDA_TYPE_Q4_K && (w.in % 256) == 0; };
    const bool gated = c.attn == 1 && v.gate_compress.data && v.gate_compress.out > 0;
    return c.attn_bf16 && q4k(v.qkv) && q4k(v.out) && q4k(v.fc1) && q4k(v.fc2) && (!gated || q4k(v.gate_compress));
}

// the contiguous row ranges of the three modalities (text | audio | video) and their pairs
struct Ranges {
    int64_t r0[3], n[3];
    int pair[3];
};
Ranges ranges(int T, int A, int V) {
    return Ranges{{0, T, static_cast<int64_t>(T) + A}, {T, A, V}, {1, 2, 0}};
}

// one trunk block on the bf16 path; pr(L, chunk, pair) is the AdaLN row
template <class RowFn>
int fused_block_run(const Fh3CudaDitCfg& c, const Fh3CudaLayerView& v, const DitBufs& b, int64_t N, const Ranges& rg,
                    const Fh3CudaSeq* seq, const float* cos_t, const float* sin_t, RowFn row, cudaStream_t s) {
    const int hid = c.hidden_size, heads = c.num_heads, hd = c.head_dim, F = c.ffn_dim;
    const int64_t inner = static_cast<int64_t>(heads) * hd;
    int rc;
    auto norm_mod = [&](const Fh3CudaW& nw, int chunk) {
        for (int m = 0; m < 3; ++m) {
            if (rg.n[m] <= 0) continue;
            const int r = fh3cuda_rmsnorm_modulate_dev(b.h + rg.r0[m] * hid, reinterpret_cast<const float*>(nw.data),
                                                       row(chunk, rg.pair[m]), row(chunk + 1, rg.pair[m]),
                                                       b.ab + rg.r0[m] * hid, static_cast<int>(rg.n[m]), hid,
                                                       c.norm_eps, s);
            if (r) return r;
        }
        return static_cast<int>(FH3_OK);
    };
    auto resid = [&](const Fh3CudaW& w, const __nv_bfloat16* x, int64_t ldx, int chunk) {
        for (int m = 0; m < 3; ++m) {
            if (rg.n[m] <= 0) continue;
            const int r = fh3cuda_gemm_q4k_dev(&w, x + rg.r0[m] * ldx, ldx, b.h + rg.r0[m] * hid, hid, rg.n[m], nullptr,
                                               row(chunk, rg.pair[m]), FH3CUDA_EPI_RESID, s);
            if (r) return r;
        }
        return static_cast<int>(FH3_OK);
    };
    if ((rc = norm_mod(v.norm1, 0))) return rc;
    if ((rc = fh3cuda_gemm_q4k_dev(&v.qkv, b.ab, hid, b.qkvb, 3 * inner, N, nullptr, nullptr, FH3CUDA_EPI_BF16, s)))
        return rc;
    for (int part = 0; part < 2; ++part) {  // q, k: per-head rmsnorm + rope3 over 96 channels, in bf16
        __nv_bfloat16* x = b.qkvb + part * inner;
        rc = fh3cuda_qk_norm_rope_dev(x, 1, 3 * inner, x, 1, 3 * inner,
                                      reinterpret_cast<const float*>(part ? v.k_norm.data : v.q_norm.data), cos_t,
                                      sin_t, static_cast<int>(N), heads, hd, 96, c.qk_norm_eps, s);
        if (rc) return rc;
    }
    const __nv_bfloat16* q = b.qkvb;
    if (c.attn == 1) {
        const bool gated = v.gate_compress.data && v.gate_compress.out > 0;
        if (gated && (rc = fh3cuda_gemm_q4k_dev(&v.gate_compress, b.ab, hid, b.gateb, inner, N, nullptr, nullptr,
                                                FH3CUDA_EPI_BF16, s)))
            return rc;
        rc = fh3cuda_vsa_attention_dev(c.vsa_tile, c.vsa_sparsity, seq, q, 3 * inner, q + inner, 3 * inner,
                                       q + 2 * inner, 3 * inner, 1, gated ? b.gateb : nullptr, inner, b.attnb, 1, inner,
                                       heads, hd, s);
    } else {
        rc = fh3cuda_attention_dev(q, 3 * inner, q + inner, 3 * inner, q + 2 * inner, 3 * inner, b.attnb, 1, inner,
                                   static_cast<int>(N), heads, hd, s);
    }
    if (rc) return rc;
    if ((rc = resid(v.out, b.attnb, inner, 2))) return rc;
    if ((rc = norm_mod(v.norm2, 3))) return rc;
    if ((rc = fh3cuda_gemm_q4k_dev(&v.fc1, b.ab, hid, b.gb, F, N, nullptr, nullptr, FH3CUDA_EPI_SWIGLU, s))) return rc;
    return resid(v.fc2, b.gb, F, 5);
}

}  // namespace

extern "C" int fh3cuda_dit_prepare_text_dev(const Fh3CudaDitCfg* cfg, const Fh3CudaDitGlobals* g,
                                            const float* text_emb, int T, float* text_rows, void* stream) {
    using namespace fh3host;
    const char* who = "fh3cuda_dit_prepare_text_dev";
    if (!ctx()) return set_error(FH3CUDA_E_NODEV, "%s: call fh3cuda_init first", who);
    if (!g || !text_emb || !text_rows || T <= 0) return set_error(FH3_ERR, "%s: bad arguments", who);
    int rc = cfg_ok(who, cfg);
    if (rc) return rc;
    const Fh3CudaDitCfg& c = *cfg;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    DitBufs b;
    if ((rc = dit_bufs(who, T, c, s, b))) return rc;
    const int hid = c.hidden_size, heads = c.num_heads, hd = c.head_dim, F = c.ffn_dim;
    const int64_t inner = static_cast<int64_t>(heads) * hd;
    // src/model/fh3_dit.c:259-320: condition projection, refiner blocks, final norm
    if ((rc = mm(g->condition_proj, text_emb, b.h, T, g->condition_proj_bias, s))) return rc;
    for (int r = 0; r < c.num_refiner_layers; ++r) {
        const Fh3CudaRefinerBlock& rb = g->refiner[r];
        if ((rc = norm(b.h, rb.norm1, b.normed, T, hid, c.norm_eps, kNoPairs, s))) return rc;
        if ((rc = mm(rb.qkv, b.normed, b.qkv, T, nullptr, s))) return rc;
        for (int part = 0; part < 2; ++part) {  // q, k: per-head rmsnorm, no rope
            float* x = b.qkv + part * inner;
            rc = fh3cuda_qk_norm_rope_dev(x, 0, 3 * inner, x, 0, 3 * inner, part ? rb.k_norm : rb.q_norm, nullptr,
                                          nullptr, T, heads, hd, 0, c.qk_norm_eps, s);
            if (rc) return rc;
        }
        if ((rc = dit_attention(c, b, T, nullptr, nullptr, s))) return rc;
        if ((rc = mm(rb.out, b.attn, b.proj, T, nullptr, s))) return rc;
        if ((rc = residual(b.h, b.proj, T, hid, kNoPairs, s))) return rc;
        if ((rc = norm(b.h, rb.norm2, b.normed, T, hid, c.norm_eps, kNoPairs, s))) return rc;
        if ((rc = mm(rb.fc1, b.normed, b.fc1, T, nullptr, s))) return rc;
        if ((rc = fh3cuda_swiglu_dev(b.fc1, b.sw, T, F, s))) return rc;
        if ((rc = mm(rb.fc2, b.sw, b.proj, T, nullptr, s))) return rc;
        if ((rc = residual(b.h, b.proj, T, hid, kNoPairs, s))) return rc;
    }
    return norm(b.h, g->refiner_final_norm, text_rows, T, hid, c.final_norm_eps, kNoPairs, s);
}

extern "C" int fh3cuda_dit_forward_dev(const Fh3CudaDitCfg* cfg, const Fh3CudaDitGlobals* g, const Fh3CudaPack* trunk,
                                       const Fh3CudaAdaln* adaln, const Fh3CudaSeq* seq, const float* cos_t,
                                       const float* sin_t, int step, const float* x_video, const float* x_audio,
                                       const float* text_rows, float* v_video, float* v_audio, void* stream) {
    using namespace fh3host;
    const char* who = "fh3cuda_dit_forward_dev";
    if (!ctx()) return set_error(FH3CUDA_E_NODEV, "%s: call fh3cuda_init first", who);
    if (!g || !trunk || !adaln || !seq || !cos_t || !sin_t || !x_video || !x_audio || !text_rows || !v_video ||
        !v_audio)
        return set_error(FH3_ERR, "%s: bad arguments", who);
    int rc = cfg_ok(who, cfg);
    if (rc) return rc;
    const Fh3CudaDitCfg& c = *cfg;
    int n_steps = 0, pairs = 0, a_hidden = 0;
    fh3cuda_adaln_dims(adaln, &n_steps, nullptr, &pairs, &a_hidden);
    if (step < 0 || step >= n_steps) return set_error(FH3_E_INVALID, "%s: step %d outside the table", who, step);
    const int N = seq->seq_len, T = seq->num_text, A = seq->num_audio, V = seq->num_video;
    if (N <= 0 || T < 0 || A < 0 || V < 0 || T + A + V != N || pairs < 3 || a_hidden != c.hidden_size ||
        fh3cuda_pack_num_layers(trunk) < c.num_layers)
        return set_error(FH3_E_INVALID, "%s: sequence, AdaLN table and trunk do not fit the configuration", who);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    DitBufs b;
    if ((rc = dit_bufs(who, N, c, s, b))) return rc;
    const int hid = c.hidden_size, heads = c.num_heads, hd = c.head_dim, F = c.ffn_dim;
    const int64_t inner = static_cast<int64_t>(heads) * hd;
    // AdaLN rows of block L (chunks c0, c0+1) for the three pairs; -1 = final layer
    auto pair_rows = [&](int L, int c0, PairRows& pr) {
        pr.T = T;
        pr.A = A;
        for (int p = 0; p < 3; ++p) {
            pr.a[p] = fh3cuda_adaln_row(adaln, step, L, p, c0);
            pr.b[p] = c0 + 1 < (L < 0 ? 2 : 6) ? fh3cuda_adaln_row(adaln, step, L, p, c0 + 1) : nullptr;
            if (!pr.a[p]) return set_error(FH3_E_INVALID, "%s: AdaLN row missing (block %d)", who, L);
        }
        return static_cast<int>(FH3_OK);
    };

    // 1. patch embedding scatter (src/model/fh3_dit.c:350-353)
    if (T > 0 && (rc = check_cuda(cudaMemcpyAsync(b.h, text_rows, static_cast<size_t>(T) * hid * 4,
                                                  cudaMemcpyDeviceToDevice, s), "dit text rows")))
        return rc;
    if ((rc = mm(g->audio_patch_proj, x_audio, b.h + static_cast<int64_t>(T) * hid, A, g->audio_patch_proj_bias, s)))
        return rc;
    if ((rc = mm(g->video_patch_proj, x_video, b.h + static_cast<int64_t>(T + A) * hid, V, g->video_patch_proj_bias,
                 s)))
        return rc;
    // 2. trunk blocks (:356-449)
    for (int L = 0; L < c.num_layers; ++L) {
        Fh3CudaLayerView v;
        if ((rc = fh3cuda_pack_layer(trunk, L, &v))) return rc;
        if (v.norm1.type != FH3CUDA_TYPE_F32 || v.norm2.type != FH3CUDA_TYPE_F32 || v.q_norm.type != FH3CUDA_TYPE_F32 ||
            v.k_norm.type != FH3CUDA_TYPE_F32)
            return set_error(FH3_E_INVALID, "%s: layer %d norm weights are not F32", who, L);
        PairRows pr;
        if ((rc = pair_rows(L, 0, pr))) return rc;
        if (fused_block(c, v)) {
            auto row = [&](int chunk, int pair) { return fh3cuda_adaln_row(adaln, step, L, pair, chunk); };
            if ((rc = fused_block_run(c, v, b, N, ranges(T, A, V), seq, cos_t, sin_t, row, s))) return rc;
            continue;
        }
        if ((rc = norm(b.h, reinterpret_cast<const float*>(v.norm1.data), b.normed, N, hid, c.norm_eps, pr, s))) return rc;
        if ((rc = mm(v.qkv, b.normed, b.qkv, N, nullptr, s))) return rc;
        for (int part = 0; part < 2; ++part) {  // q, k: per-head rmsnorm + rope3 over 96 channels
            float* x = b.qkv + part * inner;
            rc = fh3cuda_qk_norm_rope_dev(x, 0, 3 * inner, x, 0, 3 * inner,
                                          reinterpret_cast<const float*>(part ? v.k_norm.data : v.q_norm.data), cos_t,
                                          sin_t, N, heads, hd, 96, c.qk_norm_eps, s);
            if (rc) return rc;
        }
        const float* gate = nullptr;
        if (c.attn == 1 && v.gate_compress.data && v.gate_compress.out > 0) {
            if ((rc = mm(v.gate_compress, b.normed, b.gatec, N, nullptr, s))) return rc;
            gate = b.gatec;
        }
        if ((rc = dit_attention(c, b, N, c.attn == 1 ? seq : nullptr, gate, s))) return rc;
        if ((rc = mm(v.out, b.attn, b.proj, N, nullptr, s))) return rc;
        if ((rc = pair_rows(L, 2, pr))) return rc;
        if ((rc = residual(b.h, b.proj, N, hid, pr, s))) return rc;
        if ((rc = pair_rows(L, 3, pr))) return rc;
        if ((rc = norm(b.h, reinterpret_cast<const float*>(v.norm2.data), b.normed, N, hid, c.norm_eps, pr, s))) return rc;
        if ((rc = mm(v.fc1, b.normed, b.fc1, N, nullptr, s))) return rc;
        if ((rc = fh3cuda_swiglu_dev(b.fc1, b.sw, N, F, s))) return rc;
        if ((rc = mm(v.fc2, b.sw, b.proj, N, nullptr, s))) return rc;
        if ((rc = pair_rows(L, 5, pr))) return rc;
        if ((rc = residual(b.h, b.proj, N, hid, pr, s))) return rc;
    }
    // 3. final norm and modulation, 4. output heads (:451-462)
    PairRows pr;
    if ((rc = pair_rows(-1, 0, pr))) return rc;
    if ((rc = norm(b.h, g->final_norm, b.normed, N, hid, c.final_norm_eps, pr, s))) return rc;
    if ((rc = mm(g->video_out, b.normed + static_cast<int64_t>(T + A) * hid, v_video, V, g->video_out_bias, s)))
        return rc;
    return mm(g->audio_out, b.normed + static_cast<int64_t>(T) * hid, v_audio, A, g->audio_out_bias, s);
}
