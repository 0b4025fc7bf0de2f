// vsa.cu -- video sparse attention, fh3_vsa_attention (src/core/fh3_vsa.c:186-507).
//
// The sequence is cut into tiles (src/core/fh3_vsa.c:32-161): text and audio runs of
// `tile` tokens ("prefix" tiles), then 4x4x4 cells of the video grid.  Per head:
// the tile means of q and k give tile-level scores; a video query tile attends to
// the prefix key tiles and to the top-k video key tiles by that score, a prefix
// query tile to every key tile (the "fine" pass); with a gate, a coarse pass adds
// softmax(tile scores) . (tile means of v), times the gate, to every token.
//
// Launches (all on the caller's stream, scratch reused between calls):
//   vsa_perm_kernel    tile order: perm[offset(i) + r] = token r of tile i (closed form)
//   vsa_pool_kernel    tile means, fp32, in the reference's order and rounding
//   vsa_score_kernel   tile scores, sequential fp32 dot products (bit-identical)
//   vsa_select_kernel  per (head, query tile): radix select of the top-k video key
//                      tiles, ties to the lower index; the kept list in ascending order
//   vsa_coarse_kernel  softmax over every tile score of a row . v tile means
//   vsa_fine_kernel    flash attention of 64 query rows over the kept key tiles,
//                      gathered by token index (cp.async, zero-filled past a tile's
//                      end); the coarse term times the gate is added in the epilogue.
// The tile mask is therefore exactly the reference's; with bf16 operands the fine pass
// runs on tensor cores (fh3flash::WarpFlash, flash.cuh) with fp32 softmax and
// accumulation, with fp32 operands in fp32 (attention_f32.cu).
//
// Operands: element (token t, head h, channel d) of q at q[t*ldq + h*head_dim + d]
// (likewise k, v, gate, o), fp32 or bf16.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "flash.cuh"

namespace {

using namespace fh3flash;

struct VsaGeo {
    int n, T, A, V, tile;
    int nT, nA, npre;  // text tiles, audio tiles, prefix tiles
    int gt, gh, gw;    // video grid (tokens)
    int ct, ch, cw;    // video cells per grid axis
    int nvid, ntiles;
};

// build_vsa_geometry's fallbacks (src/core/fh3_vsa.c:42-64): counts that do not add
// up to n make the whole sequence video; a grid whose product is not V is (1, 1, V)
bool make_geo(VsaGeo& g, const Fh3CudaSeq& s, int tile) {
    g = VsaGeo{};
    if (s.seq_len <= 0) return false;
    g.tile = tile > 0 ? tile : 64;
    g.n = s.seq_len;
    int T = s.num_text > 0 ? s.num_text : 0, A = s.num_audio > 0 ? s.num_audio : 0;
    int V = s.num_video > 0 ? s.num_video : 0;
    if (static_cast<int64_t>(T) + A + V != g.n) {
        T = 0;
        A = 0;
        V = g.n;
    }
    int gt = s.grid_t, gh = s.grid_h, gw = s.grid_w;
    if (gt <= 0 || gh <= 0 || gw <= 0 || static_cast<int64_t>(gt) * gh * gw != V) {
        gt = 1;
        gh = 1;
        gw = V;
    }
    g.T = T;
    g.A = A;
    g.V = V;
    g.nT = (T + g.tile - 1) / g.tile;
    g.nA = (A + g.tile - 1) / g.tile;
    g.npre = g.nT + g.nA;
    g.gt = gt;
    g.gh = gh;
    g.gw = gw;
    g.ct = (gt + 3) / 4;
    g.ch = (gh + 3) / 4;
    g.cw = (gw + 3) / 4;
    g.nvid = V > 0 ? g.ct * g.ch * g.cw : 0;
    g.ntiles = g.npre + g.nvid;
    return g.ntiles > 0;
}

// compute_topk (src/core/fh3_vsa.c:163-169), float arithmetic as there
int topk(float sparsity, int nblocks) {
    if (nblocks <= 0) return 0;
    const int k = static_cast<int>(ceilf((1.0f - sparsity) * static_cast<float>(nblocks)));
    return k < 1 ? 1 : (k > nblocks ? nblocks : k);
}

__device__ __forceinline__ int ext4(int grid, int cell) { return grid - 4 * cell < 4 ? grid - 4 * cell : 4; }

// tile i: token count, offset in tile order, token of its r-th member
__device__ __forceinline__ int tile_count(const VsaGeo& g, int i) {
    if (i < g.nT) return min(g.tile, g.T - i * g.tile);
    if (i < g.npre) return min(g.tile, g.A - (i - g.nT) * g.tile);
    const int v = i - g.npre, tt = v / (g.ch * g.cw), hh = (v / g.cw) % g.ch, ww = v % g.cw;
    return ext4(g.gt, tt) * ext4(g.gh, hh) * ext4(g.gw, ww);
}
__device__ __forceinline__ int tile_offset(const VsaGeo& g, int i) {
    if (i < g.nT) return i * g.tile;
    if (i < g.npre) return g.T + (i - g.nT) * g.tile;
    const int v = i - g.npre, tt = v / (g.ch * g.cw), hh = (v / g.cw) % g.ch, ww = v % g.cw;
    const int et = ext4(g.gt, tt), eh = ext4(g.gh, hh);
    // earlier t-slabs, earlier h-rows of this slab, earlier cells of this row
    return g.T + g.A + 4 * tt * g.gh * g.gw + et * 4 * hh * g.gw + et * eh * 4 * ww;
}
__device__ __forceinline__ int tile_token(const VsaGeo& g, int i, int r) {
    if (i < g.npre) return tile_offset(g, i) + r;  // prefix tiles are runs
    const int v = i - g.npre, tt = v / (g.ch * g.cw), hh = (v / g.cw) % g.ch, ww = v % g.cw;
    const int eh = ext4(g.gh, hh), ew = ext4(g.gw, ww);
    const int dt = r / (eh * ew), dh = (r / ew) % eh, dw = r % ew;
    return g.T + g.A + ((4 * tt + dt) * g.gh + 4 * hh + dh) * g.gw + 4 * ww + dw;
}

__global__ void vsa_perm_kernel(VsaGeo g, int* __restrict__ perm, int* __restrict__ toff) {
    const int i = blockIdx.x;
    const int off = tile_offset(g, i), cnt = tile_count(g, i);
    for (int r = threadIdx.x; r < cnt; r += blockDim.x) perm[off + r] = tile_token(g, i, r);
    if (threadIdx.x == 0) {
        toff[i] = off;
        if (i == g.ntiles - 1) toff[g.ntiles] = off + cnt;
    }
}

__device__ __forceinline__ float ldf(const float* p) { return __ldg(p); }
__device__ __forceinline__ float ldf(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// tile means (src/core/fh3_vsa.c:230-256): m += x * (1/count) over the tile's
// tokens in tile order, each product and sum rounded once.  grid (tiles, heads).
template <typename T>
__global__ void vsa_pool_kernel(const int* __restrict__ perm, const int* __restrict__ toff, int nt,
                                const T* __restrict__ q, int64_t ldq, const T* __restrict__ k, int64_t ldk,
                                const T* __restrict__ v, int64_t ldv, float* __restrict__ qp, float* __restrict__ kp,
                                float* __restrict__ vp, int hd) {
    const int i = blockIdx.x, h = blockIdx.y;
    const int off = toff[i], cnt = toff[i + 1] - off;
    const float inv = __fdiv_rn(1.0f, static_cast<float>(cnt));
    const size_t dst = (static_cast<size_t>(h) * nt + i) * hd;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float aq = 0.0f, ak = 0.0f, av = 0.0f;
        for (int r = 0; r < cnt; ++r) {
            const int64_t t = perm[off + r];
            const int64_t c = static_cast<int64_t>(h) * hd + d;
            aq = __fadd_rn(aq, __fmul_rn(ldf(q + t * ldq + c), inv));
            ak = __fadd_rn(ak, __fmul_rn(ldf(k + t * ldk + c), inv));
            if (vp) av = __fadd_rn(av, __fmul_rn(ldf(v + t * ldv + c), inv));
        }
        qp[dst + d] = aq;
        kp[dst + d] = ak;
        if (vp) vp[dst + d] = av;
    }
}

// tile scores (src/core/fh3_vsa.c:268-281): S[h][i][j] = (sequential sum over d of
// qp[i][d]*kp[j][d]) * scale.  grid (ceil(nt/32), ceil(nt/32), heads), 256 threads;
// a thread owns rows ty, ty+8, ty+16, ty+24 of column tx.
constexpr int kScoreTile = 32;

__global__ void __launch_bounds__(256) vsa_score_kernel(const float* __restrict__ qp, const float* __restrict__ kp,
                                                        float* __restrict__ S, int nt, int hd, float scale) {
    extern __shared__ float sc_smem[];
    float* sq = sc_smem;                     // [32][hd]
    float* sk = sc_smem + kScoreTile * hd;   // [hd][33], transposed
    const int h = blockIdx.z, i0 = blockIdx.y * kScoreTile, j0 = blockIdx.x * kScoreTile;
    const float* qb = qp + static_cast<size_t>(h) * nt * hd;
    const float* kb = kp + static_cast<size_t>(h) * nt * hd;
    for (int e = threadIdx.x; e < kScoreTile * hd; e += blockDim.x) {
        const int r = e / hd, d = e - r * hd;
        sq[e] = i0 + r < nt ? qb[static_cast<size_t>(i0 + r) * hd + d] : 0.0f;
        sk[d * (kScoreTile + 1) + r] = j0 + r < nt ? kb[static_cast<size_t>(j0 + r) * hd + d] : 0.0f;
    }
    __syncthreads();
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int d = 0; d < hd; ++d) {
        const float kv = sk[d * (kScoreTile + 1) + tx];
#pragma unroll
        for (int m = 0; m < 4; ++m) acc[m] = __fadd_rn(acc[m], __fmul_rn(sq[(ty + 8 * m) * hd + d], kv));
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const int i = i0 + ty + 8 * m, j = j0 + tx;
        if (i < nt && j < nt) S[(static_cast<size_t>(h) * nt + i) * nt + j] = __fmul_rn(acc[m], scale);
    }
}

// float -> unsigned key with the same order; -0 and +0 map to one key (they compare
// equal in the reference's qsort comparator, so its index tie-break decides)
__device__ __forceinline__ uint32_t order_key(float s) {
    uint32_t b = __float_as_uint(s);
    if ((b << 1) == 0u) b = 0u;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// exclusive count of set flags over the block (thread order) and the block total;
// every thread of the block calls it
__device__ __forceinline__ int block_excl_count(bool f, int& total, int* wsum) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const uint32_t b = __ballot_sync(0xffffffffu, f);
    if (lane == 0) wsum[warp] = __popc(b);
    __syncthreads();
    int before = 0;
    total = 0;
    for (int w = 0; w < nw; ++w) {
        const int c = wsum[w];
        if (w < warp) before += c;
        total += c;
    }
    __syncthreads();  // wsum is rewritten by the next call
    return before + __popc(b & ((1u << lane) - 1u));
}

// Kept key tiles of row (h, i), ascending (src/core/fh3_vsa.c:295-356).  A video
// query row keeps the prefix tiles and the kv video tiles first in (score desc,
// index asc) order: an MSB-first radix select (8 bits a pass) finds the kv-th key
// tau, then every key above tau and the lowest-index keys equal to tau are kept.
// grid (tiles, heads), 256 threads; dynamic shared memory: nvid keys.
constexpr int kSelThreads = 256;

__global__ void __launch_bounds__(kSelThreads) vsa_select_kernel(const float* __restrict__ S, int* __restrict__ sel,
                                                                 int* __restrict__ selcnt, int nt, int npre, int nvid,
                                                                 int kv, int dense) {
    extern __shared__ uint32_t su[];
    __shared__ int hist[256];
    __shared__ int wsum[kSelThreads / 32];
    __shared__ int sh_bin, sh_need;
    const int i = blockIdx.x, h = blockIdx.y;
    const size_t row = static_cast<size_t>(h) * nt + i;
    int* out = sel + row * nt;
    if (i < npre || dense) {
        for (int j = threadIdx.x; j < nt; j += blockDim.x) out[j] = j;
        if (threadIdx.x == 0) selcnt[row] = nt;
        return;
    }
    const float* s = S + row * nt + npre;
    for (int j = threadIdx.x; j < nvid; j += blockDim.x) su[j] = order_key(s[j]);
    for (int j = threadIdx.x; j < npre; j += blockDim.x) out[j] = j;
    uint32_t prefix = 0u, pmask = 0u;
    int need = kv;  // keys still to take inside the current prefix bucket (>= 1)
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0;
        __syncthreads();
        for (int j = threadIdx.x; j < nvid; j += blockDim.x) {
            const uint32_t u = su[j];
            if ((u & pmask) == prefix) atomicAdd(&hist[(u >> shift) & 255u], 1);
        }
        __syncthreads();
        if (threadIdx.x < 32) {  // lane L: bins 255-8L down to 248-8L; the bin where the count from the top reaches need
            const int lane = threadIdx.x;
            int c[8], tot = 0;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                c[e] = hist[255 - 8 * lane - e];
                tot += c[e];
            }
            int incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const int excl = incl - tot;
            if (excl < need && incl >= need) {
                int run = excl;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    if (run + c[e] >= need) {
                        sh_bin = 255 - 8 * lane - e;
                        sh_need = need - run;
                        break;
                    }
                    run += c[e];
                }
            }
        }
        __syncthreads();
        prefix |= static_cast<uint32_t>(sh_bin) << shift;
        pmask |= 255u << shift;
        need = sh_need;
        __syncthreads();
    }
    int carry_eq = 0, carry_sel = 0;
    for (int base = 0; base < nvid; base += blockDim.x) {
        const int j = base + threadIdx.x;
        const uint32_t u = j < nvid ? su[j] : 0u;
        const bool eq = j < nvid && u == prefix;
        int eq_total, sel_total;
        const int eq_rank = carry_eq + block_excl_count(eq, eq_total, wsum);
        const bool take = j < nvid && (u > prefix || (eq && eq_rank < need));
        const int pos = carry_sel + block_excl_count(take, sel_total, wsum);
        if (take) out[npre + pos] = npre + j;
        carry_eq += eq_total;
        carry_sel += sel_total;
    }
    if (threadIdx.x == 0) selcnt[row] = npre + carry_sel;
}

// coarse pass (src/core/fh3_vsa.c:442-473): c[i][h] = sum_j softmax(S[h][i])_j * vp[h][j].
// grid (ceil(nt/R), heads), 128 threads; R query tiles a CTA so that every v tile
// mean read serves R rows.  Dynamic shared memory: R x nt weights.
constexpr int kCoarseRows = 8;

__global__ void __launch_bounds__(128) vsa_coarse_kernel(const float* __restrict__ S, const float* __restrict__ vp,
                                                         float* __restrict__ outc, int nt, int heads, int hd, int R) {
    extern __shared__ float wts[];
    const int h = blockIdx.y, i0 = blockIdx.x * R;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int r = warp; r < R; r += nw) {  // a warp per row: max, exp, sum
        const int i = i0 + r;
        float* w = wts + static_cast<size_t>(r) * nt;
        if (i >= nt) continue;
        const float* s = S + (static_cast<size_t>(h) * nt + i) * nt;
        float mx = -1e30f;
        for (int j = lane; j < nt; j += 32) mx = fmaxf(mx, s[j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.0f;
        for (int j = lane; j < nt; j += 32) {
            const float e = expf(s[j] - mx);
            w[j] = e;
            sum += e;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float inv = 1.0f / sum;
        __syncwarp();
        for (int j = lane; j < nt; j += 32) w[j] *= inv;
    }
    __syncthreads();
    const float* vb = vp + static_cast<size_t>(h) * nt * hd;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float c[kCoarseRows];
#pragma unroll
        for (int r = 0; r < kCoarseRows; ++r) c[r] = 0.0f;
        for (int j = 0; j < nt; ++j) {
            const float x = vb[static_cast<size_t>(j) * hd + d];
#pragma unroll
            for (int r = 0; r < kCoarseRows; ++r)
                if (r < R) c[r] = fmaf(wts[static_cast<size_t>(r) * nt + j], x, c[r]);
        }
#pragma unroll
        for (int r = 0; r < kCoarseRows; ++r)
            if (r < R && i0 + r < nt) outc[(static_cast<size_t>(i0 + r) * heads + h) * hd + d] = c[r];
    }
}

// rows of a gathered tile: row r < rows is token toks[r] (head h), later rows are zero
template <int HD>
__device__ __forceinline__ void load_rows(uint32_t tile, const __nv_bfloat16* __restrict__ base, int64_t ld, int h,
                                          const int* __restrict__ toks, int rows) {
    constexpr int CH = HD / 8;  // 16-byte chunks of a row
    for (int idx = threadIdx.x; idx < kKeys * CH; idx += blockDim.x) {
        const int r = idx / CH, c = idx % CH;
        const bool ok = r < rows;
        const int64_t t = ok ? __ldg(toks + r) : 0;
        cp_async16_zfill(tile + swz<HD>(r, c), base + t * ld + h * HD + c * 8, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// the same with the tokens listed in shared memory
template <int HD>
__device__ __forceinline__ void load_rows_smem(uint32_t tile, const __nv_bfloat16* __restrict__ base, int64_t ld,
                                               int h, const int* toks, int rows) {
    constexpr int CH = HD / 8;
    for (int idx = threadIdx.x; idx < kKeys * CH; idx += blockDim.x) {
        const int r = idx / CH, c = idx % CH;
        const bool ok = r < rows;
        const int64_t t = ok ? toks[r] : 0;
        cp_async16_zfill(tile + swz<HD>(r, c), base + t * ld + h * HD + c * 8, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

constexpr int kFineWarps = 4;  // 64 query rows a CTA

// Fine pass (src/core/fh3_vsa.c:372-432) and the combination with the coarse term
// (:476-487).  grid (tiles * qsplit, heads): CTA (i, sub) owns rows 64*sub.. of query
// tile i and walks the keys of the tiles kept for (h, i), packed into 64-key chunks
// across tile boundaries, the next chunk's K and V in flight while this one is used.
// Dynamic shared memory: Q + 2 x (K, V).
template <int HD, bool OUT_BF16>
__global__ void __launch_bounds__(kFineWarps * 32, 2) vsa_fine_kernel(
    const int* __restrict__ perm, const int* __restrict__ toff, const int* __restrict__ sel,
    const int* __restrict__ selcnt, int nt, int qsplit, const __nv_bfloat16* __restrict__ q, int64_t ldq,
    const __nv_bfloat16* __restrict__ k, int64_t ldk, const __nv_bfloat16* __restrict__ v, int64_t ldv,
    const void* __restrict__ gate, int64_t ldg, int gate_bf16, const float* __restrict__ outc, int heads,
    void* __restrict__ o, int64_t ldo, float scale_log2) {
    extern __shared__ __align__(128) uint8_t vsa_smem[];
    constexpr uint32_t TB = kKeys * HD * 2;
    const uint32_t sb = fh3::smem_u32(vsa_smem);
    const uint32_t sQ = sb;
    const uint32_t sK[2] = {sb + TB, sb + 2 * TB};
    const uint32_t sV[2] = {sb + 3 * TB, sb + 4 * TB};
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, tq = lane & 3;
    const int i = blockIdx.x / qsplit, sub = blockIdx.x - i * qsplit, h = blockIdx.y;
    const int qoff = toff[i] + sub * kKeys;
    const int qrows = min(kKeys, toff[i + 1] - qoff);
    if (qrows <= 0) return;  // CTA-uniform
    const size_t row = static_cast<size_t>(h) * nt + i;
    const int* lst = sel + row * nt;
    const int L = selcnt[row];  // >= 1

    // The kept key tiles' tokens, concatenated, are cut into chunks of 64 keys (only the
    // last one partial).  Warp 0 lists chunk t's tokens in s_tok[t % 3] two chunks ahead;
    // s_cnt holds how many of the 64 slots are filled (0: no chunk).
    __shared__ int s_tok[3][kKeys];
    __shared__ int s_cnt[3];
    int cl = 0, cr = 0;  // warp 0: next key = token cr of kept tile cl
    auto fill = [&](int buf) {  // warp 0 only
        int filled = 0;
        while (filled < kKeys && cl < L) {  // warp-uniform; one pass unless tiles are tiny
            const int e = cl + lane;
            int cnt = 0, off = 0;
            if (e < L) {
                const int j = lst[e];
                off = toff[j];
                cnt = toff[j + 1] - off;
            }
            if (lane == 0) {
                off += cr;
                cnt -= cr;
            }
            int incl = cnt;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, d);
                if (lane >= d) incl += y;
            }
            const int take = min(kKeys - filled, __shfl_sync(0xffffffffu, incl, 31));
            const int excl = incl - cnt;
            for (int kk = 0; kk < 32; ++kk) {  // the entries this chunk reaches, in order
                const int ek = __shfl_sync(0xffffffffu, excl, kk);
                if (ek >= take) break;
                const int ck = __shfl_sync(0xffffffffu, cnt, kk), ok = __shfl_sync(0xffffffffu, off, kk);
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int pslot = lane + 32 * half;
                    if (pslot >= ek && pslot < ek + ck && pslot < take) s_tok[buf][filled + pslot] = perm[ok + pslot - ek];
                }
            }
            // entries used up (the scan is monotone), and where the next chunk starts
            const int used = __popc(__ballot_sync(0xffffffffu, incl <= take));
            if (used == 32) {
                cl = min(cl + 32, L);
                cr = 0;
            } else {
                const int ex = __shfl_sync(0xffffffffu, excl, used);
                cr = (used == 0 ? cr : 0) + take - ex;
                cl = min(cl + used, L);
            }
            filled += take;
        }
        if (lane == 0) s_cnt[buf] = filled;
    };

    if (warp == 0) {
        fill(0);
        fill(1);
    }
    load_rows<HD>(sQ, q, ldq, h, perm + qoff, qrows);
    __syncthreads();
    load_rows_smem<HD>(sK[0], k, ldk, h, s_tok[0], s_cnt[0]);
    load_rows_smem<HD>(sV[0], v, ldv, h, s_tok[0], s_cnt[0]);

    // warps whose 16 query rows all lie past the tile's end skip the arithmetic
    const bool busy = warp * 16 < qrows;
    WarpFlash<HD> wf;
    wf.init();
    for (int t = 0;; ++t) {
        const int st = t & 1, nb = (t + 1) % 3;
        const int rows = s_cnt[t % 3], nrows = s_cnt[nb];
        const bool more = nrows > 0;
        if (more) {
            load_rows_smem<HD>(sK[st ^ 1], k, ldk, h, s_tok[nb], nrows);
            load_rows_smem<HD>(sV[st ^ 1], v, ldv, h, s_tok[nb], nrows);
            asm volatile("cp.async.wait_group 2;" ::: "memory");  // all but the two newest groups
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        if (busy) {
            if (t == 0) wf.load_q(sQ, warp * 16, lane);
            wf.step(sK[st], sV[st], rows, scale_log2, lane);
        }
        if (warp == 0 && more) fill((t + 2) % 3);  // chunk t+2
        __syncthreads();  // the next iteration's prefetch overwrites this stage
        if (!more) break;
    }

    float i0, i1;
    wf.inv_sums(i0, i1);
    const int r0 = warp * 16 + g, r1 = r0 + 8;
    const int64_t t0 = r0 < qrows ? perm[qoff + r0] : -1;
    const int64_t t1 = r1 < qrows ? perm[qoff + r1] : -1;
    const float* cb = gate ? outc + (static_cast<size_t>(i) * heads + h) * HD : nullptr;
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
        const int d = j * 8 + 2 * tq;
        const int64_t col = static_cast<int64_t>(h) * HD + d;
        float v0 = wf.o[j][0] * i0, v1 = wf.o[j][1] * i0, v2 = wf.o[j][2] * i1, v3 = wf.o[j][3] * i1;
        if (cb) {
            const float2 cc = *reinterpret_cast<const float2*>(cb + d);
            float2 g0 = make_float2(0.0f, 0.0f), g1 = g0;
            if (gate_bf16) {
                const __nv_bfloat16* gb = static_cast<const __nv_bfloat16*>(gate);
                if (t0 >= 0) g0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(gb + t0 * ldg + col));
                if (t1 >= 0) g1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(gb + t1 * ldg + col));
            } else {
                const float* gf = static_cast<const float*>(gate);
                if (t0 >= 0) g0 = *reinterpret_cast<const float2*>(gf + t0 * ldg + col);
                if (t1 >= 0) g1 = *reinterpret_cast<const float2*>(gf + t1 * ldg + col);
            }
            v0 += cc.x * g0.x;
            v1 += cc.y * g0.y;
            v2 += cc.x * g1.x;
            v3 += cc.y * g1.y;
        }
        if (OUT_BF16) {
            __nv_bfloat16* ob = static_cast<__nv_bfloat16*>(o);
            if (t0 >= 0) *reinterpret_cast<uint32_t*>(ob + t0 * ldo + col) = pack_bf16(v0, v1);
            if (t1 >= 0) *reinterpret_cast<uint32_t*>(ob + t1 * ldo + col) = pack_bf16(v2, v3);
        } else {
            float* of = static_cast<float*>(o);
            if (t0 >= 0) *reinterpret_cast<float2*>(of + t0 * ldo + col) = make_float2(v0, v1);
            if (t1 >= 0) *reinterpret_cast<float2*>(of + t1 * ldo + col) = make_float2(v2, v3);
        }
    }
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// scratch layout of one call (slot 9)
struct VsaBufs {
    int* perm;
    int* toff;
    float *qp, *kp, *vp;
    float* S;
    int* sel;
    int* selcnt;
    float* outc;
};

size_t vsa_layout(const VsaGeo& g, int heads, int hd, bool gate, uint8_t* base, VsaBufs* b) {
    const size_t nt = g.ntiles, pool = static_cast<size_t>(heads) * nt * hd * 4;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        uint8_t* p = base ? base + off : nullptr;
        off += align256(bytes);
        return p;
    };
    VsaBufs x{};
    x.perm = reinterpret_cast<int*>(take(static_cast<size_t>(g.n) * 4));
    x.toff = reinterpret_cast<int*>(take((nt + 1) * 4));
    x.qp = reinterpret_cast<float*>(take(pool));
    x.kp = reinterpret_cast<float*>(take(pool));
    x.vp = gate ? reinterpret_cast<float*>(take(pool)) : nullptr;
    x.S = reinterpret_cast<float*>(take(static_cast<size_t>(heads) * nt * nt * 4));
    x.sel = reinterpret_cast<int*>(take(static_cast<size_t>(heads) * nt * nt * 4));
    x.selcnt = reinterpret_cast<int*>(take(static_cast<size_t>(heads) * nt * 4));
    x.outc = gate ? reinterpret_cast<float*>(take(nt * heads * hd * 4)) : nullptr;
    if (b) *b = x;
    return off;
}

constexpr int kVsaSlot = 9;

// geometry, tile means, scores and kept lists; returns FH3_OK or an error code
int vsa_prepare(const char* who, int tile, float sparsity, const Fh3CudaSeq* seq, const void* q, int64_t ldq,
                const void* k, int64_t ldk, const void* v, int64_t ldv, int in_bf16, bool with_gate, int heads,
                int head_dim, cudaStream_t s, VsaGeo& g, VsaBufs& b) {
    using namespace fh3host;
    if (!ctx()) return set_error(FH3CUDA_E_NODEV, "%s: call fh3cuda_init first", who);
    if (!seq || !q || !k || (with_gate && !v) || heads <= 0 || heads > 65535)
        return set_error(FH3_E_INVALID, "%s: bad arguments", who);
    if (head_dim != 64 && head_dim != 128)
        return set_error(FH3_E_INVALID, "%s: head_dim must be 64 or 128 (got %d)", who, head_dim);
    if (!make_geo(g, *seq, tile)) return set_error(FH3_E_INVALID, "%s: empty sequence", who);
    const int64_t row = static_cast<int64_t>(heads) * head_dim;
    if (ldq < row || ldk < row || (v && ldv < row))
        return set_error(FH3_E_INVALID, "%s: rows must hold heads*head_dim elements", who);
    if (g.nvid > 48 * 1024) return set_error(FH3_E_INVALID, "%s: more than 49152 video tiles", who);
    const size_t bytes = vsa_layout(g, heads, head_dim, with_gate, nullptr, nullptr);
    uint8_t* base = static_cast<uint8_t*>(scratch(ctx(), kVsaSlot, bytes, s));
    if (!base) return FH3_E_NOMEM;
    vsa_layout(g, heads, head_dim, with_gate, base, &b);
    const int nt = g.ntiles;

    vsa_perm_kernel<<<nt, 64, 0, s>>>(g, b.perm, b.toff);
    const dim3 pg(static_cast<unsigned>(nt), static_cast<unsigned>(heads));
    if (in_bf16)
        vsa_pool_kernel<__nv_bfloat16><<<pg, head_dim, 0, s>>>(
            b.perm, b.toff, nt, static_cast<const __nv_bfloat16*>(q), ldq, static_cast<const __nv_bfloat16*>(k), ldk,
            static_cast<const __nv_bfloat16*>(v), ldv, b.qp, b.kp, with_gate ? b.vp : nullptr, head_dim);
    else
        vsa_pool_kernel<float><<<pg, head_dim, 0, s>>>(b.perm, b.toff, nt, static_cast<const float*>(q), ldq,
                                                       static_cast<const float*>(k), ldk,
                                                       static_cast<const float*>(v), ldv, b.qp, b.kp,
                                                       with_gate ? b.vp : nullptr, head_dim);
    const float scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    const unsigned st = static_cast<unsigned>((nt + kScoreTile - 1) / kScoreTile);
    const size_t ssm = static_cast<size_t>(kScoreTile) * head_dim * 4 + static_cast<size_t>(head_dim) * (kScoreTile + 1) * 4;
    vsa_score_kernel<<<dim3(st, st, static_cast<unsigned>(heads)), 256, ssm, s>>>(b.qp, b.kp, b.S, nt, head_dim,
                                                                                  scale);
    const int kv = topk(sparsity, g.nvid);
    const int dense = sparsity <= 0.0f || kv == g.nvid;
    const size_t selsm = static_cast<size_t>(g.nvid) * 4;
    if (selsm > 48 * 1024) {
        const int rc = check_cuda(cudaFuncSetAttribute(vsa_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       static_cast<int>(selsm)), "vsa select smem attribute");
        if (rc) return rc;
    }
    vsa_select_kernel<<<pg, kSelThreads, selsm, s>>>(b.S, b.sel, b.selcnt, nt, g.npre, g.nvid, kv, dense);
    return check_cuda(cudaGetLastError(), "vsa prepare launches");
}

bool aligned16(const void* p) { return !(reinterpret_cast<uintptr_t>(p) & 15); }

}  // namespace

extern "C" int fh3cuda_vsa_num_tiles(const Fh3CudaSeq* seq, int tile, int* num_tiles, int* num_prefix,
                                     int* num_video) {
    VsaGeo g;
    if (!seq || !make_geo(g, *seq, tile)) return fh3host::set_error(FH3_E_INVALID, "fh3cuda_vsa_num_tiles: empty sequence");
    if (num_tiles) *num_tiles = g.ntiles;
    if (num_prefix) *num_prefix = g.npre;
    if (num_video) *num_video = g.nvid;
    return FH3_OK;
}

extern "C" int fh3cuda_vsa_tiles_dev(int tile, float sparsity, const Fh3CudaSeq* seq, const void* q, int64_t ldq,
                                     const void* k, int64_t ldk, int in_bf16, int heads, int head_dim, float* scores,
                                     uint8_t* mask, void* stream) {
    using namespace fh3host;
    const char* who = "fh3cuda_vsa_tiles_dev";
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    VsaGeo g;
    VsaBufs b;
    int rc = vsa_prepare(who, tile, sparsity, seq, q, ldq, k, ldk, nullptr, 0, in_bf16, false, heads, head_dim, s,
                         g, b);
    if (rc) return rc;
    const size_t nn = static_cast<size_t>(heads) * g.ntiles * g.ntiles;
    if (scores) {
        rc = check_cuda(cudaMemcpyAsync(scores, b.S, nn * 4, cudaMemcpyDeviceToDevice, s), "vsa scores copy");
        if (rc) return rc;
    }
    if (mask) {
        std::vector<int> cnt(static_cast<size_t>(heads) * g.ntiles);
        std::vector<int> lst(nn);
        rc = check_cuda(cudaMemcpyAsync(cnt.data(), b.selcnt, cnt.size() * 4, cudaMemcpyDeviceToHost, s), "vsa copy");
        if (!rc) rc = check_cuda(cudaMemcpyAsync(lst.data(), b.sel, nn * 4, cudaMemcpyDeviceToHost, s), "vsa copy");
        if (!rc) rc = check_cuda(cudaStreamSynchronize(s), "vsa sync");
        if (rc) return rc;
        std::vector<uint8_t> m(nn, 0);
        for (size_t r = 0; r < cnt.size(); ++r)
            for (int e = 0; e < cnt[r]; ++e) m[r * g.ntiles + lst[r * g.ntiles + e]] = 1;
        rc = check_cuda(cudaMemcpyAsync(mask, m.data(), nn, cudaMemcpyHostToDevice, s), "vsa mask copy");
        if (!rc) rc = check_cuda(cudaStreamSynchronize(s), "vsa sync");
        if (rc) return rc;
    }
    return FH3_OK;
}

extern "C" int fh3cuda_vsa_attention_dev(int tile, float sparsity, const Fh3CudaSeq* seq, const void* q, int64_t ldq,
                                         const void* k, int64_t ldk, const void* v, int64_t ldv, int in_bf16,
                                         const void* gate, int64_t ldg, void* o, int o_bf16, int64_t ldo, int heads,
                                         int head_dim, void* stream) {
    using namespace fh3host;
    const char* who = "fh3cuda_vsa_attention_dev";
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!q || !k || !v || !o) return set_error(FH3_E_INVALID, "%s: bad arguments", who);
    const int64_t rowe = static_cast<int64_t>(heads) * head_dim;
    if (in_bf16) {
        if (ldo < rowe || (ldo % 8) || !aligned16(o) || (gate && (ldg < rowe || (ldg % 8) || !aligned16(gate))) ||
            (ldq % 8) || (ldk % 8) || (ldv % 8) || !aligned16(q) || !aligned16(k) || !aligned16(v))
            return set_error(FH3_E_INVALID, "%s: bf16 operands need strides that are multiples of 8 elements and "
                             "16-byte aligned pointers (q, k, v, gate, o)", who);
    } else if (o_bf16 || ldo < rowe || (gate && ldg < rowe)) {
        return set_error(FH3_E_INVALID, "%s: fp32 operands give an fp32 output (o_bf16 = 0); rows must hold "
                         "heads*head_dim elements", who);
    }
    VsaGeo g;
    VsaBufs b;
    int rc = vsa_prepare(who, tile, sparsity, seq, q, ldq, k, ldk, v, ldv, in_bf16, gate != nullptr, heads,
                         head_dim, s, g, b);
    if (rc) return rc;
    const int nt = g.ntiles;
    if (gate) {
        const int R = static_cast<int>(std::min<int64_t>(kCoarseRows, std::max<int64_t>(1, (200 * 1024) / (4 * nt))));
        const size_t csm = static_cast<size_t>(R) * nt * 4;
        if (csm > 227 * 1024) return set_error(FH3_E_INVALID, "%s: too many tiles for the coarse pass", who);
        if (csm > 48 * 1024) {
            rc = check_cuda(cudaFuncSetAttribute(vsa_coarse_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(csm)), "vsa coarse smem attribute");
            if (rc) return rc;
        }
        vsa_coarse_kernel<<<dim3(static_cast<unsigned>((nt + R - 1) / R), static_cast<unsigned>(heads)), 128, csm,
                            s>>>(b.S, b.vp, b.outc, nt, heads, head_dim, R);
    }
    if (!in_bf16)  // fp32 operands: the fine pass in fp32 (attention_f32.cu)
        return attention_f32_launch(static_cast<const float*>(q), ldq, static_cast<const float*>(k), ldk,
                                    static_cast<const float*>(v), ldv, static_cast<float*>(o), ldo, g.n, heads,
                                    head_dim, b.perm, b.toff, b.sel, b.selcnt, nt, static_cast<const float*>(gate),
                                    ldg, b.outc, s);
    const auto* qb = static_cast<const __nv_bfloat16*>(q);
    const auto* kb = static_cast<const __nv_bfloat16*>(k);
    const auto* vb = static_cast<const __nv_bfloat16*>(v);
    const int64_t lq = ldq, lk = ldk, lv = ldv;
    const int max_rows = std::max(64, g.npre > 0 ? std::min(g.tile, std::max(g.T, g.A)) : 64);
    const int qsplit = (max_rows + kKeys - 1) / kKeys;
    // tcgen05 fine pass (vsa_tc.cu) for tiles of at most 64 tokens and head_dim 128;
    // FH3CUDA_VSA_KERNEL=mma selects the mma.sync kernel below
    const char* vk = getenv("FH3CUDA_VSA_KERNEL");
    if (head_dim == 128 && qsplit == 1 && !(vk && strcmp(vk, "mma") == 0))
        return vsa_fine_tc(b.perm, b.toff, b.sel, b.selcnt, nt, g.n, qb, lq, kb, lk, vb, lv,
                           static_cast<const __nv_bfloat16*>(gate), ldg, b.outc, heads, o, o_bf16 != 0, ldo, s);
    const float scale_log2 = (1.0f / sqrtf(static_cast<float>(head_dim))) * 1.4426950408889634f;
    const dim3 grid(static_cast<unsigned>(nt * qsplit), static_cast<unsigned>(heads));
    const int smem = 5 * kKeys * head_dim * 2;
    auto launch = [&](auto kern) -> int {
        int r = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                           "vsa fine smem attribute");
        if (r) return r;
        kern<<<grid, kFineWarps * 32, smem, s>>>(b.perm, b.toff, b.sel, b.selcnt, nt, qsplit, qb, lq, kb, lk, vb, lv,
                                                 gate, ldg, in_bf16, b.outc, heads, o, ldo, scale_log2);
        return FH3_OK;
    };
    if (head_dim == 64)
        rc = o_bf16 ? launch(vsa_fine_kernel<64, true>) : launch(vsa_fine_kernel<64, false>);
    else
        rc = o_bf16 ? launch(vsa_fine_kernel<128, true>) : launch(vsa_fine_kernel<128, false>);
    if (rc) return rc;
    return check_cuda(cudaGetLastError(), "vsa launches");
}
