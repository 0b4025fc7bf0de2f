// common.cuh -- shared device helpers of libfh3cuda (sm_100a only).
//
// Q4_K format helpers, bounded mbarrier waits, TMA and tcgen05 wrappers in
// inline PTX.  Every spin-wait here has a time limit: on expiry it records
// FH3CUDA_E_TIMEOUT in the caller's device status word and returns false, so
// a kernel never hangs its GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/fh3cuda.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libfh3cuda targets sm_100a only"
#endif

namespace fh3 {

constexpr int kQ4KBlock = 256;  // weights per super-block
constexpr int kQ4KBytes = 144;  // bytes per super-block

// ---------------------------------------------------------------------------
// Q4_K super-block: bytes 0-1 d (fp16), 2-3 dmin (fp16), 4-15 packed 6-bit
// scales/mins of the eight 32-weight sub-blocks, 16-143 nibbles.  32-byte
// chunk c of the nibbles holds sub-block 2c in its low nibbles and 2c+1 in its
// high nibbles (src/core/fh3_quant.c:154-196).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void q4k_scale_min(const uint8_t* s, int j, int& sc, int& m) {
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// Same unpacking from the 12 scale bytes held in three 32-bit words
// (w0 = bytes 4-7, w1 = bytes 8-11, w2 = bytes 12-15 of the block).
__device__ __forceinline__ void q4k_scale_min_words(uint32_t w0, uint32_t w1, uint32_t w2, int j,
                                                    int& sc, int& m) {
    if (j < 4) {
        sc = (w0 >> (8 * j)) & 63;
        m = (w1 >> (8 * j)) & 63;
    } else {
        const int jj = j - 4;
        const uint32_t b8 = (w2 >> (8 * jj)) & 0xFF;       // byte j+4
        sc = (b8 & 0x0F) | (((w0 >> (8 * jj + 6)) & 3) << 4);
        m = (b8 >> 4) | (((w1 >> (8 * jj + 6)) & 3) << 4);
    }
}

__device__ __forceinline__ float h2f_bits(uint32_t h) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h & 0xFFFF)));
}

// Four nibbles (bytes of `v`, each 0x80|q) -> floats 1 + q/128, exact.
// byte_perm picks {0x00, 0x00, 0x80|q, 0x3F}: the fp32 pattern 0x3F80_0000 | q<<16.
__device__ __forceinline__ float nib_f(uint32_t v, uint32_t sel) {
    return __uint_as_float(__byte_perm(v, 0x3F000000u, sel));
}
constexpr uint32_t kSel0 = 0x7044, kSel1 = 0x7144, kSel2 = 0x7244, kSel3 = 0x7344;

// ---------------------------------------------------------------------------
// packed fp32x2 arithmetic (sm_100): two IEEE fp32 operations per instruction
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// ---------------------------------------------------------------------------
// timing / status
// ---------------------------------------------------------------------------
constexpr uint64_t kWaitLimitNs = 4000000000ull;  // 4 s: far above any legitimate wait

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void record_status(int* status, int code) {
    if (status) atomicCAS(status, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
            smem_u32(bar)),
        "r"(bytes)
        : "memory");
}
// A waiting thread may stay suspended in try_wait up to this many ns (it resumes as
// soon as the phase completes): fewer polling iterations of waiting warps leave more
// issue slots to the warps doing the work (measured: +4 % on the GEMM).
constexpr uint32_t kTryWaitSuspendNs = 20000;

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kTryWaitSuspendNs)
        : "memory");
    return ok != 0;
}

// try_wait without the suspend-time hint: for waits on the critical path (the softmax
// and MMA roles of the attention kernels), where a suspended thread's wake-up delay costs
__device__ __forceinline__ bool mbar_try_wait_spin(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` to complete.  Gives up when `abort` (a
// shared flag other roles raise on their own timeout) is set, or after
// kWaitLimitNs; then records FH3CUDA_E_TIMEOUT and returns false.
// mbar_wait_for takes the limit as an argument (the self-test of the wait, which has
// to run out in milliseconds, is its other caller).
template <bool SPIN = false>
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, volatile int* abort, int* status,
                                              uint64_t limit_ns) {
    auto probe = [&]() { return SPIN ? mbar_try_wait_spin(bar, parity) : mbar_try_wait(bar, parity); };
    if (probe()) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (probe()) return true;
        if ((it & 63) == 0) {
            if (*abort) return false;
            if (globaltimer() - t0 > limit_ns) {
                *abort = 1;
                record_status(status, FH3CUDA_E_TIMEOUT);
                return false;
            }
        }
    }
}
template <bool SPIN = false>
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          int* status) {
    return mbar_wait_for<SPIN>(bar, parity, abort, status, kWaitLimitNs);
}

// ---------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x,
                                            int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}
// 1-D bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16),
// completion bytes counted on `bar`.  No multicast.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// generic-proxy smem writes -> visible to the async proxy (tcgen05.mma reads)
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (cta_group::1)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 here), one thread.
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive (once) on `bar` when all tcgen05.mma issued so far by this thread finish.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// ---------------------------------------------------------------------------
// clusters and the 2-SM (cta_group::2) forms
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
// arrive on an mbarrier given by its shared::cluster address (any CTA of the cluster),
// with cluster-scope release (orders every prior memory access of this thread)
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// arrive on the peer CTA's mbarrier with the default (CTA-scope) release: the protocol
// CUTLASS's sm100 2-SM pipelines use after fence.proxy.async for shared-memory operands
// a transform stage wrote for the pair's MMA; about 1000 cycles cheaper per arrival
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kTryWaitSuspendNs)
        : "memory");
    return ok != 0;
}
// Bounded wait with cluster-scope acquire (for phases completed by the peer CTA).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort,
                                                  int* status) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((it & 63) == 0) {
            if (*abort) return false;
            if (globaltimer() - t0 > kWaitLimitNs) {
                *abort = 1;
                record_status(status, FH3CUDA_E_TIMEOUT);
                return false;
            }
        }
    }
}
// TMA load whose completion bytes are counted on an mbarrier that may live in the
// peer CTA of the pair (`bar_cluster` is a shared::cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem of both CTAs] (+)= A[smem of both CTAs] * B[smem of both CTAs]^T, issued by the leader CTA.
__device__ __forceinline__ void umma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive once on the mbarrier at the same offset in every CTA of `cta_mask` when the
// pair's outstanding MMAs finish.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(cta_mask)
        : "memory");
}

// 2^x by the hardware approximation (the MUFU instruction; a result below 2^-126 is
// flushed to zero, which a softmax weight may be)
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 32 lanes x 32 consecutive fp32 columns (one row per thread).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// tcgen05.ld fills its destination registers asynchronously: they hold the data only
// after tcgen05.wait::ld, but the compiler sees them as written by the ld itself and may
// schedule arithmetic on them ahead of the wait.  Passing them through an empty asm
// after the wait makes every use depend on a definition that follows it.
template <int W>
__device__ __forceinline__ void tmem_regs_ready(uint32_t (&r)[W]) {
#pragma unroll
    for (int i = 0; i < W; ++i) asm volatile("" : "+r"(r[i]));
}
// 32 lanes x 32 consecutive fp32 columns written back (one row per thread).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns written (one row per thread).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// out[c][p] = in[row_of(p)][c] over one 64-column x 64-position tile (columns c0.., positions
// p0..): 16-byte loads of 8 columns and 16-byte stores of 8 positions (eight lanes write one
// 128-byte run of an output row) through a shared tile of 33-word rows, so the transposed
// reads meet at most two-way bank conflicts.  row_of(p) < 0 reads zeros; nothing is stored at
// positions >= np.  256 threads.  Every in + row * ldi + c0 and out + c * ldo + p (p a
// multiple of 8) must be 16-byte aligned.
template <typename RowOf>
__device__ __forceinline__ void transpose64_bf16(const __nv_bfloat16* __restrict__ in, int64_t ldi, RowOf row_of,
                                                 int c0, int p0, int np, __nv_bfloat16* __restrict__ out,
                                                 int64_t ldo) {
    __shared__ uint32_t tile[64][33];  // [position][column pair]
    const int tid = threadIdx.x;
    for (int e = tid; e < 512; e += 256) {
        const int r = e >> 3, ch = e & 7;
        const int p = p0 + r;
        const int64_t row = p < np ? static_cast<int64_t>(row_of(p)) : -1;
        uint4 val = make_uint4(0u, 0u, 0u, 0u);
        if (row >= 0) val = __ldg(reinterpret_cast<const uint4*>(in + row * ldi + c0 + 8 * ch));
        tile[r][4 * ch + 0] = val.x;
        tile[r][4 * ch + 1] = val.y;
        tile[r][4 * ch + 2] = val.z;
        tile[r][4 * ch + 3] = val.w;
    }
    __syncthreads();
    for (int e = tid; e < 512; e += 256) {
        const int c = e >> 3, ch = e & 7;  // column c0 + c, positions p0 + 8ch .. +7
        const int p = p0 + 8 * ch;
        if (p >= np) continue;
        uint32_t h[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t w = tile[8 * ch + j][c >> 1];
            h[j] = (c & 1) ? (w >> 16) : (w & 0xFFFFu);
        }
        __nv_bfloat16* dst = out + static_cast<int64_t>(c0 + c) * ldo + p;
        if (p + 8 <= np) {
            *reinterpret_cast<uint4*>(dst) =
                make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
        } else {
            for (int j = 0; j < 8 && p + j < np; ++j)
                reinterpret_cast<unsigned short*>(dst)[j] = static_cast<unsigned short>(h[j]);
        }
    }
}

// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle
// layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B: rows of 128 B (64 bf16),
// 8-row atoms of 1024 B (stride-byte-offset), version 1, layout 2 (SW128).
// The tile base must be 1024-byte aligned; a K offset inside the 128-byte row
// is applied by adding bytes>>4 to the start-address field.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFF) >> 4);
    d |= static_cast<uint64_t>(1) << 16;           // leading-byte-offset (unused for SW128 K-major)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;   // stride-byte-offset: 8 rows x 128 B
    d |= static_cast<uint64_t>(1) << 46;           // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2) << 61;           // SWIZZLE_128B
    return d;
}

// Instruction descriptor: kind::f16 with bf16 A and B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n) {
    return (1u << 4)                                  // D format: f32
           | (1u << 7)                                // A format: bf16
           | (1u << 10)                               // B format: bf16
           | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
           | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

}  // namespace fh3

// Host-side helpers shared by the translation units (defined in api.cu).
namespace fh3host {
struct DevCtx;
DevCtx* ctx();                       // context of the current device (nullptr if not initialised)
int* ctx_status(DevCtx* c);          // device status word
int ctx_sms(DevCtx* c);
int ctx_device(DevCtx* c);               // CUDA ordinal of the context (-1 if none)
int set_error(int code, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);
// cuTensorMapEncodeTiled through the runtime's driver entry point
CUresult encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, cuuint32_t rank, void* gaddr,
                      const cuuint64_t* gdim, const cuuint64_t* gstride, const cuuint32_t* box,
                      const cuuint32_t* estride, CUtensorMapSwizzle swz);
// scratch of at least `bytes` for slot `slot` (cached, grows)
void* scratch(DevCtx* c, int slot, size_t bytes, cudaStream_t s);
// the same, zero-filled whenever it is (re)allocated; users keep it zero between calls
void* scratch_zeroed(DevCtx* c, int slot, size_t bytes, cudaStream_t s);
// 1..16-token Q4_K GEMV on warp-level tensor-core MMAs (gemv_mma.cu); arguments
// already validated by the caller
int gemv_mma(const Fh3CudaW* w, const float* x, float* y, int n_tok, const float* bias, cudaStream_t s);
// 1..16-token Q4_K GEMV on tcgen05 MMAs (gemv_tc.cu); returns 1 without launching
// when the shape or pointers do not suit it
int gemv_tc(const Fh3CudaW* w, const float* x, float* y, int n_tok, const float* bias, cudaStream_t s);
// the fp32 CUDA-core GEMV (gemv.cu): uses no memory beyond x, y, bias and the weights
int gemv_fp32(const Fh3CudaW* w, const float* x, float* y, int n_tok, const float* bias, cudaStream_t s);
// dense attention on tcgen05, head_dim 128 (attention_tc.cu); arguments already validated
int attention_tc(const __nv_bfloat16* q, int64_t ldq, const __nv_bfloat16* k, int64_t ldk, const __nv_bfloat16* v,
                 int64_t ldv, void* o, bool o_bf16, int64_t ldo, int n, int heads, cudaStream_t s);
// video sparse attention's fine pass + coarse * gate on tcgen05 (vsa_tc.cu): tiles of at most
// 64 tokens, head_dim 128, bf16 operands; the tile-stage arrays come from vsa.cu
int vsa_fine_tc(const int* perm, const int* toff, const int* sel, const int* selcnt, int nt, int n,
                const __nv_bfloat16* q, int64_t ldq, const __nv_bfloat16* k, int64_t ldk, const __nv_bfloat16* v,
                int64_t ldv, const __nv_bfloat16* gate, int64_t ldg, const float* outc, int heads, void* o, bool o_bf16,
                int64_t ldo, cudaStream_t s);
// fp32 softmax attention (attention_f32.cu): dense over n keys when sel is null, else
// the fine pass of video sparse attention over the kept key tiles (+ outc * gate)
int attention_f32_launch(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv,
                         float* o, int64_t ldo, int n, int heads, int head_dim, const int* perm, const int* toff,
                         const int* sel, const int* selcnt, int nt, const float* gate, int64_t ldg,
                         const float* outc, cudaStream_t s);
// argument checks shared by the GEMV entry points (FH3_OK or the error code, message set)
int gemv_args_ok(const Fh3CudaW* w, const float* x, const float* y, int n_tok, const char* who);
// fh3cuda_gemm_q4k_dev's body (gemm.cu); fused_only never takes the two-pass path,
// which is the one GEMM path that needs scratch (its bf16 weight copy)
int gemm_q4k(const Fh3CudaW* w, const void* x_bf16, int64_t ldx, void* y, int64_t ldy, int64_t n_tok,
             const float* bias, const float* gate, int epi, void* stream, bool fused_only);
// fh3cuda_gemm_bf16w_dev with a weight row stride (ldw elements, >= in, a multiple of 8)
int gemm_bf16w(const void* w_bf16, int64_t ldw, int64_t out, int64_t in, const void* x_bf16, int64_t ldx, void* y,
               int64_t ldy, int64_t n_tok, const float* bias, const float* gate, int epi, int flags, cudaStream_t s);
// fh3_matmul for the formats other than Q4_K (formats.cu): arguments checked by the caller
// except the format and block rules
int matmul_formats(DevCtx* c, const Fh3CudaW* w, const float* x, float* y, int n_tok, const float* bias,
                   cudaStream_t s);
// cudaMalloc that the library counts (fh3cuda_alloc_stats) and that honours the scratch
// limit when `limited` (FH3_E_NOMEM with the message set on failure or refusal)
int dev_alloc(void** p, size_t bytes, bool limited, const char* who);
void dev_free(void* p, size_t bytes, bool limited);
}  // namespace fh3host
