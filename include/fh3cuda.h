/*
 * fh3cuda.h -- C ABI of libfh3cuda, the sm_100a (B200) implementation of fh3's
 * Q4_K dequantise-and-multiply path.
 *
 * The reference engine (fh3, C99, CPU only) sends every DiT projection through
 *     void fh3_matmul(const Fh3W *w, const float *x, float *y, int n_tok,
 *                     const float *bias_or_null);          (include/fh3/fh3.h:107)
 * which dequantises Q4_K weight tiles (src/core/fh3_quant.c:154-196) and runs
 * AVX2/FMA dot products under OpenMP (src/core/fh3_ops.c:317-404).  This
 * library replaces that function.  Plain pointers and sizes only: no C++ or
 * torch types cross this boundary.
 *
 * Conventions
 *   - Every entry point except the void drop-in returns an int status:
 *     FH3_OK (0) or a negative code.  The codes reuse fh3's values
 *     (include/fh3/fh3.h:218-226) and add three of their own.
 *   - "_dev" entry points take device pointers and a cudaStream_t passed as
 *     void* (NULL = the legacy default stream); they are asynchronous.
 *   - Weights are fh3 rows: row o of a matrix of type t with `in` columns
 *     starts at data + o * fh3cuda_row_bytes(t, in); for block formats `in`
 *     must be a multiple of the block (256 for the K-quants, 32 for Q8_0).
 *   - Device-side waits inside the kernels are bounded; a wait that gives up
 *     records FH3CUDA_E_TIMEOUT in the device status word, read by
 *     fh3cuda_device_status().
 *   - Stream order: the GEMV and GEMM kernels are launched as programmatic
 *     dependents of the previous kernel on their stream and start reading
 *     their Q4_K weights before that kernel has finished (activations, bias,
 *     gate and outputs only after it).  Weights written by a copy, or by a
 *     kernel that runs to completion before its dependents start (every
 *     kernel of this library that writes weights does), are safe; weights
 *     written by a foreign kernel that signals its dependents early
 *     (griddepcontrol.launch_dependents) must be ordered with an event or a
 *     synchronisation before the call.
 */
#ifndef FH3CUDA_H
#define FH3CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FH3CUDA_API __attribute__((visibility("default")))
#else
#define FH3CUDA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (values of include/fh3/fh3.h:218-226, plus three). */
#define FH3_OK              0
#define FH3_ERR           (-1)
#define FH3_E_IO          (-2)
#define FH3_E_TRUNCATED   (-3)
#define FH3_E_BAD_MAGIC   (-4)
#define FH3_E_BAD_VERSION (-5)
#define FH3_E_NOMEM       (-7)
#define FH3_E_INVALID     (-8)
#define FH3CUDA_E_CUDA    (-20)  /* a CUDA runtime/driver call failed        */
#define FH3CUDA_E_TIMEOUT (-21)  /* a bounded device-side wait gave up       */
#define FH3CUDA_E_NODEV   (-22)  /* no usable sm_100 device / not initialised */

/* Weight types this path accepts (GGML ids, include/fh3/fh3.h:63-79). */
#define FH3CUDA_TYPE_F32  0   /* fh3's enum values, include/fh3/fh3.h:64-78 */
#define FH3CUDA_TYPE_F16  1
#define FH3CUDA_TYPE_Q8_0 8
#define FH3CUDA_TYPE_Q2_K 10
#define FH3CUDA_TYPE_Q3_K 11
#define FH3CUDA_TYPE_Q4_K 12
#define FH3CUDA_TYPE_Q5_K 13
#define FH3CUDA_TYPE_Q6_K 14
#define FH3CUDA_TYPE_BF16 30

/* Same layout as the reference's weight descriptor Fh3W
 * (include/fh3/fh3.h:82-87), so a pointer to one may be passed as the other. */
typedef struct Fh3CudaW {
    int type;
    int64_t in;
    int64_t out;
    const uint8_t *data;
} Fh3CudaW;

/* ---- library state --------------------------------------------------- */

/* Select `device` for the calling thread and set up its context (streams,
 * status word, tensor-map entry point).  Replaces nothing in fh3 (it has no
 * device); must precede the other calls on that device. */
FH3CUDA_API int fh3cuda_init(int device);

/* Message of the most recent failure on the calling thread ("" if none). */
FH3CUDA_API const char *fh3cuda_last_error(void);

/* Sticky status of the void drop-in (fh3cuda_matmul / __wrap_fh3_matmul),
 * which cannot return one: the first failure since the last call, then
 * cleared.  fh3_matmul itself returns silently on bad arguments
 * (src/core/fh3_ops.c:318-321); the drop-in records FH3_E_INVALID instead. */
FH3CUDA_API int fh3cuda_take_status(void);

/* Synchronise `stream` and read (then clear) the device status word that
 * bounded device-side waits write.  FH3_OK, FH3CUDA_E_TIMEOUT or
 * FH3CUDA_E_CUDA. */
FH3CUDA_API int fh3cuda_device_status(void *stream);

/* Number of SMs of the current device (0 before fh3cuda_init). */
FH3CUDA_API int fh3cuda_sm_count(void);

/* Device-memory budget for the library's scratch (0 = unlimited, the default), over
 * all devices.  A call whose scratch would grow past it fails with FH3_E_NOMEM and
 * computes nothing (the void drop-in records it as its sticky status).  No counterpart
 * in the reference, whose nearest equivalent is the host-memory plan preflight of the
 * trunk streamer (src/io/fh3_trunk.c:101-129). */
FH3CUDA_API void fh3cuda_set_scratch_limit(uint64_t bytes);

/* Self-test of the bounded device-side wait that every kernel's mbarrier waits use:
 * launches one thread that waits on an mbarrier nobody arrives at, with a limit of
 * limit_ns (at most 2 s) instead of the kernels' 4 s.  Nothing else is in flight; the
 * wait gives up, the kernel returns and fh3cuda_device_status then reports
 * FH3CUDA_E_TIMEOUT, with the context still usable.  No counterpart in the reference
 * (its CPU code has no device waits). */
FH3CUDA_API int fh3cuda_wait_selftest_dev(uint64_t limit_ns, void *stream);

/* Library allocation counters: cudaMalloc calls made so far (scratch growth, context
 * set-up, weight uploads, trunk and table uploads) and scratch bytes currently held.
 * No counterpart in the reference (diagnostics). */
FH3CUDA_API void fh3cuda_alloc_stats(uint64_t *alloc_calls, uint64_t *scratch_bytes);

/* ---- format ------------------------------------------------------------ */

/* Bytes of one weight row: replaces fh3_row_bytes (include/fh3/fh3.h:103,
 * src/core/fh3_quant.c:14-34) for the formats fh3_dequant expands (F32, F16,
 * BF16, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K); 0 for other types. */
FH3CUDA_API size_t fh3cuda_row_bytes(int type, int64_t n);

/* Dequantise `rows` rows of `n` weights of any format above to fp32,
 * bit-exact with fh3_dequant (include/fh3/fh3.h:104, src/core/fh3_quant.c:36-318):
 * dst[r*n + k].  Like the reference, only whole blocks are written; a partial
 * trailing block of a row is left untouched.  Q4_K sources must be 16-byte
 * aligned. */
FH3CUDA_API int fh3cuda_dequant_dev(int type, const void *src, float *dst, int64_t rows, int64_t n,
                        void *stream);

/* ---- the matmul ------------------------------------------------------------ */

/* y[t][o] = sum_k x[t][k] * W[o][k] (+ bias[o]), all pointers on the device.
 * Replaces fh3_matmul (include/fh3/fh3.h:107, src/core/fh3_ops.c:317-404) on
 * device buffers.  Q4_K (the DiT trunk): n_tok <= 16 runs the GEMV (relative
 * Frobenius error <= 1e-5 against fh3_matmul); larger n_tok runs the tcgen05
 * GEMM on bf16 operands with fp32 accumulation (<= 5e-3).  Every other format
 * fh3_dequant expands (the text encoder's Q5_K / Q6_K, F16 / F32 globals, ...):
 * weights formed bit-exactly as fh3_dequant's fp32 values, then up to 16 tokens an
 * fp32 CUDA-core GEMV, above that the tcgen05 GEMM on the four bf16 products of
 * weights and activations split into high and low bf16 parts (<= 1e-5 both).
 * Internal scratch is cached per device and grows on demand. */
FH3CUDA_API int fh3cuda_matmul_dev(const Fh3CudaW *w, const float *x, float *y, int n_tok,
                       const float *bias_or_null, void *stream);

/* fh3cuda_matmul_dev without device allocation on the call path: no counterpart in
 * the reference.  For callers that cannot let a library call cudaMalloc while they
 * run: hosts that budget device memory once up front, processes whose device memory
 * belongs to another allocator, and latency-critical loops that cannot afford the
 * device synchronisation cudaMalloc/cudaFree may cause.  The bf16 activation scratch
 * is a fixed 8 MiB static device array (n_tok * in <= 4,194,304 when n_tok > 16;
 * larger calls return FH3_E_INVALID), held by every GPU that loads the library.
 * Set-up: fh3cuda_init(device), then the first call on a device resolves the array's
 * address (make that first call before any stream capture).  All calls share the
 * array: calls that overlap on the GPU race and must be serialised.  More than 16
 * tokens always run the fused GEMM kernels (never the two-pass path with its bf16
 * weight copy, whatever FH3CUDA_GEMM_KERNEL says), so no row count allocates.  The
 * library's per-device state, this array's cached address included, does not survive
 * cudaDeviceReset. */
FH3CUDA_API int fh3cuda_matmul_noalloc_dev(const Fh3CudaW *w, const float *x, float *y, int n_tok,
                                           const float *bias_or_null, void *stream);

/* The drop-in: same signature and meaning as fh3_matmul
 * (include/fh3/fh3.h:107) on HOST buffers.  w->data is looked up in the
 * registered weight ranges (fh3cuda_register_weights); an unregistered
 * pointer is staged to the device for this call.  x is copied in, y copied
 * out; the call returns when y is written.  Failures are recorded for
 * fh3cuda_take_status() and printed to stderr once.  If the calling thread's
 * current device has no context yet, the first call sets it up (fh3cuda_init),
 * so an unmodified fh3 program needs no added call. */
FH3CUDA_API void fh3cuda_matmul(const Fh3CudaW *w, const float *x, float *y, int n_tok,
                    const float *bias_or_null);

/* Link-time interposer for the unmodified reference objects: link the fh3
 * application with -Wl,--wrap=fh3_matmul and this library, and every call of
 * fh3_matmul (src/model/fh3_dit.c:388-461, src/model/fh3_te.c:455-487) lands
 * here.  Identical to fh3cuda_matmul. */
FH3CUDA_API void __wrap_fh3_matmul(const Fh3CudaW *w, const float *x, float *y, int n_tok,
                       const float *bias_or_null);

/* Map the host range [host, host+bytes) to the device range starting at
 * `dev` for the drop-in's weight lookup.  This stands in for the reference's
 * trunk ring (src/io/fh3_trunk.c:409-501): weights are uploaded once and
 * stay resident in HBM. */
FH3CUDA_API int fh3cuda_register_weights(const void *host, size_t bytes, const void *dev);
FH3CUDA_API int fh3cuda_unregister_weights(const void *host);

/* cudaMalloc + copy + register in one call; *dev_out receives the device
 * copy, owned by the library until fh3cuda_release_weights(host). */
FH3CUDA_API int fh3cuda_upload_weights(const void *host, size_t bytes, void **dev_out);
FH3CUDA_API int fh3cuda_release_weights(const void *host);

/* ---- explicit kernels (tests, benchmarks, fused trunk) ----------------- */

/* Q4_K GEMV, 1 <= n_tok <= 16; same contract as fh3cuda_matmul_dev.  Tensor-core
 * kernels: warp-level integer MMAs of the nibbles against base-256 digits of x at 1-2
 * tokens, and at 3-4 when out > in; otherwise tcgen05 MMAs (integer MMAs of the nibbles up
 * to 5 tokens; from 6, f16 MMAs of sc*q against x in two f16 pieces).
 * FH3CUDA_GEMV_KERNEL in the environment selects one: tc (tcgen05 for every shape),
 * mma-i8 (the integer warp-level kernels, 1-4 tokens), mma-stream / mma-cta (warp-level
 * f16 MMAs), fp32 (the fp32 CUDA-core kernel). */
FH3CUDA_API int fh3cuda_gemv_q4k_dev(const Fh3CudaW *w, const float *x, float *y, int n_tok,
                         const float *bias_or_null, void *stream);

/* Epilogues of the tcgen05 GEMM. */
#define FH3CUDA_EPI_F32      0  /* y (fp32)  = acc + bias                              */
#define FH3CUDA_EPI_BF16     1  /* y (bf16)  = acc + bias                              */
#define FH3CUDA_EPI_SWIGLU   2  /* y (bf16)[t][f] = v * silu(g) of the fused [up;gate]
                                   weight, value-first halves (src/core/fh3_ops.c:507-527) */
#define FH3CUDA_EPI_RESID    3  /* y (fp32) += gate[o] * (acc + bias), as fh3_gate_residual
                                   (src/core/fh3_ops.c:559-585)                         */

/* tcgen05 GEMM on bf16 activations: y = epi(x_bf16 . W^T), x_bf16 holding
 * n_tok rows of K = w->in values with row stride ldx elements (ldx >= K, a
 * multiple of 8).  W is Q4_K, dequantised to bf16 in shared memory by the GEMM
 * (fewer than 2048 rows), or from 2048 rows on expanded once per call to a bf16
 * copy in device scratch that a TMA-fed kernel reads (each weight is then
 * dequantised once per call instead of once per 256-row tile; same bf16 values,
 * same results).  ldy is the row stride of y in elements.  gate is used by FH3CUDA_EPI_RESID only.
 * For FH3CUDA_EPI_SWIGLU, W holds 2F rows ([up; gate]) and y has F columns. */
FH3CUDA_API int fh3cuda_gemm_q4k_dev(const Fh3CudaW *w, const void *x_bf16, int64_t ldx, void *y,
                                     int64_t ldy, int64_t n_tok, const float *bias_or_null,
                                     const float *gate, int epilogue, void *stream);

/* The two halves of the two-pass path, for callers that schedule them themselves (the
 * trunk runner expands the next projection's weights on a second stream while the
 * current GEMM runs).  fh3cuda_q4k_to_bf16_dev writes w's Q4_K rows as bf16 [out][in]
 * (fh3's fp32 weight, dequant_q4_k of src/core/fh3_quant.c:154-196, rounded once to
 * bf16: the values the fused GEMM dequantisers feed the tensor cores); w_bf16 holds
 * out * in elements, 16-byte aligned.  fh3cuda_gemm_bf16w_dev is
 * fh3cuda_gemm_q4k_dev's GEMM on such a bf16 [out][in] weight matrix (in a multiple of
 * 64): same epilogues, same results as the Q4_K entry point on the matrix it expands
 * to.  Together they replace fh3_matmul's large-M regime (src/core/fh3_ops.c:317-404).
 * The GEMM is launched as a programmatic dependent of the previous kernel on `stream`
 * (its set-up overlaps that kernel's end; it reads and writes activations only after
 * that kernel has finished).  flags: FH3CUDA_GEMM_WEIGHTS_READY when w_bf16 was
 * complete before the previous kernel on `stream` began (written on another stream
 * and waited for with an event, or earlier on this stream): the GEMM may then load
 * its first weight tiles while that kernel still runs; 0 otherwise. */
#define FH3CUDA_GEMM_WEIGHTS_READY 1
FH3CUDA_API int fh3cuda_q4k_to_bf16_dev(const Fh3CudaW *w, void *w_bf16, void *stream);
FH3CUDA_API int fh3cuda_gemm_bf16w_dev(const void *w_bf16, int64_t out, int64_t in, const void *x_bf16,
                                       int64_t ldx, void *y, int64_t ldy, int64_t n_tok,
                                       const float *bias_or_null, const float *gate, int epilogue,
                                       int flags, void *stream);

/* Kernel launches one fh3cuda_gemm_q4k_dev call of n_tok rows makes: 1 for the
 * fused kernels, 2 from 2048 rows on, where the weights are first expanded to a
 * bf16 copy (the same bf16 values the fused dequantisers produce) and a TMA-fed
 * bf16 pair kernel runs the tiles.  FH3CUDA_GEMM_KERNEL=2sm / 1sm / two-pass in the
 * environment forces a path.  A call whose tiles would keep at most half of the CTA
 * pairs busy (small n_tok and out, not SwiGLU) splits each tile's K range on the fused
 * pair kernel and adds one reduction launch, not counted here
 * (FH3CUDA_GEMM_SPLITK=0 keeps whole tiles). */
FH3CUDA_API int fh3cuda_gemm_launches(int64_t n_tok);

/* fp32 -> bf16 (round to nearest even), n elements. */
FH3CUDA_API int fh3cuda_f32_to_bf16_dev(const float *x, void *y_bf16, int64_t n, void *stream);

/* Fused GEMM prologue: y_bf16 = bf16(modulate(rmsnorm(x, w, eps), shift, scale))
 * per row, as fh3_rmsnorm (src/core/fh3_ops.c:410-456) then fh3_modulate
 * (:529-557) with shift/scale broadcast from [dim] vectors.  norm_w may be
 * NULL (all ones). */
FH3CUDA_API int fh3cuda_rmsnorm_modulate_dev(const float *x, const float *norm_w, const float *shift,
                                 const float *scale, void *y_bf16, int n, int dim, float eps,
                                 void *stream);

/* fh3_swiglu (src/core/fh3_ops.c:507-527) on device fp32 buffers. */
FH3CUDA_API int fh3cuda_swiglu_dev(const float *in, float *out, int n, int F, void *stream);

/* q or k after the QKV projection, as fh3_dit.c:397-401: fh3_rmsnorm over each
 * head (src/core/fh3_ops.c:410-456, rows = n*heads, dim = head_dim, weights
 * norm_w[head_dim]) then fh3_rope3 (:458-505, cos/sin [n][rot_dim]), fused and
 * bit-exact with the reference.  Row i of src / dst starts at i*ld_src / i*ld_dst
 * elements and holds heads*head_dim elements (a strided view of the QKV output
 * works); element types fp32 or bf16 (flags src_bf16 / dst_bf16; a bf16 output
 * is the fp32 result rounded once).  head_dim a multiple of 32 up to 256;
 * rot_dim even, 0 (normalisation only) .. head_dim; strides multiples of 8,
 * pointers 16-byte aligned.  src == dst (in place) needs the same type and
 * stride; other overlaps are not allowed. */
FH3CUDA_API int fh3cuda_qk_norm_rope_dev(const void *src, int src_bf16, int64_t ld_src, void *dst, int dst_bf16,
                                         int64_t ld_dst, const float *norm_w, const float *cos_t,
                                         const float *sin_t, int n, int heads, int head_dim, int rot_dim,
                                         float eps, void *stream);

/* Dense, non-causal softmax attention, fh3_attention (include/fh3/fh3.h:117,
 * src/core/fh3_ops.c:587-695): o = softmax(q k^T / sqrt(128)) v per head, on
 * bf16 q/k/v with fp32 softmax and accumulation (rel. error of bf16 operands,
 * not bit-exact).  head_dim 128.  Element (token i, head h, channel d) of q is
 * q[i*ldq + h*128 + d] (likewise k, v; o with ldo), so the thirds of a bf16
 * QKV output can be passed directly.  o is fp32 (o_bf16 = 0) or bf16.  Strides
 * multiples of 8, pointers 16-byte aligned.  Kernel: tcgen05 with two query tiles a
 * CTA. */
FH3CUDA_API int fh3cuda_attention_dev(const void *q, int64_t ldq, const void *k, int64_t ldk, const void *v,
                                      int64_t ldv, void *o, int o_bf16, int64_t ldo, int n, int heads,
                                      int head_dim, void *stream);

/* The fields of the reference's struct Fh3Seq (src/model/fh3_seq.h:31-38) that
 * video sparse attention reads: N = text + audio + video tokens in that order,
 * and the video grid (t, h, w) in tokens.  Counts that do not add up to seq_len
 * make the whole sequence video; a grid whose product is not num_video is taken
 * as (1, 1, num_video) (src/core/fh3_vsa.c:42-64). */
typedef struct Fh3CudaSeq {
    int32_t seq_len;
    int32_t num_text;
    int32_t num_audio;
    int32_t num_video;
    int32_t grid_t;
    int32_t grid_h;
    int32_t grid_w;
} Fh3CudaSeq;

/* Tile counts of a sequence for video sparse attention (build_vsa_geometry,
 * src/core/fh3_vsa.c:32-161): text and audio runs of `tile` tokens (tile <= 0:
 * 64) and 4x4x4 cells of the video grid.  Any output pointer may be NULL. */
FH3CUDA_API int fh3cuda_vsa_num_tiles(const Fh3CudaSeq *seq, int tile, int *num_tiles, int *num_prefix,
                                      int *num_video);

/* Video sparse attention, fh3_vsa_attention (include/fh3/fh3.h:118,
 * src/core/fh3_vsa.c:186-507), with Fh3VsaCfg's fields (tile, sparsity) passed
 * directly.  Element (token t, head h, channel d) of q is q[t*ldq + h*head_dim
 * + d]; likewise k, v, gate and o.  q, k, v and gate are fp32 (in_bf16 = 0) or
 * bf16; o is fp32 (o_bf16 = 0) or bf16.  gate may be NULL (no coarse branch, as
 * in the reference).  The tile means, tile scores and the kept key tiles are
 * computed in fp32 in the reference's order, so the tile mask is the
 * reference's bit for bit.  With bf16 operands the fine attention runs on
 * tensor cores with fp32 softmax and accumulation (bf16 operand error, not
 * bit-exact); their strides must be multiples of 8 and the pointers (q, k, v,
 * gate, o) 16-byte aligned.  With fp32 operands it runs in fp32 (the CPU
 * path's accuracy) and o must be fp32.  head_dim 64 or 128.  bf16 fine pass: tcgen05
 * with M = 64 query tiles (head_dim 128, tiles of at most 64 tokens), mma.sync
 * otherwise; FH3CUDA_VSA_KERNEL=mma in the environment forces mma.sync. */
FH3CUDA_API int fh3cuda_vsa_attention_dev(int tile, float sparsity, const Fh3CudaSeq *seq, const void *q,
                                          int64_t ldq, const void *k, int64_t ldk, const void *v, int64_t ldv,
                                          int in_bf16, const void *gate, int64_t ldg, void *o, int o_bf16,
                                          int64_t ldo, int heads, int head_dim, void *stream);

/* fh3_attention on fp32 operands in fp32 arithmetic (the CPU path's accuracy,
 * for parity work and small shapes; the bf16 tensor-core kernel above carries
 * the production shapes).  Layout as fh3cuda_attention_dev; head_dim a
 * multiple of 32 up to 256. */
FH3CUDA_API int fh3cuda_attention_f32_dev(const float *q, int64_t ldq, const float *k, int64_t ldk, const float *v,
                                          int64_t ldv, float *o, int64_t ldo, int n, int heads, int head_dim,
                                          void *stream);

/* The tile stage of fh3cuda_vsa_attention_dev alone: tile scores [heads][T][T]
 * fp32 (src/core/fh3_vsa.c:268-281) into `scores` and the 0/1 tile mask
 * [heads][T][T] (:283-356) into `mask` (device buffers; either may be NULL),
 * T = num_tiles.  Synchronises the stream when the mask is asked for. */
FH3CUDA_API int fh3cuda_vsa_tiles_dev(int tile, float sparsity, const Fh3CudaSeq *seq, const void *q, int64_t ldq,
                                      const void *k, int64_t ldk, int in_bf16, int heads, int head_dim,
                                      float *scores, uint8_t *mask, void *stream);

/* ---- packed trunk and AdaLN table, resident in HBM ------------------------ */

/* A packed DiT trunk (FH3P, src/io/fh3_pack.h:29-88) read once into device
 * memory: replaces fh3_pack_open + the NVMe ring of fh3_trunk_open /
 * fh3_trunk_acquire (src/io/fh3_pack.c:23-106, src/io/fh3_trunk.c:135-501).
 * Errors as fh3_pack_open: FH3_E_IO, FH3_E_TRUNCATED, FH3_E_BAD_MAGIC,
 * FH3_E_BAD_VERSION, FH3_E_INVALID, plus FH3_E_NOMEM. */
typedef struct Fh3CudaPack Fh3CudaPack;

/* fh3's Fh3LayerView (include/fh3/fh3.h:90-100) with device data pointers */
typedef struct Fh3CudaLayerView {
    Fh3CudaW qkv;
    Fh3CudaW gate_compress;
    Fh3CudaW out;
    Fh3CudaW fc1;
    Fh3CudaW fc2;
    Fh3CudaW norm1;
    Fh3CudaW norm2;
    Fh3CudaW q_norm;
    Fh3CudaW k_norm;
} Fh3CudaLayerView;

FH3CUDA_API int fh3cuda_pack_open(const char *path, Fh3CudaPack **out);
FH3CUDA_API int fh3cuda_pack_num_layers(const Fh3CudaPack *p);
FH3CUDA_API uint64_t fh3cuda_pack_device_bytes(const Fh3CudaPack *p);
/* fh3_pack_layer / fh3_trunk_layer (src/io/fh3_pack.c:140-205) */
FH3CUDA_API int fh3cuda_pack_layer(const Fh3CudaPack *p, int L, Fh3CudaLayerView *out);
FH3CUDA_API void fh3cuda_pack_close(Fh3CudaPack *p);

/* The folded AdaLN table (FH3A) in device memory: fh3_adaln_open (expect_hash
 * 0 skips the schedule check) and fh3_adaln_row (src/io/fh3_pack.c:188-355);
 * a row is a device pointer to hidden_size floats, NULL outside the table. */
typedef struct Fh3CudaAdaln Fh3CudaAdaln;
FH3CUDA_API int fh3cuda_adaln_open(const char *path, uint64_t expect_hash, Fh3CudaAdaln **out);
FH3CUDA_API int fh3cuda_adaln_dims(const Fh3CudaAdaln *a, int *n_steps, int *n_blocks, int *pairs_per_step,
                                   int *hidden_size);
FH3CUDA_API const float *fh3cuda_adaln_row(const Fh3CudaAdaln *a, int step, int block, int pair, int chunk);
FH3CUDA_API void fh3cuda_adaln_close(Fh3CudaAdaln *a);

/* ---- the DiT forward on the device ----------------------------------------- */

/* The fields of fh3's Fh3DitCfg (src/model/fh3_dit.h:19-39) the forward uses, and
 * one of this library's: attn_bf16 = 0 runs attention in fp32 (the CPU path's
 * accuracy), 1 on bf16 tensor cores (dense attention then needs head_dim 128). */
typedef struct Fh3CudaDitCfg {
    int32_t attn;          /* 0 dense (FH3_ATTN_DENSE), 1 video sparse (FH3_ATTN_VSA) */
    int32_t vsa_tile;      /* Fh3VsaCfg.tile (<= 0: 64) */
    float vsa_sparsity;    /* Fh3VsaCfg.sparsity */
    int32_t hidden_size;
    int32_t num_heads;
    int32_t head_dim;
    int32_t num_layers;
    int32_t num_refiner_layers;  /* 0..4 */
    int32_t ffn_dim;
    float norm_eps;
    float qk_norm_eps;
    float final_norm_eps;
    int32_t attn_bf16;
} Fh3CudaDitCfg;

/* Fh3RefinerBlock (src/model/fh3_dit.h:41-50) with device pointers */
typedef struct Fh3CudaRefinerBlock {
    const float *norm1;
    Fh3CudaW qkv;
    const float *q_norm;
    const float *k_norm;
    Fh3CudaW out;
    const float *norm2;
    Fh3CudaW fc1;
    Fh3CudaW fc2;
} Fh3CudaRefinerBlock;

/* The global weights of fh3's Fh3Dit (src/model/fh3_dit.h:52-86: patch and
 * condition projections, text refiner, final layer) as device data; a host loads
 * them from dit_globals (fh3_dit_open, src/model/fh3_dit.c:55-180) and uploads
 * them once.  Biases may be NULL. */
typedef struct Fh3CudaDitGlobals {
    Fh3CudaW video_patch_proj;
    const float *video_patch_proj_bias;
    Fh3CudaW audio_patch_proj;
    const float *audio_patch_proj_bias;
    Fh3CudaW condition_proj;
    const float *condition_proj_bias;
    Fh3CudaRefinerBlock refiner[4];
    const float *refiner_final_norm;
    const float *final_norm;
    Fh3CudaW video_out;
    const float *video_out_bias;
    Fh3CudaW audio_out;
    const float *audio_out_bias;
} Fh3CudaDitGlobals;

/* fh3_dit_prepare_text (src/model/fh3_dit.c:221-281): text_emb [T][text_dim] ->
 * text_rows [T][hidden_size], device fp32. */
FH3CUDA_API int fh3cuda_dit_prepare_text_dev(const Fh3CudaDitCfg *cfg, const Fh3CudaDitGlobals *g,
                                             const float *text_emb, int T, float *text_rows, void *stream);

/* fh3_dit_forward (src/model/fh3_dit.c:283-467) for denoising step `step`: trunk
 * layers from a resident pack, modulation from a resident AdaLN table, rows text
 * | audio | video as seq counts them, cos_t / sin_t the [seq_len][96] rope tables
 * of fh3_seq_build (src/model/fh3_seq.c:147-168); x_video [V][video patch dim],
 * x_audio [A][audio patch dim], text_rows [T][hidden] -> v_video, v_audio.  All
 * device fp32.  FH3_E_INVALID for a step outside the table (as the reference). */
FH3CUDA_API int fh3cuda_dit_forward_dev(const Fh3CudaDitCfg *cfg, const Fh3CudaDitGlobals *g,
                                        const Fh3CudaPack *trunk, const Fh3CudaAdaln *adaln,
                                        const Fh3CudaSeq *seq, const float *cos_t, const float *sin_t, int step,
                                        const float *x_video, const float *x_audio, const float *text_rows,
                                        float *v_video, float *v_audio, void *stream);

/* Seeded synthetic Q4_K weights on the device: rows x n weights drawn from
 * scale * N(0,1) (Philox4x32-10 + Box-Muller), quantised with the same
 * per-block rule as the project's CPU quantiser.  Benchmark input generator;
 * values need not match the CPU generator bit for bit. */
FH3CUDA_API int fh3cuda_make_q4k_weights_dev(uint64_t seed, uint64_t stream_id, float scale, int64_t rows,
                                 int64_t n, void *dst, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* FH3CUDA_H */
