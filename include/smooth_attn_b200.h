/*
 * smooth_attn_b200.h — C ABI of the B200 (sm_100a) smooth-attn hot path.
 *
 * Every entry point is `extern "C"`, takes plain device pointers, sizes and
 * strides (in ELEMENTS), launches on the given CUDA stream (a cudaStream_t
 * passed as void*, NULL = legacy default stream), never allocates device
 * memory, never synchronises, and returns an sa_status (0 = success).
 * Arguments are validated before anything is launched; a rejected call has
 * no side effects.  The library is stateless apart from per-device attribute
 * caches, so calls are thread-safe.
 *
 * Each declaration names the reference interface it replaces
 * (NoSelection/smooth-attn, file:line).
 */
#ifndef SMOOTH_ATTN_B200_H
#define SMOOTH_ATTN_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define SA_API __attribute__((visibility("default")))
#else
#define SA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define SA_OK 0
#define SA_ERR_ARG (-1)         /* bad size / null pointer / bad family       */
#define SA_ERR_ALIGN (-2)       /* pointer or stride alignment not supported   */
#define SA_ERR_UNSUPPORTED (-3) /* dtype / head dim / shape not implemented    */
#define SA_ERR_LAUNCH (-4)      /* CUDA launch error (cudaGetLastError)        */
#define SA_ERR_TIMEOUT (-5)     /* a bounded device-side wait gave up          */
#define SA_ERR_CUDA (-6)        /* other CUDA runtime/driver error             */
#define SA_ERR_BOUNDS (-7)      /* debug build: a device-side index check failed */

/* Element types. */
#define SA_F32 0
#define SA_F16 1
#define SA_BF16 2

/* Library version, (major << 16) | minor. */
SA_API int sa_version(void);

/* Human-readable text for a status code (static storage). */
SA_API const char* sa_status_string(int status);

/* Text of the last CUDA error seen by this thread inside the library. */
SA_API const char* sa_last_cuda_error(void);

/*
 * Device-side status of the current device: SA_ERR_TIMEOUT if any kernel of
 * this library gave up a bounded wait (an mbarrier / copy that never
 * completed) since the last reset, else SA_OK.  Synchronises the device.
 * Otherwise SA_ERR_BOUNDS if (debug library only) a device-side index check
 * failed, otherwise SA_ERR_ARG if sa_paged_decode met a block_table entry
 * outside [0, num_blocks) since the last reset.
 * reset != 0 clears the recorded status.  (No reference counterpart: the
 * reference's Triton kernels have no bounded waits.)
 */
SA_API int sa_device_status(int reset);

/*
 * sa_device_status scoped to one stream: synchronises only `stream` (not the
 * device), then reads and optionally clears the same counters through copies
 * on that stream.  The counters are per device and shared by all streams, so
 * a timeout recorded by another stream's kernel shows here too.  (No
 * reference counterpart.)
 */
SA_API int sa_stream_status(void* stream, int reset);

/*
 * Test hook for the bounded-wait path: launches one warp that waits on an
 * mbarrier nothing ever arrives on, with a limit of limit_ns (1 ns .. 2 s).
 * The wait gives up, the timeout is recorded (sa_device_status /
 * sa_stream_status then return SA_ERR_TIMEOUT until reset) and the kernel
 * exits normally, writing 1 to the device int `done` (2 had the wait
 * completed).  It faults nothing and leaves the context usable.  (No
 * reference counterpart: the reference's kernels have no bounded waits.)
 */
SA_API int sa_probe_bounded_wait(int64_t limit_ns, int* done, void* stream);

/*
 * 1 if this library was built with device-side index checks (the debug
 * library, libsmooth_attn_b200_debug.so), else 0.  Host only.  (No reference
 * counterpart: the reference has no debug build.)
 */
SA_API int sa_debug_checks(void);

/*
 * Squareplus normalization forward over rows of length `cols`.
 *   y_j = squareplus(alpha * (x_j - theta))^power,  squareplus(a) = (a + sqrt(a^2+4)) / 2
 *   out_j = y_j / (sum_j y_j + 1e-12)
 * causal = 0: every column is visible (row-wise kernel).
 * causal = 1: rows are the rows of [M, cols, cols] score matrices stacked as
 *             [M*cols, cols]; row r is query position q = r % cols and only
 *             columns j <= q are visible; out is exactly 0 for j > q.
 * rowsum (nullable, fp32 [rows]) receives sum_j y_j + 1e-12 per row.
 * x and out have the same dtype; ld_x / ld_out are row strides in elements.
 * cols must be in [1, 4096]; power in {1,2,3}.
 *
 * Replaces: softplus_norm_triton_out / _softplus_norm_fwd
 *             (src/smooth_attn/kernels.py:1006-1031, :494-531)
 *           softplus_norm_causal_triton_out and its winner / tiered / generic
 *             variants (src/smooth_attn/kernels.py:1274-1297, :565-676,
 *             :1071-1172)
 */
SA_API int sa_norm_fwd(const void* x, void* out, float* rowsum, int64_t rows, int64_t cols, int64_t ld_x,
                int64_t ld_out, int dtype, int causal, float alpha, float theta, int power, void* stream);

/*
 * Host <-> device copy of the part of causal [nmat, L, L] matrices that the
 * causal norm reads (to_device != 0) or that can be nonzero in its output
 * (to_device == 0): for every band of `band` rows (a multiple of 8; the last
 * band may be shorter), rows [r0, r1) x columns [0, min(L, r1 rounded up to
 * 16 bytes)) of every matrix.  One cudaMemcpy3DAsync per band covers all
 * nmat matrices; src and dst are contiguous [nmat, L, L] with elem_bytes-byte
 * elements, the host side pinned.  The columns past each band's width are
 * neither read nor written.  Returns the bytes one call moves through
 * *bytes_out (nullable).  (No reference counterpart: the reference has no
 * host-buffer path; smooth_attn.host uses this to move about half of the
 * matrix bytes over PCIe in each direction.)
 */
SA_API int sa_copy_causal_bands(void* dst, const void* src, int64_t nmat, int64_t L, int64_t elem_bytes,
                                int64_t band, int to_device, int64_t* bytes_out, void* stream);

/*
 * Host memory: writes zeros to the part of [nmat, L, L] matrices that
 * sa_copy_causal_bands (to_device == 0) does not write -- in each band, the
 * columns past the band's copied width -- with `nthreads` host threads
 * (<= 0: one per core, at most 32) and non-temporal stores where the CPU has
 * them.  Blocks until done.  No GPU call.  (No reference counterpart.)
 */
SA_API int sa_host_zero_causal_tail(void* out, int64_t nmat, int64_t L, int64_t elem_bytes, int64_t band,
                                    int nthreads);

/*
 * Fused backward of sa_norm_fwd.
 *   dx_j = (dy_j/dx_j / S) * (g_j - sum_k g_k y_k / S),  S = sum_k y_k + 1e-12
 *   dy/dx = alpha * power * sp^(power-1) * sp',  sp' = (1 + a / sqrt(a^2+4)) / 2
 * x and dx share `dtype`; g has `g_dtype` (any of SA_F32/SA_F16/SA_BF16).
 * rowsum (nullable): the normalizer saved by sa_norm_fwd; when NULL it is
 * recomputed.  dx is written for every column (exact 0 above the diagonal in
 * causal mode).
 *
 * Replaces: _softplus_norm_causal_backward and the causal bwd kernels
 *             (src/smooth_attn/kernels.py:1197-1230, :679-849)
 */
SA_API int sa_norm_bwd(const void* x, const void* g, const float* rowsum, void* dx, int64_t rows, int64_t cols,
                int64_t ld_x, int64_t ld_g, int64_t ld_dx, int dtype, int g_dtype, int causal, float alpha,
                float theta, int power, void* stream);

/*
 * Fused causal squareplus attention forward (tcgen05 / TMEM / TMA).
 *   s = (q . k) * scale;  a = 2 s - 1;  y = ((a + sqrt(a^2+4)) / 2)^2 on the
 *   causal (and optional sliding-window: q - k < window) prefix;
 *   R = 1e-12 + sum y;  o = (sum bf16(y) v) / R.
 * q, o: [B, Hq, T, D]; k, v: [B, Hkv, T, D]; Hq % Hkv == 0 (GQA).
 * Strides are in elements as {batch, head, seq, dim}; the dim stride must be 1
 * and the others multiples of 8 elements (16 B) with 16 B aligned bases.
 * dtype: SA_BF16 or SA_F16.  D in {32, 64, 128}.
 * rowsum: fp32 [B, Hq, T] contiguous, receives R (needed by the backward).
 * o_lo (nullable, same dtype and strides as o): receives the residual of o's
 * 16-bit rounding, o_lo = round16(o_fp32 - o).  Pass it to sa_flash_bwd,
 * which then forms delta = rowsum(dO * (o + o_lo)) from the forward's fp32
 * output instead of its rounded copy (the rounding of o alone moves dQ / dK
 * by up to ~1.3x the 2e-2 rel / 1e-2 abs bf16 tolerance).  Training callers
 * pass it; inference callers pass NULL.
 * exact_math = 0 computes sqrt(u) as u * rsqrt(u) (the reference's default).
 *
 * Replaces: _sp2norm_flash_fwd / _sp2norm_flash_fwd_with_rowsum_kernel
 *             (src/smooth_attn/kernels.py:1912-1931, :1549-1631)
 */
SA_API int sa_flash_fwd(const void* q, const void* k, const void* v, void* o, void* o_lo, float* rowsum, int64_t B,
                 int64_t Hq,
                 int64_t Hkv, int64_t T, int64_t D, const int64_t* q_strides, const int64_t* k_strides,
                 const int64_t* v_strides, const int64_t* o_strides, float scale, int64_t window_size,
                 int exact_math, int dtype, void* stream);

/*
 * Workspace size in bytes that sa_flash_bwd needs for the given problem
 * (fp32 dQ accumulator + per-row delta).  The caller allocates it.
 */
SA_API int64_t sa_flash_bwd_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D);

/*
 * Fused causal squareplus attention backward.
 *   delta = rowsum(dO * O); dP = dO V^T; dY = (dP - delta) / R;
 *   dS = dY * 4 sp sp' * scale; dQ = dS K; dK = dS^T Q; dV = (y/R)^T dO
 * (dK, dV summed over the query heads of a GQA group).
 * q, o, dout, dq: [B, Hq, T, D]; k, v, dk, dv: [B, Hkv, T, D]; strides as in
 * sa_flash_fwd (dq/dk/dv/dout may have their own strides).
 * rowsum: fp32 [B, Hq, T] from sa_flash_fwd; o_lo (nullable): the residual
 * sa_flash_fwd wrote next to o (same strides as o).  workspace: at least
 * sa_flash_bwd_workspace_size() bytes, 256 B aligned, contents undefined on
 * entry.  sa_flash_bwd_workspace_size() returns 0 for sizes whose byte
 * count overflows int64; such problems are rejected.
 * deterministic = 0: dQ is accumulated by the key-major kernel with fp32
 * atomics (fastest; the order of the adds, and so dQ's last bits, varies
 * from run to run).  deterministic != 0: the key-major kernel computes dK and
 * dV only and a query-major kernel sums each dQ row over the key tiles in a
 * fixed order inside one CTA (the reference's order, kernels.py:1680-1784):
 * bitwise reproducible, at the cost of recomputing S and dP once more.
 *
 * Replaces: _sp2norm_flash_bwd, _sp2norm_flash_bwd_dq_kernel,
 *           _sp2norm_flash_bwd_dkv_kernel
 *             (src/smooth_attn/kernels.py:1934-1989, :1680-1784, :1800-1909)
 */
SA_API int sa_flash_bwd(const void* q, const void* k, const void* v, const void* o,
                        const void* o_lo, const void* dout,
                 const float* rowsum, void* dq, void* dk, void* dv, void* workspace, int64_t workspace_bytes,
                 int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D, const int64_t* q_strides,
                 const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                 const int64_t* do_strides, const int64_t* dq_strides, const int64_t* dk_strides,
                 const int64_t* dv_strides, float scale, int64_t window_size, int exact_math, int dtype,
                 int deterministic,
                 void* stream);

/*
 * Allocation-free sa_flash_bwd, for callers that cannot allocate device
 * memory (inside a stream capture that must not allocate, host frameworks
 * that own all device memory, latency-critical loops).  No counterpart in
 * the reference: the reference always allocates its scratch with torch.
 * Same arguments and results as sa_flash_bwd, minus the workspace: the
 * scratch is a fixed file-scope device array of
 * sa_flash_bwd_noalloc_max_bytes() bytes (32 MiB) that every GPU loading the
 * library holds until exit.  Problems whose sa_flash_bwd_workspace_size()
 * exceeds it are rejected with SA_ERR_ARG before anything is launched.
 * The first call on a device looks up the array's device address (make that
 * first call before any stream capture); the address is cached per device
 * with its CUDA context and looked up again after a device reset.  All calls share the one array:
 * calls that overlap on the GPU (other streams, other threads) race and give
 * wrong results; serialise them.  Calls no cudaMalloc / cudaFree.
 */
SA_API int64_t sa_flash_bwd_noalloc_max_bytes(void);
SA_API int sa_flash_bwd_noalloc(const void* q, const void* k, const void* v, const void* o,
                                const void* o_lo, const void* dout,
                                const float* rowsum, void* dq, void* dk, void* dv, int64_t B, int64_t Hq,
                                int64_t Hkv, int64_t T, int64_t D, const int64_t* q_strides,
                                const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                                const int64_t* do_strides, const int64_t* dq_strides, const int64_t* dk_strides,
                                const int64_t* dv_strides, float scale, int64_t window_size, int exact_math,
                                int dtype, void* stream);

/*
 * Forward of a block of Tq queries at global positions q_offset ..
 * q_offset+Tq-1 against keys / values at positions 0 .. Tk-1, with
 * sa_flash_fwd's causal / window rule in global positions (a query at
 * position p sees keys k <= p, p - k < window).  q, o: [B, Hq, Tq, D];
 * k, v: [B, Hkv, Tk, D]; rowsum: fp32 [B, Hq, Tq]; other arguments as
 * sa_flash_fwd (which is this call with Tq = Tk = T, q_offset = 0).  The
 * building block of context parallelism: every rank runs its query chunks
 * against the all-gathered key prefix; with a plain-sum normalizer no
 * cross-rank rescaling is needed.  (No reference counterpart: the reference
 * has no sequence parallelism.)
 */
SA_API int sa_flash_fwd_chunk(const void* q, const void* k, const void* v, void* o, void* o_lo, float* rowsum,
                              int64_t B,
                              int64_t Hq, int64_t Hkv, int64_t Tq, int64_t Tk, int64_t q_offset, int64_t D,
                              const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                              const int64_t* o_strides, float scale, int64_t window_size, int exact_math,
                              int dtype, void* stream);

/*
 * Backward of sa_flash_fwd_chunk: gradients of a block of Tq queries at
 * global positions q_offset .. against keys / values 0 .. Tk-1.  dq:
 * [B, Hq, Tq, D] (complete for these queries); dk, dv: [B, Hkv, Tk, D] hold
 * this query block's contribution only (a context-parallel caller adds the
 * contributions of every rank's query blocks).  rowsum / o from the chunk
 * forward; workspace: sa_flash_bwd_workspace_size(B, Hq, Hkv, Tq, D) bytes.
 * Other arguments as sa_flash_bwd (which is this call with Tq = Tk = T,
 * q_offset = 0).  (No reference counterpart.)
 */
SA_API int sa_flash_bwd_chunk(const void* q, const void* k, const void* v, const void* o,
                              const void* o_lo, const void* dout,
                              const float* rowsum, void* dq, void* dk, void* dv, void* workspace,
                              int64_t workspace_bytes, int64_t B, int64_t Hq, int64_t Hkv, int64_t Tq, int64_t Tk,
                              int64_t q_offset, int64_t D, const int64_t* q_strides, const int64_t* k_strides,
                              const int64_t* v_strides, const int64_t* o_strides, const int64_t* do_strides,
                              const int64_t* dq_strides, const int64_t* dk_strides, const int64_t* dv_strides,
                              float scale, int64_t window_size, int exact_math, int dtype,
                              int deterministic, void* stream);

/*
 * Output projection of the RoPE attention (or any 16-bit GEMM of this shape):
 *   out[M, N] = a[M, K] w[K, N],  fp32 accumulation on tcgen05 tensor cores,
 *   one rounding to the 16-bit output type.
 * a, w, out row-major with row strides lda, ldw, ldo (elements, multiples of
 * 8, 16-byte aligned bases); N a multiple of 8; dtype SA_BF16 or SA_F16.
 * For the RoPE projection a = the attention output laid out [B*T, H*D] and
 * w = W_o reshaped [H*D, D_model], so the sum over heads is the contraction.
 *
 * Replaces: the W_o stage of _sp2norm_rope_flash_proj_fwd_kernel
 *             (src/smooth_attn/kernels.py:2233-2370), which adds per-head
 *             bf16 partials with atomic_add.
 */
SA_API int sa_out_proj(const void* a, const void* w, void* out, int64_t M, int64_t K, int64_t N, int64_t lda,
                int64_t ldw, int64_t ldo, int dtype, void* stream);

/*
 * Rotary position embedding, rotate-half form, rounded to the input type:
 *   out[..., i] = x1 c - x2 s,  out[..., i + D/2] = x2 c + x1 s
 * with x1 = x[..., i], x2 = x[..., i + D/2], c = cos[t, i], s = sin[t, i],
 * each product and the sum rounded separately in fp32.
 * x: [B, H, T, D] with strides {batch, head, seq, dim} (dim stride 1, others
 * multiples of 8); out: contiguous [B, H, T, D]; cos_table / sin_table:
 * contiguous [T, D/2] of cs_dtype (SA_F32, SA_BF16 or SA_F16).  dtype:
 * SA_BF16 or SA_F16; D a multiple of 16.
 *
 * Replaces: the in-register RoPE of _sp2norm_rope_flash_fwd_kernel
 *             (src/smooth_attn/kernels.py:2147-2159, :2186-2194)
 */
SA_API int sa_rope_rotate(const void* x, void* out, const void* cos_table, const void* sin_table, int cs_dtype,
                          int64_t B, int64_t H, int64_t T, int64_t D, const int64_t* x_strides, int dtype,
                          void* stream);

/* Workspace bytes of sa_rope_flash_fwd (the rotated Q and K), or < 0. */
SA_API int64_t sa_rope_flash_fwd_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D);

/*
 * RoPE + fused causal squareplus attention forward: q and k are rotated
 * (as sa_rope_rotate) into `workspace` (>= sa_rope_flash_fwd_workspace_size
 * bytes, 256-byte aligned), then sa_flash_fwd runs on the rotated tensors;
 * v, o, rowsum, strides, scale, window_size, exact_math and dtype as in
 * sa_flash_fwd.  o may have any sa_flash_fwd-legal strides, e.g. those of a
 * [B, T, Hq, D] buffer so that an output projection is one plain GEMM.
 *
 * Replaces: sp2norm_rope_flash_attention / _sp2norm_rope_flash_fwd_kernel
 *             (src/smooth_attn/kernels.py:2373-2430, :2104-2222) and the
 *           attention part of sp2norm_rope_flash_attention_proj /
 *           _sp2norm_rope_flash_proj_fwd_kernel (:2433-2490, :2230-2370)
 */
SA_API int sa_rope_flash_fwd(const void* q, const void* k, const void* v, void* o, float* rowsum,
                             const void* cos_table, const void* sin_table, int cs_dtype, void* workspace,
                             int64_t workspace_bytes, int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D,
                             const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                             const int64_t* o_strides, float scale, int64_t window_size, int exact_math,
                             int dtype, void* stream);

/*
 * Per-tensor FP8 (E4M3) quantization of q, k and v (nq / nk / nv elements,
 * contiguous, multiples of 8, dtype SA_F32 / SA_F16 / SA_BF16):
 *   scale_t = max(max|x_t| / 448, 1e-12);  x8 = e4m3(clamp(x / scale_t, +-448))
 * q8, k8: E4M3 bytes; vq: bf16 holding the E4M3-rounded v / scale_v exactly;
 * scales: device float[3] {q, k, v}; workspace: 12 bytes of device scratch.
 * Two launches, no host synchronisation.
 *
 * Replaces: _quantize_to_fp8 (src/smooth_attn/kernels.py:2592-2601)
 */
SA_API int sa_fp8_quantize(const void* q, const void* k, const void* v, int64_t nq, int64_t nk, int64_t nv,
                           int dtype, void* q8, void* k8, void* vq, float* scales, void* workspace, void* stream);

/*
 * FP8 causal squareplus attention forward: QK^T on E4M3 tensor cores
 * (tcgen05 kind::f8f6f4), scores scaled by q_scale * k_scale * scale,
 * squareplus in fp32, P (bf16) . vq on bf16 tensor cores, times v_scale.
 * q8, k8: E4M3 [B, Hq|Hkv, T, D] (strides multiples of 16 elements);
 * vq: bf16 [B, Hkv, T, D]; o: bf16; rowsum as sa_flash_fwd; scales: the
 * device float[3] written by sa_fp8_quantize.  D in {32, 64, 128}.
 *
 * Replaces: _sp2norm_fp8_flash_fwd / _sp2norm_fp8_flash_fwd_kernel
 *             (src/smooth_attn/kernels.py:2604-2627, :2498-2589)
 */
SA_API int sa_fp8_flash_fwd(const void* q8, const void* k8, const void* vq, void* o, float* rowsum,
                            const float* scales, int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D,
                            const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                            const int64_t* o_strides, float scale, int64_t window_size, void* stream);

/*
 * Workspace bytes sa_paged_decode needs for this shape (0 when the launch
 * does not split sequences over several CTAs), or a negative sa_status when
 * the shape is rejected.  Depends on the current device's SM count.
 */
SA_API int64_t sa_paged_decode_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t max_blocks,
                                              int64_t block_size, int64_t D, int dtype);

/*
 * Decode attention (one query token per sequence) over a paged KV cache.
 *   s_j = (q . k_j) * scale;  y_j = squareplus(2 s_j - 1)^2;
 *   out = sum_j y_j v_j / (sum_j y_j + 1e-12)   over j < context_lens[b]
 * q: [B, Hq, 1, D] contiguous; k_cache, v_cache: [num_blocks, Hkv,
 * block_size, D] contiguous; token j of sequence b is row j % block_size of
 * page block_table[b, j / block_size]; block_table: int32 [B, max_blocks]
 * contiguous; context_lens: int32 [B] (clamped to [0, max_blocks *
 * block_size]).  out: bf16 [B, Hq, D] contiguous.  dtype (q and caches):
 * SA_BF16 or SA_F16; D in {32, 64, 128, 256}; Hq % Hkv == 0.  Pointers
 * 16-byte aligned.  workspace: sa_paged_decode_workspace_size() bytes,
 * 256-byte aligned; its first bytes hold per-(sequence, head) arrival
 * tickets that must be zero before the first call and that every completed
 * call leaves zero again, so one zero-filled workspace can be reused by
 * calls that do not overlap on the GPU.  Page indices outside
 * [0, num_blocks) are read as page 0 and reported by sa_device_status.
 *
 * Replaces: sp2norm_paged_attention / _sp2norm_paged_attention_kernel
 *             (src/smooth_attn/kernels.py:2776-2829, :2681-2773)
 */
SA_API int sa_paged_decode(const void* q, const void* k_cache, const void* v_cache, void* out,
                           const int32_t* block_table, const int32_t* context_lens, void* workspace,
                           int64_t workspace_bytes, int64_t B, int64_t Hq, int64_t Hkv, int64_t num_blocks,
                           int64_t block_size, int64_t max_blocks, int64_t D, float scale, int dtype,
                           void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SMOOTH_ATTN_B200_H */
