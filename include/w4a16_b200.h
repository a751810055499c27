/*
 * w4a16_b200.h -- C ABI of the sm_100a (B200) W4A16 fused dequant-GEMM library.
 *
 * Plain C: raw device pointers, 64-bit sizes and an opaque stream handle (a
 * cudaStream_t passed as void*; NULL means the legacy default stream). No
 * torch or C++ types cross this boundary and no exception escapes it: every
 * entry point returns 0 on success or a negative W4A16_* status, and
 * w4a16_strerror() turns a status into text. All launches are asynchronous
 * on the given stream; nothing here allocates device memory or synchronises
 * (scratch memory, where a kernel needs it, is passed in by the caller) except
 * the peer-to-peer buffer helpers w4a16_p2p_*, which set up the multi-GPU path.
 *
 * Data format (the reference's, unchanged): W is [K, N] (K = in_features),
 * quantised in groups of G consecutive K-rows per column.
 *   qweight int32 [K/8, N]  row k = 8i+j of column n in bits [4j, 4j+4) of qweight[i, n]
 *   scales  fp16  [K/G, N]
 *   zeros   fp16  [K/G, N]  integer zero-points (0..15 as produced by w4a16_quantize)
 * All tensors are row-major and dense unless a leading dimension is given.
 */
#ifndef W4A16_B200_H_
#define W4A16_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define W4A16_OK                 0
#define W4A16_ERR_INVALID       -1  /* bad size, group size or null pointer */
#define W4A16_ERR_ALIGNMENT     -2  /* pointer/stride alignment a kernel needs is missing */
#define W4A16_ERR_LAUNCH        -3  /* the CUDA launch itself failed */
#define W4A16_ERR_DEVICE        -4  /* device is not sm_100 or cannot be queried */
#define W4A16_ERR_TIMEOUT       -5  /* a kernel's bounded wait expired (sticky device flag) */
#define W4A16_ERR_WORKSPACE     -6  /* workspace missing, too small or misaligned */

/* Input dtypes accepted by w4a16_quantize. */
#define W4A16_DTYPE_F16  0
#define W4A16_DTYPE_F32  1
#define W4A16_DTYPE_BF16 2

/* Library version, major*10000 + minor*100 + patch. */
int w4a16_version(void);

/* Human-readable text for a status code; never NULL. */
const char* w4a16_strerror(int status);

/*
 * Fused GEMM: y[m, n] = sum_k x[m, k] * dequant(qweight, scales, zeros)[k, n]
 * accumulated in fp32, rounded to fp16, then (if bias != NULL) y + bias[n]
 * rounded to fp16 again.
 *
 * Replaces the reference's w4a16_matmul (w4a16-kernel/src/w4a16/triton_kernel.py:131-200)
 * and its CUDA twin w4a16_gemm_cuda (w4a16-kernel/src/w4a16/cuda/w4a16_gemm.cu:76-115);
 * the bias add is the one W4A16Linear.forward does afterwards (linear.py:90-91).
 *
 * x: fp16 [M, K] dense. y: fp16, row m at y + m*ldy (ldy >= N), so a caller
 * can write one column shard of a wider output. Requirements (the reference's
 * assertions, triton_kernel.py:153-182): K % 8 == 0, K % group_size == 0,
 * group_size % 64 == 0. M == 0 or N == 0 is a no-op.
 * Routing: M <= 32 runs the memory-bound decode kernel, larger M the tcgen05
 * tensor-core kernel (which needs N % 8 == 0; other N fall back to decode
 * launches over 32-row slices of x).
 *
 * workspace: device scratch of at least w4a16_gemm_workspace_size() bytes,
 * 256-byte aligned, ZEROED before its first use. The decode kernel passes the
 * partial sums of column strips shared by two or more CTAs through its first
 * W4A16_NOALLOC_SCRATCH_BYTES (tagged 64-bit words) and leaves them zero again;
 * the tensor-memory-operand prefill kernel, when it splits K, keeps arrival
 * counters (left zero) and fp32 partial tiles past that offset. So one zeroed
 * buffer serves every later call on the same stream, whatever the shape;
 * launches that may run concurrently need separate workspaces. A prefill call
 * given less workspace than the query returned runs without splitting K. (A
 * launch abandoned on W4A16_ERR_TIMEOUT can leave words set: zero the buffer
 * again before reusing it.) May be NULL when the size query returned 0.
 */
int w4a16_gemm(const void* x, const int32_t* qweight, const void* scales,
               const void* zeros, const void* bias, void* y,
               int64_t M, int64_t N, int64_t K, int64_t group_size,
               int64_t ldy, void* workspace, int64_t workspace_bytes, void* stream);

/*
 * w4a16_gemm with an fp32 output and no rounding (and no bias): the partial
 * sums of a K-sharded (row-parallel) layer, summed across GPUs before the one
 * final fp16 rounding, so a sharded layer matches the unsharded result.
 * y: fp32, row m at y + m*ldy. Same requirements and workspace as w4a16_gemm.
 * No reference counterpart: the reference has no multi-GPU path.
 */
int w4a16_gemm_f32(const void* x, const int32_t* qweight, const void* scales,
                   const void* zeros, float* y, int64_t M, int64_t N, int64_t K,
                   int64_t group_size, int64_t ldy, void* workspace,
                   int64_t workspace_bytes, void* stream);

/*
 * SwiGLU of a fused gate/up projection: h[m, n] = silu(g) * u with
 * g = gate_up[m, n] and u = gate_up[m, N + n] (fp16 in, fp32 math, one fp16
 * rounding). gate_up rows have pitch ld_in >= 2N, h rows pitch ld_out >= N.
 * No reference counterpart: it joins the projections of the MLP block the
 * benchmark configuration names.
 */
int w4a16_swiglu(const void* gate_up, void* h, int64_t M, int64_t N, int64_t ld_in,
                 int64_t ld_out, void* stream);

/*
 * The gate/up projection of an MLP block fused with its SwiGLU: the GEMM's epilogue
 * writes h[m, j] = fp16(silu(g) * u) (fp32 math on the fp16-rounded g and u, one
 * rounding: the same values as w4a16_gemm followed by w4a16_swiglu) instead of the
 * [M, N] gate/up output. The weight's N columns hold the gate and up projections
 * interleaved in blocks of 16: columns 32b .. 32b+15 are gate columns 16b .. 16b+15
 * and columns 32b+16 .. 32b+31 the matching up columns, so output column j reads
 * weight columns 32(j/16) + j%16 and that + 16. h: fp16 [M, N/2], row pitch ldh >= N/2.
 * N % 32 == 0; x, qweight, scales, zeros 16-byte aligned (W4A16_ERR_ALIGNMENT
 * otherwise); the other requirements and the workspace are w4a16_gemm's. No reference
 * counterpart: it removes the [M, N] round trip between the projections of the MLP
 * block the benchmark configuration names.
 */
int w4a16_gemm_swiglu(const void* x, const int32_t* qweight, const void* scales,
                      const void* zeros, void* h, int64_t M, int64_t N, int64_t K,
                      int64_t group_size, int64_t ldh, void* workspace,
                      int64_t workspace_bytes, void* stream);

/*
 * Option bits of w4a16_gemm_ex.
 *   W4A16_FLAG_KERNEL_ORDER  qweight holds the kernel nibble order written by
 *                            w4a16_repack instead of the reference's
 *   W4A16_FLAG_SWIGLU        the w4a16_gemm_swiglu epilogue (y is h [M, N/2])
 *   W4A16_FLAG_F32_OUT       the w4a16_gemm_f32 output (fp32, unrounded, no bias)
 *   W4A16_FLAG_BF16_OUT      y (and bias) bf16: the fp32 sums rounded to bf16, then
 *                            y + bias rounded again (for bf16 models, whose
 *                            activations w4a16_convert takes to fp16 first)
 */
#define W4A16_FLAG_KERNEL_ORDER 1u
#define W4A16_FLAG_SWIGLU       2u
#define W4A16_FLAG_F32_OUT      4u
#define W4A16_FLAG_BF16_OUT     8u

/*
 * w4a16_gemm with option bits (above): one entry point for the plain, SwiGLU and
 * fp32-output GEMMs over either nibble order. SWIGLU excludes F32_OUT, BF16_OUT and a
 * bias; F32_OUT excludes BF16_OUT and a bias;
 * KERNEL_ORDER and SWIGLU need N % 8 == 0 and 16-byte-aligned x, qweight, scales and
 * zeros (W4A16_ERR_ALIGNMENT otherwise). Unknown bits: W4A16_ERR_INVALID. No
 * reference counterpart (w4a16_gemm is the reference's operator).
 */
int w4a16_gemm_ex(const void* x, const int32_t* qweight, const void* scales,
                  const void* zeros, const void* bias, void* y, int64_t M, int64_t N,
                  int64_t K, int64_t group_size, int64_t ldy, uint32_t flags,
                  void* workspace, int64_t workspace_bytes, void* stream);

/*
 * dst[i] = src[i] rounded to dst's type, n elements; src fp16, fp32 or bf16, dst fp16
 * or bf16 (W4A16_DTYPE_*). For bf16 activations: bf16 -> fp16 is exact for |x| in
 * [2^-14, 65504] (and 0), so the fp16 GEMM computes the bf16 product unchanged
 * there. No reference counterpart (the reference takes fp16 activations only).
 */
int w4a16_convert(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t n,
                  void* stream);

/*
 * Offline repack of qweight [K/8, N] between the reference's nibble order (row 8i+j in
 * nibble j of word [i, n], w4a16-kernel/src/w4a16/quant.py:45-70) and the kernel order
 * (rows k0, k2, k4, k6, k1, k3, k5, k7 in nibbles 0..7): to_kernel_order != 0 converts
 * reference -> kernel, 0 converts back. Elementwise; out may equal qweight. In the
 * kernel order the GEMMs extract a word's consecutive row pairs with one shift and four
 * masks (W4A16_FLAG_KERNEL_ORDER). No reference counterpart: a load-time layout, the
 * stored (state_dict) format stays the reference's.
 */
int w4a16_repack(const int32_t* qweight, int32_t* out, int64_t K, int64_t N,
                 int to_kernel_order, void* stream);

/*
 * dst = src, `bytes` bytes (a multiple of 16; both 16-byte aligned), as a kernel on
 * `stream` that chains with the GEMM launches around it under programmatic
 * dependent launch. No reference counterpart: it stages a step's inputs in (or its
 * outputs out) inside a CUDA-graph-captured serving loop, where a memory-copy node
 * before a GEMM would make that GEMM wait for its predecessor's completion instead
 * of overlapping the predecessor's tail. Either pointer may be device memory or
 * pinned host memory mapped into the device's address space (W4A16_ERR_INVALID
 * otherwise). src_ready != 0 promises that no earlier kernel on the stream writes
 * src (e.g. inputs the host wrote into pinned memory): the kernel then reads src
 * while the previous kernel still runs. dst is written only after the previous
 * kernel completes, and the copy completes after it.
 */
int w4a16_stage(const void* src, void* dst, int64_t bytes, int src_ready, void* stream);

/*
 * w4a16_gemm_ex on host-resident activations: x_host [M, K] fp16 is staged into the
 * device buffer x_dev, the GEMM writes the device buffer y_dev [M, n] (n = N, or N/2
 * with W4A16_FLAG_SWIGLU; fp32 with W4A16_FLAG_F32_OUT, bf16 with
 * W4A16_FLAG_BF16_OUT, else fp16), and y_dev is staged out to y_host: kernels on
 * `stream` chained under programmatic dependent launch (no copy-engine transfers
 * between them), so an eager loop of calls keeps the GEMM's start overlapped with
 * its predecessor. Up to 32 tokens the GEMM writes y_host directly (y_dev unused). x_host and y_host must be pinned host memory
 * mapped into the device's address space (W4A16_ERR_INVALID otherwise); all four
 * buffers 16-byte aligned, M*K*2 and the y bytes multiples of 16
 * (W4A16_ERR_ALIGNMENT). y_host holds the result once the stream has completed.
 * x_dev/y_dev may be reused by the next call on the same stream. No reference
 * counterpart (the reference's GEMM takes device tensors).
 */
int w4a16_gemm_host(const void* x_host, const int32_t* qweight, const void* scales, const void* zeros,
                    const void* bias, void* y_host, int64_t M, int64_t N, int64_t K, int64_t group_size,
                    uint32_t flags, void* x_dev, void* y_dev, void* workspace, int64_t workspace_bytes,
                    void* stream);

/*
 * Bytes of workspace w4a16_gemm needs for this shape on the current device
 * (0 for shapes whose kernels need none: N % 8 != 0, or a prefill shape run
 * without splitting K). Shapes that route to the decode or prefill kernels need
 * the device (its SM count); on a machine without one the query returns
 * W4A16_ERR_DEVICE. No reference counterpart: the reference's kernels never
 * split K across thread blocks.
 */
int w4a16_gemm_workspace_size(int64_t M, int64_t N, int64_t K, int64_t group_size,
                              int64_t* bytes_out);

/*
 * Group-wise asymmetric uint4 quantisation + packing of w [K, N] (dtype one of
 * W4A16_DTYPE_*), bit-exact with the reference's quantize_weight
 * (w4a16-kernel/src/w4a16/quant.py:101-144): fp32 scale (max-min)/15 (1 when
 * not > 0), zero = clamp(rint(-min/scale), 0, 15), q = clamp(rint(w/scale) + zero, 0, 15).
 * Requirements: K % 8 == 0, K % group_size == 0, group_size >= 1.
 * Non-finite weights produce unspecified codes; the caller rejects them first.
 */
int w4a16_quantize(const void* w, int w_dtype, int32_t* qweight, void* scales,
                   void* zeros, int64_t K, int64_t N, int64_t group_size,
                   void* stream);

/*
 * w4a16_quantize with option bits. W4A16_QUANT_SYMMETRIC: symmetric codes, the
 * layout GPTQ-style checkpoints use with sym=True -- per (group, column) zero = 8 and
 * scale = 2 * max|w| / 15 in fp32 (1 when not > 0), q = clamp(rint(w / scale) + 8,
 * 0, 15) -- stored in the same qweight / scales / zeros format, so every GEMM entry
 * point takes it unchanged. No reference counterpart (the reference quantises
 * asymmetrically only). Unknown bits: W4A16_ERR_INVALID.
 */
#define W4A16_QUANT_SYMMETRIC 1u
int w4a16_quantize_ex(const void* w, int w_dtype, int32_t* qweight, void* scales,
                      void* zeros, int64_t K, int64_t N, int64_t group_size,
                      uint32_t flags, void* stream);

/*
 * Pack int32 codes q [K, N] (each in 0..15) into qweight [K/8, N]
 * (w4a16-kernel/src/w4a16/quant.py:45-70). Codes are masked with 0xF; the
 * range check the reference asserts stays with the caller. K % 8 == 0.
 */
int w4a16_pack_int4(const int32_t* q, int32_t* qweight, int64_t K, int64_t N,
                    void* stream);

/* Inverse of w4a16_pack_int4: qweight [K/8, N] -> q [K, N] in 0..15
 * (w4a16-kernel/src/w4a16/quant.py:73-95). */
int w4a16_unpack_int4(const int32_t* qweight, int32_t* q, int64_t K, int64_t N,
                      void* stream);

/* w[k, n] = fp16(fp16(q - z) * s) for the group of row k, fp16 [K, N]
 * (w4a16-kernel/src/w4a16/quant.py:147-178). K % group_size == 0, K % 8 == 0. */
int w4a16_dequantize(const int32_t* qweight, const void* scales, const void* zeros,
                     void* w, int64_t K, int64_t N, int64_t group_size,
                     void* stream);

/*
 * Read and clear the device's sticky error flags for the current device
 * (bit 0: a bounded wait in a GEMM kernel ran out of its time budget and the
 * kernel abandoned its tile). Synchronises the given stream.
 * Returns W4A16_OK when no flag was set, W4A16_ERR_TIMEOUT when one was; in
 * that case it also zeroes this device's w4a16_gemm_noalloc scratch array (if
 * it has been set up) on `stream` and synchronises again, since its callers
 * cannot clear it themselves. Results of the launches since the last check are
 * unspecified after a timeout. Caller-owned workspaces and peer buffers may
 * hold stale words too: zero them (w4a16_reset_scratch) before reusing them.
 * No reference counterpart: the reference's kernels have no bounded waits.
 */
int w4a16_check_device_errors(void* stream, uint32_t* flags_out);

/*
 * Time budget, in nanoseconds, of every bounded wait in the kernels launched
 * after this call (process-wide; 0 restores the default of 4 s; otherwise
 * 1 ms <= ns <= 600 s, else W4A16_ERR_INVALID). Each launch carries the budget
 * as a kernel parameter, so launches already queued or captured in a CUDA graph
 * keep theirs. A shorter budget lets a caller (or a test) detect a lost peer
 * sooner; legitimate waits last microseconds to milliseconds. The waits that
 * keep a kernel from exiting with copies or MMAs in flight always use 4 s.
 * No reference counterpart.
 */
int w4a16_set_wait_budget_ns(int64_t ns);

/*
 * Prefill kernel (M > 32 tokens) selection, process-wide, for the launches after
 * this call. W4A16_PREFILL_AUTO (the default) picks per shape between the kernel
 * whose dequantised weights are the shared-memory B operand of tcgen05.mma
 * (W4A16_PREFILL_SMEM_B) and the one whose dequantised weights are the
 * tensor-memory A operand (W4A16_PREFILL_TMEM_A), by a cost model measured on
 * B200. Forcing one exists for tests and tuning; both give results within the
 * GEMM tolerance of each other (the same fp16 weights, fp32 sums in another order).
 * Anything else returns W4A16_ERR_INVALID. No reference counterpart.
 */
#define W4A16_PREFILL_AUTO 0
#define W4A16_PREFILL_SMEM_B 1
#define W4A16_PREFILL_TMEM_A 2
int w4a16_set_prefill_kernel(int which);
/* The prefill kernel (W4A16_PREFILL_SMEM_B or _TMEM_A) the current selection gives an
 * M x N x K GEMM with N % 8 == 0 on the current device, or W4A16_PREFILL_AUTO when M <= 32
 * (decode). For reports and tests; no reference counterpart. */
int w4a16_prefill_choice(int64_t M, int64_t N, int64_t K, int* which);
/* The plan the cost model makes for an M x N x K GEMM (K % 64 == 0) on a GPU with num_sms
 * SMs, under the current selection, without touching a device: *which as in
 * w4a16_prefill_choice; for the tensor-memory-operand kernel *tokens_per_tile (its tile
 * height, 64..192) and *splits (K split over that many CTAs for the tiles it splits: every
 * tile when the tiles do not fill one wave, else the last wave's; 1: none), else 0 and 1.
 * A launch splits K only when it is given the workspace the size query returns. For reports
 * and tests; no reference counterpart. */
int w4a16_prefill_plan(int64_t M, int64_t N, int64_t K, int num_sms, int* which, int* tokens_per_tile,
                       int* splits);

/*
 * After W4A16_ERR_TIMEOUT: zero `workspace_bytes` of a caller's GEMM workspace
 * (when `workspace` is not NULL) and this device's w4a16_gemm_noalloc scratch
 * array (when set up), asynchronously on `stream`; allocates nothing. The next
 * GEMM on that stream then starts from clean scratch. No reference counterpart.
 */
int w4a16_reset_scratch(void* workspace, int64_t workspace_bytes, void* stream);

/*
 * w4a16_gemm without a workspace argument and without allocating anything.
 * No counterpart in the reference (its kernels need no scratch at all).
 *
 * For callers that cannot allocate device memory at call time: a C or FFI
 * host with no device allocator of its own, an engine whose memory planner
 * has already handed out all device memory, or a plugin interface whose
 * launch call passes no scratch buffer. The decode kernel's scratch (the
 * partial sums of shared column strips) lives instead in one static device
 * array inside this library, W4A16_NOALLOC_SCRATCH_BYTES per device, whose
 * address the library looks up once per device. Shapes whose decode launch
 * would need more than that return W4A16_ERR_SCRATCH_LIMIT (on a 148-SM B200
 * every shape fits: the need is CTAs * M-tiles * 8 KiB, at most 148 * 4 *
 * 8 KiB = 4.6 MiB); prefill shapes need no scratch.
 *
 * The first call on each device does the set-up: it looks the array up,
 * zeroes it on `stream` and synchronises that stream. Make that first call
 * before any stream capture; a first call made while `stream` is capturing
 * returns W4A16_ERR_INVALID. The array must be zero whenever a decode launch
 * starts: set-up zeroes it and every completed launch leaves it zero; a launch
 * abandoned on a timeout may leave words set, and w4a16_check_device_errors
 * zeroes the array again when it reports W4A16_ERR_TIMEOUT (as does
 * w4a16_reset_scratch). There is ONE scratch array per device, so calls whose kernels can run
 * at the same time (different streams, threads or processes sharing a
 * context, parallel graph branches) race on it and give wrong results: keep
 * every call on one device ordered, or use w4a16_gemm with a workspace per
 * stream. Arguments, routing and results are those of w4a16_gemm.
 */
#define W4A16_NOALLOC_SCRATCH_BYTES (5 * 1024 * 1024)
#define W4A16_ERR_SCRATCH_LIMIT -7  /* shape needs more than the static scratch */
int w4a16_gemm_noalloc(const void* x, const int32_t* qweight, const void* scales,
                       const void* zeros, const void* bias, void* y,
                       int64_t M, int64_t N, int64_t K, int64_t group_size,
                       int64_t ldy, void* stream);

/*
 * Row-parallel decode GEMM fused with its all-reduce (no counterpart in the
 * reference, which has no multi-GPU path): y = fp16(sum over the `world` ranks of
 * x_r @ dequant(W_r)) [+ bias, rounded again], where each rank holds a K-slice
 * of x and of the weight. One kernel per rank: the CTA that finalises an output
 * element writes its fp32 partial, tagged with the call's epoch in one 64-bit
 * word, into this rank's slot of every rank's peer-to-peer buffer (plain stores
 * over NVLink; no fence, no flag); the last CTAs to finish read their share of
 * the elements in every slot of their own buffer until each word carries the
 * epoch's tag (bounded wait), and sum the slots in rank order into y -- the same
 * values as an fp32 all-reduce of the partials followed by one fp16 rounding.
 *
 * peers: HOST array of `world` buffer addresses as mapped on this GPU (this
 * rank's own buffer at index `rank`), each w4a16_p2p_buffer_bytes(world, slot)
 * bytes, 16-byte aligned, zeroed before first use (w4a16_p2p_alloc does); the
 * addresses are copied into the launch. ctl: this rank's two device int32
 * control words, zeroed before first use. slot >= M * N and even. Every rank
 * must issue the same sequence of calls on one stream (a call's words alternate
 * between two buffer halves by the call count kept in ctl); calls on a buffer
 * must not overlap. Requirements as w4a16_gemm plus M <= 32, N % 8 == 0,
 * 16-byte-aligned inputs, 2 <= world <= 8. The workspace is w4a16_gemm's.
 */
int w4a16_gemm_allreduce(const void* x, const int32_t* qweight, const void* scales,
                         const void* zeros, const void* bias, void* y,
                         int64_t M, int64_t N, int64_t K, int64_t group_size,
                         int64_t ldy, void* workspace, int64_t workspace_bytes,
                         const unsigned long long* peers, int world, int rank,
                         int* ctl, int64_t slot, void* stream);

/*
 * Column-parallel decode GEMM fused with its all-gather (no counterpart in the
 * reference): rank r holds columns [r*N, (r+1)*N) of the weight (and of bias) and
 * every rank receives the whole y = [M, world*N] (row pitch ldy >= world*N): the
 * CTA that finalises an element writes its fp16 value (bias added, rounded as
 * w4a16_gemm does) as a tagged 64-bit word into this rank's slot of every rank's
 * buffer, and the last CTAs to finish copy every rank's slot into y once the tags
 * of this call are in (bounded wait). The same bits as w4a16_gemm on each rank
 * followed by an all-gather of the columns. Peers, ctl, slot (>= M*N), ordering
 * and requirements as w4a16_gemm_allreduce, whose buffers it shares.
 */
int w4a16_gemm_allgather(const void* x, const int32_t* qweight, const void* scales,
                         const void* zeros, const void* bias, void* y,
                         int64_t M, int64_t N, int64_t K, int64_t group_size,
                         int64_t ldy, void* workspace, int64_t workspace_bytes,
                         const unsigned long long* peers, int world, int rank,
                         int* ctl, int64_t slot, void* stream);

/* Bytes of one rank's peer-to-peer buffer for w4a16_gemm_allreduce / _allgather. */
int w4a16_p2p_buffer_bytes(int world, int64_t slot, int64_t* bytes_out);

/* A zeroed device buffer of `bytes` on the current device and its 64-byte CUDA
 * IPC handle (for the peers' w4a16_p2p_open); release with w4a16_p2p_free. */
int w4a16_p2p_alloc(int64_t bytes, void** ptr_out, void* handle_out);

/* Map a peer's buffer from its 64-byte IPC handle; release with w4a16_p2p_close. */
int w4a16_p2p_open(const void* handle, void** ptr_out);
int w4a16_p2p_close(void* ptr);
int w4a16_p2p_free(void* ptr);

#ifdef __cplusplus
}
#endif

#endif /* W4A16_B200_H_ */
