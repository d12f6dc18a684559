/*
 * openquant_b200 C ABI.
 *
 * One shared library (openquant_b200/_lib/libopenquant_b200.so) exports the
 * INT8 / INT4 quantize, dequantize and fused INT4 dequant-matmul entry points
 * of the OpenQuant quantize-and-multiply path, as hand-written sm_100a CUDA
 * kernels.  Every entry point:
 *
 *   - borrows caller-owned DEVICE pointers (inputs are never written;
 *     oq_int4_linear_host takes page-locked HOST activations and output);
 *   - enqueues its kernels on the caller's CUDA stream (`stream`, a
 *     cudaStream_t passed as void*; NULL = the legacy default stream) and
 *     returns without synchronising (oq_int4_linear_host,
 *     oq_int4_linear_host_run and oq_take_device_error excepted, as
 *     documented there);
 *   - allocates no device memory (oq_peer_alloc excepted: allocating is
 *     its job);
 *   - returns OQ_OK (0) or an error code; oq_last_error() then returns a
 *     thread-local, NUL-terminated message.
 *
 * OQ_ERR_INVALID maps to Python's ValueError (bad shape, dtype, group size,
 * alignment), OQ_ERR_CUDA / OQ_ERR_UNSUPPORTED to RuntimeError.
 *
 * Layouts are exactly the reference's (openquant 0.5.0):
 *   per-row INT8   : q int8 [N*K] row-major, scales fp32 [N]
 *   per-row INT4   : the row-major [N*K] int4 values flattened ACROSS row
 *                    boundaries, two per byte (element 2i in the low nibble,
 *                    2i+1 in the high nibble), odd totals padded with a zero
 *                    nibble: ceil(N*K/2) bytes; scales fp32 [N]
 *   groupwise INT4 : each row zero-padded to KP = ceil(K/g)*g columns and
 *                    packed as above: N*KP/2 bytes, row r at byte r*KP/2;
 *                    scales fp32 [N][KP/g]
 * Nibbles are two's complement (-7..7 written; -8 decodes as -8).
 */
#ifndef OPENQUANT_B200_H
#define OPENQUANT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void *oq_stream_t; /* a cudaStream_t */

#if defined(__GNUC__)
#define OQ_API __attribute__((visibility("default")))
#else
#define OQ_API
#endif

/* Status codes. */
#define OQ_OK 0
#define OQ_ERR_INVALID 1     /* argument error  -> ValueError   */
#define OQ_ERR_CUDA 2        /* CUDA error       -> RuntimeError */
#define OQ_ERR_UNSUPPORTED 3 /* no sm_100 device -> RuntimeError */

/* Element types of weight / activation inputs. */
#define OQ_F32 0
#define OQ_F16 1
#define OQ_BF16 2
#define OQ_F64 3

/* Fused-matmul kernel selection (oq_int4_linear `kernel` argument). */
#define OQ_KERNEL_AUTO 0    /* choose from shape and the tile table       */
#define OQ_KERNEL_GEMV 1    /* tensor-core GEMV, M <= 64, g % 32 == 0     */
#define OQ_KERNEL_SIMT 2    /* CUDA-core kernel, any shape                */
#define OQ_KERNEL_TCGEN05 3 /* tcgen05/TMEM GEMM, M >= 1, see oq_int4_linear */

/* oq_int4_linear `config` flag: round every weight to x's dtype exactly as
 * the reference kernel does (fp32 q*scale, then fp16/bf16).  Without it an
 * fp16 GEMV with group_size % 128 == 0 multiplies x by the exact integer
 * nibbles and applies each fp32 group scale to the group's fp32 partial
 * sum -- closer to x.(q*s) than the reference, within the parity tolerance
 * of it, and ~2.5x fewer instructions per weight.  The automatic launch
 * shape (config 0) does so up to M = 16. */
#define OQ_CONFIG_EXACT_ROUNDING 16

/* oq_int4_linear `config` flag: the packed weights and scales are static --
 * written before any kernel still in flight on `stream` (e.g. quantized at
 * load time, then synchronized).  The GEMV then streams them while the
 * previous kernel in the stream drains (programmatic dependent launch)
 * instead of after it; x and y are still ordered after that kernel.  Without
 * the flag the GEMV reads nothing before the previous kernel has finished.
 * No counterpart in the reference (its Triton launch is stream-ordered). */
#define OQ_CONFIG_STATIC_WEIGHTS 32

/* oq_int4_linear / oq_int4_linear_ex `config` flag: SiLU-gate fusion of a
 * gate/up pair.  packed and scales hold the [gate; up] stack -- 2n rows,
 * gate rows first -- and y (M x n) = silu(x . Wg^T) * (x . Wu^T) with
 * silu(g) = g / (1 + exp(-g)), in one pass, no bias: the GEMV for M <= 16
 * (kernel AUTO or GEMV), else (or kernel TCGEN05) the tcgen05 GEMM, whose
 * 128-row tiles hold the gate and up rows of 64 features and whose epilogue
 * writes silu(gate) * up (never split over a workspace).  No counterpart in
 * the reference. */
#define OQ_CONFIG_SILU_GATE 64

/* Library version string ("openquant_b200 <x.y.z> sm_100a"). */
OQ_API const char *oq_version(void);

/* Message of the last failed call on this thread ("" if none). */
OQ_API const char *oq_last_error(void);

/* Number of visible CUDA devices with compute capability 10.x, or -1 when
 * the CUDA runtime cannot be initialised.  Never fails otherwise. */
OQ_API int oq_device_count(void);

/*
 * Synchronises the current device, then reads and clears the device-side
 * error word of the library's pipelined kernels: *code = 0 when none, 1 when
 * a kernel gave up waiting on one of its internal pipeline barriers (it then
 * returned early, its outputs are undefined), 2 when oq_peer_barrier gave
 * up waiting for a peer GPU.  No reference counterpart: the reference's
 * Triton kernel has no internal waits.
 */
OQ_API int oq_take_device_error(int32_t *code);

/*
 * Per-row symmetric INT8 quantize.
 * Replaces quantize(weights, bits=8), openquant/quantization.py:14-40,
 * :54-59 of the reference: scale[r] = max_c |w[r,c]| / 127 (fp32, IEEE
 * division), 1.0 for an all-zero row; q = clip(rint(w / scale), -127, 127)
 * with round-half-to-even and IEEE division; NaN quotients give 0.
 *   w      : N*K elements of type `dtype` (device)
 *   q      : N*K int8 (device, out)
 *   scales : N fp32 (device, out)
 */
OQ_API int oq_quant_int8_rowwise(const void *w, int dtype, int64_t n, int64_t k,
                          int8_t *q, float *scales, oq_stream_t stream);

/*
 * Per-row symmetric INT4 quantize with flat nibble packing.
 * Replaces quantize(weights, bits=4), openquant/quantization.py:14-37,
 * :41-52: scale[r] = max|w[r,:]| / 7; the int4 values of the whole
 * row-major matrix are packed two per byte across row boundaries.
 *   packed : ceil(N*K/2) bytes (device, out)
 *   scales : N fp32 (device, out)
 */
OQ_API int oq_quant_int4_rowwise(const void *w, int dtype, int64_t n, int64_t k,
                          uint8_t *packed, float *scales, oq_stream_t stream);

/*
 * Groupwise INT4 quantize.
 * Replaces quantize_int4_groupwise(weights, group_size),
 * openquant/groupwise.py:13-61: rows zero-padded to KP, scale = max|group| /
 * 7.0 (1.0 for an all-zero group), q = clip(rint(w/scale), -7, 7), packed.
 * group_size must be even and >= 2.
 *   packed    : N*KP/2 bytes (device, out)
 *   scales    : N*(KP/g) fp32 (device, out)
 *   nonfinite : one int32 (device, out); set to 0, then to 1 if any input
 *               element is NaN or +-Inf (the reference raises ValueError,
 *               groupwise.py:22-23; the host wrapper does the same after
 *               reading it).  May be NULL to skip the check.
 */
OQ_API int oq_quant_int4_group(const void *w, int dtype, int64_t n, int64_t k,
                        int group_size, uint8_t *packed, float *scales,
                        int32_t *nonfinite, oq_stream_t stream);

/*
 * Per-row INT8 dequantize: out[r,c] = (float)q[r,c] * scales[r].
 * Replaces dequantize() for bits=8, openquant/quantization.py:62-64, :82,
 * and decode_gpu(bits=8), openquant/gpu_benchmark.py:10-12, :30.
 */
OQ_API int oq_dequant_int8_rowwise(const int8_t *q, const float *scales, int64_t n,
                            int64_t k, float *out, oq_stream_t stream);

/*
 * Per-row INT4 (flat-packed) dequantize: out[f] = int4(f) * scales[f / K]
 * for f < N*K.  Replaces dequantize() for bits=4,
 * openquant/quantization.py:65-78, :82, and decode_gpu(bits=4),
 * openquant/gpu_benchmark.py:14-25, :30.
 */
OQ_API int oq_dequant_int4_rowwise(const uint8_t *packed, const float *scales,
                            int64_t n, int64_t k, float *out,
                            oq_stream_t stream);

/*
 * Groupwise INT4 dequantize to fp32 [N][K] (padding columns dropped).
 * Replaces dequantize_int4_groupwise(q), openquant/groupwise.py:64-89, and
 * restore_groupwise_torch(), openquant/group_benchmark.py:11-30.
 */
OQ_API int oq_dequant_int4_group(const uint8_t *packed, const float *scales,
                          int64_t n, int64_t k, int group_size, float *out,
                          oq_stream_t stream);

/*
 * Fused groupwise-INT4 dequant + matmul: y[M][N] (fp32) = x[M][K] . W^T where
 * W[n][k] = round_to_x_dtype( (float)int4(n,k) * scales[n][k/g] ) -- the
 * weight rounding of the reference kernel, openquant/triton_int4.py:62-65 --
 * and products are accumulated in fp32.
 * Replaces int4_linear(), openquant/triton_int4.py:78-138 (its Triton kernel
 * _int4_matmul, :6-75).
 *   x       : M*K fp16 or bf16, row-major, contiguous (device)
 *   packed  : N*KP/2 bytes, the groupwise layout (device)
 *   scales  : N*(KP/g) fp32 (device)
 *   y       : M*N fp32 (device, out)
 *   kernel  : OQ_KERNEL_* (AUTO picks by shape)
 *   config  : low 4 bits: launch-shape index of the chosen kernel (0 =
 *             default); for the GEMV, 1..7 select register-ring launch
 *             shapes (warps per CTA, chunks in flight per warp, CTAs per
 *             SM) = (8,4,2) (16,2,2) (12,2,2) (16,1,2) (8,2,3) (8,2,4)
 *             (8,4,4), and 8, 9, 10 the TMA-fed kernel with 8 or 16
 *             consumer warps and one CTA per SM, or 8 warps and two CTAs per
 *             SM (M <= 16), 12 one CTA per 16-row tile with four CTAs per SM
 *             (M <= 16, K <= 4096), 13 one 16-warp CTA per SM owning two
 *             16-row tiles (M <= 16, K <= 4096, at most two tiles per SM) --
 *             only the fp32 summation order changes;
 *             `openquant tune` picks it.  | OQ_CONFIG_EXACT_ROUNDING,
 *             | OQ_CONFIG_STATIC_WEIGHTS: see above.
 */
OQ_API int oq_int4_linear(const void *x, int x_dtype, const uint8_t *packed,
                   const float *scales, float *y, int64_t m, int64_t n,
                   int64_t k, int group_size, int kernel, int config,
                   oq_stream_t stream);

/* oq_int4_linear with a fused epilogue: y[m][n] = (x . W^T)[m][n] + bias[n],
 * written as fp32, fp16 or bf16 (y_dtype = OQ_F32 / OQ_F16 / OQ_BF16) --
 * the bias is added in fp32 and the sum rounded once to y_dtype.  bias may be
 * NULL (fp32 [N] otherwise, device).  Every other argument as oq_int4_linear.
 * No counterpart in the reference (its kernel writes fp32 only,
 * openquant/triton_int4.py:120-122). */
OQ_API int oq_int4_linear_ex(const void *x, int x_dtype, const uint8_t *packed,
                             const float *scales, void *y, int y_dtype,
                             const float *bias, int64_t m, int64_t n, int64_t k,
                             int group_size, int kernel, int config,
                             oq_stream_t stream);

/* oq_int4_linear_ex with a caller workspace for the tcgen05 GEMM: when the
 * tiles do not divide evenly over the SMs, the GEMM splits the work evenly
 * (stream-K: some tiles computed in pieces by two or more SMs), keeps the
 * pieces' fp32 sums in `workspace` (device, 16-byte aligned, contents
 * ignored) and adds them in k order in a second kernel on the stream -- a
 * fixed order, so the result is deterministic; it differs from the unsplit
 * kernel's only in fp32 summation order.  ws_bytes below
 * oq_int4_linear_workspace_bytes(...) (or workspace NULL) runs the unsplit
 * kernel.  The workspace is in use until the call's work on `stream` ends.
 * The same computation as int4_linear, openquant/triton_int4.py:78-138
 * (same output contract, :120-122). */
OQ_API int oq_int4_linear_ws(const void *x, int x_dtype, const uint8_t *packed,
                             const float *scales, void *y, int y_dtype,
                             const float *bias, int64_t m, int64_t n, int64_t k,
                             int group_size, int kernel, int config,
                             void *workspace, size_t ws_bytes,
                             oq_stream_t stream);

/* The fused INT4 linear layer with one fp16 scale per group: scales is
 * fp16 [N][KP/g] (device) -- e.g. the fp32 scales of quantize_int4_groupwise
 * rounded to fp16 -- and W[n][k] = int4(n, k) * (float)scales[n][k/g].  Runs
 * the decode GEMV in its scale-after mode (each group's scale applied to the
 * group's fp32 sum of x * q; the pair GEMV, else the TMA GEMV): fp16 x,
 * M <= 16, a power-of-two group_size that is a multiple of 128, K % 8 == 0,
 * 16-byte aligned x and packed, and x small enough for those kernels to stage
 * it in shared memory (OQ_ERR_INVALID otherwise).  y, y_dtype and bias as oq_int4_linear_ex;
 * config: OQ_CONFIG_STATIC_WEIGHTS only.  A variant of int4_linear,
 * openquant/triton_int4.py:78-138, whose reference requires fp32 scales
 * (:93-94): half the scale bytes per decode step. */
OQ_API int oq_int4_linear_f16s(const void *x, int x_dtype, const uint8_t *packed,
                               const void *scales, void *y, int y_dtype,
                               const float *bias, int64_t m, int64_t n, int64_t k,
                               int group_size, int config, oq_stream_t stream);

/* The fused INT4 linear layer on HOST activations and output: x (M*K fp16 or
 * bf16) and y (M*N of y_dtype) are page-locked host memory (cudaHostAlloc /
 * cudaHostRegister); packed / scales / bias are device memory and x_stage a
 * device buffer of M*K*2 bytes (16-byte aligned; contents overwritten).  One
 * small kernel copies x over the bus into x_stage and the layer kernel -- the
 * one oq_int4_linear_ex launches for these arguments, its weights streaming
 * meanwhile (programmatic dependent launch) -- writes y straight into host
 * memory through its mapped address; the call returns once y holds the
 * result (`stream` synchronized).  x must be 16-byte aligned.  Meant for
 * decode steps (the prefill GEMM's split over a workspace is not used here).
 * Every other argument as oq_int4_linear_ex, and the same result bit for bit.
 * Replaces the host round trip of a reference caller,
 * int4_linear(x.cuda(), ...).cpu() -- openquant/triton_int4.py:78-138, fed
 * from host arrays by .cuda() copies as in openquant/fused_benchmark.py:53-70. */
OQ_API int oq_int4_linear_host(const void *x, int x_dtype, const uint8_t *packed,
                               const float *scales, void *y, int y_dtype,
                               const float *bias, int64_t m, int64_t n, int64_t k,
                               int group_size, int kernel, int config,
                               void *x_stage, oq_stream_t stream);

/* oq_int4_linear_host with its arguments fixed once: the copy kernel and the
 * layer kernel are captured into a CUDA graph (on the current device), and
 * oq_int4_linear_host_run replays it on `stream` and returns once y holds
 * the result -- one graph launch and one synchronization per decode step.
 * The graph reads x and writes y, x_stage (and reads packed, scales, bias) at
 * the addresses given here each time it runs: they stay borrowed, must
 * outlive the plan and keep their page-locking; their contents may change
 * between runs.  Runs of one plan must not overlap.  *plan receives an
 * opaque handle (NULL on failure); oq_int4_linear_host_plan_free releases it
 * (NULL is a no-op).  Same validation, kernels and result as
 * oq_int4_linear_host; no counterpart in the reference. */
OQ_API int oq_int4_linear_host_plan(const void *x, int x_dtype, const uint8_t *packed,
                                    const float *scales, void *y, int y_dtype,
                                    const float *bias, int64_t m, int64_t n, int64_t k,
                                    int group_size, int kernel, int config,
                                    void *x_stage, void **plan);
OQ_API int oq_int4_linear_host_run(void *plan, oq_stream_t stream);
OQ_API int oq_int4_linear_host_plan_free(void *plan);

/* Workspace bytes oq_int4_linear_ws uses for this shape and kernel choice
 * (0: the chosen kernel takes none).  Never fails (0 for invalid shapes). */
OQ_API int64_t oq_int4_linear_workspace_bytes(int64_t m, int64_t n, int64_t k,
                                              int group_size, int kernel,
                                              int config);

/*
 * N-column-sharded fused linear layer, one process per GPU: this GPU holds
 * rows [col0, col0 + n) of the full layer's weights (a contiguous block of
 * the groupwise layout: rows of packed and of scales) and computes
 * y[:, col0:col0+n] of the full y[M][ld], and its kernels store every element
 * of that slice into the y buffers of all n_gpus GPUs of the layer --
 * y_gpus[0] this GPU's, y_gpus[1..] the peers' (mapped with oq_peer_import)
 * -- at y_gpus[i][b * ld + col0 + f], with plain stores over NVLink.  That
 * replaces the reference's fp32 (M, N) output allocation
 * (openquant/triton_int4.py:120-122) with each GPU's share of the gathered
 * output; the compute is oq_int4_linear_ex's (same kernels, same result per
 * element), y_dtype / bias as there (bias: this shard's n features).
 * workspace / ws_bytes as oq_int4_linear_ws.  Follow it with
 * oq_peer_barrier on the same stream before reading y.  n_gpus <= 8.  No
 * counterpart in the reference (single-GPU only,
 * openquant/fused_benchmark.py:53-54).
 */
OQ_API int oq_int4_linear_peers(const void *x, int x_dtype, const uint8_t *packed,
                                const float *scales, void *const *y_gpus,
                                int n_gpus, int y_dtype, const float *bias,
                                int64_t ld, int64_t col0, int64_t m, int64_t n,
                                int64_t k, int group_size, int kernel,
                                int config, void *workspace, size_t ws_bytes,
                                oq_stream_t stream);

/* Bytes of the handle that oq_peer_export writes (a CUDA IPC handle). */
#define OQ_PEER_HANDLE_BYTES 64

/* Peer-mappable device memory for the sharded layer's outputs and flags:
 * oq_peer_alloc allocates `bytes` on the current device, zeroed (it
 * synchronises the device); oq_peer_free releases it (after every peer has
 * closed its mapping).  oq_peer_export writes the buffer's handle
 * (OQ_PEER_HANDLE_BYTES) for the other processes; oq_peer_import maps a
 * peer's buffer into this process on the current device and oq_peer_close
 * unmaps it.  No counterpart in the reference. */
OQ_API int oq_peer_alloc(size_t bytes, void **ptr);
OQ_API int oq_peer_free(void *ptr);
OQ_API int oq_peer_export(const void *ptr, uint8_t *handle);
OQ_API int oq_peer_import(const uint8_t *handle, void **ptr);
OQ_API int oq_peer_close(void *ptr);

/* Words of a flag array of oq_peer_barrier (uint32). */
#define OQ_PEER_FLAG_WORDS 16

/* Flag barrier of the sharded layer, enqueued on `stream` after the
 * oq_int4_linear_peers call: flags_gpus[j] is GPU j's flag array of
 * OQ_PEER_FLAG_WORDS uint32 (zeroed by oq_peer_alloc; flags_gpus[rank] this
 * GPU's own).  After every kernel enqueued before it has finished, it counts
 * itself (epoch = 1, 2, ...: this GPU's barrier count, kept in the last word
 * of its own array, so a captured CUDA graph replays correctly), publishes
 * the earlier kernels' writes (system-scope fence) and writes `epoch` into
 * word `rank` of every GPU's array, then waits until words 0..world-1 of its
 * own array hold `epoch` or later (wrap-around compare) -- all peers have
 * finished storing into this GPU's y.  Every GPU of the layer calls it the
 * same number of times.  The wait gives up after timeout_ns (0: 5 s), sets
 * device error code 2 (oq_take_device_error) and returns.  No counterpart in
 * the reference. */
OQ_API int oq_peer_barrier(uint32_t *const *flags_gpus, int world, int rank,
                           int64_t timeout_ns, oq_stream_t stream);

/* W8A8 linear layer on the tcgen05 tensor cores (kind::i8, int32 sums):
 * y[m][n] = sx[m] * sw[n] * sum_k qx[m][k] * qw[n][k].  qx / sx and qw / sw
 * are per-row INT8 data and fp32 scales in the format of
 * oq_quant_int8_rowwise (the reference's quantize(bits=8),
 * openquant/quantization.py:14-40) -- for the activations, one row per token.
 *   qx : int8 [M][K], sx : fp32 [M]   (device)
 *   qw : int8 [N][K], sw : fp32 [N]   (device)
 *   y  : fp32 [M][N]                  (device, out)
 * K % 16 == 0, qx and qw 16-byte aligned.  No counterpart in the reference
 * (its only matmul is the INT4 one); this is the activation-side extension of
 * the same per-row INT8 format. */
OQ_API int oq_int8_gemm(const int8_t *qx, const float *sx, const int8_t *qw,
                        const float *sw, float *y, int64_t m, int64_t n,
                        int64_t k, oq_stream_t stream);

/*
 * The W8A8 linear layer without allocation: y = x . W^T with x quantized per
 * token to INT8 (as oq_quant_int8_rowwise) and multiplied by oq_int8_gemm,
 * where the quantized activations and their scales go to a fixed array that
 * the library keeps on each GPU (16 MiB + 64 KiB, held until the process
 * exits) instead of memory the caller would allocate.  For callers that
 * cannot allocate device memory when they call in -- a host runtime that
 * lends the library only the tensors it owns, or a service whose device
 * memory is fixed at start-up.  Same result as oq_quant_int8_rowwise into
 * caller buffers followed by oq_int8_gemm.
 *   x  : [M][K] fp32 / fp16 / bf16 (x_dtype)   (device)
 *   qw : int8 [N][K], sw : fp32 [N]            (device)
 *   y  : fp32 [M][N]                           (device, out)
 * K % 16 == 0; M <= 16384 and M * K <= 16 MiB, else OQ_ERR_INVALID.
 * The first call on a device looks up the array's device address, so make
 * that first call before any stream capture.  All calls on a device share
 * the one array: calls whose work overlaps on the GPU (other streams, other
 * host threads) race and must be serialised by the caller.
 * No counterpart in the reference. */
OQ_API int oq_int8_linear_noalloc(const void *x, int x_dtype, const int8_t *qw,
                                  const float *sw, float *y, int64_t m,
                                  int64_t n, int64_t k, oq_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* OPENQUANT_B200_H */
