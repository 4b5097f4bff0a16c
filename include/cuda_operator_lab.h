/*
 * C ABI of libcuda_operator_lab.so, the sm_100a (B200) build of the
 * cuda-operator-lab Transformer operator family.
 *
 * Every symbol below is `extern "C"`, takes plain device pointers, 64-bit
 * sizes and a `void* stream` (a cudaStream_t; NULL selects the legacy
 * default stream), enqueues its work asynchronously on that stream and
 * returns an `int` that is a cudaError_t value (0 = success).  No symbol
 * synchronises the host, and none takes a PyTorch type.
 *
 * The first block re-exports, with identical names and signatures, the 54
 * symbols of the reference library (paths below are inside the reference
 * project).  All versions of one operator run the same sm_100a kernel:
 * the reference's version numbers named alternative CUDA implementations of
 * one mathematical operation, and the arithmetic they specify is kept:
 *   - gemm_bias_gelu v0/v1 use the erf GELU, v2..v6 the tanh GELU
 *     (gemm_bias_gelu.cu:795-828 vs its cuBLASLt GELU_BIAS epilogue);
 *   - gemm_swiglu v5 rounds the gate/up projections to bf16 before SiLU
 *     (gemm_swiglu.cu:268-286), all other versions keep them in fp32;
 *   - fp32-input GEMMs (gemm_swiglu v0..v3, gemm_bias_gelu v0..v6) keep
 *     full fp32 products and fp32 accumulation.
 * Error behaviour follows the reference: empty work (rows == 0, m == 0 or
 * n == 0, elements == 0) succeeds before any pointer check; NULL pointers,
 * cols == 0, k == 0, eps <= 0 and sizes above INT32_MAX return
 * cudaErrorInvalidValue (1); the bf16 GEMM versions v6..v9 keep the
 * reference's shape guards (gemm_swiglu.cu:1125,1169,1213,1257).
 *
 * The second block holds entry points the reference does not have; each
 * names the workload (bf16 norms and GEMMs of a Llama-style MLP block) or the
 * multi-GPU step it serves.
 */
#ifndef CUDA_OPERATOR_LAB_H_
#define CUDA_OPERATOR_LAB_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- Global fp32 sum ------------------------------------------------------
 * out[0] = sum(input[0..n)).  Replaces csrc/reduction/reduction.cuh:8-42.
 * Accumulates in fp64 with a fixed per-CTA partition and a fixed-order final
 * combine, so the result is bit-reproducible run to run (the reference's
 * fp32 atomicAdd combine, reduction.cu:43, is not).  input may be NULL only
 * when n == 0, in which case out[0] = 0.  Scratch (8 bytes per CTA, one
 * resident wave of CTAs) is a block the library allocates once per
 * (device, stream) on the first call on that stream and keeps (the first
 * call on a device also reserves 64 blocks for captured calls and waits for
 * its stream once).  A call captured into a CUDA graph takes one of those
 * reserved blocks for good, never the stream's; beyond them, and for
 * cudaStreamPerThread, the scratch is a stream-ordered allocation from a
 * library-owned cudaMemPool (graph memory nodes under capture).  Per-stream
 * blocks are keyed by the stream's unique id (cudaStreamGetId), so a new
 * stream never inherits a destroyed stream's block; blocks are never freed
 * and live until the process exits (at most 256).  A captured call keeps its
 * block in the graph: replays of one captured reduction (the same graph exec
 * launched on two streams at once, or two instantiations of the same
 * captured graph run concurrently) share it and must not overlap on the GPU. */
int cuda_operator_reduction_v0(const float* input, float* output, uint64_t n, void* stream); /* reduction.cuh:8  */
int cuda_operator_reduction_v1(const float* input, float* output, uint64_t n, void* stream); /* reduction.cuh:14 */
int cuda_operator_reduction_v2(const float* input, float* output, uint64_t n, void* stream); /* reduction.cuh:20 */
int cuda_operator_reduction_v3(const float* input, float* output, uint64_t n, void* stream); /* reduction.cuh:26 */
int cuda_operator_reduction_v4(const float* input, float* output, uint64_t n, void* stream); /* reduction.cuh:32 */
int cuda_operator_reduction_v5(const float* input, float* output, uint64_t n, void* stream); /* reduction.cuh:38 */

/* Message for a code returned by any symbol here.  Replaces
 * csrc/reduction/reduction.cuh:44 (cudaGetErrorString for CUDA codes, plus
 * the library's own codes, which start at 10000). */
const char* cuda_operator_error_string(int code);

/* ---- Row softmax (fp32) --------------------------------------------------
 * output[r, :] = softmax(input[r, :]).  Replaces softmax.cuh:5-47. */
int cuda_operator_softmax_v0(const float* input, float* output, uint64_t rows, uint64_t cols, void* stream); /* softmax.cuh:5  */
int cuda_operator_softmax_v1(const float* input, float* output, uint64_t rows, uint64_t cols, void* stream); /* softmax.cuh:12 */
int cuda_operator_softmax_v2(const float* input, float* output, uint64_t rows, uint64_t cols, void* stream); /* softmax.cuh:19 */
int cuda_operator_softmax_v3(const float* input, float* output, uint64_t rows, uint64_t cols, void* stream); /* softmax.cuh:26 */
int cuda_operator_softmax_v4(const float* input, float* output, uint64_t rows, uint64_t cols, void* stream); /* softmax.cuh:34 */
int cuda_operator_softmax_v5(const float* input, float* output, uint64_t rows, uint64_t cols, void* stream); /* softmax.cuh:42 */

/* ---- RMSNorm (fp32) --------------------------------------------------------
 * y = x * rsqrt(mean(x^2) + eps) * weight.  Replaces rmsnorm.cuh:5-47. */
int cuda_operator_rmsnorm_v0(const float* input, const float* weight, float* output, uint64_t rows, uint64_t cols, float eps, void* stream); /* rmsnorm.cuh:5  */
int cuda_operator_rmsnorm_v1(const float* input, const float* weight, float* output, uint64_t rows, uint64_t cols, float eps, void* stream); /* rmsnorm.cuh:14 */
int cuda_operator_rmsnorm_v2(const float* input, const float* weight, float* output, uint64_t rows, uint64_t cols, float eps, void* stream); /* rmsnorm.cuh:23 */
int cuda_operator_rmsnorm_v3(const float* input, const float* weight, float* output, uint64_t rows, uint64_t cols, float eps, void* stream); /* rmsnorm.cuh:32 */
int cuda_operator_rmsnorm_v4(const float* input, const float* weight, float* output, uint64_t rows, uint64_t cols, float eps, void* stream); /* rmsnorm.cuh:41 */

/* ---- LayerNorm (fp32, biased variance) -------------------------------------
 * Replaces layernorm.cuh:5-68. */
int cuda_operator_layernorm_v0(const float* input, const float* weight, const float* bias, float* output, uint64_t rows, uint64_t cols, float eps, void* stream); /* layernorm.cuh:5  */
int cuda_operator_layernorm_v1(const float* input, const float* weight, const float* bias, float* output, uint64_t rows, uint64_t cols, float eps, void* stream); /* layernorm.cuh:16 */
int cuda_operator_layernorm_v2(const float* input, const float* weight, const float* bias, float* output, uint64_t rows, uint64_t cols, float eps, void* stream); /* layernorm.cuh:27 */
int cuda_operator_layernorm_v3(const float* input, const float* weight, const float* bias, float* output, uint64_t rows, uint64_t cols, float eps, void* stream); /* layernorm.cuh:38 */
int cuda_operator_layernorm_v4(const float* input, const float* weight, const float* bias, float* output, uint64_t rows, uint64_t cols, float eps, void* stream); /* layernorm.cuh:49 */
int cuda_operator_layernorm_v5(const float* input, const float* weight, const float* bias, float* output, uint64_t rows, uint64_t cols, float eps, void* stream); /* layernorm.cuh:60 */

/* ---- Residual add + LayerNorm (fp32) ---------------------------------------
 * output = LayerNorm(input + residual); h = input + residual is not stored.
 * Replaces fused_residual_layernorm.cuh:5-62. */
int cuda_operator_fused_residual_layernorm_v0(const float* input, const float* residual, const float* weight, const float* bias, float* output, uint64_t rows, uint64_t cols, float eps, void* stream); /* fused_residual_layernorm.cuh:5  */
int cuda_operator_fused_residual_layernorm_v1(const float* input, const float* residual, const float* weight, const float* bias, float* output, uint64_t rows, uint64_t cols, float eps, void* stream); /* fused_residual_layernorm.cuh:17 */
int cuda_operator_fused_residual_layernorm_v2(const float* input, const float* residual, const float* weight, const float* bias, float* output, uint64_t rows, uint64_t cols, float eps, void* stream); /* fused_residual_layernorm.cuh:29 */
int cuda_operator_fused_residual_layernorm_v3(const float* input, const float* residual, const float* weight, const float* bias, float* output, uint64_t rows, uint64_t cols, float eps, void* stream); /* fused_residual_layernorm.cuh:41 */
int cuda_operator_fused_residual_layernorm_v4(const float* input, const float* residual, const float* weight, const float* bias, float* output, uint64_t rows, uint64_t cols, float eps, void* stream); /* fused_residual_layernorm.cuh:53 */

/* ---- Bias + exact (erf) GELU (fp32) -----------------------------------------
 * output[r, c] = gelu_erf(input[r, c] + bias[c]).  Replaces
 * fused_bias_gelu.cuh:5-29. */
int cuda_operator_fused_bias_gelu_v0(const float* input, const float* bias, float* output, uint64_t rows, uint64_t cols, void* stream); /* fused_bias_gelu.cuh:5  */
int cuda_operator_fused_bias_gelu_v1(const float* input, const float* bias, float* output, uint64_t rows, uint64_t cols, void* stream); /* fused_bias_gelu.cuh:14 */
int cuda_operator_fused_bias_gelu_v2(const float* input, const float* bias, float* output, uint64_t rows, uint64_t cols, void* stream); /* fused_bias_gelu.cuh:23 */

/* ---- SwiGLU (fp32) -----------------------------------------------------------
 * output = gate / (1 + exp(-gate)) * up.  Replaces swiglu.cuh:5-27 (v0/v1 take
 * an element count, v2 takes rows and cols). */
int cuda_operator_swiglu_v0(const float* gate, const float* up, float* output, uint64_t elements, void* stream); /* swiglu.cuh:5  */
int cuda_operator_swiglu_v1(const float* gate, const float* up, float* output, uint64_t elements, void* stream); /* swiglu.cuh:13 */
int cuda_operator_swiglu_v2(const float* gate, const float* up, float* output, uint64_t rows, uint64_t cols, void* stream); /* swiglu.cuh:21 */

/* ---- GEMM + bias + GELU (fp32 in/out) -----------------------------------------
 * output[m, n] = gelu(sum_k input[m, k] * weight[n, k] + bias[n]); v0/v1 erf,
 * v2..v6 tanh.  Replaces gemm_bias_gelu.cuh:5-79. */
int cuda_operator_gemm_bias_gelu_v0(const float* input, const float* weight, const float* bias, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_bias_gelu.cuh:5  */
int cuda_operator_gemm_bias_gelu_v1(const float* input, const float* weight, const float* bias, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_bias_gelu.cuh:16 */
int cuda_operator_gemm_bias_gelu_v2(const float* input, const float* weight, const float* bias, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_bias_gelu.cuh:27 */
int cuda_operator_gemm_bias_gelu_v3(const float* input, const float* weight, const float* bias, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_bias_gelu.cuh:38 */
int cuda_operator_gemm_bias_gelu_v4(const float* input, const float* weight, const float* bias, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_bias_gelu.cuh:49 */
int cuda_operator_gemm_bias_gelu_v5(const float* input, const float* weight, const float* bias, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_bias_gelu.cuh:60 */
int cuda_operator_gemm_bias_gelu_v6(const float* input, const float* weight, const float* bias, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_bias_gelu.cuh:71 */

/* ---- GEMM + SwiGLU ---------------------------------------------------------------
 * output[m, j] = silu(x[m,:] . Wg[j,:]) * (x[m,:] . Wu[j,:]), fp32 output.
 * Packed versions take W[2N, K] with the N gate rows first, then the N up
 * rows.  The workspace argument is validated (non-NULL) and left untouched:
 * the sm_100a kernel keeps both projections in tensor memory, so there is no
 * [M, 2N] round trip.  Replaces gemm_swiglu.cuh:5-136. */
int cuda_operator_gemm_swiglu_v0(const float* input, const float* gate_weight, const float* up_weight, float* workspace, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_swiglu.cuh:5   */
int cuda_operator_gemm_swiglu_v1(const float* input, const float* gate_weight, const float* up_weight, float* workspace, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_swiglu.cuh:17  */
int cuda_operator_gemm_swiglu_v2(const float* input, const float* packed_weight, float* workspace, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_swiglu.cuh:29  */
int cuda_operator_gemm_swiglu_v3(const float* input, const float* packed_weight, float* workspace, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_swiglu.cuh:40  */
int cuda_operator_gemm_swiglu_v4(const void* input_bf16, const void* packed_weight_bf16, float* workspace, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_swiglu.cuh:51  */
int cuda_operator_gemm_swiglu_v5(const void* input_bf16, const void* packed_weight_bf16, void* workspace_bf16, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_swiglu.cuh:62  */
int cuda_operator_gemm_swiglu_v6(const void* input_bf16, const void* gate_weight_bf16, const void* up_weight_bf16, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_swiglu.cuh:73  */
int cuda_operator_gemm_swiglu_v7(const void* input_bf16, const void* gate_weight_bf16, const void* up_weight_bf16, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_swiglu.cuh:84  */
int cuda_operator_gemm_swiglu_v8(const void* input_bf16, const void* gate_weight_bf16, const void* up_weight_bf16, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_swiglu.cuh:95  */
int cuda_operator_gemm_swiglu_v9(const void* input_bf16, const void* gate_weight_bf16, const void* up_weight_bf16, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_swiglu.cuh:106 */
int cuda_operator_gemm_swiglu_v10(const void* input_bf16, const void* packed_weight_bf16, float* workspace, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_swiglu.cuh:117 */
int cuda_operator_gemm_swiglu_v11(const void* input_bf16, const void* packed_weight_bf16, float* workspace, float* output, uint64_t m, uint64_t k, uint64_t n, void* stream); /* gemm_swiglu.cuh:128 */

/* ====================== Entry points new in this library ====================== */

/* RMSNorm with bf16 input, weight and output, fp32 statistics:
 * y = bf16((float(x) * rsqrt(mean(float(x)^2) + eps)) * float(w)).
 * The large row-sharded RMSNorm of the Llama MLP workload (x[16384, 4096]).
 * The reference is fp32-only (python/cuda_operator_lab/references.py:36-37). */
int cuda_operator_rmsnorm_bf16(const void* input_bf16, const void* weight_bf16, void* output_bf16, uint64_t rows, uint64_t cols, float eps, void* stream);

/* Residual add + LayerNorm that also stores h = input + residual (fp32).
 * The reference variant (fused_residual_layernorm.cu:295-306) writes only
 * LayerNorm(h); a transformer block also needs h for its next residual. */
int cuda_operator_fused_residual_layernorm_h(const float* input, const float* residual, const float* weight, const float* bias, float* h_output, float* output, uint64_t rows, uint64_t cols, float eps, void* stream);

/* Residual add + RMSNorm in one pass: h = input + residual is stored to h_out
 * and y = (h * rsqrt(mean(h^2) + eps)) * weight to output; every input byte is
 * read once.  No reference counterpart (its residual fusion exists only for
 * LayerNorm, fused_residual_layernorm.cuh:5); this is the norm that feeds the
 * MLP GEMM in a decoder block.  _bf16: bf16 tensors, fp32 statistics, h rounded
 * to bf16 before the statistics (what a separate add kernel would store);
 * _h: fp32.  rows == 0 succeeds; NULL, cols == 0 or eps <= 0 return
 * cudaErrorInvalidValue. */
int cuda_operator_fused_residual_rmsnorm_bf16(const void* input_bf16, const void* residual_bf16, const void* weight_bf16, void* h_out_bf16, void* output_bf16, uint64_t rows, uint64_t cols, float eps, void* stream);
int cuda_operator_fused_residual_rmsnorm_h(const float* input, const float* residual, const float* weight, float* h_out, float* output, uint64_t rows, uint64_t cols, float eps, void* stream);

/* Per-row inverse RMS of bf16 x[rows, cols]: rstd[row] = rsqrt(mean(x[row]^2) + eps)
 * in fp32 (the statistics of references.py:46-47 without the scaling pass).
 * No reference counterpart; pairs with cuda_operator_gemm_swiglu_rowscale_bf16.
 * Same argument rules as cuda_operator_rmsnorm_bf16. */
int cuda_operator_rmsnorm_rstd_bf16(const void* input_bf16, float* rstd, uint64_t rows, uint64_t cols, float eps, void* stream);

/* RMSNorm -> packed GEMM+SwiGLU with the normalisation folded into the GEMM:
 * out[m, j] = bf16(silu(rs[m] * g) * (rs[m] * u)), g and u the fp32-accumulated
 * products of the raw bf16 x[M, K] with the packed weight [2N, K] whose columns
 * the caller multiplied by the RMSNorm weight once (W * diag(w)), rs from
 * cuda_operator_rmsnorm_rstd_bf16.  Equal to RMSNorm followed by
 * cuda_operator_gemm_swiglu_bf16 up to bf16 rounding, without writing and
 * re-reading the normalised activations.  No reference counterpart. */
int cuda_operator_gemm_swiglu_rowscale_bf16(const void* input_bf16, const float* row_scale, const void* packed_weight_bf16, void* output_bf16, uint64_t m, uint64_t k, uint64_t n, void* stream);

/* Packed GEMM + SwiGLU with bf16 output: out[m, j] = bf16(silu(g) * u), g and u
 * accumulated in fp32 from bf16 x[M, K] and packed W[2N, K].  Same arithmetic
 * as cuda_operator_gemm_swiglu_v4 up to the final rounding; no workspace. */
int cuda_operator_gemm_swiglu_bf16(const void* input_bf16, const void* packed_weight_bf16, void* output_bf16, uint64_t m, uint64_t k, uint64_t n, void* stream);

/* GEMM + bias + exact (erf) GELU with bf16 x[M, K], W[N, K], fp32 bias[N] and
 * bf16 output, fp32 accumulation.  The reference's GEMM+bias+GELU is fp32-only
 * (gemm_bias_gelu.cuh:5); this is its bf16 tensor-core counterpart. */
int cuda_operator_gemm_bias_gelu_bf16(const void* input_bf16, const void* weight_bf16, const float* bias, void* output_bf16, uint64_t m, uint64_t k, uint64_t n, void* stream);

/* Down projection with the residual add fused: out[m, n] = bf16(x[m, :] . w[n, :]
 * + residual[m, n]), fp32 accumulation, bf16 x[M, K], W[N, K], residual and
 * out [M, N].  No reference counterpart: the step after GEMM+SwiGLU in a
 * decoder MLP block (down projection back to the model width plus the block's
 * residual).  out may equal residual (in-place update).  m == 0 or n == 0
 * succeeds; NULL, k == 0 or sizes above INT32_MAX return cudaErrorInvalidValue. */
int cuda_operator_gemm_residual_bf16(const void* input_bf16, const void* weight_bf16, const void* residual_bf16, void* output_bf16, uint64_t m, uint64_t k, uint64_t n, void* stream);

/* N-sharded packed GEMM + SwiGLU with the output all-gather fused into its
 * epilogue (no reference counterpart; the column gather after the N-sharded
 * cuda_operator_gemm_swiglu_bf16 / _rowscale_bf16).  Rank r of g computes its
 * [m, n] output column block from x[m, k] and its packed weight shard [2n, k]
 * (g, u scaled by row_scale[m] first when row_scale is not NULL) and stores it
 * to each of the num_dests (1..8) destinations: dests (a HOST array of device
 * addresses) holds the block's origin in this GPU's [m, ld] bf16 output
 * first, then the same origin in the other ranks' outputs as mapped by
 * cuda_operator_lab_peer_open.  The stores to other GPUs travel over NVLink
 * while later tiles compute.  Follow it with cuda_operator_lab_peer_barrier on
 * the same stream before reading blocks written by other ranks.  Tensor-core
 * path only: k not a multiple of 8 or unaligned x / weight return 10005; NULL
 * pointers, num_dests outside 1..8 or ld < n return cudaErrorInvalidValue;
 * m == 0 or n == 0 succeeds. */
int cuda_operator_gemm_swiglu_allgather_bf16(const void* input_bf16, const float* row_scale, const void* packed_weight_bf16, void* const* dests, int num_dests, uint64_t m, uint64_t k, uint64_t n, uint64_t ld, void* stream);

/* Row-sharded bf16 RMSNorm with its row all-gather fused in (no reference
 * counterpart; the norm of the N-sharded MLP block, whose GEMM on every rank
 * reads all normalised rows).  Normalises input[rows, cols] with weight[cols]
 * exactly as cuda_operator_rmsnorm_bf16 does (bit for bit) and stores the
 * [rows, cols] result into each of the num_dests (1..8) destinations: dests
 * (a HOST array of device addresses) holds where these rows go in this GPU's
 * buffer and in the other ranks' buffers as mapped by
 * cuda_operator_lab_peer_open.  Stores to other GPUs travel over NVLink;
 * follow the call with cuda_operator_lab_peer_barrier on the same stream
 * before another rank reads them.  cols must be a multiple of 8 and at most
 * 8192 and every pointer 16-byte aligned; otherwise, and for NULL pointers,
 * num_dests outside 1..8 or eps <= 0, cudaErrorInvalidValue; rows == 0
 * succeeds first. */
int cuda_operator_rmsnorm_allgather_bf16(const void* input_bf16, const void* weight_bf16, void* const* dests, int num_dests, uint64_t rows, uint64_t cols, float eps, void* stream);

/* Peer memory for the gathering GEMM, shared by the processes of one node
 * (one per GPU) through CUDA IPC.  peer_alloc: zero-filled device allocation
 * of `bytes` on the current device; *ptr = its address, `handle` receives
 * cuda_operator_lab_peer_handle_bytes() opaque bytes to send to the other
 * processes.  peer_open: maps such a handle from another process (address
 * usable by kernels on the current device).  peer_close undoes peer_open;
 * peer_free releases a peer_alloc allocation after every mapping of it is
 * closed.  No reference counterpart. */
uint64_t cuda_operator_lab_peer_handle_bytes(void);
int cuda_operator_lab_peer_alloc(uint64_t bytes, void** ptr, void* handle);
int cuda_operator_lab_peer_open(const void* handle, void** ptr);
int cuda_operator_lab_peer_close(void* ptr);
int cuda_operator_lab_peer_free(void* ptr);

/* Device-side barrier of `world` (1..8) ranks at `epoch`, enqueued on
 * `stream`: flag_arrays (a HOST array) holds each rank's uint32[world] flag
 * array, zero-initialised, as mapped in this process.  Each rank writes epoch
 * into its slot of every array, then waits for every slot of its own array to
 * reach epoch; epochs must increase from call to call (wrap-around safe).
 * Later work on the stream sees every store the other ranks made before their
 * barrier.  A wait longer than timeout_ns stops and sets bit 1 of the peer
 * status word (never a hang).  No reference counterpart. */
int cuda_operator_lab_peer_barrier(void* const* flag_arrays, int rank, int world, uint32_t epoch, uint64_t timeout_ns, void* stream);

/* Synchronises the current device, copies the peer status word to *status
 * (0 = no barrier wait timed out) and with clear != 0 resets it. */
int cuda_operator_lab_peer_status(unsigned int* status, int clear);

/* Partial sum for the multi-GPU reduction: partial[0] = sum(input[0..n)) in
 * fp64, with the same partition and combine order as the fp32 entry points.
 * Each rank reduces its chunk; an NCCL all-reduce of the doubles then forms
 * the global sum. */
int cuda_operator_reduction_partial_f64(const float* input, double* partial, uint64_t n, void* stream);

/* Global fp32 sum that allocates no device memory.  No counterpart in the
 * reference: it is for callers that cannot let a library allocate (a server
 * that reserved the whole device for its own allocator at start-up, a host
 * whose plugins must not allocate, a loop where an allocator call could
 * synchronise).  Same kernel and accuracy as cuda_operator_reduction_v*
 * (fp64 accumulation, fixed combine order, bit-reproducible run to run), but
 * it splits the input into fixed 16384-element chunks rather than one wave
 * of CTAs, so its result may differ from cuda_operator_reduction_v* in the
 * last bits.  Its scratch is a fixed 128 KiB array inside the library image
 * (held by every GPU that loads the library until exit).
 * Accepts n <= 268435456 (2^28); larger n returns 10004 before any launch.
 * All calls on a device share that array: calls whose GPU work overlaps
 * (unordered streams) race; calls ordered on one stream are safe.  Each call
 * clears the array's counter on its stream first.  The first call on a device
 * looks up the array's device address; make it before any stream capture. */
int cuda_operator_lab_reduction_noalloc(const float* input, float* output, uint64_t n, void* stream);

/* Number of SMs of the current device and the library's build tag; lets a
 * caller check which library it loaded.  Host-only, enqueues nothing. */
int cuda_operator_lab_device_info(int* sm_count, int* cc_major, int* cc_minor);
const char* cuda_operator_lab_build_tag(void);

/* Bounded-wait status of the tensor-core GEMM on the current device.  Every
 * mbarrier wait in that kernel gives up after a fixed time limit instead of
 * hanging; when one does, the kernel ORs a code into a device-side status
 * word and exits.  This call synchronises the current device, copies that
 * word into *status (0 = no wait ever timed out) and, when clear != 0, resets
 * it. */
int cuda_operator_lab_gemm_status(unsigned int* status, int clear);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* CUDA_OPERATOR_LAB_H_ */
