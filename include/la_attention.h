/*
 * la_attention.h -- C ABI of the B200 (sm_100a) BASED / sliding-window
 * attention library (libla_attention.so).
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * passed as void*, enqueues its kernels on that stream and returns an int
 * status (LA_OK == 0).  No entry point synchronises the stream (except
 * la_take_device_error, which says so) or allocates device memory.  All
 * except la_based_chunked_fwd_noalloc keep no state between calls and are
 * safe to call from several host threads at once; that one shares a scratch
 * array compiled into the library between all its calls on a device (see
 * its comment).
 *
 * Tensor layout: every q/k/v/out is a contiguous (batch, heads, seq_len, d)
 * row-major array in the element type given by `dtype`.  q and k have width
 * d_qk, v and out have width d_v (d_v may differ from d_qk).  Inputs are never
 * written.
 *
 * Semantics (identical to the reference's PyTorch functions):
 *   s = (q . k) / sqrt(d_qk), causal mask includes the diagonal,
 *   BASED:   out_i = sum_{j<=i} (1 + s_ij + s_ij^2/2) v_j
 *                    / (sum_{j<=i} (1 + s_ij + s_ij^2/2) + eps)
 *   sliding: out_i = softmax_{i-W+1 <= j <= i}(s_ij) . v_j
 */
#ifndef LA_ATTENTION_H
#define LA_ATTENTION_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------------
 * The reference's dispatcher swallows every failure and silently falls back
 * to PyTorch (kernels/pytorch_attention.py:87-92).  This library never falls
 * back: every failure is reported to the caller.                            */
#define LA_OK                    0
#define LA_ERR_INVALID_ARGUMENT  1  /* null pointer, negative size, bad dtype ... */
#define LA_ERR_UNSUPPORTED       2  /* valid request this build has no kernel for  */
#define LA_ERR_CUDA              3  /* a CUDA runtime / launch error               */
#define LA_ERR_WORKSPACE         4  /* workspace missing, too small or misaligned  */
#define LA_ERR_NO_DEVICE         5  /* no sm_100 device is current                 */
#define LA_ERR_DEVICE_TIMEOUT    6  /* a kernel abandoned a wait that never ended  */

/* ---- element types --------------------------------------------------------*/
#define LA_DTYPE_FLOAT32   0
#define LA_DTYPE_BFLOAT16  1

/* ---- flags for the chunked entry points ------------------------------------*/
#define LA_CHUNKED_NORMALIZE        1u  /* divide by the normaliser (+eps)        */
#define LA_CHUNKED_REUSE_SEGMENTS   2u  /* workspace already holds the segment
                                           seeds written by la_based_chunked_state */
#define LA_CHUNKED_IDENTITY         4u  /* identity feature map phi(x) = x instead
                                           of the Taylor map: the reference's
                                           ref_identity_numerator (benchmarks/
                                           chunked_attention_benchmark.py:81-93);
                                           numerator only (not with NORMALIZE)   */

/* Human-readable name of a status code (static storage, never NULL). */
const char *la_status_string(int status);

/* ABI version of this header (bumped on any incompatible change). */
int la_abi_version(void);

/* Every wait inside the tensor-core kernels is bounded (2 s); a kernel that
 * gives up records it in a per-device error word and exits cleanly, leaving
 * the CUDA context usable.  This call synchronises `stream`, then returns
 * LA_ERR_DEVICE_TIMEOUT (and clears the word) if any kernel of this library
 * on the current device has given up since the last call, else LA_OK.
 * The reference has no counterpart (its dispatcher hides all failures). */
int la_take_device_error(void *stream);

/* Number of kernels this library has launched in this process (all devices,
 * all threads), for callers that account for launches; diagnostics only. */
uint64_t la_launch_count(void);

/* Width F of the Taylor feature basis for key width d_qk: 1 + d + d(d+1)/2
 * (153 at d_qk = 16).  Replaces the width computed by the reference's
 * taylor_feature_map (benchmarks/chunked_attention_benchmark.py:34-53). */
int64_t la_based_feature_dim(int64_t d_qk);

/* ---------------------------------------------------------------------------
 * Parallel (quadratic) fused BASED attention.
 *
 * Replaces solution_nki (kernels/pytorch_attention.py:44-78) together with the
 * kernel it builds, get_based_attn_kernel / _kernel (kernels/nki_attention.py:
 * 25-115): one call computes the normalised output; no padding copies and no
 * host-side num/den division.  bf16 inputs with d_qk = 16, d_v = 64 (and
 * q/k/v 16-byte, out 32-byte aligned) use the tcgen05 tensor-core kernel;
 * everything else computes in fp32 on CUDA cores.
 * ------------------------------------------------------------------------- */
int la_based_parallel_fwd(const void *q, const void *k, const void *v, void *out,
                          int64_t batch, int64_t heads, int64_t seq_len,
                          int64_t d_qk, int64_t d_v, int dtype, float eps,
                          void *stream);

/* ---------------------------------------------------------------------------
 * Chunked recurrent BASED attention.
 *
 * Replaces chunked_nki_numerator (benchmarks/chunked_attention_benchmark.py:
 * 96-126) and the kernel of get_chunked_attn_kernel (kernels/
 * nki_attention_chunked.py:20-113).  Unlike the reference, the Taylor features
 * are never materialised in HBM, the recurrent state lives on chip, and with
 * LA_CHUNKED_NORMALIZE the normaliser is carried too (the reference returns
 * the numerator only).
 *
 * With LA_CHUNKED_IDENTITY the feature map is the identity (the reference's
 * ref_identity_numerator): phi_k(k) = k, phi_q(q) = q / sqrt(d_qk), F = d_qk,
 * and only the numerator is returned (NORMALIZE is rejected).  Either map
 * runs on the tcgen05 tensor-core kernel for bf16 inputs with d_qk = 16,
 * d_v = 64 (q/k/v 16-byte, out 32-byte aligned); other shapes compute in
 * fp32 on CUDA cores (d_qk = 64 on a thread-block cluster).
 *
 * State layout (init_state / final_state / la_based_chunked_state): fp32
 * (batch*heads, F, d_v + 1) in the key-side feature basis
 *     phi_k(k) = [1, k_0 .. k_{d-1}, k_i * k_j for i <= j in row-major order]
 * i.e. state[f][e] = sum_j phi_k(k_j)[f] * v_j[e] and state[f][d_v] =
 * sum_j phi_k(k_j)[f].  The query side carries the scale factors
 * (phi_q(q) = [1, q_i/sqrt(d), q_i q_j w_ij], w_ii = 1/(2d), w_ij = 1/d), so
 * phi_q(q) . phi_k(k) = 1 + s + s^2/2 exactly as the reference's feature map.
 *
 * segments: the sequence of each head is split into this many contiguous
 * segments processed by different CTAs (0 = let the library choose).  A
 * segmented run needs a workspace of la_based_chunked_workspace_size() bytes
 * (256-byte aligned); an unsegmented run needs none (workspace may be NULL).
 * With segments = 0 the library may also split each head unequally, into a
 * short lead and a long main piece, when between half and all of the SMs
 * hold one head each (the leads run on the SMs the heads leave free); it
 * needs one state per head of workspace.  la_based_chunked_plan with
 * segments_requested = 0 reports the segment count the library picks (2 for
 * that split) and a workspace that covers it and that many equal segments.
 * chunk_size: the reference's chunk length.  The result does not depend on it
 * beyond floating-point rounding (any positive value is accepted); the
 * kernels tile the sequence at their own fixed length.
 * ------------------------------------------------------------------------- */
int la_based_chunked_plan(int64_t batch_heads, int64_t seq_len, int64_t d_qk,
                          int64_t d_v, int dtype, int segments_requested,
                          int *segments_out, size_t *workspace_bytes_out);

size_t la_based_chunked_workspace_size(int64_t batch_heads, int64_t seq_len,
                                       int64_t d_qk, int64_t d_v, int segments);

int la_based_chunked_fwd(const void *q, const void *k, const void *v, void *out,
                         int64_t batch, int64_t heads, int64_t seq_len,
                         int64_t d_qk, int64_t d_v, int dtype,
                         int64_t chunk_size, float eps, unsigned flags,
                         const float *init_state, float *final_state,
                         void *workspace, size_t workspace_bytes, int segments,
                         void *stream);

/* The chunked forward for callers that cannot allocate device memory (a
 * plugin whose host framework owns all device memory and gives it no
 * allocation hook, or a latency-critical path that must not call cudaMalloc).
 * Same arguments and results as la_based_chunked_fwd without the workspace:
 * the segment scratch comes from an 8 MiB array compiled into the library
 * (held on every device that loads it until exit), enough for 210 (head,
 * segment) states at d_qk = 16, d_v = 64.  Allocates nothing.  A request
 * needing more scratch returns LA_ERR_WORKSPACE; LA_CHUNKED_REUSE_SEGMENTS is
 * rejected (LA_ERR_INVALID_ARGUMENT).  All calls on a device share the array
 * and leave its contents behind: calls whose kernels overlap on the GPU race
 * on it.  The array's address belongs to the CUDA context: the first call in
 * each context resolves it (and caches it for that context); make that call
 * before any stream capture.  The reference has no counterpart. */
int la_based_chunked_fwd_noalloc(const void *q, const void *k, const void *v, void *out,
                                 int64_t batch, int64_t heads, int64_t seq_len,
                                 int64_t d_qk, int64_t d_v, int dtype,
                                 int64_t chunk_size, float eps, unsigned flags,
                                 const float *init_state, float *final_state,
                                 int segments, void *stream);

/* Total state sum_j phi_k(k_j) [v_j, 1]^T of every head over all seq_len
 * tokens, written to state_out (fp32, (batch*heads, F, d_v + 1)).  This is the
 * per-rank contribution exchanged by the sequence-parallel mode.  With a
 * workspace and segments > 1 the running sums of the per-segment states (the
 * seed of each later segment) are left in the workspace so that a following
 * la_based_chunked_fwd with LA_CHUNKED_REUSE_SEGMENTS (same shapes and
 * segments) skips its own state pass.  The reference has no
 * counterpart (it has no multi-device mode). */
int la_based_chunked_state(const void *k, const void *v, float *state_out,
                           int64_t batch, int64_t heads, int64_t seq_len,
                           int64_t d_qk, int64_t d_v, int dtype,
                           void *workspace, size_t workspace_bytes, int segments,
                           void *stream);

/* ---------------------------------------------------------------------------
 * The full BASED layer: causal BASED linear attention plus sliding-window
 * softmax attention over the same q, k, v,
 *     out = based(q, k, v, eps) + sliding_window(q, k, v, window),
 * the composition the reference states at kernels/nki_attention_sliding.py:
 * 4-5 (and whose two halves its module wrapper benchmarks/
 * based_attention_benchmark.py:24-69 would call separately).  bf16 inputs
 * with d_qk = 16, d_v = 64 and window <= 129 (aligned as for the chunked
 * tensor-core path) run two tensor-core kernels: the chunked kernel writes
 * the normalised BASED term to out, then the sliding-window kernel adds its
 * term in fp32 before the one rounding to bf16 (q, k and v are read twice).
 * Other shapes run in one pass over q, k and v on CUDA cores: each chunk's
 * keys and values serve the chunked recurrence and, kept on chip, the
 * windows of the next two chunks (window <= 129); states too wide for one CTA
 * (d_qk = 64) are split over a thread-block cluster as in
 * la_based_chunked_fwd.  The sliding half uses the
 * same scale 1/sqrt(d_qk), the window [i - W + 1, i] and fp32 softmax
 * accumulation.  segments and the
 * workspace work as for la_based_chunked_fwd (la_based_chunked_plan sizes
 * it); the window of a segment's first tokens reads the keys before it.
 * The reference has no kernel for the fused layer.
 * ------------------------------------------------------------------------- */
int la_based_layer_fwd(const void *q, const void *k, const void *v, void *out,
                       int64_t batch, int64_t heads, int64_t seq_len,
                       int64_t d_qk, int64_t d_v, int dtype, int64_t window,
                       float eps, void *workspace, size_t workspace_bytes,
                       int segments, void *stream);

/* ---------------------------------------------------------------------------
 * Sliding-window causal softmax attention, window [i-W+1, i].
 *
 * Replaces nki_sliding_window_attn (benchmarks/sliding_attention_benchmark.py:
 * 59-99) and get_sliding_window_kernel / _kernel (kernels/
 * nki_attention_sliding.py:30-132).  The mask is computed from indices (never
 * loaded), no padding copies are made, and any window >= 1 is accepted (the
 * reference asserts W <= 66 at block 64).  fp32 softmax accumulation.
 * ------------------------------------------------------------------------- */
int la_sliding_window_fwd(const void *q, const void *k, const void *v, void *out,
                          int64_t batch, int64_t heads, int64_t seq_len,
                          int64_t head_dim, int dtype, int64_t window,
                          void *stream);

#ifdef __cplusplus
}
#endif

#endif /* LA_ATTENTION_H */
