// Launchers of the tcgen05 / TMEM / TMA tensor-core kernels (sm_100a).
//
// Fast-path shapes: bf16 inputs, d_qk = 16 and d_v = 64 for BASED (Taylor or
// identity feature map), head_dim = 64 for the sliding window.  Every other
// request goes to the SIMT or cluster kernels.
#pragma once

#include "common.cuh"

namespace la {

// Device address of the library's error word in the current context (set by a
// kernel whose bounded wait timed out); null if it cannot be resolved.
int *device_error_word();

int launch_parallel_tc(const void *q, const void *k, const void *v, void *out, int64_t bh,
                       int64_t n, float eps, const DeviceInfo &info, cudaStream_t s);

// State pass over segments [0, n_launch) of every head (n_launch <= segments).
// States of the n_launch leading pieces of length seg_len of every head into
// seg_states[bh][0 .. n_launch) (per-head stride `segments` entries), each
// (F, 65) with F = 153 (Taylor) or 16 (identity feature map).
int launch_chunked_state_tc(const void *k, const void *v, float *seg_states, int64_t bh,
                            int64_t n, int segments, int n_launch, int64_t seg_len, bool identity,
                            const DeviceInfo &info, cudaStream_t s);

// Output of `segments` segments of length seg_len; segment g > 0 is seeded
// with init_state + seg_states[bh][g - 1] (the prefix slots written by
// launch_prefix_segments; per-head stride `segments`).  lead_len > 0 selects
// the lead/main split instead: per head a main CTA over [lead_len, n) seeded
// with init_state + seg_states[bh] (segments = 1) and a lead CTA over
// [0, lead_len); all main CTAs are dispatched before the leads.  identity:
// the identity feature map's numerator (normalize must be false).
int launch_chunked_output_tc(const void *q, const void *k, const void *v, void *out,
                             const float *init_state, float *final_state,
                             const float *seg_states, int64_t bh, int64_t n, float eps,
                             bool normalize, bool identity, int segments, int64_t seg_len,
                             int64_t lead_len, bool after_own_kernel, const DeviceInfo &info,
                             cudaStream_t s);

// d_qk = 64, d_v = 64 (F = 2145): chunked forward with the state split over a
// 16-CTA cluster (tc_cluster64.cu).  Available where the device can hold one
// such cluster (the non-portable cluster size is enabled on first use).
// Segment, seed and state conventions as launch_chunked_{state,output}_tc;
// out needs 16-byte alignment.
bool chunked64_tc_available();
int chunked64_tc_ctas_per_segment();
// Segments per head for a default (segments = 0) run: the estimated fastest
// split given how many 16-CTA clusters the device holds at once.
int chunked64_auto_segments(int64_t bh, int64_t n, int sm_count);
int launch_chunked64_state_tc(const void *k, const void *v, float *seg_states, int64_t bh,
                              int64_t n, int segments, int n_launch, int64_t seg_len,
                              cudaStream_t s);
int launch_chunked64_output_tc(const void *q, const void *k, const void *v, void *out,
                               const float *init_state, float *final_state,
                               const float *seg_states, int64_t bh, int64_t n, float eps,
                               bool normalize, int segments, int64_t seg_len, cudaStream_t s);

// Windows the tensor-core sliding kernel handles (W <= 129).  It takes d_qk
// 64 or 16 with d_v 64; addend (null, or (bh, n, 64) bf16, may be out) is
// added to the output in fp32 before its rounding to bf16.
bool sliding_tc_supported(int64_t window);
int launch_sliding_tc(const void *q, const void *k, const void *v, void *out, int64_t bh,
                      int64_t n, int64_t d_qk, int64_t window, const void *addend,
                      const DeviceInfo &info, cudaStream_t s);

// In place, per head (seg[bh][0 .. stride) holding states): slot gr becomes
// the sum of slots [0, (gr + 1) * ratio) for gr < groups, i.e. the seed of
// segment gr + 1 when each segment's state occupies `ratio` slots; total (if
// not null) receives the sum of all groups * ratio slots.  Fixed order,
// deterministic.
int launch_prefix_segments(float *seg, float *total, int64_t bh, int stride, int groups,
                           int ratio, int64_t per_head, cudaStream_t s, bool pdl = false);

}  // namespace la
