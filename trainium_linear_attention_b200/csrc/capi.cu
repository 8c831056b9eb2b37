// C ABI entry points (include/la_attention.h): argument validation, planning
// and dispatch between the tcgen05 tensor-core kernels (bf16, d_qk = 16,
// d_v = 64 on sm_100) and the SIMT kernels (fp32 and every other shape).
#include <cuda.h>
#include <math.h>
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "tc_kernels.cuh"

namespace la {

// The library's device error word (one per context that loads the library).
__device__ int la_device_error_word;

namespace {

typedef CUresult (*CtxGetCurrentFn)(CUcontext *);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long *);

void *driver_entry(const char *name) {
  void *ptr = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &ptr, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    ptr = nullptr;
  cudaGetLastError();
  return ptr;
}

}  // namespace

// Unique id (cuCtxGetId) of the context current on this thread; false if no
// context is current or the driver cannot tell.
bool current_context_id(unsigned long long *id) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    get_current = (CtxGetCurrentFn)driver_entry("cuCtxGetCurrent");
    get_id = (CtxGetIdFn)driver_entry("cuCtxGetId");
  });
  CUcontext ctx = nullptr;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx) return false;
  return get_id(ctx, id) == CUDA_SUCCESS;
}


void *context_symbol_address(const void *symbol) {
  struct Entry {
    unsigned long long ctx;
    const void *symbol;
    void *addr;
  };
  static std::mutex mu;
  static Entry cache[256];
  static int used = 0;
  unsigned long long ctx = 0;
  bool known = current_context_id(&ctx);
  if (known) {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i)
      if (cache[i].ctx == ctx && cache[i].symbol == symbol) return cache[i].addr;
  }
  // Resolve in the current context (the runtime creates the device's primary
  // context here if no context was current yet).
  void *addr = nullptr;
  if (cudaGetSymbolAddress(&addr, symbol) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (!known) known = current_context_id(&ctx);
  if (known) {
    std::lock_guard<std::mutex> lock(mu);
    if (used < 256) cache[used++] = Entry{ctx, symbol, addr};
  }
  return addr;
}

int *device_error_word() { return (int *)context_symbol_address(&la_device_error_word); }

int allow_dynamic_smem(const void *func, int bytes) {
  struct Entry {
    unsigned long long ctx;
    const void *func;
    int bytes;
  };
  static std::mutex mu;
  static Entry cache[128];
  static int used = 0;
  unsigned long long ctx = 0;
  const bool known = current_context_id(&ctx);
  if (known) {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i)
      if (cache[i].ctx == ctx && cache[i].func == func && cache[i].bytes >= bytes) return LA_OK;
  }
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess) {
    cudaGetLastError();
    return LA_ERR_CUDA;
  }
  if (known) {
    std::lock_guard<std::mutex> lock(mu);
    if (used < 128) cache[used++] = Entry{ctx, func, bytes};
  }
  return LA_OK;
}

namespace {
std::atomic<uint64_t> g_launches{0};
}  // namespace

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int current_device_info(DeviceInfo *info) {
  static std::mutex mu;
  static DeviceInfo cache[64];
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return LA_ERR_NO_DEVICE;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev].device != dev) {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, dev) != cudaSuccess) {
      cudaGetLastError();
      return LA_ERR_NO_DEVICE;
    }
    cache[dev].sm_count = p.multiProcessorCount;
    cache[dev].cc_major = p.major;
    cache[dev].cc_minor = p.minor;
    cache[dev].smem_optin = p.sharedMemPerBlockOptin;
    cache[dev].device = dev;
  }
  *info = cache[dev];
  return LA_OK;
}

namespace {

constexpr int64_t kSegmentTile = 128;     // segment boundaries are multiples of this
constexpr int64_t kMinSegmentTokens = 1024;

// The library is built for sm_100a only.
int require_sm100(DeviceInfo *info) {
  int st = current_device_info(info);
  if (st != LA_OK) return st;
  if (info->cc_major != 10) return LA_ERR_NO_DEVICE;
  return LA_OK;
}

bool valid_dtype(int dtype) { return dtype == LA_DTYPE_FLOAT32 || dtype == LA_DTYPE_BFLOAT16; }

int check_common(const void *q, const void *k, const void *v, const void *out, int64_t batch,
                 int64_t heads, int64_t n, int64_t dqk, int64_t dv, int dtype) {
  if (batch < 0 || heads < 0 || n < 0 || dqk < 1 || dv < 1) return LA_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(dtype)) return LA_ERR_INVALID_ARGUMENT;
  if (batch * heads * n == 0) return LA_OK;
  if (!q || !k || !v || !out) return LA_ERR_INVALID_ARGUMENT;
  if (batch * heads > 65535) return LA_ERR_UNSUPPORTED;
  return LA_OK;
}

int64_t segment_len(int64_t n, int segments) {
  int64_t len = (n + segments - 1) / segments;
  len = (len + kSegmentTile - 1) / kSegmentTile * kSegmentTile;
  return len < kSegmentTile ? kSegmentTile : len;
}

// Number of segments actually used (the last one may not be empty).
int effective_segments(int64_t n, int segments) {
  if (segments <= 1 || n <= 0) return 1;
  const int64_t len = segment_len(n, segments);
  return (int)((n + len - 1) / len);
}

// Segments per head for one wave of CTAs: the largest g with bh * g <= SMs
// (a second partial wave would cost more than the idle SMs of one wave), and
// at least kMinSegmentTokens tokens per segment.
int auto_segments(int64_t bh, int64_t n, int sm_count) {
  if (bh <= 0 || n <= 0) return 1;
  int64_t g = sm_count / bh;
  const int64_t max_g = (n + kMinSegmentTokens - 1) / kMinSegmentTokens;
  if (g > max_g) g = max_g;
  if (g < 1) g = 1;
  return effective_segments(n, (int)g);
}

// The same for the tensor-core chunked kernel (bf16, d_qk = 16, d_v = 64),
// which pays for segments: the state pass, the running sums and their
// launches.  Among 1 .. auto_segments(...) segments it takes the count with
// the lowest estimated time, fixed(g) + tiles per segment * per_tile(g), in
// microseconds fitted to B200 measurements (L2 flushed, one call) of 20
// shapes with 1 to 8 segments (B*H = 16..128, N = 1024..8192): unsplit 11.6 +
// 1.45 per tile; two segments 25.2 + 1.56 per tile (state pass + output);
// more 31.5 + 1.56 (plus the running-sum launch).  E.g. B=4, H=16, N=2048:
// unsplit 0.035 ms vs 0.038 with two segments; N=4096 at 32 heads: four
// segments 0.044 ms vs 0.058 unsplit.
int tc_auto_segments(int64_t bh, int64_t n, int sm_count) {
  const int g_max = auto_segments(bh, n, sm_count);
  int best = 1;
  double best_t = 0.0;
  for (int g = 1; g <= g_max; ++g) {
    const int eff = effective_segments(n, g);
    if (eff != g) continue;  // the same split as a smaller count
    const int64_t tiles = ((g > 1 ? segment_len(n, g) : n) + kSegmentTile - 1) / kSegmentTile;
    const double fixed = g == 1 ? 11.6 : g == 2 ? 25.2 : 31.5;
    const double per_tile = g == 1 ? 1.45 : 1.56;
    const double t = fixed + (double)tiles * per_tile;
    if (g == 1 || t < best_t) {
      best = g;
      best_t = t;
    }
  }
  return best;
}

// Lead/main split of the tensor-core chunked forward, for SMs / 2 < bh < SMs
// (where equal segments leave SMs - bh SMs idle): each head's main CTA covers
// [lead, n) and is seeded by a state pass over [0, lead); the bh short lead
// CTAs run in waves on the SMs - bh free SMs while the main CTAs run.  The lead
// length balances the two: (tiles - a) = waves * (a + kLeadStartTiles), in
// 128-token tiles, where kLeadStartTiles is a CTA's start-up and drain in tile
// times.  The split pays when the tiles taken off the main CTAs outweigh the
// state pass over the leads (~0.35 of a full tile each, plus its launch).
// Measured on a B200 at N = 32768: 80 and 96 heads 12% faster (two waves of
// leads), 112 heads 1% (four waves), 128 heads 4% slower (seven waves: the
// main CTAs next to SMs that keep starting lead CTAs run slower), hence at
// most kMaxLeadWaves waves.
constexpr int64_t kLeadStartTiles = 2;
constexpr int64_t kMinLeadTiles = 8;
constexpr int64_t kMaxLeadWaves = 3;

int64_t lead_tokens(int64_t bh, int64_t n, int sm_count) {
  if (bh <= 0 || 2 * bh <= sm_count || bh >= sm_count) return 0;
  const int64_t free_sms = sm_count - bh;
  const int64_t waves = (bh + free_sms - 1) / free_sms;
  if (waves > kMaxLeadWaves) return 0;
  const int64_t tiles = n / kSegmentTile;
  const int64_t a = (tiles - waves * kLeadStartTiles) / (waves + 1);
  if (a < kMinLeadTiles) return 0;
  return a * kSegmentTile;
}

bool use_tensor_cores(int dtype, int64_t dqk, int64_t dv) {
  return dtype == LA_DTYPE_BFLOAT16 && dqk == 16 && dv == 64;
}

// d_qk = 64 (F = 2145) on tensor cores: bf16, d_v = 64, the state split over a
// 16-CTA cluster (tc_cluster64.cu), where the device can hold such a cluster
bool use_tc64(int dtype, int64_t dqk, int64_t dv) {
  return dtype == LA_DTYPE_BFLOAT16 && dqk == 64 && dv == 64 && chunked64_tc_available();
}

// TMA needs 16-byte aligned inputs and the tensor-core epilogues store the
// output in 32-byte pieces; other pointers take the SIMT kernels
bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }
bool aligned32(const void *p) { return ((uintptr_t)p & 31u) == 0; }

size_t state_floats(int64_t bh, int64_t dqk, int64_t dv) {
  return (size_t)bh * (size_t)feature_dim(dqk) * (size_t)(dv + 1);
}

}  // namespace

int plan_chunked_fwd(const void *q, const void *k, const void *v, const void *out, int64_t bh,
                     int64_t n, int64_t d_qk, int64_t d_v, int dtype, int segments,
                     unsigned flags, ChunkedFwdPlan *plan) {
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != LA_OK) return st;
  ChunkedFwdPlan p;
  p.identity = (flags & LA_CHUNKED_IDENTITY) != 0;
  p.features = p.identity ? d_qk : feature_dim(d_qk);
  p.tc = use_tensor_cores(dtype, d_qk, d_v) && aligned16(q) && aligned16(k) &&
         aligned16(v) && aligned32(out);
  p.tc64 = !p.identity && use_tc64(dtype, d_qk, d_v) && aligned16(q) && aligned16(k) &&
           aligned16(v) && aligned16(out);
  if (!p.tc && !p.tc64 && !chunked_simt_supported(p.features, d_qk, d_v)) {
    if (p.identity || !cluster_chunked_supported(d_qk, d_v)) return LA_ERR_UNSUPPORTED;
    p.cluster = true;
  }
  const bool reuse = (flags & LA_CHUNKED_REUSE_SEGMENTS) != 0;
  const size_t head_state_bytes = (size_t)p.features * (size_t)(d_v + 1) * sizeof(float);
  p.lead = (segments == 0 && p.tc && !reuse && n > 0) ? lead_tokens(bh, n, info.sm_count) : 0;
  if (p.lead > 0) {
    p.g = 1;
    p.seg_len = n;
    p.scratch = ((size_t)bh * head_state_bytes + 255) / 256 * 256;
    *plan = p;
    return LA_OK;
  }
  // one wave of CTAs: a cluster run places its cluster size of CTAs on every
  // (head, segment)
  const int wave = p.cluster ? info.sm_count / cluster_chunked_ctas_per_segment() : info.sm_count;
  p.g = segments != 0 ? effective_segments(n, segments)
        : p.tc64      ? effective_segments(n, chunked64_auto_segments(bh, n, info.sm_count))
        // (by shape, not alignment: la_based_chunked_plan sizes workspaces
        // without the pointers)
        : use_tensor_cores(dtype, d_qk, d_v) ? tc_auto_segments(bh, n, info.sm_count)
                                             : auto_segments(bh, n, wave);
  p.seg_len = p.g > 1 ? segment_len(n, p.g) : n;
  // With two segments the state pass covers only the first: a long one runs
  // as two half-length pieces so that it fills as many SMs as the output
  // pass.  The two half states then need the running-sum launch; below
  // kMinSplitStateTokens per segment that launch costs more than the halving
  // saves (measured at B=4, H=16, N=2048: 0.044 ms unsplit vs 0.050 ms).
  constexpr int64_t kMinSplitStateTokens = 32 * kSegmentTile;
  p.ratio = (p.tc && p.g == 2 && !reuse && p.seg_len % (2 * kSegmentTile) == 0 &&
             p.seg_len >= kMinSplitStateTokens)
                ? 2
                : 1;
  p.scratch = p.g > 1 ? ((size_t)bh * p.g * head_state_bytes + 255) / 256 * 256 : 0;
  *plan = p;
  return LA_OK;
}
}  // namespace la

using namespace la;

extern "C" {

const char *la_status_string(int status) {
  switch (status) {
    case LA_OK: return "ok";
    case LA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case LA_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case LA_ERR_CUDA: return "CUDA error";
    case LA_ERR_WORKSPACE: return "workspace missing, too small or misaligned";
    case LA_ERR_NO_DEVICE: return "no sm_100 CUDA device is current";
    case LA_ERR_DEVICE_TIMEOUT: return "a kernel gave up on a wait that never completed";
    default: return "unknown status";
  }
}

int la_abi_version(void) { return 1; }

uint64_t la_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int la_take_device_error(void *stream) {
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != LA_OK) return st;
  if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return LA_ERR_CUDA;
  int *word = device_error_word();
  if (!word) return LA_ERR_CUDA;
  int value = 0;
  if (cudaMemcpy(&value, word, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return LA_ERR_CUDA;
  if (value != 0) {
    const int zero = 0;
    if (cudaMemcpy(word, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess)
      return LA_ERR_CUDA;
    return LA_ERR_DEVICE_TIMEOUT;
  }
  return LA_OK;
}

int64_t la_based_feature_dim(int64_t d_qk) { return d_qk < 1 ? 0 : feature_dim(d_qk); }

int la_based_parallel_fwd(const void *q, const void *k, const void *v, void *out, int64_t batch,
                          int64_t heads, int64_t seq_len, int64_t d_qk, int64_t d_v, int dtype,
                          float eps, void *stream) {
  int st = check_common(q, k, v, out, batch, heads, seq_len, d_qk, d_v, dtype);
  if (st != LA_OK || batch * heads * seq_len == 0) return st;
  DeviceInfo info;
  if ((st = require_sm100(&info)) != LA_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  if (use_tensor_cores(dtype, d_qk, d_v) && aligned16(q) &&
      aligned16(k) && aligned16(v) && aligned32(out))
    return launch_parallel_tc(q, k, v, out, batch * heads, seq_len, eps, info, s);
  return launch_parallel_simt(q, k, v, out, batch * heads, seq_len, (int)d_qk, (int)d_v, dtype,
                              eps, s);
}

int la_based_chunked_plan(int64_t batch_heads, int64_t seq_len, int64_t d_qk, int64_t d_v,
                          int dtype, int segments_requested, int *segments_out,
                          size_t *workspace_bytes_out) {
  if (batch_heads < 0 || seq_len < 0 || d_qk < 1 || d_v < 1 || segments_requested < 0 ||
      !valid_dtype(dtype))
    return LA_ERR_INVALID_ARGUMENT;
  int g = segments_requested;
  if (g == 0) {
    DeviceInfo info;
    int st = require_sm100(&info);
    if (st != LA_OK) return st;
    if (use_tensor_cores(dtype, d_qk, d_v) &&
        lead_tokens(batch_heads, seq_len, info.sm_count) > 0) {
      // the forward's lead/main split: two pieces per head.  The workspace
      // also covers two equal segments, for callers that pass segments_out
      // on explicitly (the split itself needs one state per head).
      g = 2;
    } else if (use_tc64(dtype, d_qk, d_v)) {
      g = chunked64_auto_segments(batch_heads, seq_len, info.sm_count);
    } else if (!use_tensor_cores(dtype, d_qk, d_v) &&
               !chunked_simt_supported(feature_dim(d_qk), d_qk, d_v) &&
               cluster_chunked_supported(d_qk, d_v)) {
      g = auto_segments(batch_heads, seq_len, info.sm_count / cluster_chunked_ctas_per_segment());
    } else if (use_tensor_cores(dtype, d_qk, d_v)) {
      g = tc_auto_segments(batch_heads, seq_len, info.sm_count);
    } else {
      g = auto_segments(batch_heads, seq_len, info.sm_count);
    }
  }
  g = effective_segments(seq_len, g);
  if (segments_out) *segments_out = g;
  if (workspace_bytes_out)
    *workspace_bytes_out = la_based_chunked_workspace_size(batch_heads, seq_len, d_qk, d_v, g);
  return LA_OK;
}

size_t la_based_chunked_workspace_size(int64_t batch_heads, int64_t seq_len, int64_t d_qk,
                                       int64_t d_v, int segments) {
  if (batch_heads <= 0 || d_qk < 1 || d_v < 1) return 0;
  const int g = effective_segments(seq_len, segments);
  if (g <= 1) return 0;
  size_t bytes = state_floats(batch_heads, d_qk, d_v) * (size_t)g * sizeof(float);
  return (bytes + 255) / 256 * 256;
}

int la_based_chunked_fwd(const void *q, const void *k, const void *v, void *out, int64_t batch,
                         int64_t heads, int64_t seq_len, int64_t d_qk, int64_t d_v, int dtype,
                         int64_t chunk_size, float eps, unsigned flags, const float *init_state,
                         float *final_state, void *workspace, size_t workspace_bytes,
                         int segments, void *stream) {
  int st = check_common(q, k, v, out, batch, heads, seq_len, d_qk, d_v, dtype);
  if (st != LA_OK) return st;
  if (chunk_size < 1 || segments < 0) return LA_ERR_INVALID_ARGUMENT;
  if (flags & ~(LA_CHUNKED_NORMALIZE | LA_CHUNKED_REUSE_SEGMENTS | LA_CHUNKED_IDENTITY))
    return LA_ERR_INVALID_ARGUMENT;
  // the identity feature map has no normalised form (its denominator q.z can
  // vanish); the reference defines only its numerator
  if ((flags & LA_CHUNKED_IDENTITY) && (flags & LA_CHUNKED_NORMALIZE))
    return LA_ERR_INVALID_ARGUMENT;
  const int64_t bh = batch * heads;
  if (bh == 0) return LA_OK;
  ChunkedFwdPlan plan;
  if ((st = plan_chunked_fwd(q, k, v, out, bh, seq_len, d_qk, d_v, dtype, segments, flags,
                             &plan)) != LA_OK)
    return st;
  DeviceInfo info;
  if ((st = require_sm100(&info)) != LA_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t per_head = (size_t)plan.features * (size_t)(d_v + 1);
  if (seq_len == 0) {
    // no tokens: the final state is the initial state (or zero)
    if (final_state) {
      const size_t bytes = (size_t)bh * per_head * sizeof(float);
      cudaError_t e = init_state ? cudaMemcpyAsync(final_state, init_state, bytes,
                                                   cudaMemcpyDeviceToDevice, s)
                                 : cudaMemsetAsync(final_state, 0, bytes, s);
      return cuda_status(e);
    }
    return LA_OK;
  }
  if (plan.scratch > 0 &&
      (!workspace || workspace_bytes < plan.scratch || ((uintptr_t)workspace & 255u)))
    return LA_ERR_WORKSPACE;
  const bool normalize = (flags & LA_CHUNKED_NORMALIZE) != 0;
  if (plan.lead > 0) {
    float *lead_states = (float *)workspace;
    st = launch_chunked_state_tc(k, v, lead_states, bh, seq_len, 1, 1, plan.lead, plan.identity,
                                 info, s);
    if (st != LA_OK) return st;
    return launch_chunked_output_tc(q, k, v, out, init_state, final_state, lead_states, bh,
                                    seq_len, eps, normalize, plan.identity, 1, seq_len, plan.lead,
                                    true, info, s);
  }
  const int g = plan.g;
  float *seg_states = g > 1 ? (float *)workspace : nullptr;
  if (g == 1 && (flags & LA_CHUNKED_REUSE_SEGMENTS))
    return LA_ERR_INVALID_ARGUMENT;  // nothing to reuse without segments
  if (g > 1 && !(flags & LA_CHUNKED_REUSE_SEGMENTS)) {
    // states of segments 0 .. g-2 (ratio slots each), then their prefix sums:
    // slot g - 1 seeds segment g
    st = plan.tc        ? launch_chunked_state_tc(k, v, seg_states, bh, seq_len, g,
                                                  (g - 1) * plan.ratio,
                                                  plan.seg_len / plan.ratio, plan.identity, info,
                                                  s)
         : plan.tc64    ? launch_chunked64_state_tc(k, v, seg_states, bh, seq_len, g, g - 1,
                                                    plan.seg_len, s)
         : plan.cluster ? launch_chunked_state_cluster(k, v, seg_states, bh, seq_len, (int)d_qk,
                                                       (int)d_v, dtype, g, g - 1, plan.seg_len,
                                                       s)
                        : launch_chunked_state_simt(k, v, seg_states, bh, seq_len, (int)d_qk,
                                                    (int)d_v, dtype, plan.identity, g,
                                                    plan.seg_len, s);
    if (st != LA_OK) return st;
    if ((g - 1) * plan.ratio > 1 &&
        (st = launch_prefix_segments(seg_states, nullptr, bh, g, g - 1, plan.ratio,
                                     (int64_t)per_head, s, plan.tc || plan.tc64)) != LA_OK)
      return st;
  }
  if (plan.tc64)
    return launch_chunked64_output_tc(q, k, v, out, init_state, final_state, seg_states, bh,
                                      seq_len, eps, normalize, g, plan.seg_len, s);
  const bool after_state_pass = g > 1 && !(flags & LA_CHUNKED_REUSE_SEGMENTS);
  if (plan.tc)
    return launch_chunked_output_tc(q, k, v, out, init_state, final_state, seg_states, bh,
                                    seq_len, eps, normalize, plan.identity, g, plan.seg_len, 0,
                                    after_state_pass, info, s);
  if (plan.cluster)
    return launch_chunked_output_cluster(q, k, v, out, init_state, final_state, seg_states, bh,
                                         seq_len, (int)d_qk, (int)d_v, dtype, eps, normalize, g,
                                         plan.seg_len, 0, s);
  return launch_chunked_output_simt(q, k, v, out, init_state, final_state, seg_states, bh,
                                    seq_len, (int)d_qk, (int)d_v, dtype, plan.identity, eps,
                                    normalize, g, plan.seg_len, 0, s);
}

int la_based_layer_fwd(const void *q, const void *k, const void *v, void *out, int64_t batch,
                       int64_t heads, int64_t seq_len, int64_t d_qk, int64_t d_v, int dtype,
                       int64_t window, float eps, void *workspace, size_t workspace_bytes,
                       int segments, void *stream) {
  int st = check_common(q, k, v, out, batch, heads, seq_len, d_qk, d_v, dtype);
  if (st != LA_OK) return st;
  if (window < 1 || segments < 0) return LA_ERR_INVALID_ARGUMENT;
  const int64_t bh = batch * heads;
  if (bh == 0 || seq_len == 0) return LA_OK;
  // Tensor-core shapes (bf16, d_qk = 16 or 64, d_v = 64, window <= 129): the
  // chunked kernel writes the normalised BASED term, then the sliding kernel
  // adds the window term to it in its epilogue (q, k and v are read twice; on
  // CUDA cores one pass is slower by far).
  if ((use_tensor_cores(dtype, d_qk, d_v) || use_tc64(dtype, d_qk, d_v)) &&
      sliding_tc_supported(window) && aligned16(q) && aligned16(k) && aligned16(v) &&
      aligned32(out)) {
    st = la_based_chunked_fwd(q, k, v, out, batch, heads, seq_len, d_qk, d_v, dtype, 64, eps,
                              LA_CHUNKED_NORMALIZE, nullptr, nullptr, workspace, workspace_bytes,
                              segments, stream);
    if (st != LA_OK) return st;
    DeviceInfo info;
    if ((st = require_sm100(&info)) != LA_OK) return st;
    return launch_sliding_tc(q, k, v, out, bh, seq_len, d_qk, window, out, info,
                             (cudaStream_t)stream);
  }
  // one CTA per (head, segment) holds the state and the window's two
  // previous chunks; wider states split over a cluster
  const bool simt = layer_simt_supported(d_qk, d_v, window);
  if (!simt && (window > 129 || !cluster_chunked_supported(d_qk, d_v))) return LA_ERR_UNSUPPORTED;
  DeviceInfo info;
  if ((st = require_sm100(&info)) != LA_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  const int wave = simt ? info.sm_count : info.sm_count / cluster_chunked_ctas_per_segment();
  const int g = segments == 0 ? auto_segments(bh, seq_len, wave)
                              : effective_segments(seq_len, segments);
  const int64_t seg_len = g > 1 ? segment_len(seq_len, g) : seq_len;
  const int64_t per_head = feature_dim(d_qk) * (d_v + 1);
  float *seg_states = nullptr;
  if (g > 1) {
    const size_t need = ((size_t)bh * g * per_head * sizeof(float) + 255) / 256 * 256;
    if (!workspace || workspace_bytes < need || ((uintptr_t)workspace & 255u))
      return LA_ERR_WORKSPACE;
    seg_states = (float *)workspace;
    st = simt ? launch_chunked_state_simt(k, v, seg_states, bh, seq_len, (int)d_qk, (int)d_v,
                                          dtype, false, g, seg_len, s)
              : launch_chunked_state_cluster(k, v, seg_states, bh, seq_len, (int)d_qk, (int)d_v,
                                             dtype, g, g - 1, seg_len, s);
    if (st != LA_OK) return st;
    if (g > 2 && (st = launch_prefix_segments(seg_states, nullptr, bh, g, g - 1, 1, per_head,
                                              s)) != LA_OK)
      return st;
  }
  if (!simt)
    return launch_chunked_output_cluster(q, k, v, out, nullptr, nullptr, seg_states, bh, seq_len,
                                         (int)d_qk, (int)d_v, dtype, eps, true, g, seg_len,
                                         window, s);
  return launch_chunked_output_simt(q, k, v, out, nullptr, nullptr, seg_states, bh, seq_len,
                                    (int)d_qk, (int)d_v, dtype, false, eps, true, g, seg_len,
                                    window, s);
}

int la_based_chunked_state(const void *k, const void *v, float *state_out, int64_t batch,
                           int64_t heads, int64_t seq_len, int64_t d_qk, int64_t d_v, int dtype,
                           void *workspace, size_t workspace_bytes, int segments, void *stream) {
  if (batch < 0 || heads < 0 || seq_len < 0 || d_qk < 1 || d_v < 1 || segments < 0 ||
      !valid_dtype(dtype))
    return LA_ERR_INVALID_ARGUMENT;
  const int64_t bh = batch * heads;
  if (bh == 0) return LA_OK;
  if (!state_out || (seq_len > 0 && (!k || !v))) return LA_ERR_INVALID_ARGUMENT;
  if (bh > 65535) return LA_ERR_UNSUPPORTED;
  DeviceInfo info;
  int st = require_sm100(&info);
  if (st != LA_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t state_bytes = state_floats(bh, d_qk, d_v) * sizeof(float);
  if (seq_len == 0) return cuda_status(cudaMemsetAsync(state_out, 0, state_bytes, s));
  const bool tc = use_tensor_cores(dtype, d_qk, d_v) && aligned16(k) &&
                  aligned16(v);
  const bool tc64 = use_tc64(dtype, d_qk, d_v) && aligned16(k) && aligned16(v);
  const bool cluster = !tc && !tc64 && !chunked_simt_supported(feature_dim(d_qk), d_qk, d_v);
  if (cluster && !cluster_chunked_supported(d_qk, d_v)) return LA_ERR_UNSUPPORTED;
  // the same segmentation as la_based_chunked_fwd, so that a forward with
  // LA_CHUNKED_REUSE_SEGMENTS finds the seeds it expects
  const int wave = cluster ? info.sm_count / cluster_chunked_ctas_per_segment() : info.sm_count;
  int g = segments != 0 ? effective_segments(seq_len, segments)
          : tc64        ? effective_segments(seq_len,
                                             chunked64_auto_segments(bh, seq_len, info.sm_count))
          : use_tensor_cores(dtype, d_qk, d_v) ? tc_auto_segments(bh, seq_len, info.sm_count)
                                               : auto_segments(bh, seq_len, wave);
  if (g > 1) {
    const size_t need = la_based_chunked_workspace_size(bh, seq_len, d_qk, d_v, g);
    if (!workspace || workspace_bytes < need || ((uintptr_t)workspace & 255u))
      return LA_ERR_WORKSPACE;
  }
  const int64_t seg_len = g > 1 ? segment_len(seq_len, g) : seq_len;
  float *dst = g > 1 ? (float *)workspace : state_out;
  st = tc        ? launch_chunked_state_tc(k, v, dst, bh, seq_len, g, g, seg_len, false, info, s)
       : tc64    ? launch_chunked64_state_tc(k, v, dst, bh, seq_len, g, g, seg_len, s)
       : cluster ? launch_chunked_state_cluster(k, v, dst, bh, seq_len, (int)d_qk, (int)d_v,
                                                dtype, g, g, seg_len, s)
                 : launch_chunked_state_simt(k, v, dst, bh, seq_len, (int)d_qk, (int)d_v, dtype,
                                             false, g, seg_len, s);
  if (st != LA_OK || g == 1) return st;
  // the total, and in the workspace the prefix slots a forward with
  // LA_CHUNKED_REUSE_SEGMENTS seeds its segments from
  return launch_prefix_segments(dst, state_out, bh, g, g, 1,
                                (int64_t)feature_dim(d_qk) * (d_v + 1), s, tc || tc64);
}

int la_sliding_window_fwd(const void *q, const void *k, const void *v, void *out, int64_t batch,
                          int64_t heads, int64_t seq_len, int64_t head_dim, int dtype,
                          int64_t window, void *stream) {
  int st = check_common(q, k, v, out, batch, heads, seq_len, head_dim, head_dim, dtype);
  if (st != LA_OK) return st;
  if (window < 1) return LA_ERR_INVALID_ARGUMENT;
  if (batch * heads * seq_len == 0) return LA_OK;
  DeviceInfo info;
  if ((st = require_sm100(&info)) != LA_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == LA_DTYPE_BFLOAT16 && head_dim == 64 &&
      sliding_tc_supported(window) && aligned16(q) && aligned16(k) && aligned16(v) &&
      aligned32(out))
    return launch_sliding_tc(q, k, v, out, batch * heads, seq_len, head_dim, window, nullptr,
                             info, s);
  return launch_sliding_simt(q, k, v, out, batch * heads, seq_len, (int)head_dim, dtype, window,
                             s);
}

}  // extern "C"
