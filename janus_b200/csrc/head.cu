// Readout heads fused with the decoder's final RMSNorm: a gather of the readout rows of the fp32 residual stream,
// RMSNorm (1 + w), LayerNorm, and the Scalar / Pointer projections, all fp32. HBM/latency-bound: the gathered rows
// are (options + decisions) * hidden * 4 bytes and the head weights are read once per CTA from L2.
#include <mutex>

#include "common.cuh"

namespace jb {

constexpr int kHeadThreads = 256;
constexpr int kHeadMaxH = 8192;
constexpr int kHeadMaxRank = 4096;            // projection rank bound (the released heads use 128)
constexpr int64_t kHeadMaxRows = 1 << 24;     // options + decision rows per call (grid size, int arithmetic)

// Final RMSNorm then LayerNorm of one row into shared memory `ln` (H floats); returns nothing, ln filled. A null
// final_w skips the RMSNorm (rows that are already the decoder's final-normed output).
__device__ void norm_row(const float* __restrict__ xr, int H, const __nv_bfloat16* __restrict__ final_w, float rms_eps,
                         const float* __restrict__ ln_w, const float* __restrict__ ln_b, float ln_eps, float* ln,
                         float* red) {
  float s = 0.f;
  if (final_w) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      const float v = xr[i];
      ln[i] = v;
      ss += v * v;
    }
    ss = block_sum(ss, red);
    const float r = rsqrtf(ss / (float)H + rms_eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      const float h = ln[i] * r * (1.f + bf2f(final_w[i]));
      ln[i] = h;
      s += h;
    }
  } else {
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      const float v = xr[i];
      ln[i] = v;
      s += v;
    }
  }
  __syncthreads();
  s = block_sum(s, red);
  const float mean = s / (float)H;
  float var = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float d = ln[i] - mean;
    var += d * d;
  }
  __syncthreads();
  var = block_sum(var, red);
  const float inv = rsqrtf(var / (float)H + ln_eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x) ln[i] = (ln[i] - mean) * inv * ln_w[i] + ln_b[i];
  __syncthreads();
}

__global__ void __launch_bounds__(kHeadThreads) head_scalar_kernel(const float* __restrict__ x, int H,
                                                                   const int32_t* __restrict__ rows,
                                                                   const __nv_bfloat16* __restrict__ final_w,
                                                                   float rms_eps, const float* __restrict__ ln_w,
                                                                   const float* __restrict__ ln_b, float ln_eps,
                                                                   const float* __restrict__ w_out,
                                                                   const float* __restrict__ b_out,
                                                                   float* __restrict__ logits) {
  extern __shared__ float ln[];
  __shared__ float red[32];
  const int i = blockIdx.x;
  norm_row(x + (int64_t)rows[i] * H, H, final_w, rms_eps, ln_w, ln_b, ln_eps, ln, red);
  float d = 0.f;
  for (int j = threadIdx.x; j < H; j += blockDim.x) d += ln[j] * w_out[j];
  d = block_sum(d, red);
  if (threadIdx.x == 0) logits[i] = d + b_out[0];
}

// Row i < n: option row (projected by wk); row n + q: the decision row of question q (projected by wq).
__global__ void __launch_bounds__(kHeadThreads) head_project_kernel(
    const float* __restrict__ x, int H, const int32_t* __restrict__ option_rows, int n,
    const int32_t* __restrict__ decision_rows, const __nv_bfloat16* __restrict__ final_w, float rms_eps,
    const float* __restrict__ ln_w, const float* __restrict__ ln_b, float ln_eps, const float* __restrict__ wq,
    const float* __restrict__ wk, int R, float* __restrict__ proj) {
  extern __shared__ float ln[];
  __shared__ float red[32];
  const int i = blockIdx.x;
  const int row = i < n ? option_rows[i] : decision_rows[i - n];
  const float* W = i < n ? wk : wq;
  norm_row(x + (int64_t)row * H, H, final_w, rms_eps, ln_w, ln_b, ln_eps, ln, red);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int j = warp; j < R; j += nw) {
    const float* wr = W + (int64_t)j * H;
    float d = 0.f;
    for (int c = lane; c < H; c += 32) d += ln[c] * wr[c];
    d = warp_sum(d);
    if (lane == 0) proj[(int64_t)i * R + j] = d;
  }
}

// An option whose question index lies outside [0, Q) reads nothing and gets a NaN logit (the caller's contract is
// 0 <= option_question[i] < Q; a NaN makes a broken table visible instead of reading past the projected rows).
__global__ void head_dot_kernel(const float* __restrict__ proj, int n, const int32_t* __restrict__ option_question,
                                int Q, int R, float inv_scale, float* __restrict__ logits) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= n) return;
  const int qi = option_question[w];
  if (qi < 0 || qi >= Q) {
    if (lane == 0) logits[w] = __int_as_float(0x7fc00000);
    return;
  }
  const float* a = proj + (int64_t)w * R;
  const float* b = proj + (int64_t)(n + qi) * R;
  float d = 0.f;
  for (int j = lane; j < R; j += 32) d += a[j] * b[j];
  d = warp_sum(d);
  if (lane == 0) logits[w] = d * inv_scale;
}

}  // namespace jb

using namespace jb;

extern "C" int janus_b200_head_scalar(const float* x, int64_t H, const int32_t* rows, int64_t n, const void* final_w,
                                      float rms_eps, const float* ln_w, const float* ln_b, float ln_eps,
                                      const float* w_out, const float* b_out, float* logits, void* stream) {
  JB_REQUIRE(x && rows && ln_w && ln_b && w_out && b_out && logits, JANUS_ERR_INVALID,
             "head_scalar: null pointer");
  JB_REQUIRE(H > 0 && H <= kHeadMaxH && n >= 0, JANUS_ERR_INVALID, "head_scalar: hidden %lld out of range", (long long)H);
  if (n == 0) return JANUS_OK;
  head_scalar_kernel<<<(unsigned)n, kHeadThreads, H * sizeof(float), (cudaStream_t)stream>>>(
      x, (int)H, rows, (const __nv_bfloat16*)final_w, rms_eps, ln_w, ln_b, ln_eps, w_out, b_out, logits);
  return launch_status("head_scalar");
}

extern "C" int janus_b200_head_pointer(const float* x, int64_t H, const int32_t* option_rows,
                                       const int32_t* option_question, int64_t n, const int32_t* decision_rows,
                                       int64_t Q, const void* final_w, float rms_eps, const float* ln_w,
                                       const float* ln_b, float ln_eps, const float* wq, const float* wk, int64_t R,
                                       float* workspace, size_t workspace_bytes, float* logits, void* stream) {
  JB_REQUIRE(x && option_rows && option_question && decision_rows && ln_w && ln_b && wq && wk && logits,
             JANUS_ERR_INVALID, "head_pointer: null pointer");
  JB_REQUIRE(H > 0 && H <= kHeadMaxH && n >= 0 && Q >= 0 && R > 0 && R <= kHeadMaxRank, JANUS_ERR_INVALID,
             "head_pointer: sizes (H %lld, options %lld, questions %lld, rank %lld <= %d)", (long long)H, (long long)n,
             (long long)Q, (long long)R, kHeadMaxRank);
  JB_REQUIRE(n == 0 || Q > 0, JANUS_ERR_INVALID, "head_pointer: %lld options but no question", (long long)n);
  JB_REQUIRE(n + Q <= kHeadMaxRows, JANUS_ERR_INVALID, "head_pointer: options + questions %lld > %lld",
             (long long)(n + Q), (long long)kHeadMaxRows);
  JB_REQUIRE(workspace && workspace_bytes >= (size_t)(n + Q) * R * sizeof(float), JANUS_ERR_WORKSPACE,
             "head_pointer: workspace %zu bytes < %lld", workspace_bytes, (long long)((n + Q) * R * 4));
  if (n == 0) return JANUS_OK;
  cudaStream_t s = (cudaStream_t)stream;
  head_project_kernel<<<(unsigned)(n + Q), kHeadThreads, H * sizeof(float), s>>>(
      x, (int)H, option_rows, (int)n, decision_rows, (const __nv_bfloat16*)final_w, rms_eps, ln_w, ln_b, ln_eps, wq,
      wk, (int)R, workspace);
  int st = launch_status("head_pointer/project");
  if (st) return st;
  const int th = 256;
  head_dot_kernel<<<(unsigned)((n * 32 + th - 1) / th), th, 0, s>>>(workspace, (int)n, option_question, (int)Q,
                                                                   (int)R, 1.f / sqrtf((float)R), logits);
  return launch_status("head_pointer/dot");
}

// ------------------------------------------------------------------------------------------------------------------
// PointerHead without a caller workspace. The projected rows live in a static device array of this library
// (kPointerScratchFloats fp32 = 1 MiB, held by every GPU that loads the library until the process exits). Host code
// cannot pass the array's name to a kernel (on the host it names a stand-in, not device memory), so the device address
// is looked up once per device with cudaGetSymbolAddress, with that device current, on the first call there; that
// first call on a device should come before any stream capture. Every call on a device shares the array: calls that
// overlap on the GPU (other streams, or other threads) race on it and must be serialised by the caller. The
// projection kernel writes every element it later reads, so nothing needs clearing between calls.

namespace jb {

constexpr size_t kPointerScratchFloats = size_t(1) << 18;
constexpr int kMaxDevices = 64;
static __device__ __align__(256) float g_pointer_scratch[kPointerScratchFloats];
static float* g_pointer_scratch_addr[kMaxDevices] = {};
static std::mutex g_pointer_scratch_mutex;

static int pointer_scratch(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("head_pointer_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return JANUS_ERR_CUDA;
  }
  JB_REQUIRE(dev >= 0 && dev < kMaxDevices, JANUS_ERR_UNSUPPORTED, "head_pointer_noalloc: device %d >= %d", dev,
             kMaxDevices);
  std::lock_guard<std::mutex> lock(g_pointer_scratch_mutex);
  if (!g_pointer_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_pointer_scratch);
    if (e != cudaSuccess || !p) {
      set_error("head_pointer_noalloc: cudaGetSymbolAddress on device %d: %s", dev, cudaGetErrorString(e));
      return JANUS_ERR_CUDA;
    }
    g_pointer_scratch_addr[dev] = static_cast<float*>(p);
  }
  *out = g_pointer_scratch_addr[dev];
  return JANUS_OK;
}

}  // namespace jb

extern "C" int janus_b200_head_pointer_noalloc(const float* x, int64_t H, const int32_t* option_rows,
                                               const int32_t* option_question, int64_t n,
                                               const int32_t* decision_rows, int64_t Q, const void* final_w,
                                               float rms_eps, const float* ln_w, const float* ln_b, float ln_eps,
                                               const float* wq, const float* wk, int64_t R, float* logits,
                                               void* stream) {
  JB_REQUIRE(x && option_rows && option_question && decision_rows && ln_w && ln_b && wq && wk && logits,
             JANUS_ERR_INVALID, "head_pointer_noalloc: null pointer");
  JB_REQUIRE(H > 0 && H <= kHeadMaxH && n >= 0 && Q >= 0 && R > 0 && R <= kHeadMaxRank, JANUS_ERR_INVALID,
             "head_pointer_noalloc: sizes (H %lld, options %lld, questions %lld, rank %lld <= %d)", (long long)H,
             (long long)n, (long long)Q, (long long)R, kHeadMaxRank);
  JB_REQUIRE(n == 0 || Q > 0, JANUS_ERR_INVALID, "head_pointer_noalloc: %lld options but no question", (long long)n);
  JB_REQUIRE(n + Q <= kHeadMaxRows, JANUS_ERR_INVALID, "head_pointer_noalloc: options + questions %lld > %lld",
             (long long)(n + Q), (long long)kHeadMaxRows);
  JB_REQUIRE((size_t)(n + Q) * (size_t)R <= kPointerScratchFloats, JANUS_ERR_WORKSPACE,
             "head_pointer_noalloc: (options %lld + decisions %lld) x rank %lld = %lld floats exceed the static "
             "scratch of %zu floats; split the call or use janus_b200_head_pointer with a workspace",
             (long long)n, (long long)Q, (long long)R, (long long)((n + Q) * R), kPointerScratchFloats);
  if (n == 0) return JANUS_OK;
  float* scratch = nullptr;
  int st = pointer_scratch(&scratch);
  if (st) return st;
  cudaStream_t s = (cudaStream_t)stream;
  head_project_kernel<<<(unsigned)(n + Q), kHeadThreads, H * sizeof(float), s>>>(
      x, (int)H, option_rows, (int)n, decision_rows, (const __nv_bfloat16*)final_w, rms_eps, ln_w, ln_b, ln_eps, wq,
      wk, (int)R, scratch);
  st = launch_status("head_pointer_noalloc/project");
  if (st) return st;
  const int th = 256;
  head_dot_kernel<<<(unsigned)((n * 32 + th - 1) / th), th, 0, s>>>(scratch, (int)n, option_question, (int)Q,
                                                                   (int)R, 1.f / sqrtf((float)R), logits);
  return launch_status("head_pointer_noalloc/dot");
}
