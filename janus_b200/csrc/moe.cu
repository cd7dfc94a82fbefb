// Sparse MoE feed-forward with W4A16 experts (int4 codes, one bf16 scale per 128 inputs): routing plan, permuted
// grouped GEMMs and the weighted combine.
//
// moe_route: softmax over the router logits (fp32), top-k, renormalise (Qwen3_5MoeTopKRouter), then a sync-free tile
// plan: per-expert counts (atomics), a one-CTA scan padding every expert to the tile height, and the scatter of the
// assignments (token * k + slot) into expert-sorted order. The tile count stays on the device; the GEMMs are
// launched for the worst case (every expert padded) and tiles past the count exit at once — the plan of
// janus/moe_w4a16.py:89-106, computed by three small kernels instead of argsort/bincount/searchsorted.
//
// The grouped GEMMs between the plan and the combine are in moe_tc.cu (tcgen05, int4 decoded on the fly). The first
// stores silu(gate) * up per sorted row; the second multiplies by the routing weight and stores per assignment.
// moe_combine sums the k assignments of a token in fp32 and adds the gated shared expert; moe_plan, reduce_slots and
// combine_ep are the receiving and owning sides of the expert-parallel layout.
#include <algorithm>

#include "common.cuh"

namespace jb {
namespace {

constexpr int BM = 128;  // rows per tile of the plan: the M of the grouped GEMMs' MMAs (moe_tc.cu)

// ------------------------------------------------------------------------------------------------------- routing

__global__ void route_init_kernel(int32_t* __restrict__ ws, int E, int32_t* __restrict__ sorted_ids, int64_t rows) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows; i += (int64_t)gridDim.x * blockDim.x)
    sorted_ids[i] = -1;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 3 * E; i += gridDim.x * blockDim.x) ws[i] = 0;
}

// one warp per token: softmax, top-k by k rounds of a warp argmax, renormalise, count per expert
__global__ void route_topk_kernel(const float* __restrict__ logits, int64_t S, int E, int k,
                                  int32_t* __restrict__ topk_idx, float* __restrict__ topk_w,
                                  int32_t* __restrict__ counts) {
  const int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= S) return;
  constexpr int MAXE = 16;  // experts per lane (E <= 512)
  float p[MAXE];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < MAXE; ++i) {
    const int e = lane + 32 * i;
    p[i] = e < E ? logits[t * E + e] : -INFINITY;
    mx = fmaxf(mx, p[i]);
  }
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < MAXE; ++i) {
    const int e = lane + 32 * i;
    p[i] = e < E ? expf(p[i] - mx) : 0.f;
    sum += p[i];
  }
  sum = warp_sum(sum);
  const float inv = 1.f / sum;
  float picked_sum = 0.f;
  float vals[16];
  int idxs[16];
  for (int j = 0; j < k; ++j) {
    float bv = -1.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < MAXE; ++i) {
      const int e = lane + 32 * i;
      const float v = e < E ? p[i] * inv : -1.f;
      if (v > bv || (v == bv && e < bi)) {
        bv = v;
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    vals[j] = bv;
    idxs[j] = bi;
    picked_sum += bv;
#pragma unroll
    for (int i = 0; i < MAXE; ++i)
      if (lane + 32 * i == bi) p[i] = -2.f * sum;  // removed (probabilities are >= 0)
  }
  if (lane == 0) {
    for (int j = 0; j < k; ++j) {
      topk_idx[t * k + j] = idxs[j];
      topk_w[t * k + j] = vals[j] / picked_sum;
      atomicAdd(&counts[idxs[j]], 1);
    }
  }
}

// one CTA: pad each expert's count to BM rows, exclusive scan, tile -> expert map, tile count
__global__ void route_plan_kernel(int32_t* __restrict__ ws, int E, int bm, int32_t* __restrict__ tile_expert,
                                  int64_t max_tiles, int32_t* __restrict__ n_tiles) {
  extern __shared__ int32_t sh[];  // [E] padded counts -> offsets
  int32_t* counts = ws;
  int32_t* offsets = ws + E;
  for (int e = threadIdx.x; e < E; e += blockDim.x) sh[e] = (counts[e] + bm - 1) / bm * bm;
  __syncthreads();
  if (threadIdx.x == 0) {  // E <= 1024: a serial scan is a few microseconds
    int32_t run = 0;
    for (int e = 0; e < E; ++e) {
      const int32_t c = sh[e];
      sh[e] = run;
      run += c;
    }
    n_tiles[0] = run / bm;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    offsets[e] = sh[e];
    const int32_t first = sh[e] / bm, last = (sh[e] + (counts[e] + bm - 1) / bm * bm) / bm;
    for (int32_t tt = first; tt < last; ++tt) tile_expert[tt] = e;
  }
}

__global__ void route_scatter_kernel(const int32_t* __restrict__ topk_idx, int64_t n, int32_t* __restrict__ ws, int E,
                                     int32_t* __restrict__ sorted_ids) {
  const int32_t* offsets = ws + E;
  int32_t* cursors = ws + 2 * E;
  for (int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; a < n; a += (int64_t)gridDim.x * blockDim.x) {
    const int e = topk_idx[a];
    if (e < 0 || e >= E) continue;  // a slot without an expert here (expert-parallel plans)
    const int pos = offsets[e] + atomicAdd(&cursors[e], 1);
    sorted_ids[pos] = (int32_t)a;
  }
}

// per-expert counts of explicit slot -> expert ids (negative or >= E: no expert)
__global__ void plan_count_kernel(const int32_t* __restrict__ ids, int64_t n, int E, int32_t* __restrict__ counts) {
  for (int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; a < n; a += (int64_t)gridDim.x * blockDim.x) {
    const int e = ids[a];
    if (e >= 0 && e < E) atomicAdd(&counts[e], 1);
  }
}

// out[t] = sum_j y[t*k + j] (fp32) + sigmoid(gate_logit[t]) * shared[t]
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ y, int k, const __nv_bfloat16* __restrict__ shared,
                                   const float* __restrict__ gate_logit, int64_t S, int H,
                                   __nv_bfloat16* __restrict__ out) {
  const int64_t n = S * (H / 8);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / (H / 8);
    const int c = (int)(i - t * (H / 8)) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, v[8];
    for (int j = 0; j < k; ++j) {
      load8(y + (t * k + j) * H + c, v);
#pragma unroll
      for (int u = 0; u < 8; ++u) acc[u] += v[u];
    }
    if (shared) {
      const float gsig = sigmoidf_(gate_logit[t]);
      load8(shared + t * H + c, v);
#pragma unroll
      for (int u = 0; u < 8; ++u) acc[u] += gsig * v[u];
    }
    store8(out + t * H + c, acc);
  }
}

// out[r] = sum over the slots j of row r that have an expert of y[r*k + j], in fp32 (slot order)
__global__ void reduce_slots_kernel(const __nv_bfloat16* __restrict__ y, int k, const int32_t* __restrict__ slot_expert,
                                    int64_t R, int H, float* __restrict__ out) {
  const int64_t n = R * (H / 8);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (H / 8);
    const int c = (int)(i - r * (H / 8)) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, v[8];
    for (int j = 0; j < k; ++j) {
      if (slot_expert && slot_expert[r * k + j] < 0) continue;
      load8(y + (r * k + j) * H + c, v);
#pragma unroll
      for (int u = 0; u < 8; ++u) acc[u] += v[u];
    }
    float4* o = reinterpret_cast<float4*>(out + r * H + c);
    o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
}

// out[t] = sum over the ranks w (in rank order) of partials[row_index[t, w]] (fp32) + sigmoid(gate) * shared[t]
__global__ void combine_ep_kernel(const float* __restrict__ partials, const int32_t* __restrict__ row_index, int W,
                                  const __nv_bfloat16* __restrict__ shared, const float* __restrict__ gate_logit,
                                  int64_t S, int H, __nv_bfloat16* __restrict__ out) {
  const int64_t n = S * (H / 8);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / (H / 8);
    const int c = (int)(i - t * (H / 8)) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, v[8];
    for (int w = 0; w < W; ++w) {
      const int32_t r = row_index[t * W + w];
      if (r < 0) continue;
      const float4* p = reinterpret_cast<const float4*>(partials + (int64_t)r * H + c);
      const float4 a = p[0], b = p[1];
      acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
      acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
    }
    if (shared) {
      const float gsig = sigmoidf_(gate_logit[t]);
      load8(shared + t * H + c, v);
#pragma unroll
      for (int u = 0; u < 8; ++u) acc[u] += gsig * v[u];
    }
    store8(out + t * H + c, acc);
  }
}

}  // namespace
}  // namespace jb

using namespace jb;

extern "C" int janus_b200_moe_route(const float* logits, int64_t S, int64_t E, int64_t k, int64_t tile_rows,
                                    int32_t* topk_idx, float* topk_w, int32_t* sorted_ids, int32_t* tile_expert,
                                    int64_t max_tiles, int32_t* n_tiles, int32_t* workspace, size_t workspace_bytes,
                                    void* stream) {
  JB_REQUIRE(logits && topk_idx && topk_w && sorted_ids && tile_expert && n_tiles, JANUS_ERR_INVALID,
             "moe_route: null pointer");
  JB_REQUIRE(S >= 0 && E > 0 && E <= 512 && k > 0 && k <= 16 && k <= E && tile_rows == BM, JANUS_ERR_INVALID,
             "moe_route: E %lld (<= 512), k %lld (<= 16), tile rows %lld (must be %d)", (long long)E, (long long)k,
             (long long)tile_rows, BM);
  const int64_t need_tiles = (S * k + E * (tile_rows - 1) + tile_rows - 1) / tile_rows;
  JB_REQUIRE(max_tiles >= need_tiles, JANUS_ERR_INVALID, "moe_route: max_tiles %lld < worst case %lld",
             (long long)max_tiles, (long long)need_tiles);
  JB_REQUIRE(workspace && workspace_bytes >= (size_t)(3 * E) * sizeof(int32_t), JANUS_ERR_WORKSPACE,
             "moe_route: workspace needs %lld bytes", (long long)(3 * E * 4));
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t rows = max_tiles * tile_rows;
  route_init_kernel<<<(unsigned)std::min<int64_t>(148 * 8, (rows + 255) / 256 + 1), 256, 0, s>>>(workspace, (int)E,
                                                                                                 sorted_ids, rows);
  int st = launch_status("moe_route/init");
  if (st) return st;
  if (S > 0) {
    route_topk_kernel<<<(unsigned)((S * 32 + 255) / 256), 256, 0, s>>>(logits, S, (int)E, (int)k, topk_idx, topk_w,
                                                                       workspace);
    st = launch_status("moe_route/topk");
    if (st) return st;
  }
  route_plan_kernel<<<1, 256, E * sizeof(int32_t), s>>>(workspace, (int)E, (int)tile_rows, tile_expert, max_tiles,
                                                        n_tiles);
  st = launch_status("moe_route/plan");
  if (st) return st;
  if (S > 0) {
    route_scatter_kernel<<<(unsigned)std::min<int64_t>(148 * 8, (S * k + 255) / 256), 256, 0, s>>>(
        topk_idx, S * k, workspace, (int)E, sorted_ids);
    st = launch_status("moe_route/scatter");
  }
  return st;
}

namespace jb {
int moe_router_tc(const void* x, int64_t x_stride, int64_t S, int64_t H, const void* w_router, int64_t E,
                  const void* w_gate, int64_t k, int32_t* topk_idx, float* topk_w, float* gate_logit, int32_t* counts,
                  int32_t* status, cudaStream_t stream);
}

extern "C" int janus_b200_moe_route_fused(const void* x, int64_t x_stride, int64_t S, int64_t H, const void* w_router,
                                          int64_t E, const void* w_gate, int64_t k, int64_t tile_rows,
                                          int32_t* topk_idx, float* topk_w, float* gate_logit, int32_t* sorted_ids,
                                          int32_t* tile_expert, int64_t max_tiles, int32_t* n_tiles,
                                          int32_t* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  JB_REQUIRE(x && w_router && topk_idx && topk_w && sorted_ids && tile_expert && n_tiles && (!w_gate || gate_logit),
             JANUS_ERR_INVALID, "moe_route_fused: null pointer");
  JB_REQUIRE(S >= 0 && E > 0 && k > 0 && k <= E && tile_rows == BM, JANUS_ERR_INVALID,
             "moe_route_fused: E %lld, k %lld, tile rows %lld (must be %d)", (long long)E, (long long)k,
             (long long)tile_rows, BM);
  const int64_t need_tiles = (S * k + E * (tile_rows - 1) + tile_rows - 1) / tile_rows;
  JB_REQUIRE(max_tiles >= need_tiles, JANUS_ERR_INVALID, "moe_route_fused: max_tiles %lld < worst case %lld",
             (long long)max_tiles, (long long)need_tiles);
  JB_REQUIRE(workspace && workspace_bytes >= (size_t)(3 * E) * sizeof(int32_t), JANUS_ERR_WORKSPACE,
             "moe_route_fused: workspace needs %lld bytes", (long long)(3 * E * 4));
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t rows = max_tiles * tile_rows;
  route_init_kernel<<<(unsigned)std::min<int64_t>(148 * 8, (rows + 255) / 256 + 1), 256, 0, s>>>(workspace, (int)E,
                                                                                                 sorted_ids, rows);
  int st = launch_status("moe_route_fused/init");
  if (st) return st;
  st = moe_router_tc(x, x_stride, S, H, w_router, E, w_gate, k, topk_idx, topk_w, gate_logit, workspace, status, s);
  if (st) return st;
  route_plan_kernel<<<1, 256, E * sizeof(int32_t), s>>>(workspace, (int)E, (int)tile_rows, tile_expert, max_tiles,
                                                        n_tiles);
  st = launch_status("moe_route_fused/plan");
  if (st) return st;
  if (S > 0) {
    route_scatter_kernel<<<(unsigned)std::min<int64_t>(148 * 8, (S * k + 255) / 256), 256, 0, s>>>(
        topk_idx, S * k, workspace, (int)E, sorted_ids);
    st = launch_status("moe_route_fused/scatter");
  }
  return st;
}

extern "C" int janus_b200_moe_combine(const void* y, int64_t k, const void* shared, const float* shared_gate_logit,
                                      int64_t S, int64_t H, void* out, void* stream) {
  JB_REQUIRE(y && out && k > 0 && S >= 0 && H > 0 && H % 8 == 0, JANUS_ERR_INVALID, "moe_combine: arguments");
  JB_REQUIRE(!shared || shared_gate_logit, JANUS_ERR_INVALID, "moe_combine: shared expert needs its gate logits");
  JB_REQUIRE(JB_ALIGNED(y, 16) && JB_ALIGNED(out, 16) && (!shared || JB_ALIGNED(shared, 16)), JANUS_ERR_ALIGNMENT,
             "moe_combine: alignment");
  if (S == 0) return JANUS_OK;
  const int64_t n = S * (H / 8);
  moe_combine_kernel<<<(unsigned)std::min<int64_t>(148 * 32, (n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)y, (int)k, (const __nv_bfloat16*)shared, shared_gate_logit, S, (int)H,
      (__nv_bfloat16*)out);
  return launch_status("moe_combine");
}

extern "C" int janus_b200_moe_plan(const int32_t* expert_ids, int64_t n, int64_t E, int64_t tile_rows,
                                   int32_t* sorted_ids, int32_t* tile_expert, int64_t max_tiles, int32_t* n_tiles,
                                   int32_t* workspace, size_t workspace_bytes, void* stream) {
  JB_REQUIRE((expert_ids || n == 0) && sorted_ids && tile_expert && n_tiles, JANUS_ERR_INVALID,
             "moe_plan: null pointer");
  JB_REQUIRE(n >= 0 && n <= 0x7fffffff && E > 0 && E <= 1024 && tile_rows == BM, JANUS_ERR_INVALID,
             "moe_plan: n %lld, E %lld (<= 1024), tile rows %lld (must be %d)", (long long)n, (long long)E,
             (long long)tile_rows, BM);
  const int64_t need_tiles = (n + E * (tile_rows - 1) + tile_rows - 1) / tile_rows;
  JB_REQUIRE(max_tiles >= need_tiles, JANUS_ERR_INVALID, "moe_plan: max_tiles %lld < worst case %lld",
             (long long)max_tiles, (long long)need_tiles);
  JB_REQUIRE(workspace && workspace_bytes >= (size_t)(3 * E) * sizeof(int32_t), JANUS_ERR_WORKSPACE,
             "moe_plan: workspace needs %lld bytes", (long long)(3 * E * 4));
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t rows = max_tiles * tile_rows;
  route_init_kernel<<<(unsigned)std::min<int64_t>(148 * 8, (rows + 255) / 256 + 1), 256, 0, s>>>(workspace, (int)E,
                                                                                                 sorted_ids, rows);
  int st = launch_status("moe_plan/init");
  if (st) return st;
  if (n > 0) {
    plan_count_kernel<<<(unsigned)std::min<int64_t>(148 * 8, (n + 255) / 256), 256, 0, s>>>(expert_ids, n, (int)E,
                                                                                             workspace);
    st = launch_status("moe_plan/count");
    if (st) return st;
  }
  route_plan_kernel<<<1, 256, E * sizeof(int32_t), s>>>(workspace, (int)E, (int)tile_rows, tile_expert, max_tiles,
                                                        n_tiles);
  st = launch_status("moe_plan/plan");
  if (st) return st;
  if (n > 0) {
    route_scatter_kernel<<<(unsigned)std::min<int64_t>(148 * 8, (n + 255) / 256), 256, 0, s>>>(expert_ids, n,
                                                                                               workspace, (int)E,
                                                                                               sorted_ids);
    st = launch_status("moe_plan/scatter");
  }
  return st;
}

extern "C" int janus_b200_moe_reduce_slots(const void* y, int64_t k, const int32_t* slot_expert, int64_t R, int64_t H,
                                           float* out, void* stream) {
  JB_REQUIRE(out && (y || R == 0) && k > 0 && R >= 0 && H > 0 && H % 8 == 0, JANUS_ERR_INVALID,
             "moe_reduce_slots: arguments");
  JB_REQUIRE(JB_ALIGNED(y, 16) && JB_ALIGNED(out, 16), JANUS_ERR_ALIGNMENT, "moe_reduce_slots: alignment");
  if (R == 0) return JANUS_OK;
  const int64_t n = R * (H / 8);
  reduce_slots_kernel<<<(unsigned)std::min<int64_t>(148 * 32, (n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)y, (int)k, slot_expert, R, (int)H, out);
  return launch_status("moe_reduce_slots");
}

extern "C" int janus_b200_moe_combine_ep(const float* partials, const int32_t* row_index, int64_t W, const void* shared,
                                         const float* shared_gate_logit, int64_t S, int64_t H, void* out,
                                         void* stream) {
  JB_REQUIRE(out && row_index && W > 0 && S >= 0 && H > 0 && H % 8 == 0, JANUS_ERR_INVALID,
             "moe_combine_ep: arguments");
  JB_REQUIRE(!shared || shared_gate_logit, JANUS_ERR_INVALID, "moe_combine_ep: shared expert needs its gate logits");
  JB_REQUIRE(JB_ALIGNED(partials, 16) && JB_ALIGNED(out, 16) && (!shared || JB_ALIGNED(shared, 16)),
             JANUS_ERR_ALIGNMENT, "moe_combine_ep: alignment");
  if (S == 0) return JANUS_OK;
  const int64_t n = S * (H / 8);
  combine_ep_kernel<<<(unsigned)std::min<int64_t>(148 * 32, (n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      partials, row_index, (int)W, (const __nv_bfloat16*)shared, shared_gate_logit, S, (int)H, (__nv_bfloat16*)out);
  return launch_status("moe_combine_ep");
}
