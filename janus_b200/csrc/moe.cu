// Sparse MoE feed-forward with W4A16 experts (int4 codes, one bf16 scale per 128 inputs): routing plan, permuted
// grouped GEMMs and the weighted combine.
//
// moe_route: softmax over the router logits (fp32), top-k, renormalise (Qwen3_5MoeTopKRouter), then a sync-free tile
// plan: per-expert counts (atomics), a one-CTA scan padding every expert to the tile height, and the scatter of the
// assignments (token * k + slot) into expert-sorted order. The tile count stays on the device; the GEMMs are
// launched for the worst case (every expert padded) and tiles past the count exit at once — the plan of
// janus/moe_w4a16.py:89-106, computed by three small kernels instead of argsort/bincount/searchsorted.
//
// moe_gemm: one CTA per (tile of 64 expert-sorted rows, 64 output columns). Per 128-deep k-block the CTA stages the
// activation rows (gathered by token for the first GEMM), the packed int4 weight rows and their scales with
// cp.async (double-buffered), decodes the codes once into a bf16 tile in shared memory (code * scale in fp32, one
// rounding to bf16: the value the reference's dequantise path feeds its GEMM) and runs mma.sync on it. The first
// GEMM computes gate and up columns together and stores silu(gate) * up per sorted row; the second multiplies by the
// routing weight and stores per assignment. moe_combine sums the k assignments of a token in fp32 and adds the gated
// shared expert.
#include <algorithm>

#include "common.cuh"

namespace jb {
namespace {

constexpr int BM = 64, BN = 64, BK = 128, GROUP = 128;
constexpr int NT = 128;
constexpr int PACKED_ROW = BK / 2 + 16;  // bytes per packed weight row in shared memory (16-byte aligned, padded)

__device__ __forceinline__ uint32_t s32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void cpa16(void* dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s32(dst)), "l"(src), "r"(ok ? 16 : 0));
}
__device__ __forceinline__ void ldx4(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(s32(p)));
}
__device__ __forceinline__ void mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// swizzled bf16 tile [rows][BK]
__device__ __forceinline__ int sw(int r, int c) { return r * BK + (((c >> 3) ^ (r & 7)) << 3) + (c & 7); }

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

// ---------------------------------------------------------------------------------------------- grouped GEMM

struct MoeSmem {
  __nv_bfloat16 a[2][BM * BK];
  uint8_t wq[2][2][BN * PACKED_ROW];  // [stage][gate/up][row][bytes]
  __nv_bfloat16 ws[2][2][BN];         // scales of the k-block
  __nv_bfloat16 b[2][BN * BK];        // decoded weights [gate/up][n][k]
  int32_t rows[BM];
};

template <bool GATED>
__global__ void __launch_bounds__(NT) moe_gemm_kernel(const __nv_bfloat16* __restrict__ A, int64_t lda,
                                                      const uint8_t* __restrict__ W, const __nv_bfloat16* __restrict__ Ws,
                                                      const int32_t* __restrict__ sorted_ids,
                                                      const int32_t* __restrict__ tile_expert,
                                                      const int32_t* __restrict__ n_tiles, int N, int K, int topk,
                                                      const float* __restrict__ topk_w, __nv_bfloat16* __restrict__ out,
                                                      int64_t ldo) {
  extern __shared__ __align__(16) unsigned char raw[];
  MoeSmem& sm = *reinterpret_cast<MoeSmem*>(raw);
  const int tile = blockIdx.x;
  if (tile >= n_tiles[0]) return;
  const int e = tile_expert[tile];
  const int n0 = blockIdx.y * BN;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int NW = GATED ? 2 * N : N;  // weight rows of the expert
  const uint8_t* We = W + (int64_t)e * NW * (K / 2);
  const __nv_bfloat16* Wse = Ws + (int64_t)e * NW * (K / GROUP);
  if (tid < BM) {
    const int id = sorted_ids[(int64_t)tile * BM + tid];
    // GEMM 1 gathers the token of the assignment; GEMM 2 reads its own sorted row
    sm.rows[tid] = GATED ? (id >= 0 ? id / topk : -1) : (id >= 0 ? tile * BM + tid : -1);
  }
  __syncthreads();
  const int nkb = K / BK;
  auto load = [&](int kb, int st) {
    const int k0 = kb * BK;
    for (int x = tid; x < BM * (BK / 8); x += NT) {
      const int r = x / (BK / 8), c = (x % (BK / 8)) * 8;
      const int row = sm.rows[r];
      cpa16(&sm.a[st][sw(r, c)], A + (int64_t)(row >= 0 ? row : 0) * lda + k0 + c, row >= 0);
    }
    for (int x = tid; x < (GATED ? 2 : 1) * BN * (BK / 32); x += NT) {
      const int half = x / (BN * (BK / 32));
      const int y = x % (BN * (BK / 32));
      const int r = y / (BK / 32), c = (y % (BK / 32)) * 16;
      const int wrow = n0 + r + half * N;
      cpa16(&sm.wq[st][half][r * PACKED_ROW + c], We + (int64_t)wrow * (K / 2) + k0 / 2 + c, true);
    }
    if (tid < (GATED ? 2 : 1) * BN) {
      const int half = tid / BN, r = tid % BN;
      sm.ws[st][half][r] = Wse[(int64_t)(n0 + r + half * N) * (K / GROUP) + k0 / GROUP];
    }
  };
  float acc[2][BN / 8][4];
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int n = 0; n < BN / 8; ++n) acc[h][n][0] = acc[h][n][1] = acc[h][n][2] = acc[h][n][3] = 0.f;
  load(0, 0);
  asm volatile("cp.async.commit_group;\n" ::);
  for (int kb = 0; kb < nkb; ++kb) {
    const int st = kb & 1;
    if (kb + 1 < nkb) {
      load(kb + 1, st ^ 1);
      asm volatile("cp.async.commit_group;\n" ::);
      asm volatile("cp.async.wait_group 1;\n" ::);
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::);
    }
    __syncthreads();
    // decode: byte j of a row holds k = 2j (low nibble) and 2j + 1 (high nibble); value = code * scale, rounded once
    for (int x = tid; x < (GATED ? 2 : 1) * BN * (BK / 2); x += NT) {
      const int half = x / (BN * (BK / 2));
      const int y = x % (BN * (BK / 2));
      const int r = y / (BK / 2), j = y % (BK / 2);
      const uint32_t byte = sm.wq[st][half][r * PACKED_ROW + j];
      const float sc = bf2f(sm.ws[st][half][r]);
      const float lo = (float)((int)((byte & 15u) ^ 8u) - 8) * sc;
      const float hi = (float)((int)((byte >> 4) ^ 8u) - 8) * sc;
      *reinterpret_cast<__nv_bfloat162*>(&sm.b[half][sw(r, 2 * j)]) = __floats2bfloat162_rn(lo, hi);
    }
    __syncthreads();
#pragma unroll
    for (int ks = 0; ks < BK; ks += 16) {
      uint32_t a[4];
      ldx4(a, &sm.a[st][sw(warp * 16 + (lane & 15), ks + ((lane >> 4) << 3))]);
#pragma unroll
      for (int h = 0; h < (GATED ? 2 : 1); ++h) {
#pragma unroll
        for (int np = 0; np < BN / 16; ++np) {
          uint32_t b[4];
          ldx4(b, &sm.b[h][sw(np * 16 + (lane & 7) + ((lane >> 4) << 3), ks + (((lane >> 3) & 1) << 3))]);
          mma(acc[h][2 * np], a, b[0], b[1]);
          mma(acc[h][2 * np + 1], a, b[2], b[3]);
        }
      }
    }
    __syncthreads();  // sm.b and the stage are free for the next k-block
  }
  // epilogue
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = warp * 16 + (lane >> 2) + i * 8;
    const int id = sorted_ids[(int64_t)tile * BM + r];
    if (id < 0) continue;
    const int64_t orow = GATED ? (int64_t)tile * BM + r : (int64_t)id;
    const float wgt = GATED ? 1.f : topk_w[id];
#pragma unroll
    for (int n = 0; n < BN / 8; ++n) {
      const int c = n0 + n * 8 + (lane & 3) * 2;
      float v0, v1;
      if (GATED) {
        v0 = silu(acc[0][n][2 * i]) * acc[1][n][2 * i];
        v1 = silu(acc[0][n][2 * i + 1]) * acc[1][n][2 * i + 1];
      } else {
        v0 = acc[0][n][2 * i] * wgt;
        v1 = acc[0][n][2 * i + 1] * wgt;
      }
      *reinterpret_cast<__nv_bfloat162*>(out + orow * ldo + c) = __floats2bfloat162_rn(v0, v1);
    }
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

extern "C" int janus_b200_moe_grouped_w4a16(const void* x, int64_t ldx, const uint8_t* codes, const void* scales,
                                            int64_t E, int64_t N, int64_t K, int32_t gated, const int32_t* sorted_ids,
                                            const int32_t* tile_expert, const int32_t* n_tiles, int64_t max_tiles,
                                            int64_t topk, const float* topk_w, void* out, int64_t ldo, void* stream) {
  JB_REQUIRE(x && codes && scales && sorted_ids && tile_expert && n_tiles && out, JANUS_ERR_INVALID,
             "moe_grouped_w4a16: null pointer");
  JB_REQUIRE(E > 0 && N > 0 && N % BN == 0 && K > 0 && K % BK == 0 && topk > 0, JANUS_ERR_UNSUPPORTED,
             "moe_grouped_w4a16: N %lld must be a multiple of %d and K %lld of %d", (long long)N, BN, (long long)K, BK);
  JB_REQUIRE(gated || topk_w, JANUS_ERR_INVALID, "moe_grouped_w4a16: the down projection needs routing weights");
  JB_REQUIRE(ldx % 8 == 0 && ldo % 2 == 0 && JB_ALIGNED(x, 16) && JB_ALIGNED(codes, 16) && JB_ALIGNED(out, 4),
             JANUS_ERR_ALIGNMENT, "moe_grouped_w4a16: alignment");
  if (max_tiles == 0) return JANUS_OK;
  const size_t smem = sizeof(MoeSmem);
  cudaStream_t s = (cudaStream_t)stream;
  dim3 grid((unsigned)max_tiles, (unsigned)(N / BN));
  cudaError_t e;
  if (gated) {
    e = cudaFuncSetAttribute(moe_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
      moe_gemm_kernel<true><<<grid, NT, smem, s>>>((const __nv_bfloat16*)x, ldx, codes, (const __nv_bfloat16*)scales,
                                                   sorted_ids, tile_expert, n_tiles, (int)N, (int)K, (int)topk, topk_w,
                                                   (__nv_bfloat16*)out, ldo);
  } else {
    e = cudaFuncSetAttribute(moe_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
      moe_gemm_kernel<false><<<grid, NT, smem, s>>>((const __nv_bfloat16*)x, ldx, codes, (const __nv_bfloat16*)scales,
                                                    sorted_ids, tile_expert, n_tiles, (int)N, (int)K, (int)topk, topk_w,
                                                    (__nv_bfloat16*)out, ldo);
  }
  if (e != cudaSuccess) {
    set_error("moe_grouped_w4a16: smem attribute: %s", cudaGetErrorString(e));
    return JANUS_ERR_CUDA;
  }
  return launch_status("moe_grouped_w4a16");
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
