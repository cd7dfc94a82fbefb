// The MoE router fused with its routing (Qwen3_5MoeTopKRouter, transformers qwen3_5_moe :754-770, and the shared
// expert's gate logit, :778-791): logits = x W_r^T on the 5th-generation tensor cores, fp32 in TMEM, never written to
// HBM; then per token softmax (fp32), top-k, renormalisation and the per-expert counts of the routing plan. One CTA
// per 128 tokens: x rows and W_r / w_g k-blocks of 64 stream through a TMA ring (no multicast); one thread issues an
// M=128, N=round16(E) MMA for the router and an M=128, N=16 MMA for the gate row (rows past E or past the one gate
// row are zero-filled by the loads). Warps: 0 TMA producer, 1 TMEM owner and MMA issuer, 2-5 epilogue (one token per
// thread, TMEM lane = token). The epilogue repeats the arithmetic of route_topk_kernel (moe.cu) operation for
// operation: max, e^(l - max), the sum in that kernel's order (32 lane partials over experts e = lane + 32 i, then
// its xor butterfly), p = e^(l - max) / sum, top-k by (p descending, expert ascending), weights p / sum of the picked
// p; so given the same logits both pick the same experts with the same weights. Every wait is bounded: one that runs
// out sets the status word and the CTA winds down (loads landed, MMAs drained, TMEM released).
#include "tcgen05.cuh"

namespace jb {
namespace rtc {
using namespace tcx;

constexpr int BM = 128, BK = 64, S = 3, NT = 192;
constexpr int kMaxE = 256, kMaxK = 8;
constexpr uint32_t kA = BM * BK * 2;       // 16 KB
constexpr uint32_t kB = kMaxE * BK * 2;    // 32 KB (router rows)
constexpr uint32_t kG = 16 * BK * 2;       // 2 KB (gate row + 15 zero rows)
constexpr uint32_t kStage = kA + kB + kG;  // 50 KB, a multiple of 1024
constexpr uint32_t kSmem = S * kStage;
constexpr uint32_t kColL = 0, kColG = 256, kTmemCols = 512;

struct Params {
  CUtensorMap xmap, wmap, gmap;  // x [S][H], W_r [E][H], w_g [1][H] bf16; boxes of 64 columns x 128 / NB / 16 rows
  int32_t* topk_idx;
  float* topk_w;
  float* gate_logit;
  int32_t* counts;
  int32_t* err;
  int S, H, E, NB, k;
};

struct Bars {
  uint64_t full[S], empty[S], acc, drain;
};

template <int K>
__global__ void __launch_bounds__(NT, 1) moe_router_kernel(const __grid_constant__ Params p) {
  extern __shared__ unsigned char raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = s32(base);
  __shared__ Bars bars;
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.x * BM;
  const int nkb = (p.H + BK - 1) / BK;

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(&tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      bar_init(&bars.full[s], 1);
      bar_init(&bars.empty[s], 1);
    }
    bar_init(&bars.acc, 1);
    bar_init(&bars.drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tm = tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      const uint32_t bytes = kA + (uint32_t)p.NB * BK * 2 + kG;
      for (int kb = 0; kb < nkb && ok; ++kb) {
        const int s = kb % S;
        if (kb >= S) ok = wait_bar(&bars.empty[s], (kb / S - 1) & 1, p.err);
        if (!ok) break;
        bar_expect_tx(&bars.full[s], bytes);
        const uint32_t st = sbase + s * kStage;
        tma_load2(st, &p.xmap, kb * BK, m0, &bars.full[s]);
        tma_load2(st + kA, &p.wmap, kb * BK, 0, &bars.full[s]);
        tma_load2(st + kA + kB, &p.gmap, kb * BK, 0, &bars.full[s]);
        issued = kb + 1;
      }
      for (int kb = issued - S < 0 ? 0 : issued - S; kb < issued; ++kb)  // the loads land before the CTA leaves
        wait_bar_quiet(&bars.full[kb % S], (kb / S) & 1, p.err);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t id_l = idesc(BM, p.NB, 0, 0), id_g = idesc(BM, 16, 0, 0);
      bool ok = true;
      for (int kb = 0; kb < nkb && ok; ++kb) {
        const int s = kb % S;
        ok = wait_bar(&bars.full[s], (kb / S) & 1, p.err);
        if (!ok) break;
        fence_after();
        const uint32_t st = sbase + s * kStage;
#pragma unroll
        for (int ks = 0; ks < BK / 16; ++ks) {
          const uint64_t da = sdesc(st + ks * 32, 16, 1024);
          mma(tm + kColL, da, sdesc(st + kA + ks * 32, 16, 1024), id_l, (kb | ks) != 0);
          mma(tm + kColG, da, sdesc(st + kA + kB + ks * 32, 16, 1024), id_g, (kb | ks) != 0);
        }
        commit(&bars.empty[s]);
      }
      if (ok) commit(&bars.acc);
      commit(&bars.drain);
    }
  } else {
    // ------------------------------------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter
    const int r = 32 * q + lane;
    const int t = m0 + r;
    const uint32_t la = tm + ((uint32_t)(32 * q) << 16);
    const bool ok = __all_sync(kFull, wait_bar_sleep(&bars.acc, 0, p.err));
    fence_after();
    if (ok) {
      const int E = p.E;
      // max over the experts
      float mx = -INFINITY;
      for (int c = 0; c < p.NB; c += 32) {
        float l[32];
        tld32f(la + kColL + c, l);
#pragma unroll
        for (int x = 0; x < 32; ++x)
          if (c + x < E) mx = fmaxf(mx, l[x]);
      }
      // the sum of e^(l - max): partial x holds experts x, x + 32, ... in order (route_topk's lane x), then the
      // butterfly over the 32 partials in route_topk's order (offsets 16, 8, 4, 2, 1; own value first)
      float part[32];
#pragma unroll
      for (int x = 0; x < 32; ++x) part[x] = 0.f;
      for (int c = 0; c < p.NB; c += 32) {
        float l[32];
        tld32f(la + kColL + c, l);
#pragma unroll
        for (int x = 0; x < 32; ++x) part[x] += (c + x < E) ? expf(l[x] - mx) : 0.f;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int x = 0; x < o; ++x) part[x] = part[x] + part[x + o];
      const float sum = part[0];
      const float inv = 1.f / sum;
      // top-k of p = e^(l - max) * inv by (p descending, expert ascending): a sorted list of K; an expert enters only
      // when its p beats the K-th (experts arrive in ascending order, so an equal p never displaces an earlier one)
      float bv[K];
      int bi[K];
#pragma unroll
      for (int j = 0; j < K; ++j) {
        bv[j] = -1.f;
        bi[j] = 0x7fffffff;
      }
      for (int c = 0; c < p.NB; c += 32) {
        float l[32];
        tld32f(la + kColL + c, l);
#pragma unroll
        for (int x = 0; x < 32; ++x) {
          float v = c + x < E ? expf(l[x] - mx) * inv : -1.f;
          if (v > bv[K - 1]) {
            int vi = c + x;
#pragma unroll
            for (int j = 0; j < K; ++j) {
              const bool better = v > bv[j];
              const float tv = bv[j];
              const int ti = bi[j];
              bv[j] = better ? v : tv;
              bi[j] = better ? vi : ti;
              v = better ? tv : v;
              vi = better ? ti : vi;
            }
          }
        }
      }
      float gl[16];
      tld16f(la + kColG, gl);
      if (t < p.S) {
        float picked = 0.f;
#pragma unroll
        for (int j = 0; j < K; ++j) picked += bv[j];
#pragma unroll
        for (int j = 0; j < K; ++j) {
          p.topk_idx[(int64_t)t * K + j] = bi[j];
          p.topk_w[(int64_t)t * K + j] = bv[j] / picked;
          atomicAdd(&p.counts[bi[j]], 1);
        }
        if (p.gate_logit) p.gate_logit[t] = gl[0];
      }
    }
  }
  // wind down: every MMA issued has completed before TMEM is released
  fence_before();
  __syncthreads();
  fence_after();
  wait_bar_quiet(&bars.drain, 0, p.err);
  fence_before();
  __syncthreads();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(kTmemCols));
}

// row-major [rows][cols] bf16 with row stride ld elements, boxes of 64 columns x box_rows rows, 128B swizzle, zero fill
static int router_map(CUtensorMap* m, const void* ptr, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_rows) {
  EncodeTiled enc = encode_tiled_fn();
  if (!enc) {
    set_error("moe_router: cuTensorMapEncodeTiled unavailable");
    return JANUS_ERR_CUDA;
  }
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("moe_router: tensor map encode failed (%d)", (int)r);
    return JANUS_ERR_INVALID;
  }
  return JANUS_OK;
}

template <int K>
int launch(const Params& p, cudaStream_t stream) {
  const size_t smem = kSmem + 1024;
  cudaError_t e = cudaFuncSetAttribute(moe_router_kernel<K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    set_error("moe_router: smem attribute %s", cudaGetErrorString(e));
    return JANUS_ERR_CUDA;
  }
  moe_router_kernel<K><<<(unsigned)((p.S + BM - 1) / BM), NT, smem, stream>>>(p);
  return launch_status("moe_router");
}

}  // namespace rtc

// the router and top-k of moe_route_fused (moe.cu): topk_idx, topk_w, the per-expert counts (added onto `counts`) and
// the shared expert's gate logit (if w_gate)
int moe_router_tc(const void* x, int64_t x_stride, int64_t S, int64_t H, const void* w_router, int64_t E,
                  const void* w_gate, int64_t k, int32_t* topk_idx, float* topk_w, float* gate_logit, int32_t* counts,
                  int32_t* status, cudaStream_t stream) {
  JB_REQUIRE(E > 0 && E <= rtc::kMaxE && k > 0 && k <= rtc::kMaxK && k <= E && H > 0 && H % 8 == 0 &&
                 x_stride >= H && x_stride % 8 == 0 && S >= 0 && S < (1ll << 31),
             JANUS_ERR_UNSUPPORTED, "moe_router: E %lld (<= %d), k %lld (<= %d), H %lld (multiple of 8)",
             (long long)E, rtc::kMaxE, (long long)k, rtc::kMaxK, (long long)H);
  JB_REQUIRE(JB_ALIGNED(x, 16) && JB_ALIGNED(w_router, 16) && (!w_gate || JB_ALIGNED(w_gate, 16)), JANUS_ERR_ALIGNMENT,
             "moe_router: 16-byte aligned x and weights");
  if (S == 0) return JANUS_OK;
  rtc::Params p{};
  const int NB = (int)((E + 15) / 16 * 16);
  // without a gate row the gate MMA reads the router's first rows (its result is not stored)
  int st = rtc::router_map(&p.xmap, x, (uint64_t)H, (uint64_t)S, (uint64_t)x_stride, rtc::BM);
  if (!st) st = rtc::router_map(&p.wmap, w_router, (uint64_t)H, (uint64_t)E, (uint64_t)H, (uint32_t)NB);
  if (!st) st = rtc::router_map(&p.gmap, w_gate ? w_gate : w_router, (uint64_t)H, 1, (uint64_t)H, 16);
  if (st) return st;
  p.topk_idx = topk_idx;
  p.topk_w = topk_w;
  p.gate_logit = w_gate ? gate_logit : nullptr;
  p.counts = counts;
  p.err = status;
  p.S = (int)S;
  p.H = (int)H;
  p.E = (int)E;
  p.NB = NB;
  p.k = (int)k;
  switch (k) {
    case 1: return rtc::launch<1>(p, stream);
    case 2: return rtc::launch<2>(p, stream);
    case 4: return rtc::launch<4>(p, stream);
    case 6: return rtc::launch<6>(p, stream);
    case 8: return rtc::launch<8>(p, stream);
    default:
      set_error("moe_router: top-k %lld not compiled (1, 2, 4, 6, 8)", (long long)k);
      return JANUS_ERR_UNSUPPORTED;
  }
}

}  // namespace jb
