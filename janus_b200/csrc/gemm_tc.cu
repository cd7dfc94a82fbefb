// Dense bf16 GEMMs of the dense projections on the 5th-generation tensor cores: out[M, N] = A[M, K] W[N, K]^T (the
// torch F.linear of the reference's merged projections, janus/hybrid.py:1108-1133), fp32 accumulation in TMEM.
//
// Epilogues:
//   plain   out bf16 [M, N] = the accumulator rounded once;
//   swiglu  W's rows come in 256-row blocks of 128 gate rows followed by the 128 matching up rows (janus_b200
//           ops.swiglu_weight builds that order from gate_proj / up_proj); out bf16 [M, N / 2] =
//           silu(gate) * up from the fp32 accumulators, rounded once: the MLP's gate/up GEMM and its SwiGLU
//           (`_silu_mul`, janus/hybrid.py:263) in one pass, the 2N-wide intermediate never written.
//
// Tiles of 128 rows x 256 columns, one M=128, N=256 MMA per 16-deep k step. A stage holds a 128-deep k-block (two
// 128-byte swizzle atoms of bf16) of A (32 KB) and W (64 KB), loaded by TMA (no multicast) into a 2-stage ring: the
// MMA thread waits once per 8 MMAs (a wait costs the tensor pipe a few hundred cycles even when the phase is
// already complete, so waiting once per 64-deep block left it idle a quarter of the time). Persistent
// CTAs, one per SM, walk the (m-tile, n-block) items with the n-block fastest: the CTAs of a wave share one or two
// A tiles and the whole weight matrix stays resident in L2 across waves, so A and W are read from HBM about once.
// The fp32 accumulator is double-buffered in TMEM (2 x 256 columns), so an item's epilogue overlaps the next item's
// main loop. Warps: 0 TMA producer, 1 TMEM owner and MMA issuer, 2-3 idle, 4-7 epilogue (warp w reads TMEM lanes
// 32 (w % 4) .. +31). Rows past M and columns past N are zero-filled by the loads and not stored. Every hand-off is
// an mbarrier with a bounded wait: a wait that runs out sets the status word and the CTA winds down (loads in
// flight waited for, MMAs drained, TMEM released).
#include "tcgen05.cuh"

namespace jb {
namespace gtc {
using namespace tcx;

constexpr int BM = 128, BN = 256, BK = 64;  // BK: one swizzle atom
constexpr int AT = 2;    // atoms per stage: a stage is a 128-deep k-block
constexpr int S = 2;     // stages
constexpr int NT = 256;  // 8 warps
constexpr uint32_t kAtomA = BM * BK * 2;  // 16 KB
constexpr uint32_t kAtomB = BN * BK * 2;  // 32 KB
constexpr uint32_t kA = AT * kAtomA;
constexpr uint32_t kB = AT * kAtomB;
constexpr uint32_t kStage = kA + kB;
constexpr uint32_t kOut = S * kStage;              // epilogue staging: 4 warps x 32 rows x 64 bytes
constexpr uint32_t kSmem = kOut + 4 * 32 * 64;

struct Params {
  CUtensorMap amap, bmap;  // A [M][K], W [N][K] bf16, boxes of 64 columns x 128 / 256 rows, 128B swizzle
  __nv_bfloat16* out;
  int64_t ldo;
  int32_t* err;
  int M, N, K, nblk, n_items, swiglu;
};

struct Bars {
  uint64_t full[S], empty[S], acc_full[2], acc_empty[2], drain;
};

__global__ void __launch_bounds__(NT, 1) gemm_bf16_tc_kernel(const __grid_constant__ Params p) {
  extern __shared__ unsigned char raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = s32(base);
  __shared__ Bars bars;
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x;
  const int nkb = (p.K + AT * BK - 1) / (AT * BK);  // stages per item (the last one zero-filled past K)

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(&tmem_base)),
                 "r"(2 * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      bar_init(&bars.full[s], 1);   // the producer's expect_tx, then the TMA bytes
      bar_init(&bars.empty[s], 1);  // the stage's MMAs (commit)
    }
    for (int a = 0; a < 2; ++a) {
      bar_init(&bars.acc_full[a], 1);   // the item's last MMAs (commit)
      bar_init(&bars.acc_empty[a], 4);  // one arrival per epilogue warp
    }
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
      int q = 0, issued = 0;
      for (int it = blockIdx.x; it < p.n_items && ok; it += G) {
        const int m0 = (it / p.nblk) * BM, n0 = (it % p.nblk) * BN;
        for (int kb = 0; kb < nkb; ++kb, ++q) {
          const int s = q % S;
          if (q >= S) ok = wait_bar(&bars.empty[s], ((q / S) - 1) & 1, p.err);
          if (!ok) break;
          bar_expect_tx(&bars.full[s], kStage);
#pragma unroll
          for (int t = 0; t < AT; ++t) {
            tma_load2(sbase + s * kStage + t * kAtomA, &p.amap, (kb * AT + t) * BK, m0, &bars.full[s]);
            tma_load2(sbase + s * kStage + kA + t * kAtomB, &p.bmap, (kb * AT + t) * BK, n0, &bars.full[s]);
          }
          issued = q + 1;
        }
      }
      // every issued load has landed before the CTA may leave (on the normal path the MMAs consumed them all)
      for (int j = issued - S < 0 ? 0 : issued - S; j < issued; ++j)
        wait_bar_quiet(&bars.full[j % S], (j / S) & 1, p.err);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID = idesc(BM, BN, 0, 0);
      bool ok = true;
      int q = 0, i = 0;
      for (int it = blockIdx.x; it < p.n_items && ok; it += G, ++i) {
        const int ab = i & 1;
        if (i >= 2) ok = wait_bar(&bars.acc_empty[ab], ((i >> 1) - 1) & 1, p.err);
        if (!ok) break;
        fence_after();
        const uint32_t acc = tm + ab * BN;
        for (int kb = 0; kb < nkb; ++kb, ++q) {
          const int s = q % S;
          ok = wait_bar(&bars.full[s], (q / S) & 1, p.err);
          if (!ok) break;
          fence_after();
          const uint32_t a = sbase + s * kStage, b = a + kA;
#pragma unroll
          for (int ks = 0; ks < AT * BK / 16; ++ks) {
            const uint32_t off = (ks / (BK / 16)), in = (ks % (BK / 16)) * 32;
            mma(acc, sdesc(a + off * kAtomA + in, 16, 1024), sdesc(b + off * kAtomB + in, 16, 1024), ID,
                (kb | ks) != 0);
          }
          commit(&bars.empty[s]);
        }
        if (ok) commit(&bars.acc_full[ab]);
      }
      commit(&bars.drain);  // completes once every MMA issued above has finished
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------------------------------- epilogue
    // thread = accumulator row (TMEM lane 32 (warp % 4) + lane). Each 32-column slice of the warp's rows goes through
    // a small shared-memory buffer so the global stores cover 8 rows x 64 bytes per instruction instead of 32 rows x
    // 16 bytes.
    const int eq = warp & 3;
    unsigned char* stg = base + kOut + eq * (32 * 64);  // [32 rows][64 bytes], 16-byte units swizzled by row
    const int outc = p.swiglu ? BN / 2 : BN;            // output columns of an item
    const int out_n = p.swiglu ? p.N / 2 : p.N;
    bool ok = true;
    int i = 0;
    for (int it = blockIdx.x; it < p.n_items && ok; it += G, ++i) {
      const int ab = i & 1;
      const int m0 = (it / p.nblk) * BM, c0 = (it % p.nblk) * outc;
      ok = __all_sync(kFull, wait_bar_sleep(&bars.acc_full[ab], (i >> 1) & 1, p.err));
      if (!ok) break;
      fence_after();
      const uint32_t la = tm + ((uint32_t)(32 * eq) << 16) + ab * BN;
#pragma unroll 1
      for (int cc = 0; cc < outc; cc += 32) {
        uint32_t o[16];
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          float a[16];
          tld16f(la + cc + 16 * h2, a);
          if (p.swiglu) {  // silu(gate) * up: gate in accumulator columns 0..127, up in 128..255
            float u[16];
            tld16f(la + 128 + cc + 16 * h2, u);
#pragma unroll
            for (int k = 0; k < 8; ++k)
              o[8 * h2 + k] = pack_bf16(silu(a[2 * k]) * u[2 * k], silu(a[2 * k + 1]) * u[2 * k + 1]);
          } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) o[8 * h2 + k] = pack_bf16(a[2 * k], a[2 * k + 1]);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
          *reinterpret_cast<uint4*>(stg + lane * 64 + ((u ^ ((lane >> 1) & 3)) << 4)) =
              make_uint4(o[4 * u], o[4 * u + 1], o[4 * u + 2], o[4 * u + 3]);
        __syncwarp();
        const int col = c0 + cc + (lane & 3) * 8;  // the 8 columns this lane stores
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int rr = k * 8 + (lane >> 2);
          const uint4 v = *reinterpret_cast<const uint4*>(stg + rr * 64 + (((lane & 3) ^ ((rr >> 1) & 3)) << 4));
          const int row = m0 + 32 * eq + rr;
          if (row < p.M && col < out_n) *reinterpret_cast<uint4*>(p.out + (int64_t)row * p.ldo + col) = v;
        }
        __syncwarp();  // the buffer is read before the next slice overwrites it
      }
      fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&bars.acc_empty[ab]);
    }
  }

  // wind down: every MMA issued has completed before TMEM is released
  fence_before();
  __syncthreads();
  fence_after();
  wait_bar_quiet(&bars.drain, 0, p.err);
  fence_before();
  __syncthreads();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(2 * BN));
}

}  // namespace gtc

// row-major [rows][cols] bf16 with row stride ld elements, boxes of 64 columns x box_rows rows, 128B swizzle,
// zero fill past the edges
static int gemm_map(CUtensorMap* m, const void* ptr, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_rows) {
  tcx::EncodeTiled enc = tcx::encode_tiled_fn();
  if (!enc) {
    set_error("gemm_bf16: cuTensorMapEncodeTiled unavailable");
    return JANUS_ERR_CUDA;
  }
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)gtc::BK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("gemm_bf16: tensor map encode failed (%d)", (int)r);
    return JANUS_ERR_INVALID;
  }
  return JANUS_OK;
}

}  // namespace jb

using namespace jb;

extern "C" int janus_b200_gemm_bf16(const void* a, int64_t lda, const void* w, int64_t ldw, int64_t M, int64_t N,
                                    int64_t K, int32_t epilogue, void* out, int64_t ldo, int32_t* status,
                                    void* stream) {
  JB_REQUIRE(a && w && out, JANUS_ERR_INVALID, "gemm_bf16: null pointer");
  JB_REQUIRE(epilogue == 0 || epilogue == 1, JANUS_ERR_INVALID, "gemm_bf16: epilogue %d (0 plain, 1 swiglu)",
             (int)epilogue);
  JB_REQUIRE(M >= 0 && N > 0 && K > 0 && M < (1ll << 31) && N < (1ll << 24) && K < (1ll << 24),
             JANUS_ERR_INVALID, "gemm_bf16: sizes M %lld N %lld K %lld", (long long)M, (long long)N, (long long)K);
  JB_REQUIRE(N % 16 == 0 && K % 8 == 0 && (epilogue == 0 || N % 256 == 0), JANUS_ERR_UNSUPPORTED,
             "gemm_bf16: N %lld must be a multiple of 16 (256 for swiglu), K %lld of 8", (long long)N, (long long)K);
  JB_REQUIRE(lda >= K && ldw >= K && lda % 8 == 0 && ldw % 8 == 0 && ldo % 8 == 0 &&
                 ldo >= (epilogue ? N / 2 : N) && JB_ALIGNED(a, 16) && JB_ALIGNED(w, 16) && JB_ALIGNED(out, 16),
             JANUS_ERR_ALIGNMENT, "gemm_bf16: 16-byte aligned operands, leading dimensions multiples of 8");
  if (M == 0) return JANUS_OK;
  gtc::Params p{};
  int st = gemm_map(&p.amap, a, (uint64_t)K, (uint64_t)M, (uint64_t)lda, gtc::BM);
  if (!st) st = gemm_map(&p.bmap, w, (uint64_t)K, (uint64_t)N, (uint64_t)ldw, gtc::BN);
  if (st) return st;
  const int64_t mt = (M + gtc::BM - 1) / gtc::BM, nblk = (N + gtc::BN - 1) / gtc::BN;
  JB_REQUIRE(mt * nblk < (1ll << 31), JANUS_ERR_UNSUPPORTED, "gemm_bf16: too many tiles");
  p.out = (__nv_bfloat16*)out;
  p.ldo = ldo;
  p.err = status;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.nblk = (int)nblk;
  p.n_items = (int)(mt * nblk);
  p.swiglu = epilogue;
  const size_t smem = gtc::kSmem + 1024;
  cudaError_t e =
      cudaFuncSetAttribute(gtc::gemm_bf16_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    set_error("gemm_bf16: smem attribute: %s", cudaGetErrorString(e));
    return JANUS_ERR_CUDA;
  }
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
    set_error("gemm_bf16: device query failed");
    return JANUS_ERR_CUDA;
  }
  const int grid = (int)(p.n_items < sms ? p.n_items : sms);
  gtc::gemm_bf16_tc_kernel<<<grid, gtc::NT, smem, (cudaStream_t)stream>>>(p);
  return launch_status("gemm_bf16");
}
