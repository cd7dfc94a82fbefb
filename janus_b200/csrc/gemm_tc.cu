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
// Two tilings on CTA pairs, k-blocks of 64 (one 128-byte swizzle atom of bf16) in a TMA ring: the tall form (the
// default; 512 rows x 256 columns per pair, single-buffered accumulators, a 4-stage ring) and the 256-row form
// (256 x 256 per pair, double-buffered accumulators, a 6-stage ring; JANUS_B200_GEMM=pair). Both issue the same MMAs
// in the same k order for every output element, so their results are bit-identical. Persistent pairs walk the
// (m-tile, n-block) items with the n-block fastest: the pairs of a wave share one or two A tiles and the whole weight
// matrix stays resident in L2 across waves, so A and W are read from HBM about once. Warps: 0 TMA producer, 1 TMEM
// owner and (first CTA) MMA issuer, 2-3 idle, 4 and up epilogue (warp w reads TMEM lanes 32 (w % 4) .. +31). Rows
// past M and columns past N are zero-filled by the loads and not stored. Every hand-off is an mbarrier with a
// bounded wait: a wait that runs out sets the status word and the CTA winds down (loads in flight waited for, MMAs
// drained, TMEM released).
#include <stdlib.h>
#include <string.h>

#include "tcgen05.cuh"

namespace jb {
namespace gtc {
using namespace tcx;

struct Params {
  CUtensorMap amap, bmap;  // A [M][K], W [N][K] bf16, boxes of 64 columns x 128 / 256 rows, 128B swizzle
  __nv_bfloat16* out;
  int64_t ldo;
  int32_t* err;
  int M, N, K, nblk, n_items, swiglu;
  int mt, band;  // tall form: m-tiles, n-blocks per band (items walk a band's n-blocks for every m-tile, band by band)
};

}  // namespace gtc

// ------------------------------------------------------------------------------------------------------------------
// The 256-row form on CTA pairs (clusters of 2, cta_group::2): a pair computes a 256 x 256 tile with M=256, N=256 MMAs
// issued by the pair's first CTA; each CTA stages its own 128 rows of A and its own 128 of the tile's 256 W rows, so
// a CTA's shared memory carries 8 KB of operand reads and 8 KB of TMA writes per 128 MMA cycles (128 B per cycle,
// shared memory's rate; a single CTA with a 128 x 256 tile would carry 12 + 12 KB). Each CTA's TMEM holds the
// accumulator of its 128 rows, double-buffered (2 x 256 columns), so an item's epilogue overlaps the next item's
// main loop. Hand-offs: both CTAs' TMA loads complete on the first CTA's `full` barrier (which expects both CTAs'
// bytes); the MMA's commits arrive on the `empty`, `acc_full` and `drain` barriers of both CTAs (multicast to the
// pair); the epilogue warps of both CTAs arrive on the first CTA's `acc_empty`. A cluster barrier after the barrier
// set-up and before the exit keeps every remote arrival inside the peer's lifetime. No TMA load uses multicast.
namespace gtc2 {
using namespace tcx;

constexpr int BM = 128, BN = 256, BK = 64;  // per CTA: 128 rows of A, 128 of the 256 W rows of the tile
constexpr int S = 6;
constexpr int NT = 256;
constexpr uint32_t kA = BM * BK * 2;         // 16 KB
constexpr uint32_t kB = (BN / 2) * BK * 2;   // 16 KB
constexpr uint32_t kStage = kA + kB;
constexpr uint32_t kOut = S * kStage;
constexpr uint32_t kSmem = kOut + 4 * 32 * 64;

struct Bars {
  uint64_t full[S], empty[S], acc_full[2], acc_empty[2], drain;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t n_clusters() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// the shared::cluster address of this CTA's shared variable at `saddr` in the pair's CTA `rank`
__device__ __forceinline__ uint32_t peer_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void remote_arrive(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA tile load into this CTA's shared memory, completing on a barrier of the pair (cluster address); no multicast
__device__ __forceinline__ void tma_load2_pair(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}
// D (both CTAs' TMEM, 128 lanes each) (+)= A (both CTAs' shared memory) x B (both CTAs' halves)
__device__ __forceinline__ void mma2(uint32_t tm, uint64_t da, uint64_t db, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n}\n" ::"r"(tm),
      "l"(da), "l"(db), "r"(id), "r"(acc), "r"(0));
}
// completion of this CTA's MMAs issued so far, arriving on the barrier at the same offset in both CTAs of the pair
__device__ __forceinline__ void commit2(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          s32(bar)),
      "h"((uint16_t)3)
      : "memory");
}

__global__ void __launch_bounds__(NT, 1) gemm_bf16_pair_kernel(const __grid_constant__ gtc::Params p) {
  extern __shared__ unsigned char raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = s32(base);
  __shared__ Bars bars;
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const int G = (int)n_clusters(), c = (int)cluster_id();
  const int nkb = (p.K + BK - 1) / BK;

  if (warp == 1) {  // both CTAs' warp 1: the pair's TMEM, same columns in both
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(&tmem_base)),
                 "r"(2 * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::);
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      bar_init(&bars.full[s], 1);   // the first CTA's expect_tx, then both CTAs' TMA bytes
      bar_init(&bars.empty[s], 1);  // the stage's MMAs (commit, multicast)
    }
    for (int a = 0; a < 2; ++a) {
      bar_init(&bars.acc_full[a], 1);   // the item's last MMAs (commit, multicast)
      bar_init(&bars.acc_empty[a], 8);  // the 4 epilogue warps of each CTA (first CTA's barrier)
    }
    bar_init(&bars.drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote arrival
  fence_after();
  const uint32_t tm = tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------------------------------ TMA producers
    if (lane == 0) {
      bool ok = true;
      int q = 0, issued = 0;
      for (int it = c; it < p.n_items && ok; it += G) {
        const int m0 = (it / p.nblk) * (2 * BM) + (int)rank * BM, n0 = (it % p.nblk) * BN + (int)rank * (BN / 2);
        for (int kb = 0; kb < nkb; ++kb, ++q) {
          const int s = q % S;
          if (q >= S) ok = wait_bar(&bars.empty[s], ((q / S) - 1) & 1, p.err);
          if (!ok) break;
          if (rank == 0) bar_expect_tx(&bars.full[s], 2 * kStage);
          const uint32_t fb = peer_addr(s32(&bars.full[s]), 0);
          tma_load2_pair(sbase + s * kStage, &p.amap, kb * BK, m0, fb);
          tma_load2_pair(sbase + s * kStage + kA, &p.bmap, kb * BK, n0, fb);
          issued = q + 1;
        }
      }
      // every load landed before the CTA may leave: the first CTA's full barriers count both CTAs' bytes; the
      // second waits for the MMAs that read its last stages
      if (rank == 0) {
        for (int j = issued - S < 0 ? 0 : issued - S; j < issued; ++j)
          wait_bar_quiet(&bars.full[j % S], (j / S) & 1, p.err);
      } else {
        for (int j = issued - S < 0 ? 0 : issued - S; j < issued; ++j)
          wait_bar_quiet(&bars.empty[j % S], (j / S) & 1, p.err);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------- MMA issuer (first CTA)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t ID = idesc(2 * BM, BN, 0, 0);
      bool ok = true;
      int q = 0, i = 0;
      for (int it = c; it < p.n_items && ok; it += G, ++i) {
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
          for (int ks = 0; ks < BK / 16; ++ks)
            mma2(acc, sdesc(a + ks * 32, 16, 1024), sdesc(b + ks * 32, 16, 1024), ID, (kb | ks) != 0);
          commit2(&bars.empty[s]);
        }
        if (ok) commit2(&bars.acc_full[ab]);
      }
      commit2(&bars.drain);  // completes once every MMA issued above has finished
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------------------------ epilogue (both CTAs)
    const int eq = warp & 3;
    unsigned char* stg = base + kOut + eq * (32 * 64);
    const int outc = p.swiglu ? BN / 2 : BN;
    const int out_n = p.swiglu ? p.N / 2 : p.N;
    bool ok = true;
    int i = 0;
    for (int it = c; it < p.n_items && ok; it += G, ++i) {
      const int ab = i & 1;
      const int m0 = (it / p.nblk) * (2 * BM) + (int)rank * BM, c0 = (it % p.nblk) * outc;
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
          if (p.swiglu) {
            float u[16];
            tld16f(la + 128 + cc + 16 * h2, u);
#pragma unroll
            for (int k = 0; k < 8; ++k)
              o[8 * h2 + k] = pack_bf16(silu_fast(a[2 * k]) * u[2 * k], silu_fast(a[2 * k + 1]) * u[2 * k + 1]);
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
        const int col = c0 + cc + (lane & 3) * 8;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int rr = k * 8 + (lane >> 2);
          const uint4 v = *reinterpret_cast<const uint4*>(stg + rr * 64 + (((lane & 3) ^ ((rr >> 1) & 3)) << 4));
          const int row = m0 + 32 * eq + rr;
          if (row < p.M && col < out_n) *reinterpret_cast<uint4*>(p.out + (int64_t)row * p.ldo + col) = v;
        }
        __syncwarp();
      }
      fence_before();
      __syncwarp();
      if (lane == 0) remote_arrive(peer_addr(s32(&bars.acc_empty[ab]), 0));
    }
  }

  // wind down: the pair's MMAs have completed (drain, multicast) before either CTA releases TMEM, and neither CTA
  // leaves while the other may still arrive on its barriers
  fence_before();
  __syncthreads();
  fence_after();
  wait_bar_quiet(&bars.drain, 0, p.err);
  fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(2 * BN));
}

}  // namespace gtc2

// ------------------------------------------------------------------------------------------------------------------
// The tall-tile form: each CTA of the pair stages TWO 128-row A tiles against its 128 W rows, and the pair issues two
// M=256, N=256 MMAs per k-step (one per A tile) into two accumulators that fill TMEM (2 x 256 columns), so a pair
// computes a 512 x 256 tile. Per CTA and 64-deep k-block that is 48 KB of TMA loads for 1024 MMA cycles (48 B per
// cycle) against the 256-row form's 32 KB per 512 cycles (64 B per cycle): the L2-to-shared-memory path, which
// bounds the 256-row form at about two thirds of the tensor peak, carries a quarter fewer bytes per FLOP. The
// accumulators are single-buffered. The 8 epilogue warps (two per TMEM lane quarter, splitting the columns) read
// accumulator 0 into registers as bf16 pairs and release it before storing, then accumulator 1; the next item starts
// skewed: its first 4 staged k-blocks go into accumulator 0 while accumulator 1 is read, then into accumulator 1, and
// only then are their stages released; the stores run under the next item's MMAs.
// Meanwhile the 4-stage ring holds the next k-blocks. Hand-offs and the wind-down as in the 256-row form. No TMA
// load uses multicast.
namespace gtc4 {
using namespace tcx;
using gtc2::cluster_rank;
using gtc2::cluster_id;
using gtc2::n_clusters;
using gtc2::cluster_sync;
using gtc2::peer_addr;
using gtc2::remote_arrive;
using gtc2::tma_load2_pair;
using gtc2::mma2;
using gtc2::commit2;

constexpr int BM = 128, BN = 256, BK = 64;   // per CTA: 2 x 128 rows of A, 128 of the 256 W rows of the tile
constexpr int S = 4;
constexpr int NT = 384;                      // warps 0 TMA, 1 TMEM / MMA, 2-3 idle, 4-11 epilogue
constexpr uint32_t kA = BM * BK * 2;         // 16 KB per A tile
constexpr uint32_t kB = (BN / 2) * BK * 2;   // 16 KB
constexpr uint32_t kStage = 2 * kA + kB;     // 48 KB
constexpr uint32_t kOut = S * kStage;
constexpr uint32_t kSmem = kOut + 8 * 32 * 64;

struct Bars {
  uint64_t full[S], empty[S], acc_full, acc_empty[2], drain;
};

// item -> (m-tile, n-block): the n-blocks come in bands of p.band (the last one narrower); a band's items run its
// n-blocks fastest for every m-tile before the next band starts, so the band's weight rows stay in L2 while A streams
__device__ __forceinline__ void item_tile(const gtc::Params& p, int it, int& mi, int& ni) {
  const int per_band = p.mt * p.band, b = it / per_band, r = it - b * per_band;
  const int w = min(p.band, p.nblk - b * p.band);
  mi = r / w;
  ni = b * p.band + (r - mi * w);
}

// One accumulator's share of an epilogue warp (32 TMEM lanes x 128 accumulator columns): TMEM -> bf16 pairs in
// registers (plain: 128 output columns, 64 registers; SwiGLU: 64 output columns from 64 gate and 64 up columns, 32
// registers), then the accumulator is released to the next item's MMAs, and only then go the stores (staged through
// the warp's 2 KB of shared memory for 16-byte row segments), so the stores run under the next item's MMAs.
template <bool SW>
__device__ __forceinline__ void drain_acc(const gtc::Params& p, uint32_t la, int h, int eq, int lane, int m0, int c0,
                                          int out_n, unsigned char* stg, uint64_t* acc_empty) {
  constexpr int kChunks = SW ? 2 : 4;  // 32-column output chunks of this warp
  constexpr int kHalf = 32 * kChunks;  // output columns of this warp
  uint32_t pk[kChunks][16];
#pragma unroll
  for (int ch = 0; ch < kChunks; ++ch) {
    const int cc = h * kHalf + 32 * ch;
    float a[32];
    tld32f(la + cc, a);
    if (SW) {
      float u[32];
      tld32f(la + 128 + cc, u);
#pragma unroll
      for (int k = 0; k < 16; ++k)
        pk[ch][k] = pack_bf16(silu_fast(a[2 * k]) * u[2 * k], silu_fast(a[2 * k + 1]) * u[2 * k + 1]);
    } else {
#pragma unroll
      for (int k = 0; k < 16; ++k) pk[ch][k] = pack_bf16(a[2 * k], a[2 * k + 1]);
    }
  }
  fence_before();
  __syncwarp();
  if (lane == 0) remote_arrive(peer_addr(s32(acc_empty), 0));
#pragma unroll
  for (int ch = 0; ch < kChunks; ++ch) {
#pragma unroll
    for (int u = 0; u < 4; ++u)
      *reinterpret_cast<uint4*>(stg + lane * 64 + ((u ^ ((lane >> 1) & 3)) << 4)) =
          make_uint4(pk[ch][4 * u], pk[ch][4 * u + 1], pk[ch][4 * u + 2], pk[ch][4 * u + 3]);
    __syncwarp();
    const int col = c0 + h * kHalf + 32 * ch + (lane & 3) * 8;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int rr = k * 8 + (lane >> 2);
      const uint4 v = *reinterpret_cast<const uint4*>(stg + rr * 64 + (((lane & 3) ^ ((rr >> 1) & 3)) << 4));
      const int row = m0 + 32 * eq + rr;
      if (row < p.M && col < out_n) *reinterpret_cast<uint4*>(p.out + (int64_t)row * p.ldo + col) = v;
    }
    __syncwarp();
  }
}

__global__ void __launch_bounds__(NT, 1) gemm_bf16_tall_kernel(const __grid_constant__ gtc::Params p) {
  extern __shared__ unsigned char raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = s32(base);
  __shared__ Bars bars;
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const int G = (int)n_clusters(), c = (int)cluster_id();
  const int nkb = (p.K + BK - 1) / BK;

  if (warp == 1) {  // both CTAs' warp 1: the pair's TMEM, same columns in both
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(&tmem_base)),
                 "r"(2 * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::);
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      bar_init(&bars.full[s], 1);   // the first CTA's expect_tx, then both CTAs' TMA bytes
      bar_init(&bars.empty[s], 1);  // the stage's MMAs (commit, multicast)
    }
    bar_init(&bars.acc_full, 1);  // the item's last MMAs (commit, multicast)
    for (int a = 0; a < 2; ++a) bar_init(&bars.acc_empty[a], 16);  // 8 epilogue warps x 2 CTAs (first CTA's)
    bar_init(&bars.drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote arrival
  fence_after();
  const uint32_t tm = tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------------------------------ TMA producers
    if (lane == 0) {
      bool ok = true;
      int q = 0, issued = 0;
      for (int it = c; it < p.n_items && ok; it += G) {
        int mi, ni;
        item_tile(p, it, mi, ni);
        const int m0 = mi * (4 * BM) + (int)rank * (2 * BM), n0 = ni * BN + (int)rank * (BN / 2);
        for (int kb = 0; kb < nkb; ++kb, ++q) {
          const int s = q % S;
          if (q >= S) ok = wait_bar(&bars.empty[s], ((q / S) - 1) & 1, p.err);
          if (!ok) break;
          if (rank == 0) bar_expect_tx(&bars.full[s], 2 * kStage);
          const uint32_t fb = peer_addr(s32(&bars.full[s]), 0), st = sbase + s * kStage;
          tma_load2_pair(st, &p.amap, kb * BK, m0, fb);
          tma_load2_pair(st + kA, &p.amap, kb * BK, m0 + BM, fb);
          tma_load2_pair(st + 2 * kA, &p.bmap, kb * BK, n0, fb);
          issued = q + 1;
        }
      }
      // every load landed before the CTA may leave (as in the 256-row form)
      if (rank == 0) {
        for (int j = issued - S < 0 ? 0 : issued - S; j < issued; ++j)
          wait_bar_quiet(&bars.full[j % S], (j / S) & 1, p.err);
      } else {
        for (int j = issued - S < 0 ? 0 : issued - S; j < issued; ++j)
          wait_bar_quiet(&bars.empty[j % S], (j / S) & 1, p.err);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------- MMA issuer (first CTA)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t ID = idesc(2 * BM, BN, 0, 0);
      bool ok = true;
      int q = 0, i = 0;
      const int P = nkb < S ? nkb : S;  // the k-blocks of an item's skewed start
      for (int it = c; it < p.n_items && ok; it += G, ++i) {
        // skewed start: the first P staged k-blocks go into accumulator 0 as soon as the epilogue has drained it,
        // then into accumulator 1 once that is drained too (the stages are released only then)
        if (i >= 1) ok = wait_bar(&bars.acc_empty[0], (i - 1) & 1, p.err);
        if (!ok) break;
        fence_after();
        for (int kb = 0; kb < P && ok; ++kb) {
          const int s = (q + kb) % S;
          ok = wait_bar(&bars.full[s], ((q + kb) / S) & 1, p.err);
          if (!ok) break;
          fence_after();
          const uint32_t a0 = sbase + s * kStage, b = a0 + 2 * kA;
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks)
            mma2(tm, sdesc(a0 + ks * 32, 16, 1024), sdesc(b + ks * 32, 16, 1024), ID, (kb | ks) != 0);
        }
        if (ok && i >= 1) ok = wait_bar(&bars.acc_empty[1], (i - 1) & 1, p.err);
        if (!ok) break;
        fence_after();
        for (int kb = 0; kb < P; ++kb, ++q) {
          const int s = q % S;
          const uint32_t a1 = sbase + s * kStage + kA, b = a1 + kA;
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks)
            mma2(tm + BN, sdesc(a1 + ks * 32, 16, 1024), sdesc(b + ks * 32, 16, 1024), ID, (kb | ks) != 0);
          commit2(&bars.empty[s]);
        }
        for (int kb = P; kb < nkb; ++kb, ++q) {
          const int s = q % S;
          ok = wait_bar(&bars.full[s], (q / S) & 1, p.err);
          if (!ok) break;
          fence_after();
          const uint32_t a0 = sbase + s * kStage, a1 = a0 + kA, b = a0 + 2 * kA;
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks) {
            const uint64_t db = sdesc(b + ks * 32, 16, 1024);
            mma2(tm, sdesc(a0 + ks * 32, 16, 1024), db, ID, 1);
            mma2(tm + BN, sdesc(a1 + ks * 32, 16, 1024), db, ID, 1);
          }
          commit2(&bars.empty[s]);
        }
        if (ok) commit2(&bars.acc_full);
      }
      commit2(&bars.drain);  // completes once every MMA issued above has finished
    }
  } else if (warp >= 4) {
    // ----------------------------------------------- epilogue (both CTAs): accumulator 0, then accumulator 1, each
    // split between the two warps of a TMEM lane quarter by columns (warp group h takes the h-th half of the outputs)
    const int eq = warp & 3, h = (warp - 4) >> 2;
    unsigned char* stg = base + kOut + (warp - 4) * (32 * 64);
    const int outc = p.swiglu ? BN / 2 : BN;
    const int out_n = p.swiglu ? p.N / 2 : p.N;
    bool ok = true;
    int i = 0;
    for (int it = c; it < p.n_items && ok; it += G, ++i) {
      ok = __all_sync(kFull, wait_bar_sleep(&bars.acc_full, i & 1, p.err));
      if (!ok) break;
      fence_after();
      int mi, ni;
      item_tile(p, it, mi, ni);
#pragma unroll 1
      for (int g = 0; g < 2; ++g) {
        const int m0 = mi * (4 * BM) + (int)rank * (2 * BM) + g * BM, c0 = ni * outc;
        const uint32_t la = tm + ((uint32_t)(32 * eq) << 16) + g * BN;
        if (p.swiglu)
          drain_acc<true>(p, la, h, eq, lane, m0, c0, out_n, stg, &bars.acc_empty[g]);
        else
          drain_acc<false>(p, la, h, eq, lane, m0, c0, out_n, stg, &bars.acc_empty[g]);
      }
    }
  }

  // wind down (as in the 256-row form)
  fence_before();
  __syncthreads();
  fence_after();
  wait_bar_quiet(&bars.drain, 0, p.err);
  fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(2 * BN));
}

}  // namespace gtc4

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
  const cuuint32_t box[2] = {(cuuint32_t)gtc2::BK, box_rows};
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
  int st = gemm_map(&p.amap, a, (uint64_t)K, (uint64_t)M, (uint64_t)lda, gtc2::BM);
  if (!st) st = gemm_map(&p.bmap, w, (uint64_t)K, (uint64_t)N, (uint64_t)ldw, gtc2::BN / 2);
  if (st) return st;
  // the tall-tile form unless JANUS_B200_GEMM=pair asks for the 256-row one
  const char* form = getenv("JANUS_B200_GEMM");
  const bool tall = !(form && strcmp(form, "pair") == 0);
  const int64_t rows_per_item = tall ? 4 * gtc4::BM : 2 * gtc2::BM;
  const int64_t mt = (M + rows_per_item - 1) / rows_per_item, nblk = (N + gtc2::BN - 1) / gtc2::BN;
  JB_REQUIRE(mt * nblk < (1ll << 31), JANUS_ERR_UNSUPPORTED, "gemm_bf16: too many tiles");
  p.out = (__nv_bfloat16*)out;
  p.ldo = ldo;
  p.err = status;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.nblk = (int)nblk;
  p.n_items = (int)(mt * nblk);
  p.mt = (int)mt;
  // bands of at most 48 MB of weight rows: one band's rows plus the A tiles and outputs that stream past between
  // two uses of a weight tile stay within L2 (126 MB), at the price of reading A once per band
  const int64_t w_bytes = N * K * 2, band_cap = 48ll << 20;
  const int64_t nbands = tall ? (w_bytes + band_cap - 1) / band_cap : 1;
  p.band = (int)((nblk + nbands - 1) / nbands);
  p.swiglu = epilogue;
  const size_t smem = (tall ? gtc4::kSmem : gtc2::kSmem) + 1024;
  void (*kernel)(const gtc::Params) = tall ? gtc4::gemm_bf16_tall_kernel : gtc2::gemm_bf16_pair_kernel;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    set_error("gemm_bf16: smem attribute: %s", cudaGetErrorString(e));
    return JANUS_ERR_CUDA;
  }
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 1) {
    set_error("gemm_bf16: device query failed");
    return JANUS_ERR_CUDA;
  }
  const int pairs = (int)(p.n_items < sms / 2 ? p.n_items : sms / 2);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  cfg.blockDim = dim3(tall ? gtc4::NT : gtc2::NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kernel, p);
  if (e != cudaSuccess) {
    set_error("gemm_bf16: launch: %s", cudaGetErrorString(e));
    return JANUS_ERR_CUDA;
  }
  return launch_status("gemm_bf16");
}
