// Tree attention on CTA pairs (clusters of 2, tcgen05 cta_group::2) for head dims 128 and 256: the same rule and
// arithmetic as tree_attention_tc_kernel (attn_tc.cu), with the two CTAs of a pair sharing every K/V block.
//
// A pair owns two query tiles of 128 rows (tile 2c in CTA 0, tile 2c+1 in CTA 1; rows = tokens x the G query heads of
// one kv head, row r in TMEM lane r of its CTA). The pair walks the union of the two tiles' key ranges per level in
// blocks of 128 keys, and one thread of CTA 0 issues M = 256 MMAs for both tiles:
//   S = Q K_j^T     A = Q (each CTA's TMEM), B = K_j split by keys: each CTA stages 64 keys x D dims
//   O += P_j V_j    A = P_j (each CTA's shared memory), B = V_j split by dims: each CTA stages 128 keys x D/2 dims
// so a CTA's shared memory receives half of every K and V block: its ring of 160 KB holds twice the blocks of the
// single-CTA kernel's, which gives each TMA load that much more lead, and each CTA pulls half the bytes from L2.
// TMEM per CTA as in the single-CTA kernel: O [0, D) fp32, S [256, 384) fp32, Q [384, 384 + D/2) bf16 pairs.
// Roles per CTA: warps 0-7 softmax over the CTA's own rows (identical to the single-CTA kernel: mask by the tree
// rule, running max refreshed only on growth by more than 2^8, P_j to shared memory, normalise, gate, store);
// warp 8 the TMA producer of the CTA's halves; in CTA 0, warp 9 the S issuer and warp 10 the PV issuer.
// Hand-offs across the pair: both CTAs' TMA loads complete on CTA 0's `full` barrier; the softmax warps of both CTAs
// arrive (one arrival per warp, release at cluster scope) on CTA 0's q_full / s_empty / p_full; the MMA commits arrive
// on the barriers at the same offset in both CTAs (multicast: empty, s_full, pv_done, drain). A cluster barrier after
// the barrier set-up and before the exit keeps every remote arrival inside the peer's lifetime. No TMA load uses
// multicast. Every wait is bounded: one that runs out sets the status word and the pair winds down (loads landed,
// MMAs drained, TMEM released).
//
// Measured on B200 it is the slower form (the 4B state level of 16 requests x 8192 tokens: 144 ms of attention per
// step against 106 ms for single CTAs): the deeper ring is not what bounds a block, the chain S_j -> softmax -> P_j ->
// P_j V_j is, and the pair adds a cross-CTA hand-off to two of its links (both CTAs' softmax warps must have read S_j
// before S_{j+1} is issued, and must have written P_j before P_j V_j). The host runs it only when asked
// (JANUS_B200_ATTN=pairs); outputs agree with the single-CTA form's to fp32 summation order.
#include "tcgen05.cuh"

namespace jb {
namespace tcp {
using namespace tcx;

constexpr int BM = 128, BN = 128;
constexpr int kSoftmaxThreads = 256;
constexpr int kProducerWarp = 8, kMmaSWarp = 9, kMmaPvWarp = 10;
constexpr int NT = kSoftmaxThreads + 96;
constexpr int kMaxLevels = 4;
constexpr int kMaxSegs = 2 * kMaxLevels;  // per level the two tiles' key ranges, merged when they overlap
constexpr uint32_t kRingBytes = 160 * 1024;
// an item's full barrier is re-armed for the item kItemBars later, once the ring slot of the item SLOTS later is free;
// the V items' issuer trails the K items' by up to two items, so kItemBars >= SLOTS + 4 keeps every re-arm behind the
// wait on the barrier's previous phase
constexpr int kItemBars = 16;
constexpr uint32_t kColO = 0, kColS = 256, kColQ = 384, kTmemCols = 512;
constexpr int kArrivals = 16;  // one per softmax warp of the pair

template <int D>
struct Layout {
  static constexpr uint32_t SLOT = D * 128;  // one item: K half (64 keys x D dims) or V half (128 keys x D/2 dims)
  static constexpr int SLOTS = kRingBytes / SLOT;
  static constexpr uint32_t RING = 0;
  static constexpr uint32_t P = RING + SLOTS * SLOT;  // 128 rows x 128 keys bf16: two [128 rows][64 keys] atoms
  static constexpr uint32_t BYTES = P + BM * BN * 2;
};

struct Params {
  CUtensorMap kmap[kMaxLevels], vmap[kMaxLevels];  // K boxes 64 dims x 1 head x 64 keys, V boxes ... x 128 keys
  const __nv_bfloat16* q;
  const int32_t* lo[kMaxLevels];
  const int32_t* hi[kMaxLevels];
  const int32_t* row_start;
  const int32_t* row_of_token;
  const int32_t* tiles;
  const __nv_bfloat16* gate;
  __nv_bfloat16* out;
  int32_t* err;
  int64_t gate_stride, gate_head_stride;
  int Hq, Hkv, G, n_levels, n_tiles;
  float scale_log2;
};

struct Bars {
  uint64_t full[kItemBars], empty[16], s_full, s_empty, p_full, pv_done, q_full, drain;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
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
// one arrival on CTA 0's barrier at the offset of `bar`, ordered after this thread's earlier memory operations
__device__ __forceinline__ void arrive_first(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(peer_addr(s32(bar), 0))
               : "memory");
}
// bounded wait on a barrier that the other CTA arrives on too: acquire at cluster scope
__device__ __forceinline__ bool wait_bar_cl(uint64_t* bar, uint32_t parity, int32_t* err) {
  uint32_t done = 0;
  uint64_t t0 = 0;
  for (long it = 0; !done; ++it) {
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(s32(bar)), "r"(parity)
        : "memory");
    if (!done && (it & 1023) == 1023) {
      const uint64_t now = global_ns();
      if (t0 == 0) t0 = now;
      const bool other = err && *reinterpret_cast<volatile int32_t*>(err) != 0;
      if (other || now - t0 > kWaitNs || it > kSpinLimit) break;
    }
  }
  if (!done && err) atomicExch(err, 1);
  return done != 0;
}
// TMA tile load into this CTA's shared memory, completing on CTA 0's barrier (cluster address); no multicast
__device__ __forceinline__ void tma_load3_pair(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                               uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}
// D (both CTAs' TMEM) (+)= A (both CTAs' TMEM) x B (both CTAs' shared memory halves)
__device__ __forceinline__ void mma2_ts(uint32_t tm, uint32_t ta, uint64_t db, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n}\n" ::"r"(tm),
      "r"(ta), "l"(db), "r"(id), "r"(acc), "r"(0));
}
// D (+)= A (both CTAs' shared memory) x B (both CTAs' shared memory halves)
__device__ __forceinline__ void mma2(uint32_t tm, uint64_t da, uint64_t db, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n}\n" ::"r"(tm),
      "l"(da), "l"(db), "r"(id), "r"(acc), "r"(0));
}
// completion of the MMAs issued so far, arriving on the barrier at the same offset in both CTAs of the pair
__device__ __forceinline__ void commit2(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          s32(bar)),
      "h"((uint16_t)3)
      : "memory");
}
// 32 consecutive fp32 TMEM columns of this thread's lane, waited for inside the same statement
__device__ __forceinline__ void tld32(uint32_t addr, float* f) {
  uint32_t v[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(addr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]);
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void pair_sync(int quarter) {  // the two softmax warps of a TMEM lane quarter
  asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
}

// item i of the ring sequence K_0, K_1, V_0, K_2, V_1, ..., K_{n-1}, V_{n-2}, V_{n-1} (the order the MMAs use them)
__device__ __forceinline__ bool item_is_k(int i, int n) { return i == 0 || (i % 2 == 1 && (i + 1) / 2 < n); }
__device__ __forceinline__ int item_block(int i, int n) {
  if (i == 0) return 0;
  if (i % 2 == 1 && (i + 1) / 2 < n) return (i + 1) / 2;
  return i % 2 == 0 ? i / 2 - 1 : (i - 1) / 2;
}
__device__ __forceinline__ int k_item(int j) { return j == 0 ? 0 : 2 * j - 1; }
__device__ __forceinline__ int v_item(int j, int n) { return j + 1 < n ? 2 * j + 2 : 2 * n - 1; }

template <int D>
__global__ void __launch_bounds__(NT, 1) tree_attention_pair_kernel(const __grid_constant__ Params p) {
  using Lay = Layout<D>;
  constexpr int SLOTS = Lay::SLOTS;
  static_assert(SLOTS + 4 <= kItemBars && SLOTS <= 16, "ring barriers");
  extern __shared__ unsigned char raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = s32(base);
  __shared__ Bars bars;
  __shared__ uint32_t tmem_base;
  __shared__ int s_tok[BM], s_own[BM];
  __shared__ int s_lo[kMaxLevels - 1][BM], s_hi[kMaxLevels - 1][BM];
  __shared__ int s_rng[2][kMaxLevels][2];  // [tile of the pair][level]: the tile's key range [lo, hi)
  __shared__ int s_seg_lo[kMaxSegs], s_seg_n[kMaxSegs], s_seg_lvl[kMaxSegs];
  __shared__ int s_total;
  __shared__ float s_red[2][2][BM];  // [block parity][key half][row]: partial row maxima
  __shared__ float s_sum[2][BM];     // [key half][row]: partial row sums
  __shared__ int s_ok[2][2][4];      // [block parity][key half][lane quarter]: the warp is still on track

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const int hkv = blockIdx.y;
  const int G = p.G, TQ = BM / G, L = p.n_levels;
  const int pair_tile = blockIdx.x & ~1;  // the pair's tiles: pair_tile (CTA 0) and pair_tile + 1 (CTA 1)
  auto bounds = [&](int t, int& a, int& b) {  // tiles past the list are empty (an odd count is padded)
    a = 0;
    b = 0;
    if (t < p.n_tiles) {
      a = p.tiles[2 * t];
      b = p.tiles[2 * t + 1];
      if (b - a > TQ) b = a + TQ;  // tiles longer than the kernel's tile are truncated (the host never makes them)
    }
  };
  int q0, q1;
  bounds(pair_tile + (int)rank, q0, q1);
  const int ntok = q1 - q0;

  if (tid < 2 * kMaxLevels * 2) (&s_rng[0][0][0])[tid] = (tid & 1) ? -1 : 0x7fffffff;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(&tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::);
  }
  if (tid == 32 * kProducerWarp) {
    for (int s = 0; s < kItemBars; ++s) bar_init(&bars.full[s], 1);
    for (int s = 0; s < SLOTS; ++s) bar_init(&bars.empty[s], 1);
    bar_init(&bars.s_full, 1);
    bar_init(&bars.s_empty, kArrivals);
    bar_init(&bars.p_full, kArrivals);
    bar_init(&bars.pv_done, 1);
    bar_init(&bars.q_full, kArrivals);
    bar_init(&bars.drain, 2);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid < 2 * TQ) {  // one thread per token of the pair's two tiles: the tiles' key ranges per level
    const int u = tid / TQ, x = tid % TQ;
    int a, b;
    bounds(pair_tile + u, a, b);
    const bool live = x < b - a;
    const int t = live ? a + x : 0;
    const int row = live ? p.row_of_token[t] : 0;
    if (live) {
      for (int l = 0; l < L - 1; ++l) {
        const int lo = p.lo[l][row], hi = p.hi[l][row];
        if (lo < hi) {
          atomicMin(&s_rng[u][l][0], lo);
          atomicMax(&s_rng[u][l][1], hi);
        }
      }
      atomicMin(&s_rng[u][L - 1][0], p.row_start[row]);  // the own level: the row's tokens up to this one
      atomicMax(&s_rng[u][L - 1][1], t + 1);
    }
    if (u == (int)rank) {  // this CTA's rows
      s_tok[x] = live ? t : -1;
      s_own[x] = live ? p.row_start[row] : 0;
      for (int l = 0; l < L - 1; ++l) {
        s_lo[l][x] = live ? p.lo[l][row] : 0x7fffffff;
        s_hi[l][x] = live ? p.hi[l][row] : -1;
      }
    }
  }
  __syncthreads();
  if (tid == 0) {  // the key segments both CTAs walk: per level the two ranges, merged unless that costs blocks
    int ns = 0, tot = 0;
    auto add = [&](int lo, int hi, int l) {
      s_seg_lo[ns] = lo;
      s_seg_n[ns] = (hi - lo + BN - 1) / BN;
      s_seg_lvl[ns] = l;
      tot += s_seg_n[ns];
      ++ns;
    };
    for (int l = 0; l < L; ++l) {
      const int a0 = s_rng[0][l][0], b0 = s_rng[0][l][1], a1 = s_rng[1][l][0], b1 = s_rng[1][l][1];
      const bool e0 = a0 >= b0, e1 = a1 >= b1;
      if (e0 && e1) continue;
      if (e0 || e1) {
        add(e0 ? a1 : a0, e0 ? b1 : b0, l);
        continue;
      }
      const int lo = min(a0, a1), hi = max(b0, b1);
      const int merged = (hi - lo + BN - 1) / BN, apart = (b0 - a0 + BN - 1) / BN + (b1 - a1 + BN - 1) / BN;
      if (merged <= apart) {
        add(lo, hi, l);
      } else if (a0 <= a1) {
        add(a0, b0, l);
        add(a1, b1, l);
      } else {
        add(a1, b1, l);
        add(a0, b0, l);
      }
    }
    for (int s = ns; s < kMaxSegs; ++s) s_seg_n[s] = 0x7fffffff;  // a walk never passes the last segment
    s_total = tot;
  }
  fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote arrival or complete_tx
  fence_after();
  const uint32_t tm = tmem_base;
  const int total = s_total;
  const int n_items = 2 * total;

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      for (int i = 0; i < n_items && ok; ++i) {
        const bool is_k = item_is_k(i, total);
        int blk = item_block(i, total), seg = 0;
        while (blk >= s_seg_n[seg]) {
          blk -= s_seg_n[seg];
          ++seg;
        }
        const int lvl = s_seg_lvl[seg];
        const int ks = s_seg_lo[seg] + blk * BN;
        const int slot = i % SLOTS;
        if (i >= SLOTS) ok = wait_bar(&bars.empty[slot], (i / SLOTS - 1) & 1, p.err);  // its MMAs are done
        if (!ok) break;
        uint64_t* fb = &bars.full[i % kItemBars];
        if (rank == 0) bar_expect_tx(fb, 2 * Lay::SLOT);  // both CTAs' halves
        const uint32_t fba = peer_addr(s32(fb), 0);
        const uint32_t dst = sbase + Lay::RING + slot * Lay::SLOT;
        if (is_k) {  // keys ks + 64 rank .. +63, every head dim: D/64 boxes of [64 keys][64 dims]
#pragma unroll
          for (int a = 0; a < D / 64; ++a)
            tma_load3_pair(dst + a * 8192, &p.kmap[lvl], a * 64, hkv, ks + 64 * (int)rank, fba);
        } else {  // head dims D/2 rank .. +D/2-1 of keys ks .. +127: D/128 boxes of [128 keys][64 dims]
#pragma unroll
          for (int a = 0; a < D / 128; ++a)
            tma_load3_pair(dst + a * 16384, &p.vmap[lvl], (D / 2) * (int)rank + a * 64, hkv, ks, fba);
        }
        issued = i + 1;
      }
      // every issued load has landed before the CTA may leave: CTA 0's full barriers count both CTAs' bytes; CTA 1
      // waits for the MMAs that read its last slots
      if (rank == 0) {
        for (int i = issued - kItemBars < 0 ? 0 : issued - kItemBars; i < issued; ++i)
          wait_bar_quiet(&bars.full[i % kItemBars], (i / kItemBars) & 1, p.err);
      } else {
        for (int i = issued - SLOTS < 0 ? 0 : issued - SLOTS; i < issued; ++i)
          wait_bar_quiet(&bars.empty[i % SLOTS], (i / SLOTS) & 1, p.err);
      }
    }
  } else if (warp == kMmaSWarp) {
    // ------------------------------------------------------------------------------- S issuer (CTA 0)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t ID_S = idesc(2 * BM, BN, 0, 0);
      bool ok = wait_bar_cl(&bars.q_full, 0, p.err);
      for (int j = 0; j < total && ok; ++j) {
        const int item = k_item(j);
        if (j > 0) ok = wait_bar_cl(&bars.s_empty, (j - 1) & 1, p.err);  // both CTAs read S_{j-1}
        ok = ok && wait_bar_cl(&bars.full[item % kItemBars], (item / kItemBars) & 1, p.err);
        if (!ok) break;
        fence_after();
        const uint32_t kb = sbase + Lay::RING + (item % SLOTS) * Lay::SLOT;
#pragma unroll
        for (int s = 0; s < D / 16; ++s)  // 16 head dims per step
          mma2_ts(tm + kColS, tm + kColQ + s * 8, sdesc(kb + (s >> 2) * 8192 + (s & 3) * 32, 16, 1024), ID_S,
                  s ? 1u : 0u);
        commit2(&bars.empty[item % SLOTS]);
        commit2(&bars.s_full);
      }
      commit2(&bars.drain);  // completes once every MMA issued by this thread has finished
    }
  } else if (warp == kMmaPvWarp) {
    // ------------------------------------------------------------------------------ PV issuer (CTA 0)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t ID_PV = idesc(2 * BM, D, 0, 1);
      bool ok = true;
      for (int j = 0; j < total && ok; ++j) {
        const int item = v_item(j, total);
        ok = wait_bar_cl(&bars.p_full, j & 1, p.err) &&
             wait_bar_cl(&bars.full[item % kItemBars], (item / kItemBars) & 1, p.err);
        if (!ok) break;
        fence_after();
        const uint32_t vb = sbase + Lay::RING + (item % SLOTS) * Lay::SLOT;
#pragma unroll
        for (int s = 0; s < BN / 16; ++s)  // 16 keys per step; O[:, every dim] += P_j V_j
          mma2(tm + kColO, sdesc(sbase + Lay::P + (s >> 2) * (BM * 128) + (s & 3) * 32, 16, 1024),
               sdesc(vb + s * 16 * 128, 16384, 1024), ID_PV, (j > 0 || s > 0) ? 1u : 0u);
        commit2(&bars.empty[item % SLOTS]);
        commit2(&bars.pv_done);
      }
      commit2(&bars.drain);
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------------------------------------ softmax warps
    constexpr int HC = BN / 2, HD = D / 2;
    const int quarter = warp & 3, half = warp >> 2;
    const int r = 32 * quarter + lane;  // query row = TMEM lane
    const int tq = r / G;
    const uint32_t lane_addr = tm + ((uint32_t)(32 * quarter) << 16);
    {  // this warp's half of the Q row into TMEM (bf16 pairs, even dim in the low half)
      const bool live = tq < ntok;
      const __nv_bfloat16* qr = p.q + ((int64_t)(live ? q0 + tq : 0) * p.Hq + hkv * G + r % G) * D + half * HD;
      uint32_t v[HD / 2];
#pragma unroll
      for (int i = 0; i < HD / 2; i += 4) {
        const uint4 x = live ? *reinterpret_cast<const uint4*>(qr + 2 * i) : make_uint4(0, 0, 0, 0);
        v[i] = x.x;
        v[i + 1] = x.y;
        v[i + 2] = x.z;
        v[i + 3] = x.w;
      }
#pragma unroll
      for (int c = 0; c < HD / 2; c += 16) tst16(lane_addr + kColQ + half * (HD / 2) + c, v + c);
      tst_wait();
      fence_before();
      __syncwarp();
      if (lane == 0) arrive_first(&bars.q_full);
    }
    const float sc = p.scale_log2;
    float m_used = -INFINITY, l_sum = 0.f;
    bool ok = true;  // warp-uniform; the two warps of a pair agree on it at every pair barrier
    int seg = 0, b = 0;
    for (int j = 0; j < total; ++j, ++b) {
      while (b >= s_seg_n[seg]) {
        b = 0;
        ++seg;
      }
      const int lvl = s_seg_lvl[seg];
      const int ks = s_seg_lo[seg] + b * BN + half * HC;  // first key of this warp's columns
      int lo, hi;
      if (tq >= ntok) {
        lo = 0;
        hi = -1;
      } else if (lvl == L - 1) {
        lo = s_own[tq];
        hi = s_tok[tq] + 1;
      } else {
        lo = s_lo[lvl][tq];
        hi = s_hi[lvl][tq];
      }
      const bool mine = ok && __all_sync(kFull, wait_bar(&bars.s_full, j & 1, p.err));
      float s[HC], mx = -INFINITY;
      if (mine) {
        fence_after();
        tld32(lane_addr + kColS + half * HC, s);
        tld32(lane_addr + kColS + half * HC + 32, s + 32);
        fence_before();
        __syncwarp();
        if (lane == 0) arrive_first(&bars.s_empty);  // S may be overwritten by the next block's scores
        if (!(ks >= lo && ks + HC <= hi)) {  // not every column of this half is visible to this row
#pragma unroll
          for (int c = 0; c < HC; ++c) {
            const int kk = ks + c;
            s[c] = (kk >= lo && kk < hi) ? s[c] : -INFINITY;
          }
        }
        float mx4[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
        for (int c = 4; c < HC; c += 4)
#pragma unroll
          for (int i = 0; i < 4; ++i) mx4[i] = fmaxf(mx4[i], s[c + i]);
        mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      }
      // exchange the half-row maxima (and whether both warps are still on track) with the partner warp
      const int par = j & 1;
      s_red[par][half][r] = mx;
      if (lane == 0) s_ok[par][half][quarter] = mine;
      pair_sync(quarter);
      ok = mine && s_ok[par][half ^ 1][quarter];
      if (!ok) break;
      mx = fmaxf(mx, s_red[par][half ^ 1][r]) * sc;
      const bool grow = mx > m_used + 8.f;
      const float m_new = grow ? mx : m_used;
      const bool rescale = grow && m_used != -INFINITY;
      const float alpha = rescale ? exp2f(m_used - m_new) : 1.f;
      l_sum *= alpha;
      m_used = m_new;
      const float mref = m_used == -INFINITY ? 0.f : m_used;
      uint32_t pk[HC / 2];
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < HC; c += 2) {
        const float e0 = ex2(fmaf(s[c], sc, -mref)), e1 = ex2(fmaf(s[c + 1], sc, -mref));
        ls[(c >> 1) & 3] += e0 + e1;
        pk[c / 2] = pack_bf16(e0, e1);
      }
      l_sum += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      if (j > 0) ok = __all_sync(kFull, wait_bar(&bars.pv_done, (j - 1) & 1, p.err));  // P free, O final
      if (ok) {  // (a wait that ran out is handed to the partner at the next pair barrier)
        fence_after();
        if (__any_sync(kFull, rescale)) {
#pragma unroll 1
          for (int c = 0; c < HD; c += 16) {
            float o[16];
            tld16f(lane_addr + kColO + half * HD + c, o);
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] *= alpha;
            tst16f(lane_addr + kColO + half * HD + c, o);
          }
          tst_wait();  // the rescaled O is in TMEM before the next P V accumulates onto it
        }
        unsigned char* prow = base + Lay::P + half * (BM * 128) + r * 128;  // atom `half`: keys half*64 ..
#pragma unroll
        for (int c = 0; c < HC / 8; ++c)
          *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) =
              make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        fence_async_smem();
        fence_before();
        __syncwarp();
        if (lane == 0) arrive_first(&bars.p_full);
      }
    }
    if (total > 0 && ok) ok = __all_sync(kFull, wait_bar(&bars.pv_done, (total - 1) & 1, p.err));
    fence_after();
    // the row's normaliser: this half's sum plus the partner's (both warps reach this barrier exactly once)
    s_sum[half][r] = l_sum;
    pair_sync(quarter);
    l_sum += s_sum[half ^ 1][r];
    // epilogue: warp-collective TMEM loads of this warp's half of O, stores by the live rows
    if (__all_sync(kFull, ok)) {
      const bool live = tq < ntok;
      const int g = r % G;
      const int64_t t = live ? q0 + tq : 0;
      const int h = hkv * G + g;
      const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
      const __nv_bfloat16* gr = p.gate + t * p.gate_stride + (int64_t)h * p.gate_head_stride + half * HD;
      __nv_bfloat16* orow = p.out + (t * p.Hq + h) * D + half * HD;
      bf16x8 gate[HD / 8];
#pragma unroll
      for (int c = 0; c < HD / 8; ++c) gate[c] = live ? *reinterpret_cast<const bf16x8*>(gr + 8 * c) : bf16x8{};
#pragma unroll
      for (int c = 0; c < HD; c += 16) {
        float o[16];
        tld16f(lane_addr + kColO + half * HD + c, o);
        if (live) {
          float res[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const __nv_bfloat162 gp = gate[(c + i) / 8].h[((c + i) % 8) / 2];
            const float gv = (i & 1) ? __high2float(gp) : __low2float(gp);
            res[i] = o[i] * inv * sigmoidf_(gv);
          }
          store8(orow + c, res);
          store8(orow + c + 8, res + 8);
        }
      }
    }
  }
  // wind down: the pair's MMAs have completed (drain, multicast) before either CTA releases TMEM, and neither CTA
  // leaves while the other may still arrive on its barriers or complete loads on them
  fence_before();
  __syncthreads();
  fence_after();
  wait_bar_quiet(&bars.drain, 0, p.err);
  fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(kTmemCols));
}

// ------------------------------------------------------------------------------------------------ host side

// K or V of one level: [T keys][Hkv][D] bf16, boxes of 64 dims x 1 head x box_keys keys, 128B swizzle; keys past T
// read as zeros (and are masked)
static int make_map(CUtensorMap* map, const void* ptr, int64_t T, int64_t Hkv, int64_t D, uint32_t box_keys) {
  EncodeTiled enc = encode_tiled_fn();
  if (!enc) {
    set_error("tree_attention(pairs): cuTensorMapEncodeTiled unavailable");
    return JANUS_ERR_CUDA;
  }
  const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)Hkv, (cuuint64_t)T};
  const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)(Hkv * D * 2)};
  const cuuint32_t box[3] = {64, 1, box_keys};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("tree_attention(pairs): cuTensorMapEncodeTiled failed (%d)", (int)r);
    return JANUS_ERR_INVALID;
  }
  return JANUS_OK;
}

template <int D>
int launch(const Params& p, cudaStream_t s) {
  const size_t smem = Layout<D>::BYTES + 1024;
  cudaError_t e =
      cudaFuncSetAttribute(tree_attention_pair_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    set_error("tree_attention(pairs): smem attribute %s", cudaGetErrorString(e));
    return JANUS_ERR_CUDA;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(2 * ((p.n_tiles + 1) / 2)), (unsigned)p.Hkv);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, tree_attention_pair_kernel<D>, p);
  if (e != cudaSuccess) {
    set_error("tree_attention(pairs): launch %s", cudaGetErrorString(e));
    return JANUS_ERR_CUDA;
  }
  return launch_status("tree_attention(pairs)");
}

}  // namespace tcp

int tree_attention_pair(const void* q, int64_t Hq, int64_t Hkv, int64_t D, int32_t n_levels,
                        const void* const* k_levels, const void* const* v_levels, const int64_t* level_tokens,
                        const int32_t* const* anc_lo, const int32_t* const* anc_hi, const int32_t* row_start,
                        const int32_t* row_of_token, const int32_t* tiles, int64_t n_tiles, const void* gate,
                        int64_t gate_stride, int64_t gate_head_stride, float scale, void* out, int32_t* err,
                        cudaStream_t stream) {
  JB_REQUIRE(n_levels >= 1 && n_levels <= tcp::kMaxLevels && n_tiles < (1ll << 30) && Hkv <= 65535,
             JANUS_ERR_INVALID, "tree_attention(pairs): %d levels, %lld tiles", (int)n_levels, (long long)n_tiles);
  tcp::Params p{};
  for (int l = 0; l < n_levels; ++l) {
    if (level_tokens[l] > 0) {  // an empty level is never read (every row's range on it is empty)
      int st = tcp::make_map(&p.kmap[l], k_levels[l], level_tokens[l], Hkv, D, 64);
      if (!st) st = tcp::make_map(&p.vmap[l], v_levels[l], level_tokens[l], Hkv, D, 128);
      if (st) return st;
    }
    if (l < n_levels - 1) {
      p.lo[l] = anc_lo[l];
      p.hi[l] = anc_hi[l];
    }
  }
  p.q = (const __nv_bfloat16*)q;
  p.row_start = row_start;
  p.row_of_token = row_of_token;
  p.tiles = tiles;
  p.gate = (const __nv_bfloat16*)gate;
  p.out = (__nv_bfloat16*)out;
  p.err = err;
  p.gate_stride = gate_stride;
  p.gate_head_stride = gate_head_stride;
  p.Hq = (int)Hq;
  p.Hkv = (int)Hkv;
  p.G = (int)(Hq / Hkv);
  p.n_levels = n_levels;
  p.n_tiles = (int)n_tiles;
  p.scale_log2 = scale * 1.4426950408889634f;
  if (n_tiles == 0) return JANUS_OK;
  if (D == 256) return tcp::launch<256>(p, stream);
  if (D == 128) return tcp::launch<128>(p, stream);
  set_error("tree_attention(pairs): head dim %lld", (long long)D);
  return JANUS_ERR_UNSUPPORTED;
}

}  // namespace jb
