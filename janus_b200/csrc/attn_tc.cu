// Tree attention on the 5th-generation tensor cores (tcgen05, accumulators in TMEM) for head dims 128 and 256.
//
// A CTA owns one kv head and 128 query rows = (128 / G) tokens x G query heads (GQA folded into M): row r lives in
// TMEM lane r. Keys go in blocks of 128 (the MMA shape M=128 x N=128 runs at the full tensor rate; N=64 at half).
// TMEM (512 columns): O [0, D) fp32, S [256, 384) fp32 (one block of scores), Q [384, 384 + D/2) bf16 pairs; Q is
// the A operand of S = Q K^T straight from TMEM, so shared memory holds only K/V and P. Four roles, eleven warps:
//   warps 0-7  softmax, two warps per TMEM lane quarter (warp w: rows 32*(w%4).., key half w/4 of every S block and
//              column half w/4 of O): write the Q rows into TMEM; per block read S_j, mask it by the tree rule
//              (ancestor key ranges, own row causal), agree with the partner warp on the row max (shared memory + a
//              64-thread named barrier), compute P_j = exp2(S_j*c - m) in registers, then (once P_{j-1} V_{j-1} is
//              done) rescale O when needed and write P_j to shared memory (bf16, K-major, 128B-swizzled); at the end
//              normalise, gate and store O;
//   warp 8     producer: TMA loads (no multicast) of K/V into a ring of 5 slots of 128 keys x 128 head dims
//              (128B swizzle, zero fill past the level's end), in the order the MMAs consume them:
//              K_0, K_1, V_0, K_2, V_1, ..., V_{n-1} (a K or V block is D/128 slots);
//   warp 9     S issuer (one thread): S_{j+1} = Q K_{j+1}^T as soon as S_j has been read and K_{j+1} landed;
//   warp 10    PV issuer (one thread): O += P_j V_j (two N=128 halves, V as the MN-major operand) once P_j is
//              written and V_j landed. An mbarrier wait idles its issuing thread for a few hundred cycles; with two
//              issuers the tensor pipe runs one's MMAs while the other waits, and it computes S_{j+1} while the
//              softmax warps work on block j. Each ring slot is released by a tcgen05.commit after the MMAs that
//              read it; one full barrier covers all slots of a K/V item.
// The running max m is refreshed only when a row's max grows by more than 2^8 (the row's O is then rescaled in
// TMEM), so P stays <= 256 and the normaliser l uses the same m: the exact softmax. Every mbarrier wait is bounded;
// a wait that runs out sets the status word and the CTA winds down (its TMA loads and MMAs drained first).
#include "tcgen05.cuh"

namespace jb {
namespace tc {
using namespace tcx;

constexpr int BM = 128, BN = 128;
constexpr int kSoftmaxThreads = 256;              // 8 softmax warps: two per TMEM lane quarter
constexpr int kProducerWarp = 8, kMmaSWarp = 9, kMmaPvWarp = 10;
constexpr int NT = kSoftmaxThreads + 96;          // + 1 producer warp + 2 MMA-issuing warps
constexpr int kMaxLevels = 4;
constexpr int kSlots = 5;                         // K/V ring slots
constexpr uint32_t kSlotBytes = BN * 128 * 2;     // 128 keys x 128 head dims (two [128 keys][64 dims] TMA boxes)
constexpr uint32_t kBoxBytes = BN * 128;          // one [128 keys][64 dims] box: 16 KB
constexpr int kItemBars = 9;                      // >= the K/V items in flight (at most kSlots) + 4: the V
                                                  // items' issuer trails the K items' by up to two items
constexpr uint32_t kColO = 0, kColS = 256, kColQ = 384, kTmemCols = 512;

struct Params {
  CUtensorMap kmap[kMaxLevels], vmap[kMaxLevels];  // [T_l keys][Hkv][D] bf16, box 64 dims x 1 head x 128 keys
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
  int Hq, Hkv, G, n_levels;
  float scale_log2;
};

// 32 consecutive fp32 TMEM columns of this thread's lane, waited for inside the same statement
__device__ __forceinline__ void tld32(uint32_t addr, float* f) {
  uint32_t v[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
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
__device__ __forceinline__ float ex2(float x) {  // 2^x on the MUFU unit, flush-to-zero (irrelevant for weights)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// named barrier of the two softmax warps that share a TMEM lane quarter
__device__ __forceinline__ void pair_sync(int quarter) {
  asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
}

template <int D>
struct Layout {
  static constexpr int SPT = D / 128;                      // ring slots per K or V block
  static constexpr uint32_t RING = 0;                      // kSlots x 32 KB
  static constexpr uint32_t P = RING + kSlots * kSlotBytes;  // 128 rows x 128 keys: two [128 rows][64 keys] atoms
  static constexpr uint32_t BYTES = P + BM * BN * 2;
};

// full[i % kItemBars]: K/V item i (all its slots) has landed; empty[slot]: the MMAs reading a ring slot are done
struct Bars {
  uint64_t full[kItemBars], empty[kSlots], s_full, s_empty, p_full, pv_done, q_full, drain;
};

// The ring position sequence shared by the producer and the MMA issuer: block item i (0-based) of
// K_0, K_1, V_0, K_2, V_1, ..., K_{n-1}, V_{n-2}, V_{n-1} is K_{kv_block(i)} when is_k(i); each item is SPT slots.
__device__ __forceinline__ bool item_is_k(int i, int n) { return i == 0 || (i % 2 == 1 && (i + 1) / 2 < n); }
__device__ __forceinline__ int item_block(int i, int n) {
  if (i == 0) return 0;
  if (i % 2 == 1 && (i + 1) / 2 < n) return (i + 1) / 2;  // K_{(i+1)/2}
  // V blocks: V_j follows K_{j+1} (item 2j+2) while there is a K_{j+1}; after the last K they run in order
  return i % 2 == 0 ? i / 2 - 1 : (i - 1) / 2;
}

// the item indices of K_j and V_j in that sequence
__device__ __forceinline__ int k_item(int j) { return j == 0 ? 0 : 2 * j - 1; }
__device__ __forceinline__ int v_item(int j, int n) { return j + 1 < n ? 2 * j + 2 : 2 * n - 1; }

template <int D>
__global__ void __launch_bounds__(NT, 1) tree_attention_tc_kernel(const __grid_constant__ Params p) {
  using Lay = Layout<D>;
  constexpr int SPT = Lay::SPT;
  extern __shared__ unsigned char raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = s32(base);
  __shared__ Bars bars;
  __shared__ uint32_t tmem_base;
  __shared__ int s_tok[BM], s_own[BM];
  __shared__ int s_lo[kMaxLevels - 1][BM], s_hi[kMaxLevels - 1][BM];
  __shared__ int s_klo[kMaxLevels], s_nblk[kMaxLevels];
  __shared__ float s_red[2][2][BM];  // [block parity][key half][row]: partial row maxima
  __shared__ float s_sum[2][BM];     // [key half][row]: partial row sums
  __shared__ int s_ok[2][2][4];      // [block parity][key half][lane quarter]: the warp is still on track

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hkv = blockIdx.y;
  const int G = p.G, TQ = BM / G, L = p.n_levels;
  const int q0 = p.tiles[2 * blockIdx.x];
  int ntok = p.tiles[2 * blockIdx.x + 1] - q0;
  if (ntok > TQ) ntok = TQ;  // tiles longer than the kernel's tile are truncated (the host never makes them)
  const int q1 = q0 + ntok;

  if (tid < TQ) {
    const bool live = tid < ntok;
    const int t = live ? q0 + tid : q0;
    const int row = p.row_of_token[t];
    s_tok[tid] = live ? t : -1;
    s_own[tid] = p.row_start[row];
    for (int l = 0; l < L - 1; ++l) {
      s_lo[l][tid] = live ? p.lo[l][row] : 0x7fffffff;
      s_hi[l][tid] = live ? p.hi[l][row] : -1;
    }
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(&tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  if (tid == 32 * kProducerWarp) {
    for (int s = 0; s < kItemBars; ++s) bar_init(&bars.full[s], 1);
    for (int s = 0; s < kSlots; ++s) bar_init(&bars.empty[s], 1);
    bar_init(&bars.s_full, 1);
    bar_init(&bars.s_empty, kSoftmaxThreads);
    bar_init(&bars.p_full, kSoftmaxThreads);
    bar_init(&bars.pv_done, 1);
    bar_init(&bars.q_full, kSoftmaxThreads);
    bar_init(&bars.drain, 2);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0) {
    for (int l = 0; l < L - 1; ++l) {
      int a = 0x7fffffff, b = -1;
      for (int tq = 0; tq < ntok; ++tq) {
        a = min(a, s_lo[l][tq]);
        b = max(b, s_hi[l][tq]);
      }
      s_klo[l] = a < b ? a : 0;
      s_nblk[l] = a < b ? (b - a + BN - 1) / BN : 0;
    }
    s_klo[L - 1] = s_own[0];
    s_nblk[L - 1] = (q1 - s_own[0] + BN - 1) / BN;
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tm = tmem_base;
  int total = 0;
  for (int l = 0; l < L; ++l) total += s_nblk[l];
  const int n_items = 2 * total;

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      int issued = 0;  // items whose loads went out
      for (int i = 0; i < n_items && ok; ++i) {
        const bool is_k = item_is_k(i, total);
        int blk = item_block(i, total), lvl = 0;
        while (blk >= s_nblk[lvl]) {
          blk -= s_nblk[lvl];
          ++lvl;
        }
        const int ks = s_klo[lvl] + blk * BN;
        const CUtensorMap* map = is_k ? &p.kmap[lvl] : &p.vmap[lvl];
        for (int h = 0; h < SPT && ok; ++h) {  // every slot of the item is free
          const int pos = i * SPT + h;
          if (pos >= kSlots) ok = wait_bar(&bars.empty[pos % kSlots], (pos / kSlots - 1) & 1, p.err);
        }
        if (!ok) break;
        uint64_t* fb = &bars.full[i % kItemBars];
        bar_expect_tx(fb, SPT * kSlotBytes);
        for (int h = 0; h < SPT; ++h) {
          const uint32_t dst = sbase + Lay::RING + ((i * SPT + h) % kSlots) * kSlotBytes;
          tma_load3(dst, map, h * 128, hkv, ks, fb);
          tma_load3(dst + kBoxBytes, map, h * 128 + 64, hkv, ks, fb);
        }
        issued = i + 1;
      }
      // every issued load has landed before the CTA may leave (no-ops on the normal path: all consumed)
      for (int i = issued - kItemBars < 0 ? 0 : issued - kItemBars; i < issued; ++i)
        wait_bar_quiet(&bars.full[i % kItemBars], (i / kItemBars) & 1, p.err);
    }
  } else if (warp == kMmaSWarp) {
    // ------------------------------------------------------------------------------------------ S issuer
    // Two issuing threads, one for S and one for PV: any mbarrier wait of an issuing thread idles it for a few
    // hundred cycles, and with two of them the tensor pipe runs one's MMAs while the other waits.
    if (lane == 0) {
      constexpr uint32_t ID_QK = idesc(BM, BN, 0, 0);
      bool ok = wait_bar(&bars.q_full, 0, p.err);
      for (int j = 0; j < total && ok; ++j) {
        const int item = k_item(j);
        if (j > 0) ok = wait_bar(&bars.s_empty, (j - 1) & 1, p.err);  // S_{j-1} has been read
        ok = ok && wait_bar(&bars.full[item % kItemBars], (item / kItemBars) & 1, p.err);
        if (!ok) break;
        fence_after();
        for (int h = 0; h < SPT; ++h) {
          const int slot = (item * SPT + h) % kSlots;
          const uint32_t kb = sbase + Lay::RING + slot * kSlotBytes;
#pragma unroll
          for (int s = 0; s < 8; ++s)  // 16 head dims per step: dims h*128 + 16 s
            mma_ts(tm + kColS, tm + kColQ + (h * 8 + s) * 8, sdesc(kb + (s >> 2) * kBoxBytes + (s & 3) * 32, 16, 1024),
                   ID_QK, (h | s) ? 1u : 0u);
          commit(&bars.empty[slot]);
        }
        commit(&bars.s_full);
      }
      commit(&bars.drain);  // completes once every MMA issued by this thread has finished
    }
  } else if (warp == kMmaPvWarp) {
    // ------------------------------------------------------------------------------------------ PV issuer
    if (lane == 0) {
      constexpr uint32_t ID_PV = idesc(BM, 128, 0, 1);
      bool ok = true;
      for (int j = 0; j < total && ok; ++j) {
        const int item = v_item(j, total);
        ok = wait_bar(&bars.p_full, j & 1, p.err) &&
             wait_bar(&bars.full[item % kItemBars], (item / kItemBars) & 1, p.err);
        if (!ok) break;
        fence_after();
        for (int h = 0; h < SPT; ++h) {  // O[:, h*128 ..] += P_j V_j[:, h*128 ..]
          const int slot = (item * SPT + h) % kSlots;
          const uint32_t vb = sbase + Lay::RING + slot * kSlotBytes;
#pragma unroll
          for (int s = 0; s < BN / 16; ++s)  // 16 keys per step
            mma(tm + kColO + h * 128, sdesc(sbase + Lay::P + (s >> 2) * (BM * 128) + (s & 3) * 32, 16, 1024),
                sdesc(vb + s * 16 * 128, kBoxBytes, 1024), ID_PV, (j > 0 || s > 0) ? 1u : 0u);
          commit(&bars.empty[slot]);
        }
        commit(&bars.pv_done);
      }
      commit(&bars.drain);
    }
  } else {
    // ------------------------------------------------------------------------------------------ softmax warps
    constexpr int HC = BN / 2, HD = D / 2;
    const int quarter = warp & 3, half = warp >> 2;
    const int r = 32 * quarter + lane;  // query row = TMEM lane
    const int tq = r / G;
    const uint32_t lane_addr = tm + ((uint32_t)(32 * quarter) << 16);
    {  // this warp's half of the Q row into TMEM (bf16 pairs, even dim in the low half)
      const bool live = tq < ntok;
      const __nv_bfloat16* qr = p.q + ((int64_t)(live ? q0 + tq : q0) * p.Hq + hkv * G + r % G) * D + half * HD;
      uint32_t v[HD / 2];  // every load before the first TMEM store (which orders after all earlier memory ops)
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
      bar_arrive(&bars.q_full);
    }
    const float sc = p.scale_log2;
    float m_used = -INFINITY, l_sum = 0.f;
    bool ok = true;  // warp-uniform; the two warps of a pair agree on it at every pair barrier
    int lvl = 0, b = 0;
    for (int j = 0; j < total; ++j, ++b) {
      while (b >= s_nblk[lvl]) {
        b = 0;
        ++lvl;
      }
      const int ks = s_klo[lvl] + b * BN + half * HC;  // first key of this warp's columns
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
        bar_arrive(&bars.s_empty);  // S may be overwritten by the next block's scores
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
        bar_arrive(&bars.p_full);
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
      const int64_t t = q0 + (live ? tq : 0);
      const int h = hkv * G + g;
      const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
      const __nv_bfloat16* gr = p.gate + t * p.gate_stride + (int64_t)h * p.gate_head_stride + half * HD;
      __nv_bfloat16* orow = p.out + (t * p.Hq + h) * D + half * HD;
      // the whole gate row first: the output stores could alias it as far as the compiler knows, so loads issued
      // between them would each wait for the one before
      bf16x8 gate[HD / 8];
#pragma unroll
      for (int c = 0; c < HD / 8; ++c)
        gate[c] = live ? *reinterpret_cast<const bf16x8*>(gr + 8 * c) : bf16x8{};
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
  // wind down: the producer has seen its last loads land; every MMA issued has completed before TMEM is released
  fence_before();
  __syncthreads();
  fence_after();
  wait_bar_quiet(&bars.drain, 0, p.err);
  fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(kTmemCols));
}

// Self-test of the bounded wait used above: one thread waits on an mbarrier phase that nothing completes; the
// wait gives up after kWaitNs, sets the status word and the kernel returns (no trap, no fault; the context stays
// usable).
__global__ void wait_timeout_selftest_kernel(int32_t* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    bar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    wait_bar(&bar, 0, status);  // phase 0 never completes: nobody arrives
  }
}

// ------------------------------------------------------------------------------------------------ host side

// K or V of one level: [T keys][Hkv][D] bf16, boxes of 64 dims x 1 head x 128 keys, 128B swizzle; keys past T
// read as zeros (and are masked)
static int make_kv_map(CUtensorMap* map, const void* ptr, int64_t T, int64_t Hkv, int64_t D) {
  EncodeTiled enc = encode_tiled_fn();
  if (!enc) {
    set_error("tree_attention(tcgen05): cuTensorMapEncodeTiled unavailable");
    return JANUS_ERR_CUDA;
  }
  const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)Hkv, (cuuint64_t)T};
  const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)(Hkv * D * 2)};
  const cuuint32_t box[3] = {64, 1, (cuuint32_t)BN};  // 64 dims x 1 head x 128 keys
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("tree_attention(tcgen05): cuTensorMapEncodeTiled failed (%d)", (int)r);
    return JANUS_ERR_INVALID;
  }
  return JANUS_OK;
}

template <int D>
int launch(const Params& p, int64_t n_tiles, cudaStream_t s) {
  const size_t smem = Layout<D>::BYTES + 1024;
  cudaError_t e =
      cudaFuncSetAttribute(tree_attention_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    set_error("tree_attention(tcgen05): smem attribute %s", cudaGetErrorString(e));
    return JANUS_ERR_CUDA;
  }
  dim3 grid((unsigned)n_tiles, (unsigned)p.Hkv);
  tree_attention_tc_kernel<D><<<grid, NT, smem, s>>>(p);
  return launch_status("tree_attention(tcgen05)");
}

}  // namespace tc

int wait_timeout_selftest(int32_t* status, cudaStream_t stream) {
  tc::wait_timeout_selftest_kernel<<<1, 32, 0, stream>>>(status);
  return launch_status("wait_timeout_selftest");
}

int tree_attention_tc(const void* q, int64_t Hq, int64_t Hkv, int64_t D, int32_t n_levels, const void* const* k_levels,
                      const void* const* v_levels, const int64_t* level_tokens, const int32_t* const* anc_lo,
                      const int32_t* const* anc_hi, const int32_t* row_start, const int32_t* row_of_token,
                      const int32_t* tiles, int64_t n_tiles, const void* gate, int64_t gate_stride,
                      int64_t gate_head_stride, float scale, void* out, int32_t* err, cudaStream_t stream) {
  tc::Params p{};
  for (int l = 0; l < n_levels; ++l) {
    if (level_tokens[l] > 0) {  // an empty level is never read (every row's range on it is empty)
      int st = tc::make_kv_map(&p.kmap[l], k_levels[l], level_tokens[l], Hkv, D);
      if (!st) st = tc::make_kv_map(&p.vmap[l], v_levels[l], level_tokens[l], Hkv, D);
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
  p.scale_log2 = scale * 1.4426950408889634f;
  if (D == 256) return tc::launch<256>(p, n_tiles, stream);
  if (D == 128) return tc::launch<128>(p, n_tiles, stream);
  set_error("tree_attention(tcgen05): head dim %lld", (long long)D);
  return JANUS_ERR_UNSUPPORTED;
}

}  // namespace jb
