// Tree attention on the 5th-generation tensor cores (tcgen05, accumulators in TMEM) for head dims 128 and 256.
//
// A CTA owns one kv head and 128 query rows = (128 / G) tokens x G query heads (GQA folded into M), one row per
// softmax thread: row r lives in TMEM lane r, so the softmax of a row is thread-local. Three roles, six warps:
//   warps 0-3  softmax: read S_j from TMEM, mask it by the tree rule (ancestor key ranges, own row causal),
//              compute P_j = exp2(S_j*c - m) in registers, then (once O_{j-1} is final) rescale O when needed and
//              write P_j to shared memory (bf16, K-major, 128B-swizzled); at the end normalise, gate and store O;
//   warp 4     producer: TMA loads of the K_j and V_j tiles (64 keys x D, 128B swizzle, zero fill past the level's
//              end) into two-stage rings;
//   warp 5     MMA issuer (one thread): S_j = Q K_j^T into one of two TMEM S buffers (M=128, N=64), and
//              O += P_j V_j (M=128, N=D, V as the MN-major operand) into the D TMEM columns of O.
// Hand-offs are mbarriers: TMA completion (expect-tx), tcgen05.commit for MMA completion, thread arrivals for the
// softmax. The MMA thread issues S_{j+1} before it waits for P_j, so the tensor core computes the next scores while
// the softmax warps work on the current ones, and the exponentials of block j overlap P_{j-1} V_{j-1}.
// The running max m is refreshed only when a row's max grows by more than 2^8 (the row's O is then rescaled in
// TMEM), so P stays <= 256 and the normaliser l uses the same m: the exact softmax. Every mbarrier wait is bounded;
// a wait that runs out sets the status word and the CTA winds down (its TMA loads and MMAs drained first).
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace jb {
namespace tc {

constexpr int BM = 128, BN = 64;
constexpr int NT = 192;  // 4 softmax warps, 1 producer warp, 1 MMA warp
constexpr int kMaxLevels = 4;
constexpr long kSpinLimit = 1L << 24;
constexpr unsigned kFull = 0xffffffffu;

struct Params {
  CUtensorMap kmap[kMaxLevels], vmap[kMaxLevels];  // [T_l keys][Hkv][D] bf16, box 64 keys x 1 head x 64 elements
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

__device__ __forceinline__ uint32_t s32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void cpa16(uint32_t dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0));
}
// UMMA shared-memory descriptor, 128B swizzle, sm_100 version bits
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// UMMA instruction descriptor: bf16 x bf16 -> f32, M x N, operand majors (0 = K-major, 1 = MN-major)
__host__ __device__ constexpr uint32_t idesc(int M, int N, int amaj, int bmaj) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)amaj << 15) | ((uint32_t)bmaj << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void mma(uint32_t tm, uint64_t da, uint64_t db, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n" ::"r"(tm),
      "l"(da), "l"(db), "r"(id), "r"(acc), "r"(0));
}
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(s32(bar))
               : "memory");
}
__device__ __forceinline__ void bar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(s32(bar)), "r"(count));
}
__device__ __forceinline__ void bar_arrive(uint64_t* bar) {
  asm volatile("{\n.reg .b64 st;\nmbarrier.arrive.shared::cta.b64 st, [%0];\n}\n" ::"r"(s32(bar)) : "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n.reg .b64 st;\nmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}\n" ::"r"(s32(bar)),
               "r"(bytes)
               : "memory");
}
// bounded wait for the completion of the mbarrier phase of this parity; false (and the status word set) when the
// limit ran out
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, int32_t* err) {
  uint32_t done = 0;
  for (long it = 0; it < kSpinLimit && !done; ++it)
    asm volatile("{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(done)
                 : "r"(s32(bar)), "r"(parity)
                 : "memory");
  if (!done && err) atomicExch(err, 1);
  return done != 0;
}
// TMA tile load (no multicast) of a 3D tensor map into this CTA's shared memory, completing on `bar`
__device__ __forceinline__ void tma_load3(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(s32(bar))
      : "memory");
}
__device__ __forceinline__ void tld16(uint32_t addr, float* f) {
  uint32_t v[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(addr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) f[i] = __uint_as_float(v[i]);
}
// 64 consecutive fp32 TMEM columns of this thread's lane, waited for inside the same statement so no use of the
// registers can be scheduled before the load has completed
__device__ __forceinline__ void tld64(uint32_t addr, float* f) {
  uint32_t v[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31]),
        "=r"(v[32]), "=r"(v[33]), "=r"(v[34]), "=r"(v[35]), "=r"(v[36]), "=r"(v[37]), "=r"(v[38]), "=r"(v[39]),
        "=r"(v[40]), "=r"(v[41]), "=r"(v[42]), "=r"(v[43]), "=r"(v[44]), "=r"(v[45]), "=r"(v[46]), "=r"(v[47]),
        "=r"(v[48]), "=r"(v[49]), "=r"(v[50]), "=r"(v[51]), "=r"(v[52]), "=r"(v[53]), "=r"(v[54]), "=r"(v[55]),
        "=r"(v[56]), "=r"(v[57]), "=r"(v[58]), "=r"(v[59]), "=r"(v[60]), "=r"(v[61]), "=r"(v[62]), "=r"(v[63])
      : "r"(addr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) f[i] = __uint_as_float(v[i]);
}
__device__ __forceinline__ void tst16(uint32_t addr, const float* f) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
          addr),
      "r"(__float_as_uint(f[0])), "r"(__float_as_uint(f[1])), "r"(__float_as_uint(f[2])), "r"(__float_as_uint(f[3])),
      "r"(__float_as_uint(f[4])), "r"(__float_as_uint(f[5])), "r"(__float_as_uint(f[6])), "r"(__float_as_uint(f[7])),
      "r"(__float_as_uint(f[8])), "r"(__float_as_uint(f[9])), "r"(__float_as_uint(f[10])),
      "r"(__float_as_uint(f[11])), "r"(__float_as_uint(f[12])), "r"(__float_as_uint(f[13])),
      "r"(__float_as_uint(f[14])), "r"(__float_as_uint(f[15])));
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ float ex2(float x) {  // 2^x on the MUFU unit, flush-to-zero (irrelevant for weights)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// byte offset of (row, element d) in a K-major 128B-swizzled tile of `rows` rows: atoms of 64 elements (the layout
// TMA writes with CU_TENSOR_MAP_SWIZZLE_128B into a 1024-byte aligned destination)
__device__ __forceinline__ uint32_t swz(int row, int d, int rows) {
  return (uint32_t)((d >> 6) * rows * 128 + row * 128 + ((((d & 63) >> 3) ^ (row & 7)) << 4));
}

template <int D>
struct Layout {
  static constexpr uint32_t Q = 0;                   // 128 rows x D
  static constexpr uint32_t K = Q + BM * D * 2;      // 2 stages of 64 keys x D
  static constexpr uint32_t V = K + 2 * BN * D * 2;  // 2 stages of 64 keys x D
  static constexpr uint32_t P = V + 2 * BN * D * 2;  // 128 rows x 64 keys
  static constexpr uint32_t BYTES = P + BM * BN * 2;
  static constexpr uint32_t STAGE = BN * D * 2;
  static constexpr uint32_t TMEM_COLS = 512;  // S0 [0,64) S1 [64,128) O [128, 128+D)
};

struct Bars {
  uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2], s_empty[2], p_full, pv_done, q_full, drain;
};

template <int D>
__global__ void __launch_bounds__(NT, 1) tree_attention_tc_kernel(const __grid_constant__ Params p) {
  using Lay = Layout<D>;
  extern __shared__ unsigned char raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = s32(base);
  __shared__ Bars bars;
  __shared__ uint32_t tmem_base;
  __shared__ int s_tok[BM], s_own[BM];
  __shared__ int s_lo[kMaxLevels - 1][BM], s_hi[kMaxLevels - 1][BM];
  __shared__ int s_klo[kMaxLevels], s_nblk[kMaxLevels];

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
                 "r"(Lay::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  if (tid == 160) {
    for (int s = 0; s < 2; ++s) {
      bar_init(&bars.k_full[s], 1);
      bar_init(&bars.k_empty[s], 1);
      bar_init(&bars.v_full[s], 1);
      bar_init(&bars.v_empty[s], 1);
      bar_init(&bars.s_full[s], 1);
      bar_init(&bars.s_empty[s], 128);
    }
    bar_init(&bars.p_full, 128);
    bar_init(&bars.pv_done, 1);
    bar_init(&bars.q_full, 128);
    bar_init(&bars.drain, 1);
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

  if (warp == 4) {
    // ------------------------------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      int issued = 0;  // K/V tiles issued: each has a pending or consumed full-barrier phase
      int lvl = 0, b = 0;
      for (int j = 0; j < total && ok; ++j, ++b) {
        while (b >= s_nblk[lvl]) {
          b = 0;
          ++lvl;
        }
        const int st = j & 1, ks = s_klo[lvl] + b * BN;
        if (j >= 2) ok = wait_bar(&bars.k_empty[st], ((j >> 1) - 1) & 1, p.err);
        if (!ok) break;
        bar_expect_tx(&bars.k_full[st], Lay::STAGE);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load3(sbase + Lay::K + st * Lay::STAGE + c * BN * 128, &p.kmap[lvl], c * 64, hkv, ks, &bars.k_full[st]);
        if (j >= 2) ok = wait_bar(&bars.v_empty[st], ((j >> 1) - 1) & 1, p.err);
        if (ok) {
          bar_expect_tx(&bars.v_full[st], Lay::STAGE);
#pragma unroll
          for (int c = 0; c < D / 64; ++c)
            tma_load3(sbase + Lay::V + st * Lay::STAGE + c * BN * 128, &p.vmap[lvl], c * 64, hkv, ks,
                      &bars.v_full[st]);
        }
        issued = j + 1;
        if (!ok) {  // K_j went out without V_j: wait for K_j alone below
          wait_bar(&bars.k_full[st], (j >> 1) & 1, p.err);
          issued = j;
        }
      }
      // the last tile of each stage has landed before the CTA may leave (no-ops on the normal path: consumed)
      for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; ++j) {
        wait_bar(&bars.k_full[j & 1], (j >> 1) & 1, p.err);
        wait_bar(&bars.v_full[j & 1], (j >> 1) & 1, p.err);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_QK = idesc(BM, BN, 0, 0);
      constexpr uint32_t ID_PV = idesc(BM, D, 0, 1);
      auto issue_s = [&](int j) -> bool {  // S_j = Q K_j^T into S buffer j & 1
        const int st = j & 1;
        if (!wait_bar(&bars.k_full[st], (j >> 1) & 1, p.err)) return false;
        if (j >= 2 && !wait_bar(&bars.s_empty[st], ((j >> 1) - 1) & 1, p.err)) return false;
        fence_after();
        const uint32_t kb = sbase + Lay::K + st * Lay::STAGE;
#pragma unroll
        for (int s = 0; s < D / 16; ++s)
          mma(tm + st * BN, sdesc(sbase + Lay::Q + (s >> 2) * BM * 128 + (s & 3) * 32, 16, 1024),
              sdesc(kb + (s >> 2) * BN * 128 + (s & 3) * 32, 16, 1024), ID_QK, s > 0);
        commit(&bars.s_full[st]);
        commit(&bars.k_empty[st]);
        return true;
      };
      bool ok = wait_bar(&bars.q_full, 0, p.err);
      if (ok && total > 0) ok = issue_s(0);
      for (int j = 0; j < total && ok; ++j) {
        if (j + 1 < total) ok = issue_s(j + 1);
        if (!ok) break;
        const int st = j & 1;
        ok = wait_bar(&bars.p_full, j & 1, p.err) && wait_bar(&bars.v_full[st], (j >> 1) & 1, p.err);
        if (!ok) break;
        fence_after();
        const uint32_t vb = sbase + Lay::V + st * Lay::STAGE;
#pragma unroll
        for (int s = 0; s < BN / 16; ++s)
          mma(tm + 2 * BN, sdesc(sbase + Lay::P + s * 32, 16, 1024), sdesc(vb + s * 16 * 128, BN * 128, 1024), ID_PV,
              (j > 0 || s > 0) ? 1u : 0u);
        commit(&bars.pv_done);
        commit(&bars.v_empty[st]);
      }
      commit(&bars.drain);  // completes once every MMA issued above has finished
    }
  } else {
    // ------------------------------------------------------------------------------------------ softmax warps
    const int r = tid;  // query row = TMEM lane
    const int tq = r / G;
    const uint32_t lane_addr = tm + ((uint32_t)(32 * warp) << 16);
    for (int c = tid; c < BM * (D / 8); c += 128) {  // Q tile: row rr = tq * G + g
      const int rr = c / (D / 8), d = (c % (D / 8)) * 8;
      const int tqq = rr / G, g = rr % G;
      const bool live = tqq < ntok;
      cpa16(sbase + Lay::Q + swz(rr, d, BM), p.q + ((int64_t)(live ? q0 + tqq : q0) * p.Hq + hkv * G + g) * D + d,
            live);
    }
    asm volatile("cp.async.commit_group;\n" ::);
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    fence_async_smem();
    bar_arrive(&bars.q_full);
    const float sc = p.scale_log2;
    float m_used = -INFINITY, l_sum = 0.f;
    bool ok = true;
    int lvl = 0, b = 0;
    for (int j = 0; j < total && ok; ++j, ++b) {
      while (b >= s_nblk[lvl]) {
        b = 0;
        ++lvl;
      }
      const int sb = j & 1, ks = s_klo[lvl] + b * BN;
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
      ok = __all_sync(kFull, wait_bar(&bars.s_full[sb], (j >> 1) & 1, p.err));
      if (!ok) break;
      fence_after();
      float s[BN];
      tld64(lane_addr + sb * BN, s);
      fence_before();
      bar_arrive(&bars.s_empty[sb]);  // the S buffer may be overwritten
      float mx = -INFINITY;
      if (ks >= lo && ks + BN <= hi) {  // the whole block is visible to this row
#pragma unroll
        for (int c = 0; c < BN; ++c) mx = fmaxf(mx, s[c]);
      } else {
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          const int kk = ks + c;
          s[c] = (kk >= lo && kk < hi) ? s[c] : -INFINITY;
          mx = fmaxf(mx, s[c]);
        }
      }
      mx *= sc;
      const bool grow = mx > m_used + 8.f;
      const float m_new = grow ? mx : m_used;
      const bool rescale = grow && m_used != -INFINITY;
      const float alpha = rescale ? exp2f(m_used - m_new) : 1.f;
      l_sum *= alpha;
      m_used = m_new;
      const float mref = m_used == -INFINITY ? 0.f : m_used;
      uint32_t pk[BN / 2];
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const float e0 = ex2(fmaf(s[c], sc, -mref)), e1 = ex2(fmaf(s[c + 1], sc, -mref));
        l_sum += e0 + e1;
        pk[c / 2] = pack_bf16(e0, e1);
      }
      if (j > 0) ok = __all_sync(kFull, wait_bar(&bars.pv_done, (j - 1) & 1, p.err));  // P free, O final
      if (!ok) break;
      fence_after();
      if (__any_sync(kFull, rescale)) {
#pragma unroll 1
        for (int c = 0; c < D; c += 16) {
          float o[16];
          tld16(lane_addr + 2 * BN + c, o);
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] *= alpha;
          tst16(lane_addr + 2 * BN + c, o);
        }
      }
      unsigned char* prow = base + Lay::P + r * 128;
#pragma unroll
      for (int c = 0; c < BN / 8; ++c)
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      fence_async_smem();
      fence_before();
      bar_arrive(&bars.p_full);
    }
    if (total > 0 && ok) ok = __all_sync(kFull, wait_bar(&bars.pv_done, (total - 1) & 1, p.err));
    fence_after();
    // epilogue: warp-collective TMEM loads by every softmax thread, stores by the live rows
    if (ok) {
      const bool live = tq < ntok;
      const int g = r % G;
      const int64_t t = q0 + (live ? tq : 0);
      const int h = hkv * G + g;
      const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
      const __nv_bfloat16* gr = p.gate + t * p.gate_stride + (int64_t)h * p.gate_head_stride;
      __nv_bfloat16* orow = p.out + (t * p.Hq + h) * D;
#pragma unroll 1
      for (int c = 0; c < D; c += 16) {
        float o[16];
        tld16(lane_addr + 2 * BN + c, o);
        if (live) {
          float gv[16], res[16];
#pragma unroll
          for (int i = 0; i < 16; i += 8) load8(gr + c + i, gv + i);
#pragma unroll
          for (int i = 0; i < 16; ++i) res[i] = o[i] * inv * sigmoidf_(gv[i]);
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
  wait_bar(&bars.drain, 0, p.err);
  fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(Lay::TMEM_COLS));
}

// ------------------------------------------------------------------------------------------------ host side

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(ptr);
  });
  return fn;
}

// K or V of one level: [T keys][Hkv][D] bf16, boxes of 64 keys x 1 head x 64 elements, 128B swizzle; keys past T
// read as zeros (and are masked)
static int make_kv_map(CUtensorMap* map, const void* ptr, int64_t T, int64_t Hkv, int64_t D) {
  EncodeTiled enc = encode_fn();
  if (!enc) {
    set_error("tree_attention(tcgen05): cuTensorMapEncodeTiled unavailable");
    return JANUS_ERR_CUDA;
  }
  const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)Hkv, (cuuint64_t)T};
  const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)(Hkv * D * 2)};
  const cuuint32_t box[3] = {64, 1, (cuuint32_t)BN};
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
