// Tree attention on the 5th-generation tensor cores (tcgen05, accumulators in TMEM) for head dims 128 and 256.
//
// A CTA owns one kv head and 128 query rows = (128 / G) tokens x G query heads (GQA folded into M), one row per
// thread: row r lives in TMEM lane r, so the softmax of a row is thread-local. Per key block of 64:
//   S_j = Q K_j^T            tcgen05.mma M=128 N=64, A = Q and B = K_j from 128B-swizzled shared memory (K-major),
//                            into one of two TMEM S buffers (64 columns each)
//   P_j = exp2(S_j*c - m)    read from TMEM by the owning thread, masked by the tree rule (ancestor key ranges,
//                            own row causal), written to shared memory as bf16 (K-major, swizzled)
//   O  += P_j V_j            tcgen05.mma M=128 N=D, B = V_j MN-major (the same swizzled [key][d] tiles as K)
// O (D fp32 columns) stays in TMEM for the whole key range. The running max m is refreshed only when a row's max
// grows by more than 2^8 (then the row's O is rescaled in TMEM), so P stays <= 256 and the exact softmax is kept:
// the normaliser l uses the same m. One elected thread issues the MMAs; completion is tracked by mbarriers fed by
// tcgen05.commit. The QK^T of block j+1 is issued before the softmax of block j, so the tensor core works on it
// while the CUDA cores do the softmax. Loads use cp.async into the swizzled layouts (K/V double-buffered).
// Every mbarrier wait is bounded; a wait that runs out sets the error word and the CTA stops issuing work.
#include "common.cuh"

namespace jb {
namespace tc {

constexpr int BM = 128, BN = 64, NT = 128;
constexpr int kMaxLevels = 4;
constexpr long kSpinLimit = 1L << 26;

struct Params {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k[kMaxLevels];
  const __nv_bfloat16* v[kMaxLevels];
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
// bounded wait on an mbarrier phase; false when the limit ran out (the error word is set)
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, int32_t* err) {
  uint32_t done = 0;
  for (long it = 0; it < kSpinLimit && !done; ++it)
    asm volatile("{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(done)
                 : "r"(s32(bar)), "r"(parity));
  if (!done && err) atomicExch(err, 1);
  return done != 0;
}
__device__ __forceinline__ void tld16(uint32_t addr, float* f) {
  uint32_t v[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) f[i] = __uint_as_float(v[i]);
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
// 2^x on the MUFU unit, flush-to-zero (results below 2^-126 are 0: irrelevant for softmax weights)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// byte offset of (row, element d) in a K-major 128B-swizzled tile of `rows` rows: atoms of 64 elements
__device__ __forceinline__ uint32_t swz(int row, int d, int rows) {
  return (uint32_t)((d >> 6) * rows * 128 + row * 128 + ((((d & 63) >> 3) ^ (row & 7)) << 4));
}

template <int D>
struct Layout {
  static constexpr uint32_t Q = 0;                       // 128 rows x D
  static constexpr uint32_t K = Q + BM * D * 2;          // 2 stages of 64 keys x D
  static constexpr uint32_t V = K + 2 * BN * D * 2;      // 2 stages of 64 keys x D
  static constexpr uint32_t P = V + 2 * BN * D * 2;      // 128 rows x 64 keys
  static constexpr uint32_t BYTES = P + BM * BN * 2;
  static constexpr uint32_t STAGE = BN * D * 2;
  static constexpr uint32_t TMEM_COLS = 512;             // S0 [0,64) S1 [64,128) O [128, 128+D)
};

template <int D>
__global__ void __launch_bounds__(NT, 1) tree_attention_tc_kernel(Params p) {
  using Lay = Layout<D>;
  extern __shared__ unsigned char raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = s32(base);
  __shared__ uint64_t bar_s[2], bar_pv, bar_drain;
  __shared__ uint32_t tmem_base;
  __shared__ int s_tok[BM], s_own[BM];
  __shared__ int s_lo[kMaxLevels][BM], s_hi[kMaxLevels][BM];
  __shared__ int s_klo[kMaxLevels], s_khi[kMaxLevels], s_nblk[kMaxLevels];

  const int tid = threadIdx.x, warp = tid >> 5;
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
  if (tid == 32) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s32(&bar_s[0])));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s32(&bar_s[1])));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s32(&bar_pv)));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s32(&bar_drain)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::);
  }
  __syncthreads();
  if (tid == 0) {
    for (int l = 0; l < L - 1; ++l) {
      int a = 0x7fffffff, b = -1;
      for (int tq = 0; tq < ntok; ++tq) {
        a = min(a, s_lo[l][tq]);
        b = max(b, s_hi[l][tq]);
      }
      s_klo[l] = a;
      s_khi[l] = b > a ? b : a;
    }
    s_klo[L - 1] = s_own[0];
    s_khi[L - 1] = q1;
    for (int l = 0; l < L; ++l) s_nblk[l] = (s_khi[l] - s_klo[l] + BN - 1) / BN;
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tm = tmem_base;
  int total = 0;
  for (int l = 0; l < L; ++l) total += s_nblk[l];

  auto block_of = [&](int b, int& lvl, int& ks) {
    int l = 0;
    while (b >= s_nblk[l]) {
      b -= s_nblk[l];
      ++l;
    }
    lvl = l;
    ks = s_klo[l] + b * BN;
  };
  // K or V block b into stage st: [d-chunk][key][64 d], 128B swizzled by key
  auto load_kv = [&](int b, int st, bool values) {
    int lvl, ks;
    block_of(b, lvl, ks);
    const int kend = s_khi[lvl];
    const __nv_bfloat16* src = values ? p.v[lvl] : p.k[lvl];
    const uint32_t dst = sbase + (values ? Lay::V : Lay::K) + st * Lay::STAGE;
    for (int c = tid; c < BN * (D / 8); c += NT) {
      const int r = c / (D / 8), d = (c % (D / 8)) * 8;
      const int kk = ks + r;
      const bool ok = kk < kend;
      cpa16(dst + swz(r, d, BN), src + ((int64_t)(ok ? kk : ks) * p.Hkv + hkv) * D + d, ok);
    }
  };

  // Q tile: row r = tq * G + g
  for (int c = tid; c < BM * (D / 8); c += NT) {
    const int r = c / (D / 8), d = (c % (D / 8)) * 8;
    const int tq = r / G, g = r % G;
    const bool ok = tq < ntok;
    cpa16(sbase + Lay::Q + swz(r, d, BM), p.q + ((int64_t)(ok ? q0 + tq : q0) * p.Hq + hkv * G + g) * D + d, ok);
  }
  load_kv(0, 0, false);
  load_kv(0, 0, true);
  if (total > 1) load_kv(1, 1, false);
  asm volatile("cp.async.commit_group;\n" ::);
  asm volatile("cp.async.wait_group 0;\n" ::);
  fence_async_smem();
  fence_before();
  __syncthreads();
  fence_after();

  constexpr uint32_t ID_QK = idesc(BM, BN, 0, 0);
  constexpr uint32_t ID_PV = idesc(BM, D, 0, 1);
  auto issue_s = [&](int b) {  // S_b = Q K_b^T into S buffer b & 1
    const uint32_t kb = sbase + Lay::K + (b & 1) * Lay::STAGE;
#pragma unroll
    for (int s = 0; s < D / 16; ++s)
      mma(tm + (b & 1) * BN, sdesc(sbase + Lay::Q + (s >> 2) * BM * 128 + (s & 3) * 32, 16, 1024),
          sdesc(kb + (s >> 2) * BN * 128 + (s & 3) * 32, 16, 1024), ID_QK, s > 0);
    commit(&bar_s[b & 1]);
  };
  bool ok = true;
  if (tid == 0) issue_s(0);

  const int r = tid;  // this thread's query row / TMEM lane
  const int tq = r / G;
  const uint32_t lane_addr = tm + ((uint32_t)(32 * warp) << 16);
  float m_used = -INFINITY, l_sum = 0.f;

  for (int j = 0; j < total && ok; ++j) {
    const int sb = j & 1;
    if (tid == 0 && j + 1 < total) issue_s(j + 1);
    ok = wait_bar(&bar_s[sb], (j >> 1) & 1, p.err);
    fence_after();
    if (j + 2 < total) load_kv(j + 2, sb, false);  // K_j's stage: S_j is complete
    int lvl, ks;
    block_of(j, lvl, ks);
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
    float s[BN];
#pragma unroll
    for (int c = 0; c < BN; c += 16) tld16(lane_addr + sb * BN + c, s + c);
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
    mx *= p.scale_log2;  // scale > 0: the max of the scaled scores
    if (j > 0) ok = ok && wait_bar(&bar_pv, (j - 1) & 1, p.err);
    fence_after();
    // V_{j+1} into the stage PV_{j-1} has finished reading; it lands while this block and the next are processed
    if (j + 1 < total) load_kv(j + 1, sb ^ 1, true);
    asm volatile("cp.async.commit_group;\n" ::);
    // lazy max: refresh when the row's max grows by more than 2^8; rescale O then (warp-collective TMEM access)
    const bool grow = mx > m_used + 8.f;
    const float m_new = grow ? mx : m_used;
    const bool rescale = grow && m_used != -INFINITY;
    const float alpha = rescale ? exp2f(m_used - m_new) : 1.f;
    if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
      for (int c = 0; c < D; c += 16) {
        float o[16];
        tld16(lane_addr + 2 * BN + c, o);
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] *= alpha;
        tst16(lane_addr + 2 * BN + c, o);
      }
    }
    l_sum *= alpha;
    m_used = m_new;
    const float mref = m_used == -INFINITY ? 0.f : m_used;
    const float sc = p.scale_log2;
    unsigned char* prow = base + Lay::P + r * 128;
#pragma unroll
    for (int c = 0; c < BN; c += 8) {
      float e[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        e[i] = ex2(fmaf(s[c + i], sc, -mref));
        l_sum += e[i];
      }
      uint4 v;
      __nv_bfloat162 h0 = __floats2bfloat162_rn(e[0], e[1]), h1 = __floats2bfloat162_rn(e[2], e[3]);
      __nv_bfloat162 h2 = __floats2bfloat162_rn(e[4], e[5]), h3 = __floats2bfloat162_rn(e[6], e[7]);
      v.x = *reinterpret_cast<uint32_t*>(&h0);
      v.y = *reinterpret_cast<uint32_t*>(&h1);
      v.z = *reinterpret_cast<uint32_t*>(&h2);
      v.w = *reinterpret_cast<uint32_t*>(&h3);
      *reinterpret_cast<uint4*>(prow + ((((c >> 3) ^ (r & 7))) << 4)) = v;
    }
    asm volatile("cp.async.wait_group 1;\n" ::);  // the previous iteration's group: K_{j+1}, V_j
    fence_async_smem();
    fence_before();
    ok = __syncthreads_and(ok);  // CTA-uniform: a timed-out wait anywhere stops every thread at the loop head
    fence_after();
    if (tid == 0 && ok) {
      const uint32_t vb = sbase + Lay::V + sb * Lay::STAGE;
#pragma unroll
      for (int s = 0; s < BN / 16; ++s)
        mma(tm + 2 * BN, sdesc(sbase + Lay::P + s * 32, 16, 1024), sdesc(vb + s * 16 * 128, BN * 128, 1024), ID_PV,
            (j > 0 || s > 0) ? 1u : 0u);
      commit(&bar_pv);
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::);
  if (total > 0 && ok) ok = wait_bar(&bar_pv, (total - 1) & 1, p.err);
  fence_before();
  ok = __syncthreads_and(ok);
  fence_after();
  if (ok) {  // CTA-uniform; the TMEM loads below are warp-collective, only the stores depend on the row
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
  if (!ok) {  // a wait ran out: let every MMA already issued finish (bounded) before the TMEM is released
    if (tid == 0) commit(&bar_drain);
    wait_bar(&bar_drain, 0, p.err);
  }
  fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(Lay::TMEM_COLS));
}

template <int D>
int launch(const Params& p, int64_t n_tiles, cudaStream_t s) {
  const size_t smem = Layout<D>::BYTES + 1024;
  cudaError_t e = cudaFuncSetAttribute(tree_attention_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
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
                      const void* const* v_levels, const int32_t* const* anc_lo, const int32_t* const* anc_hi,
                      const int32_t* row_start, const int32_t* row_of_token, const int32_t* tiles, int64_t n_tiles,
                      const void* gate, int64_t gate_stride, int64_t gate_head_stride, float scale, void* out,
                      int32_t* err, cudaStream_t stream) {
  tc::Params p{};
  p.q = (const __nv_bfloat16*)q;
  for (int l = 0; l < n_levels; ++l) {
    p.k[l] = (const __nv_bfloat16*)k_levels[l];
    p.v[l] = (const __nv_bfloat16*)v_levels[l];
    if (l < n_levels - 1) {
      p.lo[l] = anc_lo[l];
      p.hi[l] = anc_hi[l];
    }
  }
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
