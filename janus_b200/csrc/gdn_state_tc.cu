// The sequential pass of the chunked gated delta rule on the 5th-generation tensor cores: one CTA per (row, value
// head) walks the row's 64-token chunks in order with the whole 128 x 128 state in TMEM, transposed (lane = value
// column v, TMEM column = key row k), so every product of the pass is an M=128 MMA over the value dimension:
//
//   VT  = S^T W^T          V'^T before the subtraction   A = S^T (bf16 copy in TMEM)   B = W  [tok][k] (K-major)
//   OT  = S^T Q^T          the inter-chunk output        A = S^T (bf16 copy in TMEM)   B = Q  [tok][k] (K-major)
//   O2T = V'^T QK^T        the intra-chunk output        A = V'^T (bf16, TMEM)         B = QK [i][j]   (K-major)
//   ST += (V' f_k)^T K     the state update              A = (V' f_k)^T (bf16, TMEM)   B = K  [tok][k] (MN-major)
//
// with V' = U - S W (fp32), f_k = e^(G_last - G), the state decayed by e^(G_last) before the update, and
// O = e^G scale OT + O2T: the same rounding points as the mma.sync formulation (bf16 state and V' as MMA operands,
// fp32 accumulation, the fp32 state carried in TMEM). W, U (transposed: a value column's tokens per row), QK and G
// come from the prep pass in chunk-major layout (zeros past a row's end); q and k straight from the projections
// (tokens past a row's end belong to the next row, but they meet zero rows of W, U, QK and contribute nothing, and
// their outputs are not stored).
//
// Warps: 0-3 one thread per value column v (TMEM lane v): state in/out, V', the decay, the bf16 state copy;
// warp 4 lane 0 the TMA producer (double-buffered chunk stages); warp 5 lane 0 the MMA issuer; warps 6-9 (again
// one thread per value column) the output of a chunk while the others go on with the next one (OT and O2T are
// double-buffered by chunk parity). Hand-offs are mbarriers with bounded waits; a wait that runs out sets the
// status word and the CTA winds down.
#include <mutex>

#include "tcgen05.cuh"

namespace jb {
namespace tcx {

EncodeTiled encode_tiled_fn() {
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

}  // namespace tcx

namespace gst {
using namespace tcx;

constexpr int CT = 64, DH = 128;
constexpr int NT = 320;  // 4 value-column warps, producer warp, MMA warp, 4 output warps
// TMEM columns: the state (fp32) and its bf16 copy, V'^T and (V' f_k)^T (bf16), and per chunk parity p the
// accumulators VT (then O2T, once V' has been read) and OT, so chunk c+1's products overlap chunk c's output
constexpr uint32_t cST = 0, cSB = 128, cVB = 192, cVD = 224, kTmemCols = 512;
__device__ __forceinline__ uint32_t cVT(int p) { return 256 + 128 * p; }  // VT, then O2T
__device__ __forceinline__ uint32_t cOT(int p) { return 320 + 128 * p; }
// one stage = the tiles of one chunk, 128B-swizzled [atom][64 rows][128 bytes]
constexpr uint32_t kTile = CT * 128 * 2;  // 64 rows x 128 elements bf16: 16 KB (two 8 KB atoms)
constexpr uint32_t sW = 0, sU = kTile, sQ = 2 * kTile, sK = 3 * kTile, sQK = 4 * kTile;  // QK: one 8 KB atom
constexpr uint32_t sG = sQK + CT * 128;                                                  // 64 fp32
constexpr uint32_t kStage = (sG + CT * 4 + 1023) & ~1023u;  // stages start on 1024-byte boundaries (swizzle atoms)
constexpr uint32_t kStageBytes = 4 * kTile + CT * 128 + CT * 4;  // bytes the TMA writes per stage
constexpr uint32_t kSmemBytes = 2 * kStage;

struct Params {
  CUtensorMap wmap, qkmap;  // chunk-major workspace [n_chunks*Hv*64 rows][128 | 64], boxes 64 x 64
  CUtensorMap umap;         // U^T [n_chunks*Hv*128 value columns][64 tokens], box 64 x 128
  CUtensorMap qmap, kmap;         // projections [T][Hk][128], box 64 x 1 x 64
  const float* G;                 // chunk-major [n_chunks][Hv][64]
  const int32_t* row_start;
  const int32_t* chunk_start;
  const float* state_in;
  const int32_t* state_row;
  float* state_out;
  __nv_bfloat16* o;
  int32_t* err;
  int Hk, Hv;
  float scale;
};

struct Bars {
  // st_done per chunk parity: the output warps trail the value-column warps by up to a chunk; s_upd: the state
  // update of the current chunk is done (the value-column warps' hand-off, committed before O2T is issued)
  uint64_t full[2], empty[2], sb_ready, vt_done, vb_ready, st_done[2], s_upd, drain;
};

// G -> (fq, fk) per token and the chunk's decay, in shared memory; by the 64 first value-column threads
__device__ __forceinline__ void chunk_factors(const float* G, float scale, float* fq, float* fk, float* dl, int tid) {
  const float gl = G[CT - 1];  // past a row's end G stays flat, so the last entry is the row's last token's
  if (tid < CT) {
    fq[tid] = expf(G[tid]) * scale;
    fk[tid] = expf(gl - G[tid]);
  }
  if (tid == 0) *dl = expf(gl);
}

// named barrier of the four value-column warps; vand also ANDs a flag over them, so a wait that ran out in any of
// them ends the loop in all four together (they never diverge around a named barrier)
__device__ __forceinline__ void vsync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
__device__ __forceinline__ void osync() { asm volatile("bar.sync 2, 128;" ::: "memory"); }  // the output warps
__device__ __forceinline__ bool oand(bool x) {
  uint32_t r;
  asm volatile("{\n.reg .pred p, q;\nsetp.ne.u32 q, %1, 0;\nbar.red.and.pred p, 2, 128, q;\nselp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(r)
               : "r"((uint32_t)x)
               : "memory");
  return r != 0;
}
__device__ __forceinline__ bool vand(bool x) {
  uint32_t r;
  asm volatile("{\n.reg .pred p, q;\nsetp.ne.u32 q, %1, 0;\nbar.red.and.pred p, 1, 128, q;\nselp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(r)
               : "r"((uint32_t)x)
               : "memory");
  return r != 0;
}

__global__ void __launch_bounds__(NT, 1) gdn_state_tc_kernel(const __grid_constant__ Params p) {
  extern __shared__ unsigned char raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = s32(base);
  __shared__ Bars bars;
  __shared__ uint32_t tmem_base;
  __shared__ float s_fq[2][CT], s_fk[CT], s_dl;  // s_fq per chunk parity: the output warps trail by a chunk

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x, row = blockIdx.y;
  const int hk = h / (p.Hv / p.Hk);
  const int cbeg = p.chunk_start[row], nch = p.chunk_start[row + 1] - cbeg;
  const int64_t r0 = p.row_start[row], r1 = p.row_start[row + 1];

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(&tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  if (tid == 128) {
    for (int s = 0; s < 2; ++s) {
      bar_init(&bars.full[s], 1);
      bar_init(&bars.empty[s], 1 + 128);  // the stage's last MMAs (commit) + the 128 output threads
    }
    bar_init(&bars.sb_ready, 128);
    bar_init(&bars.vt_done, 1);
    bar_init(&bars.vb_ready, 128);
    bar_init(&bars.st_done[0], 1);
    bar_init(&bars.st_done[1], 1);
    bar_init(&bars.s_upd, 1);
    bar_init(&bars.drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tm = tmem_base;

  if (warp == 4) {
    // -------------------------------------------------------------------------------------------- TMA producer
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      for (int i = 0; i < nch && ok; ++i) {
        const int st = i & 1;
        if (i >= 2) ok = wait_bar(&bars.empty[st], ((i >> 1) - 1) & 1, p.err);
        if (!ok) break;
        uint64_t* fb = &bars.full[st];
        bar_expect_tx(fb, kStageBytes);
        const int c = cbeg + i;
        const int rb = (c * p.Hv + h) * CT;  // first row of the chunk in the chunk-major maps
        const int t0 = (int)(r0 + (int64_t)i * CT);
        const uint32_t dst = sbase + st * kStage;
        tma_load2(dst + sW, &p.wmap, 0, rb, fb);
        tma_load2(dst + sW + kTile / 2, &p.wmap, 64, rb, fb);
        tma_load2(dst + sU, &p.umap, 0, 2 * rb, fb);  // U^T [128 value columns][64 tokens]: one box
        tma_load2(dst + sQK, &p.qkmap, 0, rb, fb);
        tma_load3(dst + sQ, &p.qmap, 0, hk, t0, fb);
        tma_load3(dst + sQ + kTile / 2, &p.qmap, 64, hk, t0, fb);
        tma_load3(dst + sK, &p.kmap, 0, hk, t0, fb);
        tma_load3(dst + sK + kTile / 2, &p.kmap, 64, hk, t0, fb);
        bulk_load(dst + sG, p.G + (int64_t)rb, CT * 4, fb);
        issued = i + 1;
      }
      // every issued load has landed before the CTA may leave (no-ops on the normal path: all consumed)
      for (int i = issued - 2 < 0 ? 0 : issued - 2; i < issued; ++i)
        wait_bar_quiet(&bars.full[i & 1], (i >> 1) & 1, p.err);
    }
  } else if (warp == 5) {
    // -------------------------------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_N64 = idesc(128, 64, 0, 0);    // B K-major, N = 64 tokens
      constexpr uint32_t ID_N128 = idesc(128, 128, 0, 1);  // B MN-major (K as [tok][k]), N = 128 key rows
      bool ok = true;
      for (int i = 0; i < nch && ok; ++i) {
        const int st = i & 1;
        const uint32_t stage = sbase + st * kStage;
        ok = wait_bar(&bars.sb_ready, i & 1, p.err) && wait_bar(&bars.full[st], (i >> 1) & 1, p.err);
        if (!ok) break;
        fence_after();
#pragma unroll
        for (int s = 0; s < 8; ++s)  // VT = S^T W^T, 16 key rows per step
          mma_ts(tm + cVT(st), tm + cSB + s * 8, sdesc(stage + sW + (s >> 2) * (kTile / 2) + (s & 3) * 32, 16, 1024),
                 ID_N64, s > 0);
        commit(&bars.vt_done);  // V' can start while OT runs
#pragma unroll
        for (int s = 0; s < 8; ++s)  // OT = S^T Q^T
          mma_ts(tm + cOT(st), tm + cSB + s * 8, sdesc(stage + sQ + (s >> 2) * (kTile / 2) + (s & 3) * 32, 16, 1024),
                 ID_N64, s > 0);
        ok = wait_bar(&bars.vb_ready, i & 1, p.err);
        if (!ok) break;
        fence_after();
        const uint32_t keep = s_dl != 0.f ? 1u : 0u;  // 0: the decayed state is zero, the update overwrites ST
        // the state update first (the next chunk waits on it), then the output's O2T (only the output warps do)
#pragma unroll
        for (int s = 0; s < 4; ++s)  // ST += (V' f_k)^T K, 16 tokens per step; K rows as the MN-major operand
          mma_ts(tm + cST, tm + cVD + s * 8, sdesc(stage + sK + s * 16 * 128, kTile / 2, 1024), ID_N128,
                 s > 0 ? 1u : keep);
        commit(&bars.s_upd);
#pragma unroll
        for (int s = 0; s < 4; ++s)  // O2T = V'^T QK^T, 16 tokens j per step
          mma_ts(tm + cVT(st), tm + cVB + s * 8, sdesc(stage + sQK + s * 32, 16, 1024), ID_N64, s > 0);
        commit(&bars.st_done[st]);
        commit(&bars.empty[st]);
      }
      commit(&bars.drain);  // completes once every MMA issued above has finished
    }
  } else if (warp >= 6) {
    // -------------------------------------------------------------------------------------------- output warps
    // O = e^G scale (Q S) + QK V' of chunk c, staged row-major [tok][v] in the stage's U tile (consumed by then)
    // and stored, while the value-column warps and the tensor core go on with chunk c+1
    const int v = 32 * (warp & 3) + lane;  // TMEM lane
    const uint32_t la = tm + ((uint32_t)(32 * (warp & 3)) << 16);
    bool ok = true;
    for (int i = 0; i < nch && ok; ++i) {
      const int st = i & 1;
      unsigned char* stage = base + st * kStage;
      const int64_t t0 = r0 + (int64_t)i * CT;
      const int nt = (r1 - t0) < CT ? (int)(r1 - t0) : CT;
      ok = oand(wait_bar(&bars.st_done[st], (i >> 1) & 1, p.err));
      if (!ok) break;
      fence_after();
      __nv_bfloat16* ost = reinterpret_cast<__nv_bfloat16*>(stage + sU);
      {
        float ot[CT], o2[CT];
        tld64f(la + cOT(st), ot);
        tld64f(la + cVT(st), o2);
        // every factor is read before the first store: the stores go through a generic pointer the compiler
        // cannot tell apart from s_fq, and interleaving them would serialise each load behind a store
        __nv_bfloat16 res[CT];
#pragma unroll
        for (int e = 0; e < CT; ++e) res[e] = __float2bfloat16_rn(ot[e] * s_fq[st][e] + o2[e]);
#pragma unroll
        for (int e = 0; e < CT; ++e) ost[e * DH + v] = res[e];
      }
      osync();  // the output tile is complete
      {  // 8 rows x 16 B per thread: all loads first, then the stores
        uint4 val[CT * (DH / 8) / 128];
#pragma unroll
        for (int n = 0; n < CT * (DH / 8) / 128; ++n) {
          const int x = v + 128 * n;
          val[n] = *reinterpret_cast<const uint4*>(ost + (x / (DH / 8)) * DH + (x % (DH / 8)) * 8);
        }
#pragma unroll
        for (int n = 0; n < CT * (DH / 8) / 128; ++n) {
          const int x = v + 128 * n, tok = x / (DH / 8);
          if (tok < nt)
            *reinterpret_cast<uint4*>(p.o + ((t0 + tok) * p.Hv + h) * DH + (x % (DH / 8)) * 8) = val[n];
        }
      }
      fence_before();
      bar_arrive(&bars.empty[st]);  // OT / O2T of this parity and the stage are free
    }
  } else {
    // -------------------------------------------------------------------------------------------- value columns
    const int v = tid;  // TMEM lane
    const uint32_t la = tm + ((uint32_t)(32 * warp) << 16);
    const float* s0 = p.state_in ? p.state_in + ((int64_t)(p.state_row ? p.state_row[row] : row) * p.Hv + h) * DH * DH
                                 : nullptr;
    // the initial state: ST (fp32) and its bf16 copy SB, column v of S = lane v of S^T
#pragma unroll 1
    for (int k0 = 0; k0 < DH; k0 += 64) {  // 64 loads in flight before the TMEM stores (which order after them)
      float f[64];
      uint32_t b[32];
#pragma unroll
      for (int e = 0; e < 64; ++e) f[e] = s0 ? s0[(int64_t)(k0 + e) * DH + v] : 0.f;
#pragma unroll
      for (int e = 0; e < 32; ++e) b[e] = pack_bf16(f[2 * e], f[2 * e + 1]);
      uint32_t w[64];
#pragma unroll
      for (int e = 0; e < 64; ++e) w[e] = __float_as_uint(f[e]);
      tst32(la + cST + k0, w);
      tst32(la + cST + k0 + 32, w + 32);
      tst32(la + cSB + k0 / 2, b);
    }
    tst_wait();
    fence_before();
    bar_arrive(&bars.sb_ready);
    bool ok = true;
    for (int i = 0; i < nch && ok; ++i) {
      const int st = i & 1;
      unsigned char* stage = base + st * kStage;
      ok = vand(wait_bar(&bars.full[st], (i >> 1) & 1, p.err));
      if (!ok) break;
      chunk_factors(reinterpret_cast<const float*>(stage + sG), p.scale, s_fq[st], s_fk, &s_dl, v);
      vsync();
      // the state decays by e^(G_last) before the update accumulates onto it, while VT = S^T W^T runs (the
      // products read the bf16 copy, not ST); a decay that underflowed to 0 (a fast-forgetting head: G_last < -103)
      // leaves nothing of the state, and the update MMA overwrites it instead
      const float dl = s_dl;
      if (dl != 0.f) {
#pragma unroll 1
        for (int k0 = 0; k0 < DH; k0 += 64) {
          float f[64];
          tld64f(la + cST + k0, f);
          uint32_t w[64];
#pragma unroll
          for (int e = 0; e < 64; ++e) w[e] = __float_as_uint(f[e] * dl);
          tst32(la + cST + k0, w);
          tst32(la + cST + k0 + 32, w + 32);
        }
      }
      ok = vand(wait_bar(&bars.vt_done, i & 1, p.err));
      if (!ok) break;
      fence_after();
      // V' = U - S W (fp32) -> V'^T and (V' f_k)^T as bf16 A operands
      {
        // U^T row v: the value column's 64 tokens, eight 16-byte units (swizzled by v & 7)
        const unsigned char* ut = stage + sU + v * 128;
        uint4 uu[CT / 8];
#pragma unroll
        for (int c = 0; c < CT / 8; ++c) uu[c] = *reinterpret_cast<const uint4*>(ut + ((c ^ (v & 7)) << 4));
        float vt[CT];
        tld64f(la + cVT(st), vt);
        uint32_t vb[CT / 2], vd[CT / 2];
#pragma unroll
        for (int c = 0; c < CT / 8; ++c)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 u2 = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(&uu[c])[i]);
            vt[8 * c + 2 * i] = u2.x - vt[8 * c + 2 * i];
            vt[8 * c + 2 * i + 1] = u2.y - vt[8 * c + 2 * i + 1];
          }
#pragma unroll
        for (int e = 0; e < CT / 2; ++e) {
          vb[e] = pack_bf16(vt[2 * e], vt[2 * e + 1]);
          vd[e] = pack_bf16(vt[2 * e] * s_fk[2 * e], vt[2 * e + 1] * s_fk[2 * e + 1]);
        }
        tst32(la + cVB, vb);
        tst32(la + cVD, vd);
      }
      tst_wait();
      fence_before();
      bar_arrive(&bars.vb_ready);
      ok = vand(wait_bar(&bars.s_upd, i & 1, p.err));
      if (!ok) break;
      fence_after();
      // the next chunk's bf16 state first: it releases the next chunk's products
#pragma unroll 1
      for (int k0 = 0; k0 < DH; k0 += 64) {
        float f[64];
        uint32_t b[32];
        tld64f(la + cST + k0, f);
#pragma unroll
        for (int e = 0; e < 32; ++e) b[e] = pack_bf16(f[2 * e], f[2 * e + 1]);
        tst32(la + cSB + k0 / 2, b);
      }
      tst_wait();
      fence_before();
      bar_arrive(&bars.sb_ready);
    }
    // the final state (the last update is complete: s_upd of the last chunk was waited for above)
    if (p.state_out && ok) {
      float* so = p.state_out + ((int64_t)row * p.Hv + h) * DH * DH;
#pragma unroll 1
      for (int k0 = 0; k0 < DH; k0 += 64) {
        float f[64];
        tld64f(la + cST + k0, f);
#pragma unroll
        for (int e = 0; e < 64; ++e) so[(int64_t)(k0 + e) * DH + v] = f[e];
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
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(kTmemCols));
}

}  // namespace gst

// ------------------------------------------------------------------------------------------------ host side

// row-major [rows][cols] bf16, boxes of 64 columns x box_rows rows (128B swizzle); also the chunk prep's store map
int map2d(CUtensorMap* m, const void* ptr, uint64_t cols, uint64_t rows, uint32_t box_rows) {
  tcx::EncodeTiled enc = tcx::encode_tiled_fn();
  if (!enc) {
    set_error("gdn_chunk_scan(tcgen05): cuTensorMapEncodeTiled unavailable");
    return JANUS_ERR_CUDA;
  }
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("gdn_chunk_scan(tcgen05): tensor map encode failed (%d)", (int)r);
    return JANUS_ERR_INVALID;
  }
  return JANUS_OK;
}

// [T][H][128] bf16, boxes of 64 dims x 1 head x 64 tokens (128B swizzle), zeros past T; also the chunk prep's loads
int map3d(CUtensorMap* m, const void* ptr, uint64_t T, uint64_t H) {
  tcx::EncodeTiled enc = tcx::encode_tiled_fn();
  if (!enc) {
    set_error("gdn_chunk_scan(tcgen05): cuTensorMapEncodeTiled unavailable");
    return JANUS_ERR_CUDA;
  }
  const cuuint64_t dims[3] = {128, H, T};
  const cuuint64_t strides[2] = {128 * 2, H * 128 * 2};
  const cuuint32_t box[3] = {64, 1, 64};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("gdn_chunk_scan(tcgen05): tensor map encode failed (%d)", (int)r);
    return JANUS_ERR_INVALID;
  }
  return JANUS_OK;
}

// the sequential pass over B rows x Hv heads; W, U [n_chunks*Hv*64][128], QK [n_chunks*Hv*64][64] bf16 and
// G [n_chunks*Hv*64] fp32 chunk-major from the prep pass
int gdn_state_tc(const void* q, const void* k, int64_t T, int64_t B, const int32_t* row_start,
                 const int32_t* chunk_start, int64_t n_chunks, const float* state_in, const int32_t* state_row,
                 float* state_out, int64_t Hk, int64_t Hv, float scale, const void* W, const void* U, const void* QK,
                 const float* G, int32_t* err, void* o, cudaStream_t stream) {
  gst::Params p{};
  const uint64_t rows = (uint64_t)n_chunks * Hv * 64;
  int st = map2d(&p.wmap, W, 128, rows, 64);
  if (!st) st = map2d(&p.umap, U, 64, 2 * rows, 128);  // U^T: [chunk][head][128 value columns][64 tokens]
  if (!st) st = map2d(&p.qkmap, QK, 64, rows, 64);
  if (!st) st = map3d(&p.qmap, q, (uint64_t)T, (uint64_t)Hk);
  if (!st) st = map3d(&p.kmap, k, (uint64_t)T, (uint64_t)Hk);
  if (st) return st;
  p.G = G;
  p.row_start = row_start;
  p.chunk_start = chunk_start;
  p.state_in = state_in;
  p.state_row = state_row;
  p.state_out = state_out;
  p.o = (__nv_bfloat16*)o;
  p.err = err;
  p.Hk = (int)Hk;
  p.Hv = (int)Hv;
  p.scale = scale;
  const size_t smem = gst::kSmemBytes + 1024;
  cudaError_t e =
      cudaFuncSetAttribute(gst::gdn_state_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    set_error("gdn_chunk_scan(tcgen05): smem attribute %s", cudaGetErrorString(e));
    return JANUS_ERR_CUDA;
  }
  gst::gdn_state_tc_kernel<<<dim3((unsigned)Hv, (unsigned)B), gst::NT, smem, stream>>>(p);
  return launch_status("gdn_chunk_scan/state(tcgen05)");
}

}  // namespace jb
