// The chunked gated delta rule in one launch: one CTA per (row, value head) computes each 64-token chunk's WY
// products (the prep) one chunk ahead of the sequential state pass, both on the 5th-generation tensor cores, and
// hands W, U, QK and G from one to the other through shared memory. The arithmetic, and every rounding point, is
// that of the two-launch form in gdn_chunk.cu (prep, chunk-major workspace in HBM) + gdn_state_tc.cu (the state
// pass), so the two give bit-identical outputs and states; this form drops the workspace's write and read-back
// (about two thirds of the two-launch form's DRAM traffic) and runs the prep of chunk c+1 under the state pass of
// chunk c. Rows only (no segment ids: the state fork of the leaf levels stays on the two-launch form).
//
// Measured on B200 it is the slower form (16 rows x 8192 tokens, 32 value heads: 4.2 ms against 3.1 ms; 2 rows:
// 0.99 against 0.57): per chunk the prep's chain of dependent phases takes about 14k cycles against the state
// pass's 3.7k (clock stamps per phase), one prep group per CTA cannot hide it, and the shared memory of two stages
// leaves no room for a second; the two-launch prep runs three chunks per SM side by side instead. The host calls it
// only when asked (janus_b200.ops.gdn_chunk_scan(fused=True)).
//
// Per chunk, with G the in-chunk cumulative g:
//   prep:  P1 = [K; Q] K^T (M = 128) -> N = -tril_strict(diag(beta) K K^T e^(G_i - G_j)) fp32, QK bf16
//          T = (I - N)^-1 (16x16 diagonal blocks by substitution, doubling 16 -> 32 -> 64 in tf32)
//          P2: U^T = V^T (T diag(beta))^T, W^T = K^T (T diag(beta e^G))^T, bf16
//   state: V' = U - W S;  O = scale e^G (Q S) + QK V';  S = e^(G_last) S + K^T (V' e^(G_last - G))
//
// Warps: 0-3 value columns (one thread per value column v = TMEM lane: state in/out, V', the decay, the bf16 state
// copy), 4-7 output (O of chunk c while the others go on), 8-11 prep, 12 lane 0 TMA producer, 13 lane 0 the state
// pass's MMA issuer (the prep's first thread issues the prep's MMAs). Shared memory: two chunk stages ([K; Q] by
// TMA; W, U^T, QK, G written by the prep; U^T's place then stages the output) and the prep's private region (V by
// TMA, N, T, T diag(beta), T diag(beta e^G)). TMEM: the state pass's 384 columns and the prep's 128. Every hand-off
// is an mbarrier with a bounded wait; a wait that runs out sets the status word and every role winds down (loads in
// flight landed, MMAs drained, TMEM released).
#include "gdn_inverse.cuh"
#include "tcgen05.cuh"

namespace jb {
namespace gsf {
using namespace tcx;

constexpr int CT = 64, DH = 128;
constexpr int NT = 448;
constexpr int PADF = 68;  // fp32 [64][68] tiles: tf32 A fragments hit 32 distinct banks
constexpr int PADM = 40;  // fp32 [32][40]
// TMEM columns: state (fp32) and its bf16 copy, V'^T and (V' f_k)^T (bf16), VT (then O2T), OT; the prep's P1 / P2
constexpr uint32_t cST = 0, cSB = 128, cVB = 192, cVD = 224, cVT = 256, cOT = 320, cP = 384, kTmemCols = 512;
// one stage (chunk parity): [K; Q] as [2 atoms][K rows 0-63 | Q rows 0-63][128 B] (so [K; Q] is one M = 128 operand
// and K, Q the N = 64 ones), W [2 atoms][64 tokens][128 B], U^T [128 value columns][128 B] (then the output tile
// [64 tokens][128] bf16), QK [64][128 B], G fp32 [64]; 128B-swizzled tiles on 1024-byte boundaries
constexpr uint32_t oKQ = 0, oW = 32768, oU = 49152, oQK = 65536, oG = 73728, kStage = 74752;
// the prep's region
constexpr uint32_t oV = 2 * kStage;              // V [2 atoms][64 tokens][128 B]
constexpr uint32_t oN = oV + 16384;              // N fp32 [64][PADF]
constexpr uint32_t oTF = oN + CT * PADF * 4;     // T fp32 [64][PADF]
constexpr uint32_t oT1 = oTF + CT * PADF * 4;    // T diag(beta) bf16 [64][128 B]; during the inverse M fp32 [32][PADM]
constexpr uint32_t oT2 = oT1 + 8192;             // T diag(beta e^G) bf16 [64][128 B]
constexpr uint32_t oVec = oT2 + 8192;            // G, e^G, beta, raw g: fp32 [64] each
constexpr uint32_t kSmem = oVec + 4 * CT * 4;
static_assert(kStage % 1024 == 0 && oG + CT * 4 <= kStage && oV % 1024 == 0 && oT1 % 1024 == 0 && oT2 % 1024 == 0,
              "swizzled tiles on 1024-byte boundaries");
static_assert(32 * PADM * 4 <= 8192, "M fits in T diag(beta)'s place");
static_assert(kSmem + 1024 <= 227 * 1024, "shared memory");

struct Params {
  CUtensorMap qmap, kmap, vmap;  // [T][H][128] bf16, boxes 64 dims x 1 head x 64 tokens
  const float* g;
  const float* beta;
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
  uint64_t kq_full[2], v_full, p1_done, p2_done, prep_done[2], sb_ready, vt_done, vb_ready, st_done, acc_free,
      stage_free[2], drain, pdrain;
};

// named barriers of the 128-thread groups (id 1 value columns, 2 output, 3 prep); the *and forms AND a flag over the
// group, so a wait that ran out in any thread ends the loop in the whole group together
__device__ __forceinline__ void vsync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
__device__ __forceinline__ void osync() { asm volatile("bar.sync 2, 128;" ::: "memory"); }
__device__ __forceinline__ void psync() { asm volatile("bar.sync 3, 128;" ::: "memory"); }
template <int ID>
__device__ __forceinline__ bool group_and(bool x) {
  uint32_t r;
  asm volatile("{\n.reg .pred p, q;\nsetp.ne.u32 q, %1, 0;\nbar.red.and.pred p, %2, 128, q;\nselp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(r)
               : "r"((uint32_t)x), "n"(ID)
               : "memory");
  return r != 0;
}

__device__ __forceinline__ uint32_t tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
// C[16 x 8] += A[16 x K] B[K x 8] (row-major fp32), K a multiple of 8
__device__ __forceinline__ void tile_mma_tf32(float* c, const float* A, int lda, const float* B, int ldb, int K,
                                              int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int k0 = 0; k0 < K; k0 += 8) {
    const uint32_t a0 = tf32(A[g * lda + k0 + t]), a1 = tf32(A[(g + 8) * lda + k0 + t]);
    const uint32_t a2 = tf32(A[g * lda + k0 + t + 4]), a3 = tf32(A[(g + 8) * lda + k0 + t + 4]);
    const uint32_t b0 = tf32(B[(k0 + t) * ldb + g]), b1 = tf32(B[(k0 + t + 4) * ldb + g]);
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}
__device__ __forceinline__ void store_tile(const float* c, float* D, int ldd, int lane) {
  const int g = lane >> 2, t = lane & 3;
  D[g * ldd + 2 * t] = c[0];
  D[g * ldd + 2 * t + 1] = c[1];
  D[(g + 8) * ldd + 2 * t] = c[2];
  D[(g + 8) * ldd + 2 * t + 1] = c[3];
}
// byte offset of element (r, c) of a 64-column swizzled atom [rows][128 B]
__device__ __forceinline__ uint32_t swz(int r, int c) { return r * 128 + ((((c >> 3) ^ r) & 7) << 4) + (c & 7) * 2; }

__global__ void __launch_bounds__(NT, 1) gdn_scan_fused_kernel(const __grid_constant__ Params p) {
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
      bar_init(&bars.kq_full[s], 1);
      bar_init(&bars.prep_done[s], 128);   // every prep thread, after its W / U / QK / G writes
      bar_init(&bars.stage_free[s], 128);  // every output thread, after the chunk's output left the stage
    }
    bar_init(&bars.v_full, 1);
    bar_init(&bars.p1_done, 1);
    bar_init(&bars.p2_done, 1);
    bar_init(&bars.sb_ready, 128);
    bar_init(&bars.vt_done, 1);
    bar_init(&bars.vb_ready, 128);
    bar_init(&bars.st_done, 1);
    bar_init(&bars.acc_free, 128);
    bar_init(&bars.drain, 1);
    bar_init(&bars.pdrain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tm = tmem_base;

  if (warp == 12) {
    // ------------------------------------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      int issued = 0, issued_v = 0;
      for (int i = 0; i < nch && ok; ++i) {
        const int st = i & 1;
        const int t0 = (int)(r0 + (int64_t)i * CT);
        const uint32_t stage = sbase + st * kStage;
        if (i >= 2) ok = wait_bar(&bars.stage_free[st], ((i >> 1) - 1) & 1, p.err);
        if (!ok) break;
        bar_expect_tx(&bars.kq_full[st], 2 * 2 * CT * 128);
#pragma unroll
        for (int a = 0; a < 2; ++a) {
          tma_load3(stage + oKQ + a * 16384, &p.kmap, 64 * a, hk, t0, &bars.kq_full[st]);
          tma_load3(stage + oKQ + a * 16384 + 8192, &p.qmap, 64 * a, hk, t0, &bars.kq_full[st]);
        }
        issued = i + 1;
        if (i >= 1) ok = wait_bar(&bars.p2_done, (i - 1) & 1, p.err);  // the previous chunk's V is consumed
        if (!ok) break;
        bar_expect_tx(&bars.v_full, 2 * CT * 128);
        tma_load3(sbase + oV, &p.vmap, 0, h, t0, &bars.v_full);
        tma_load3(sbase + oV + 8192, &p.vmap, 64, h, t0, &bars.v_full);
        issued_v = i + 1;
      }
      // every issued load has landed before the CTA may leave (no-ops on the normal path: all consumed)
      for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; ++j)
        wait_bar_quiet(&bars.kq_full[j & 1], (j >> 1) & 1, p.err);
      if (issued_v > 0) wait_bar_quiet(&bars.v_full, (issued_v - 1) & 1, p.err);
    }
  } else if (warp == 13) {
    // ------------------------------------------------------------------------------- MMA issuer of the state pass
    if (lane == 0) {
      constexpr uint32_t ID_N64 = idesc(128, 64, 0, 0);    // B K-major, N = 64 tokens
      constexpr uint32_t ID_N128 = idesc(128, 128, 0, 1);  // B MN-major (K as [tok][k]), N = 128 key rows
      bool ok = true;
      for (int i = 0; i < nch && ok; ++i) {
        const int st = i & 1;
        const uint32_t stage = sbase + st * kStage;
        ok = wait_bar(&bars.sb_ready, i & 1, p.err) && wait_bar(&bars.prep_done[st], (i >> 1) & 1, p.err) &&
             (i == 0 || wait_bar(&bars.acc_free, (i - 1) & 1, p.err));
        if (!ok) break;
        fence_after();
#pragma unroll
        for (int s = 0; s < 8; ++s)  // VT = S^T W^T, 16 key rows per step
          mma_ts(tm + cVT, tm + cSB + s * 8, sdesc(stage + oW + (s >> 2) * 8192 + (s & 3) * 32, 16, 1024), ID_N64,
                 s > 0);
        commit(&bars.vt_done);  // V' can start while OT runs
#pragma unroll
        for (int s = 0; s < 8; ++s)  // OT = S^T Q^T
          mma_ts(tm + cOT, tm + cSB + s * 8, sdesc(stage + oKQ + 8192 + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024),
                 ID_N64, s > 0);
        ok = wait_bar(&bars.vb_ready, i & 1, p.err);
        if (!ok) break;
        fence_after();
        const uint32_t keep = s_dl != 0.f ? 1u : 0u;  // 0: the decayed state is zero, the update overwrites ST
#pragma unroll
        for (int s = 0; s < 4; ++s)  // O2T = V'^T QK^T, 16 tokens j per step
          mma_ts(tm + cVT, tm + cVB + s * 8, sdesc(stage + oQK + s * 32, 16, 1024), ID_N64, s > 0);
#pragma unroll
        for (int s = 0; s < 4; ++s)  // ST += (V' f_k)^T K, 16 tokens per step; K rows as the MN-major operand
          mma_ts(tm + cST, tm + cVD + s * 8, sdesc(stage + oKQ + s * 16 * 128, 16384, 1024), ID_N128,
                 s > 0 ? 1u : keep);
        commit(&bars.st_done);
      }
      commit(&bars.drain);  // completes once every MMA issued above has finished
    }
  } else if (warp >= 8) {
    // -------------------------------------------------------------------------------------------------------- prep
    const int pt = tid - 256, pw = pt >> 5;
    float* sN = reinterpret_cast<float*>(base + oN);
    float* sTF = reinterpret_cast<float*>(base + oTF);
    float* sM = reinterpret_cast<float*>(base + oT1);
    float* sG = reinterpret_cast<float*>(base + oVec);
    float* seG = sG + CT;
    float* sBeta = sG + 2 * CT;
    float* sGraw = sG + 3 * CT;
    float* sGl = sGraw;  // G log2(e), between the chunk's scan and the next chunk's raw g
    const uint32_t la = tm + ((uint32_t)(32 * pw) << 16) + cP;  // this warp's TMEM lanes, the prep's columns
    // g and beta of the chunk after the one in hand, in registers (their loads overlap a chunk's work)
    float g_next = 0.f, b_next = 0.f;
    if (pt < CT && nch > 0 && r0 + pt < r1) {
      g_next = p.g[(r0 + pt) * p.Hv + h];
      b_next = p.beta[(r0 + pt) * p.Hv + h];
    }
    bool ok = true;
    for (int i = 0; i < nch && ok; ++i) {
      const int st = i & 1;
      const uint32_t stage = sbase + st * kStage;
      unsigned char* stg = base + st * kStage;
      const int64_t t0 = r0 + (int64_t)i * CT;
      const int nt = (r1 - t0) < CT ? (int)(r1 - t0) : CT;
      if (pt < CT) {  // tokens past the row's end: g = beta = 0 (they touch nothing)
        sGraw[pt] = g_next;
        sBeta[pt] = b_next;
        const int64_t tn = t0 + CT + pt;
        const bool in = i + 1 < nch && tn < r1;
        g_next = in ? p.g[tn * p.Hv + h] : 0.f;
        b_next = in ? p.beta[tn * p.Hv + h] : 0.f;
      }
      if (pt == 0) {  // P1: [K; Q] K^T (M = 128, N = 64): lanes 0-63 K K^T, lanes 64-127 Q K^T
        if (wait_bar(&bars.kq_full[st], (i >> 1) & 1, p.err)) {
          fence_after();
#pragma unroll
          for (int s = 0; s < DH / 16; ++s) {
            const uint32_t off = stage + oKQ + (s >> 2) * 16384 + (s & 3) * 32;
            mma(tm + cP, sdesc(off, 16, 1024), sdesc(off, 16, 1024), idesc(128, 64, 0, 0), s > 0);
          }
          commit(&bars.p1_done);
        }
      }
      psync();
      if (pw == 1) {  // in-chunk cumulative sum of g (two values per lane)
        const float a = sGraw[2 * lane], b = a + sGraw[2 * lane + 1];
        float inc = b;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, inc, off);
          if (lane >= off) inc += y;
        }
        const float excl = inc - b;
        sG[2 * lane] = excl + a;
        sG[2 * lane + 1] = excl + b;
      }
      psync();
      if (pt < CT) {
        seG[pt] = expf(sG[pt]);
        sGl[pt] = sG[pt] * kLog2e;
      }
      ok = group_and<3>(wait_bar(&bars.p1_done, i & 1, p.err));
      if (!ok) break;
      fence_after();
      if (pt < CT) reinterpret_cast<float*>(stg + oG)[pt] = sG[pt];  // the stage is free: its [K; Q] load landed
      // P1 epilogue, warp pw: TMEM lanes 32 pw .. +31, all 64 columns. Lanes 0-63: N = -beta_i (K K^T)_ij
      // e^(G_i - G_j) for j < i (fp32); lanes 64-127: QK = scale (Q K^T)_ij e^(G_i - G_j) for j <= i, rows past the
      // row's end zero (bf16, the stage's QK tile)
      {
        const int ii = 32 * (pw & 1) + lane;
        const float gli = sGl[ii];
        if (!(pw & 1)) {  // rows 0-31 against columns 32-63 lie wholly above the diagonal: both masks are zero
          if (pw < 2) {
#pragma unroll
            for (int x = 32; x < CT; x += 4) *reinterpret_cast<float4*>(&sN[ii * PADF + x]) = make_float4(0, 0, 0, 0);
          } else {
#pragma unroll
            for (int u = 0; u < 4; ++u) *reinterpret_cast<uint4*>(stg + oQK + swz(ii, 32 + 8 * u)) = make_uint4(0, 0, 0, 0);
          }
        }
#pragma unroll 1
        for (int j0 = 0; j0 < ((pw & 1) ? CT : 32); j0 += 32) {
          float d[32];
          tld16f(la + j0, d);
          tld16f(la + j0 + 16, d + 16);
          if (pw < 2) {
            const float nb = -sBeta[ii];
            float nv[32];
#pragma unroll
            for (int x = 0; x < 32; ++x) nv[x] = n_entry(d[x], nb, gli, sGl[j0 + x], j0 + x < ii);
#pragma unroll
            for (int x = 0; x < 32; x += 4)
              *reinterpret_cast<float4*>(&sN[ii * PADF + j0 + x]) = make_float4(nv[x], nv[x + 1], nv[x + 2], nv[x + 3]);
          } else {
            uint32_t qv[16];
#pragma unroll
            for (int x = 0; x < 32; x += 2) {
              float e[2];
#pragma unroll
              for (int u = 0; u < 2; ++u)
                e[u] = qk_entry(d[x + u], p.scale, gli, sGl[j0 + x + u], (j0 + x + u <= ii) & (ii < nt));
              qv[x / 2] = pack_bf16(e[0], e[1]);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
              *reinterpret_cast<uint4*>(stg + oQK + swz(ii, j0 + 8 * u)) =
                  make_uint4(qv[4 * u], qv[4 * u + 1], qv[4 * u + 2], qv[4 * u + 3]);
          }
        }
      }
      fence_async_smem();  // the QK tile is an MMA operand
      // T = (I - N)^-1. The zeros above the block diagonal that the full-length products below read
      // (T[0:16, 16:32], T[32:48, 48:64]), then the diagonal 16x16 blocks (warp w: block w, lane c < 16 column c)
      for (int x = pt; x < 512; x += 128) {
        const int blk = x >> 8, r = (x >> 4) & 15, cc = x & 15;
        sTF[(blk * 32 + r) * PADF + blk * 32 + 16 + cc] = 0.f;
      }
      psync();  // N complete
      diag_inverse16<PADF>(sN, sTF, pw * 16, lane);
      psync();
      // stage 1: T[2b+1, 2b] = T[2b+1, 2b+1] N[2b+1, 2b] T[2b, 2b] (16x16 blocks, tf32; warp: block b = w >> 1,
      // 8 columns (w & 1) * 8)
      {
        const int hb = pw >> 1, ntile = pw & 1;
        const int bi = (2 * hb + 1) * 16, bj = 2 * hb * 16;
        float cacc[4] = {0.f, 0.f, 0.f, 0.f};
        tile_mma_tf32(cacc, &sN[bi * PADF + bj], PADF, &sTF[bj * PADF + bj + 8 * ntile], PADF, 16, lane);
        store_tile(cacc, &sM[(hb * 16) * PADM + 8 * ntile], PADM, lane);
      }
      psync();
      {
        const int hb = pw >> 1, ntile = pw & 1;
        const int bi = (2 * hb + 1) * 16, bj = 2 * hb * 16;
        float cacc[4] = {0.f, 0.f, 0.f, 0.f};
        tile_mma_tf32(cacc, &sTF[bi * PADF + bi], PADF, &sM[(hb * 16) * PADM + 8 * ntile], PADM, 16, lane);
        store_tile(cacc, &sTF[bi * PADF + bj + 8 * ntile], PADF, lane);
      }
      psync();
      // stage 2: T[32:, :32] = T[32:, 32:] N[32:, :32] T[:32, :32] (32x32 blocks, tf32; warp w: 8 columns w * 8,
      // both 16-row halves)
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        float cacc[4] = {0.f, 0.f, 0.f, 0.f};
        tile_mma_tf32(cacc, &sN[(32 + 16 * mt) * PADF], PADF, &sTF[8 * pw], PADF, 32, lane);
        store_tile(cacc, &sM[(16 * mt) * PADM + 8 * pw], PADM, lane);
      }
      psync();
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        float cacc[4] = {0.f, 0.f, 0.f, 0.f};
        tile_mma_tf32(cacc, &sTF[(32 + 16 * mt) * PADF + 32], PADF, &sM[8 * pw], PADM, 32, lane);
        store_tile(cacc, &sTF[(32 + 16 * mt) * PADF + 8 * pw], PADF, lane);
      }
      psync();
      // the beta and beta e^G factors go on T's columns: T1, T2 bf16 in the swizzled K-major layout (B operands of the
      // U, W products); T1's place held M until the psync above
      {
        const int j = (pt & 31) * 2, i0 = pt >> 5;  // thread: columns j, j+1 of rows i0, i0 + 4, ...
        const float b0 = sBeta[j], b1 = sBeta[j + 1], e0 = seG[j], e1 = seG[j + 1];
#pragma unroll
        for (int it = 0; it < CT / 4; ++it) {
          const int ii = i0 + 4 * it;
          const float2 t = *reinterpret_cast<const float2*>(&sTF[ii * PADF + j]);
          const float v0 = (j <= ii) ? t.x * b0 : 0.f, v1 = (j + 1 <= ii) ? t.y * b1 : 0.f;
          *reinterpret_cast<uint32_t*>(base + oT1 + swz(ii, j)) = pack_bf16(v0, v1);
          *reinterpret_cast<uint32_t*>(base + oT2 + swz(ii, j)) = pack_bf16(v0 * e0, v1 * e1);
        }
      }
      fence_async_smem();
      fence_before();
      psync();
      fence_after();
      // P2: U^T = V^T (T diag(beta))^T and W^T = K^T (T diag(beta e^G))^T (M = 128 value / key columns, N = 64 tokens
      // i, K = 64 tokens j): A = the V / K tile read MN-major (its two 64-column atoms LBO apart), B = T1 / T2
      if (pt == 0) {
        if (wait_bar(&bars.v_full, i & 1, p.err)) {
          fence_after();
#pragma unroll
          for (int s = 0; s < CT / 16; ++s) {
            mma(tm + cP, sdesc(sbase + oV + s * 16 * 128, 8192, 1024), sdesc(sbase + oT1 + s * 32, 16, 1024),
                idesc(128, 64, 1, 0), s > 0);
            mma(tm + cP + 64, sdesc(stage + oKQ + s * 16 * 128, 16384, 1024), sdesc(sbase + oT2 + s * 32, 16, 1024),
                idesc(128, 64, 1, 0), s > 0);
          }
          commit(&bars.p2_done);
        }
      }
      ok = group_and<3>(wait_bar(&bars.p2_done, i & 1, p.err));
      if (!ok) break;
      fence_after();
      // P2 epilogue, warp pw: lane d = 32 pw + lane holds value column d of U^T and key column d of W^T for the 64
      // tokens. U^T row d goes to the stage as eight swizzled 16-byte units; W [token][k]: lanes d and d^1 swap one
      // token of each pair, so every lane stores two columns of one token
      {
        const int d = 32 * pw + lane, odd = lane & 1, kk = d & ~1;
#pragma unroll 1
        for (int tb = 0; tb < CT; tb += 32) {
          float u[32];
          tld32f(la + tb, u);
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            const int c = tb / 8 + c4;
            *reinterpret_cast<uint4*>(stg + oU + d * 128 + ((c ^ (d & 7)) << 4)) =
                make_uint4(pack_bf16(u[8 * c4], u[8 * c4 + 1]), pack_bf16(u[8 * c4 + 2], u[8 * c4 + 3]),
                           pack_bf16(u[8 * c4 + 4], u[8 * c4 + 5]), pack_bf16(u[8 * c4 + 6], u[8 * c4 + 7]));
          }
          float w[32];
          tld32f(la + 64 + tb, w);
#pragma unroll
          for (int t = 0; t < 32; t += 2) {
            const float mine = odd ? w[t + 1] : w[t];  // this lane's column at the token it stores
            const float give = odd ? w[t] : w[t + 1];  // the partner's token
            const float got = __shfl_xor_sync(0xffffffffu, give, 1);
            const int tok = tb + t + odd;
            *reinterpret_cast<uint32_t*>(stg + oW + (kk >> 6) * 8192 + swz(tok, kk & 63)) =
                odd ? pack_bf16(got, mine) : pack_bf16(mine, got);
          }
        }
      }
      fence_async_smem();  // W is an MMA operand
      fence_before();
      bar_arrive(&bars.prep_done[st]);
      psync();  // every TMEM read of this chunk's P2 precedes the next chunk's P1
    }
    // no prep MMA in flight at the wind-down (the loop waits for every one it issues, unless a wait ran out)
    if (pt == 0) {
      commit(&bars.pdrain);
      wait_bar_quiet(&bars.pdrain, 0, p.err);
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------------------------------------- output warps
    // O = e^G scale (Q S) + QK V' of chunk c, staged row-major [tok][v] in the stage's U^T tile (consumed by then)
    // and stored, while the value-column warps and the tensor core go on with chunk c+1
    const int v = 32 * (warp & 3) + lane;  // TMEM lane
    const uint32_t la = tm + ((uint32_t)(32 * (warp & 3)) << 16);
    bool ok = true;
    for (int i = 0; i < nch && ok; ++i) {
      const int st = i & 1;
      unsigned char* stg = base + st * kStage;
      const int64_t t0 = r0 + (int64_t)i * CT;
      const int nt = (r1 - t0) < CT ? (int)(r1 - t0) : CT;
      ok = group_and<2>(wait_bar(&bars.st_done, i & 1, p.err));
      if (!ok) break;
      fence_after();
      __nv_bfloat16* ost = reinterpret_cast<__nv_bfloat16*>(stg + oU);
      uint32_t res[CT / 2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float ot[32], o2[32];
        tld32f(la + cOT + 32 * hh, ot);
        tld32f(la + cVT + 32 * hh, o2);
#pragma unroll
        for (int e = 0; e < 32; e += 2)
          res[16 * hh + e / 2] = pack_bf16(ot[e] * s_fq[st][32 * hh + e] + o2[e],
                                           ot[e + 1] * s_fq[st][32 * hh + e + 1] + o2[e + 1]);
      }
      fence_before();
      bar_arrive(&bars.acc_free);  // OT and O2T are read: the next chunk's products may overwrite them
#pragma unroll
      for (int e = 0; e < CT; e += 2) {
        const __nv_bfloat162 pr = *reinterpret_cast<const __nv_bfloat162*>(&res[e / 2]);
        ost[e * DH + v] = pr.x;
        ost[(e + 1) * DH + v] = pr.y;
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
      bar_arrive(&bars.stage_free[st]);  // the stage may take chunk c+2
    }
  } else {
    // -------------------------------------------------------------------------------------------- value columns
    const int v = tid;  // TMEM lane
    const uint32_t la = tm + ((uint32_t)(32 * warp) << 16);
    const float* s0 = p.state_in ? p.state_in + ((int64_t)(p.state_row ? p.state_row[row] : row) * p.Hv + h) * DH * DH
                                 : nullptr;
    // the initial state: ST (fp32) and its bf16 copy SB, column v of S = lane v of S^T (32 rows at a time: this
    // kernel's threads have 128 registers)
#pragma unroll 1
    for (int k0 = 0; k0 < DH; k0 += 32) {
      uint32_t w[32], b[16];
#pragma unroll
      for (int e = 0; e < 32; ++e) w[e] = __float_as_uint(s0 ? s0[(int64_t)(k0 + e) * DH + v] : 0.f);
#pragma unroll
      for (int e = 0; e < 16; ++e) b[e] = pack_bf16(__uint_as_float(w[2 * e]), __uint_as_float(w[2 * e + 1]));
      tst16(la + cST + k0, w);
      tst16(la + cST + k0 + 16, w + 16);
      tst16(la + cSB + k0 / 2, b);
    }
    tst_wait();
    fence_before();
    bar_arrive(&bars.sb_ready);
    bool ok = true;
    for (int i = 0; i < nch && ok; ++i) {
      const int st = i & 1;
      unsigned char* stg = base + st * kStage;
      ok = group_and<1>(wait_bar(&bars.prep_done[st], (i >> 1) & 1, p.err));
      if (!ok) break;
      {  // G -> (fq, fk) per token and the chunk's decay
        const float* G = reinterpret_cast<const float*>(stg + oG);
        const float gl = G[CT - 1];  // past a row's end G stays flat, so the last entry is the row's last token's
        if (v < CT) {
          s_fq[st][v] = expf(G[v]) * p.scale;
          s_fk[v] = expf(gl - G[v]);
        }
        if (v == 0) s_dl = expf(gl);
      }
      vsync();
      // the state decays by e^(G_last) before the update accumulates onto it, while VT = S^T W^T runs (the
      // products read the bf16 copy, not ST); a decay that underflowed to 0 leaves nothing of the state, and the
      // update MMA overwrites it instead
      const float dl = s_dl;
      if (dl != 0.f) {
#pragma unroll 1
        for (int k0 = 0; k0 < DH; k0 += 32) {
          float f[32];
          tld32f(la + cST + k0, f);
          uint32_t w[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) w[e] = __float_as_uint(f[e] * dl);
          tst16(la + cST + k0, w);
          tst16(la + cST + k0 + 16, w + 16);
        }
      }
      ok = group_and<1>(wait_bar(&bars.vt_done, i & 1, p.err));
      if (!ok) break;
      fence_after();
      // V' = U - S W (fp32) -> V'^T and (V' f_k)^T as bf16 A operands, 32 tokens at a time
      {
        const unsigned char* ut = stg + oU + v * 128;  // U^T row v: eight 16-byte units, swizzled by v & 7
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint4 uu[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) uu[c] = *reinterpret_cast<const uint4*>(ut + (((4 * hh + c) ^ (v & 7)) << 4));
          float vt[32];
          tld32f(la + cVT + 32 * hh, vt);
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float2 u2 = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(&uu[c])[q]);
              vt[8 * c + 2 * q] = u2.x - vt[8 * c + 2 * q];
              vt[8 * c + 2 * q + 1] = u2.y - vt[8 * c + 2 * q + 1];
            }
          uint32_t vb[16], vd[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            vb[e] = pack_bf16(vt[2 * e], vt[2 * e + 1]);
            vd[e] = pack_bf16(vt[2 * e] * s_fk[32 * hh + 2 * e], vt[2 * e + 1] * s_fk[32 * hh + 2 * e + 1]);
          }
          tst16(la + cVB + 16 * hh, vb);
          tst16(la + cVD + 16 * hh, vd);
        }
      }
      tst_wait();
      fence_before();
      bar_arrive(&bars.vb_ready);
      ok = group_and<1>(wait_bar(&bars.st_done, i & 1, p.err));
      if (!ok) break;
      fence_after();
      // the next chunk's bf16 state first: it releases the next chunk's products
#pragma unroll 1
      for (int k0 = 0; k0 < DH; k0 += 32) {
        float f[32];
        uint32_t b[16];
        tld32f(la + cST + k0, f);
#pragma unroll
        for (int e = 0; e < 16; ++e) b[e] = pack_bf16(f[2 * e], f[2 * e + 1]);
        tst16(la + cSB + k0 / 2, b);
      }
      tst_wait();
      fence_before();
      bar_arrive(&bars.sb_ready);
    }
    // the final state (the last update is complete: st_done of the last chunk was waited for above)
    if (p.state_out && ok) {
      float* so = p.state_out + ((int64_t)row * p.Hv + h) * DH * DH;
#pragma unroll 1
      for (int k0 = 0; k0 < DH; k0 += 32) {
        float f[32];
        tld32f(la + cST + k0, f);
#pragma unroll
        for (int e = 0; e < 32; ++e) so[(int64_t)(k0 + e) * DH + v] = f[e];
      }
    }
  }
  // wind down: every MMA of the state pass has completed before TMEM is released
  fence_before();
  __syncthreads();
  fence_after();
  wait_bar_quiet(&bars.drain, 0, p.err);
  fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(kTmemCols));
}

}  // namespace gsf

int map3d(CUtensorMap* m, const void* ptr, uint64_t T, uint64_t H);

}  // namespace jb

using namespace jb;

extern "C" int janus_b200_gdn_chunk_scan_fused(const void* q, const void* k, const void* v, const float* g,
                                               const float* beta, int64_t T, int64_t B, const int32_t* row_start,
                                               const int32_t* chunk_start, int64_t n_chunks, const float* state_in,
                                               const int32_t* state_row, float* state_out, int64_t Hk, int64_t Hv,
                                               int64_t Dk, int64_t Dv, float scale, void* o, int32_t* status,
                                               void* stream) {
  JB_REQUIRE(q && k && v && g && beta && row_start && chunk_start && o, JANUS_ERR_INVALID,
             "gdn_chunk_scan_fused: null pointer");
  JB_REQUIRE(Dk == gsf::DH && Dv == gsf::DH, JANUS_ERR_UNSUPPORTED,
             "gdn_chunk_scan_fused: Dk = Dv = 128 only (got %lld, %lld)", (long long)Dk, (long long)Dv);
  JB_REQUIRE(T >= 0 && T <= 0x7fffffff && B >= 0 && B <= 65535 && n_chunks >= 0 && Hk > 0 && Hv > 0 &&
                 Hv % Hk == 0 && Hv <= 65535,
             JANUS_ERR_INVALID, "gdn_chunk_scan_fused: sizes");
  JB_REQUIRE(JB_ALIGNED(q, 16) && JB_ALIGNED(k, 16) && JB_ALIGNED(v, 16) && JB_ALIGNED(o, 16), JANUS_ERR_ALIGNMENT,
             "gdn_chunk_scan_fused: q, k, v, o must be 16-byte aligned");
  if (B == 0) return JANUS_OK;
  gsf::Params p{};
  int st = map3d(&p.qmap, q, (uint64_t)(T > 0 ? T : 1), (uint64_t)Hk);
  if (!st) st = map3d(&p.kmap, k, (uint64_t)(T > 0 ? T : 1), (uint64_t)Hk);
  if (!st) st = map3d(&p.vmap, v, (uint64_t)(T > 0 ? T : 1), (uint64_t)Hv);
  if (st) return st;
  p.g = g;
  p.beta = beta;
  p.row_start = row_start;
  p.chunk_start = chunk_start;
  p.state_in = state_in;
  p.state_row = state_row;
  p.state_out = state_out;
  p.o = (__nv_bfloat16*)o;
  p.err = status;
  p.Hk = (int)Hk;
  p.Hv = (int)Hv;
  p.scale = scale;
  const size_t smem = gsf::kSmem + 1024;
  cudaError_t e =
      cudaFuncSetAttribute(gsf::gdn_scan_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    set_error("gdn_chunk_scan_fused: smem attribute %s", cudaGetErrorString(e));
    return JANUS_ERR_CUDA;
  }
  gsf::gdn_scan_fused_kernel<<<dim3((unsigned)Hv, (unsigned)B), gsf::NT, smem, (cudaStream_t)stream>>>(p);
  return launch_status("gdn_chunk_scan_fused");
}
