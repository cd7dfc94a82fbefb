// Gated delta rule over long rows in 64-token chunks (the state level), in two launches.
//
// 1. gdn_chunk_prep: one CTA per (chunk, value head), all chunks of all rows in parallel. With G the in-chunk
//    cumulative g (every exponential is of a difference of G, so nothing overflows):
//      N  = -tril_strict(diag(beta) K K^T * e^(G_i - G_j))          tcgen05 (M = 128: [K; Q] K^T), fp32 in TMEM
//      QK = tril(scale Q K^T * e^(G_i - G_j))                        the same product's lower half, stored bf16
//      T  = (I - N)^-1                                               fp32: 16x16 diagonal blocks by substitution,
//                                                                    then doubling stages 16 -> 32 -> 64 (tf32 MMAs)
//      U  = (T diag(beta)) V,  W = (T diag(beta e^G)) K              tcgen05 as U^T = V^T (T diag(beta))^T and
//                                                                    W^T = K^T (T diag(beta e^G))^T (M = 128
//                                                                    value / key columns), stored bf16
//    K, Q, V arrive by TMA; U, W, QK leave by TMA stores from swizzled staging tiles.
// 2. the sequential pass (gdn_state_tc.cu, tcgen05): one CTA per (row, value head) walking the row's chunks in
//    order with the fp32 state in TMEM:
//      V' = U - W S;   O = scale e^G (Q S) + QK V';   S = e^(G_last) S + K^T (V' * e^(G_last - G))
//    (S rounded to bf16 for the products, as fla's chunk kernels do; the e^G factors scale rows of fp32 results
//    instead of the bf16 operands, so q and k are used as loaded). The WY form of transformers'
//    torch_chunk_gated_delta_rule (the reference's CPU rule) and of fla's chunk kernels (its GPU rule). A row's last
//    chunk is ragged: the tokens past its end get g = beta = 0 and are masked, which leaves the state untouched.
// With a segment id per token (the state fork packed into chunks: sibling rows of one parent share a chunk), G is a
// cumulative sum within each segment and every mask also requires the same segment, so each segment runs from the
// chunk's initial state on its own.
// The prep writes W, QK and G chunk-major ([chunk][value head][64 tokens], zeros past a row's end) and U transposed
// ([chunk][value head][128 value columns][64 tokens], the rows the sequential pass's value threads read) for the
// sequential pass's TMA loads.
#include "gdn_inverse.cuh"
#include "tcgen05.cuh"

namespace jb {
namespace {

constexpr int CT = 64;   // chunk tokens
constexpr int DH = 128;  // Dk = Dv
constexpr int PADF = 68;  // fp32 [64][68] tiles: row stride = 4 banks, tf32 A fragments hit 32 distinct banks
constexpr int PADM = 40;  // fp32 [32][40]: stride = 8 banks, the B fragments read from it hit 32 distinct banks

// tf32 tensor-core products on fp32 shared tiles, for the blocks of the triangular inverse (tf32 keeps 10 mantissa
// bits, more than the bf16 that T is rounded to afterwards; fla's Triton solve multiplies its fp32 blocks in tf32 too)
__device__ __forceinline__ uint32_t tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
// C[16 x 8] += A[16 x K] B[K x 8] (row-major fp32, leading dimensions lda, ldb), K a multiple of 8
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
// the 16 x 8 accumulator tile to a row-major fp32 matrix
__device__ __forceinline__ void store_tile(const float* c, float* D, int ldd, int lane) {
  const int g = lane >> 2, t = lane & 3;
  D[g * ldd + 2 * t] = c[0];
  D[g * ldd + 2 * t + 1] = c[1];
  D[(g + 8) * ldd + 2 * t] = c[2];
  D[(g + 8) * ldd + 2 * t + 1] = c[3];
}

// the row of global chunk c (chunk_start: prefix sum of the rows' chunk counts, rows with no chunk skipped over)
__device__ __forceinline__ int chunk_row(const int32_t* chunk_start, int B, int c) {
  int lo = 0, hi = B;  // invariant: chunk_start[lo] <= c < chunk_start[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (chunk_start[mid] <= c) lo = mid; else hi = mid;
  }
  return lo;
}

// ------------------------------------------------------------------------------------------------ chunk prep

// Shared memory of the prep (byte offsets from a 1024-aligned base), small enough for four CTAs per SM: regions are
// reused as their contents die. Operand tiles are in the UMMA 128B-swizzled K-major layout: [64-column atom][rows]
// [128 bytes], the 16-byte unit u of row r at (u ^ (r & 7)) * 16.
//   KQ [2 atoms][128 rows]: rows 0-63 the chunk's K, rows 64-127 its Q, so [K; Q] is one M=128 operand and K alone
//      (rows 0-63) the N=64 one. Once Q is consumed, the Q half of atom 0 stages QK for its TMA store and then holds
//      T1 = T diag(beta); the Q half of atom 1 holds the fp32 scratch M of the inverse, then T2 = T diag(beta e^G)
//   NV fp32 N [64][PADF], inverted in place into T = (I - N)^-1 block by block; once T is consumed (T1, T2 built),
//      the chunk's V [2 atoms][64 rows] (a second TMA load)
constexpr uint32_t kOffKQ = 0, kOffT1 = 8192, kOffM = 16384 + 8192, kOffT2 = 16384 + 8192;
constexpr uint32_t kOffNV = 32768;  // 1024-byte boundary
constexpr uint32_t kOffVec = kOffNV + CT * PADF * 4;  // G, eG, beta, graw (fp32 [64]), seg (int [64])
constexpr uint32_t kOffBar = kOffVec + 5 * CT * 4;
constexpr uint32_t kPrepSmem = kOffBar + 32 + 1024;  // + alignment slack
constexpr uint32_t kPrepTmemCols = 128;  // P1 (KK^T | QK^T) cols 0-63, then U^T cols 0-63 and W^T cols 64-127
// after P2 the [K; Q] region holds the staged W (two [64 tokens][64 columns] boxes) and U^T ([128][64 tokens])
constexpr uint32_t kOffWst = 0, kOffUst = 16384;
static_assert(CT * PADF * 4 >= 2 * CT * 64 * 2 && 32 * PADM * 4 <= 8192, "prep shared-memory regions");
static_assert(4 * (kPrepSmem + 1024) <= 228 * 1024, "four prep CTAs per SM");

struct PrepParams {
  CUtensorMap qmap, kmap, vmap;       // [T][H][128] bf16 loads, boxes 64 dims x 1 head x 64 tokens
  CUtensorMap qkmap;                  // chunk-major QK store, boxes 64 x 64
  CUtensorMap wmap;                   // W store: chunk-major [chunk][head][64 tokens][128], boxes 64 x 64
  CUtensorMap umap;                   // U^T store: [chunk][head][128 value columns][64 tokens], boxes 64 x 128
  const float* g;
  const float* beta;
  const int32_t* row_start;
  const int32_t* chunk_start;
  const int32_t* segment;
  float* Gg;
  int32_t* err;
  int B, Hk, Hv;
  float scale;
};

// 2D TMA tile store from this CTA's shared memory (no multicast); x is a multiple of 64 elements (16-byte rule)
__device__ __forceinline__ void tma_store2(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
// byte offset of element (r, c) of a 64-column swizzled atom [rows][128 B]
__device__ __forceinline__ uint32_t swz(int r, int c) { return r * 128 + ((((c >> 3) ^ r) & 7) << 4) + (c & 7) * 2; }

__global__ void __launch_bounds__(256, 4) gdn_chunk_prep_kernel(const __grid_constant__ PrepParams p) {
  extern __shared__ unsigned char raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = tcx::s32(base);
  float* sN = reinterpret_cast<float*>(base + kOffNV);
  float* sTF = sN;  // T overwrites N block by block
  float* sM = reinterpret_cast<float*>(base + kOffM);
  float* sG = reinterpret_cast<float*>(base + kOffVec);
  float* seG = sG + CT;
  float* sBeta = sG + 2 * CT;
  float* sGraw = sG + 3 * CT;
  float* sGl = sGraw;  // G log2(e), once the scan is done
  int32_t* sSeg = reinterpret_cast<int32_t*>(sG + 4 * CT);
  uint64_t* bar_load = reinterpret_cast<uint64_t*>(base + kOffBar);
  uint64_t* bar_mma = bar_load + 1;
  __shared__ uint32_t tmem_base;
  __shared__ int s_ok;

  const int h = blockIdx.x, c = blockIdx.y;  // heads fastest: the Hv/Hk heads sharing q and k run together
  const int hk = h / (p.Hv / p.Hk);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = chunk_row(p.chunk_start, p.B, c);
  const int64_t t0 = p.row_start[row] + (int64_t)(c - p.chunk_start[row]) * CT;
  const int64_t rend = p.row_start[row + 1];
  const int nt = (rend - t0) < CT ? (int)(rend - t0) : CT;
  const int rb = (c * p.Hv + h) * CT;  // first row of the chunk in the chunk-major workspace

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tcx::s32(&tmem_base)),
                 "r"(kPrepTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  if (tid == 0) {  // the barriers, then at once the K, Q, V tiles of the chunk (rows past the row's end meet
                   // beta = 0 and the masks)
    tcx::bar_init(bar_load, 1);
    tcx::bar_init(bar_mma, 1);
    s_ok = 1;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tcx::bar_expect_tx(bar_load, 2 * 2 * CT * 64 * 2);
#pragma unroll
    for (int a = 0; a < 2; ++a) {
      tcx::tma_load3(sbase + kOffKQ + a * 16384, &p.kmap, 64 * a, hk, (int)t0, bar_load);
      tcx::tma_load3(sbase + kOffKQ + a * 16384 + 8192, &p.qmap, 64 * a, hk, (int)t0, bar_load);
    }
  }
  if (tid < CT) {
    const bool in = tid < nt;  // tokens past the row's end: g = beta = 0 (they touch nothing)
    sGraw[tid] = in ? p.g[(t0 + tid) * p.Hv + h] : 0.f;
    sBeta[tid] = in ? p.beta[(t0 + tid) * p.Hv + h] : 0.f;
    sSeg[tid] = p.segment ? (in ? p.segment[t0 + tid] : -1) : 0;
  }
  tcx::fence_before();
  __syncthreads();
  tcx::fence_after();
  const uint32_t tm = tmem_base;
  if (tid == 0) {
    // P1: [K; Q] K^T (M = 128, N = 64, K = 128): lanes 0-63 K K^T, lanes 64-127 Q K^T, columns 0-63
    bool ok = tcx::wait_bar(bar_load, 0, p.err);
    if (ok) {
      tcx::fence_after();
#pragma unroll
      for (int s = 0; s < DH / 16; ++s) {
        const uint32_t off = kOffKQ + (s >> 2) * 16384 + (s & 3) * 32;
        tcx::mma(tm, tcx::sdesc(sbase + off, 16, 1024), tcx::sdesc(sbase + off, 16, 1024), tcx::idesc(128, 64, 0, 0),
                 s > 0);
      }
      tcx::commit(bar_mma);
    } else {
      s_ok = 0;
      tcx::wait_bar_quiet(bar_load, 0, p.err);  // the loads land before the CTA may leave
    }
  }
  if (warp == 1 && p.segment) {  // cumulative sum of g within each segment (a segmented scan, two tokens per lane)
    const float ga = sGraw[2 * lane], gb = sGraw[2 * lane + 1];
    const int sa = sSeg[2 * lane], sb = sSeg[2 * lane + 1], sp = lane > 0 ? sSeg[2 * lane - 1] : -2;
    const bool ha = sa != sp, hb = sb != sa;  // the token starts a segment
    float v = hb ? gb : ga + gb;               // the pair's sum within the segment its last token belongs to
    int f = (ha || hb) ? 1 : 0;                // a segment starts inside the range v covers
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, v, off);
      const int yf = __shfl_up_sync(0xffffffffu, f, off);
      if (lane >= off && !f) v += y;
      if (lane >= off) f |= yf;
    }
    const float prev = __shfl_up_sync(0xffffffffu, v, 1);  // up to the previous lane's last token
    const float Ga = ha ? ga : prev + ga;
    sG[2 * lane] = Ga;
    sG[2 * lane + 1] = hb ? gb : Ga + gb;
  } else if (warp == 1) {  // in-chunk cumulative sum of g (two values per lane)
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
  __syncthreads();
  if (tid < CT) {
    seG[tid] = expf(sG[tid]);
    sGl[tid] = sG[tid] * kLog2e;  // in the raw g's place (the scan has read it)
    p.Gg[(int64_t)rb + tid] = sG[tid];  // chunk-major; past the row's end G stays at G[nt - 1]
  }
  __syncthreads();
  const bool live = s_ok != 0;
  // P1 epilogue: warp w reads TMEM lanes 32 (w & 3) .. +31, columns 32 (w >> 2) .. +31. Lanes 0-63: N = -beta_i
  // (K K^T)_ij e^(G_i - G_j) for j < i in the same segment (fp32, shared); lanes 64-127: QK = scale (Q K^T)_ij
  // e^(G_i - G_j) for j <= i in the same segment, rows past the row's end zero (bf16, staged for the TMA store)
  if (live) {
    const bool done = __all_sync(0xffffffffu, tcx::wait_bar(bar_mma, 0, p.err));
    tcx::fence_after();
    const int qw = warp & 3, j0 = (warp >> 2) * 32;
    const int i = 32 * (qw & 1) + lane;
    const uint32_t la = tm + ((uint32_t)(32 * qw) << 16) + j0;
    // rows 0-31 against columns 32-63 lie wholly above the diagonal: both masks are zero there (warps 4 and 6)
    const bool none = (qw & 1) == 0 && j0 == 32;
    float d[32];
    if (!none) {
      tcx::tld16f(la, d);
      tcx::tld16f(la + 16, d + 16);
    }
    if (done && none) {
      if (qw < 2) {
#pragma unroll
        for (int x = 0; x < 32; x += 4) *reinterpret_cast<float4*>(&sN[i * PADF + j0 + x]) = make_float4(0, 0, 0, 0);
      } else {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          *reinterpret_cast<uint4*>(base + kOffKQ + 8192 + swz(i, j0 + 8 * u)) = make_uint4(0, 0, 0, 0);
        tcx::fence_async_smem();
      }
    } else if (done) {
      // branch-free: the masks select (a divergent branch per element is slow); the segment compare only runs for a
      // segmented scan; G log2(e) of the columns four at a time
      const float gli = sGl[i];
      const int si = sSeg[i];
      const bool segs = p.segment != nullptr;
      const float4* gl4 = reinterpret_cast<const float4*>(sGl + j0);
      const int4* sg4 = reinterpret_cast<const int4*>(sSeg + j0);
      if (qw < 2) {
        const float nb = -sBeta[i];
#pragma unroll
        for (int x = 0; x < 32; x += 4) {  // each group of 4 entries stored as it is made (few live registers)
          const float4 g = gl4[x / 4];
          const int4 sg = segs ? sg4[x / 4] : make_int4(si, si, si, si);
          const float gj[4] = {g.x, g.y, g.z, g.w};
          const int sj[4] = {sg.x, sg.y, sg.z, sg.w};
          float nv[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) nv[u] = n_entry(d[x + u], nb, gli, gj[u], (j0 + x + u < i) & (sj[u] == si));
          *reinterpret_cast<float4*>(&sN[i * PADF + j0 + x]) = make_float4(nv[0], nv[1], nv[2], nv[3]);
        }
      } else {
        const bool il = i < nt;
#pragma unroll
        for (int x = 0; x < 32; x += 8) {  // each 16-byte unit stored as it is made
          uint32_t qv[4];
#pragma unroll
          for (int y = 0; y < 8; y += 4) {
            const float4 g = gl4[(x + y) / 4];
            const int4 sg = segs ? sg4[(x + y) / 4] : make_int4(si, si, si, si);
            const float gj[4] = {g.x, g.y, g.z, g.w};
            const int sj[4] = {sg.x, sg.y, sg.z, sg.w};
            float e[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
              e[u] = qk_entry(d[x + y + u], p.scale, gli, gj[u], (j0 + x + y + u <= i) & il & (sj[u] == si));
            qv[y / 2] = tcx::pack_bf16(e[0], e[1]);
            qv[y / 2 + 1] = tcx::pack_bf16(e[2], e[3]);
          }
          *reinterpret_cast<uint4*>(base + kOffKQ + 8192 + swz(i, j0 + x)) = make_uint4(qv[0], qv[1], qv[2], qv[3]);
        }
        tcx::fence_async_smem();  // the staged QK is read by the TMA store
      }
    }
  }
  __syncthreads();  // N complete
  if (tid == 0 && live) {  // the staged QK leaves while the inverse runs (its read is waited for before T1)
    tma_store2(&p.qkmap, sbase + kOffKQ + 8192, 0, rb);
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  }
  // T = (I - N)^-1 in place: diagonal 16x16 blocks (warps 0-3, lane c < 16 owns column c). The zeros above the block
  // diagonal that the full-length products below read (T[0:16, 16:32], T[32:48, 48:64]) are N's, already in place.
  if (warp < 4) diag_inverse16<PADF>(sN, sTF, warp * 16, lane);
  __syncthreads();
  // stage 1: T[2h+1, 2h] = T[2h+1, 2h+1] N[2h+1, 2h] T[2h, 2h] (16x16 blocks), h = 0, 1, on the tensor cores in
  // tf32 (warps 0-3: block h = w >> 1, 8 columns (w & 1) * 8). The triangular zeros of N and T make full-length
  // products exact.
  if (warp < 4) {
    const int hb = warp >> 1, ntile = warp & 1;
    const int bi = (2 * hb + 1) * 16, bj = 2 * hb * 16;
    float cacc[4] = {0.f, 0.f, 0.f, 0.f};
    tile_mma_tf32(cacc, &sN[bi * PADF + bj], PADF, &sTF[bj * PADF + bj + 8 * ntile], PADF, 16, lane);
    store_tile(cacc, &sM[(hb * 16) * PADM + 8 * ntile], PADM, lane);
  }
  __syncthreads();
  if (warp < 4) {
    const int hb = warp >> 1, ntile = warp & 1;
    const int bi = (2 * hb + 1) * 16, bj = 2 * hb * 16;
    float cacc[4] = {0.f, 0.f, 0.f, 0.f};
    tile_mma_tf32(cacc, &sTF[bi * PADF + bi], PADF, &sM[(hb * 16) * PADM + 8 * ntile], PADM, 16, lane);
    store_tile(cacc, &sTF[bi * PADF + bj + 8 * ntile], PADF, lane);
  }
  __syncthreads();
  // stage 2: T[32:, :32] = T[32:, 32:] N[32:, :32] T[:32, :32] (32x32 blocks, tf32; warp: rows 16 (w >> 2), 8 columns
  // (w & 3) * 8)
  {
    const int mt = warp >> 2, ntile = warp & 3;
    float cacc[4] = {0.f, 0.f, 0.f, 0.f};
    tile_mma_tf32(cacc, &sN[(32 + 16 * mt) * PADF], PADF, &sTF[8 * ntile], PADF, 32, lane);
    store_tile(cacc, &sM[(16 * mt) * PADM + 8 * ntile], PADM, lane);
    __syncthreads();
    cacc[0] = cacc[1] = cacc[2] = cacc[3] = 0.f;
    tile_mma_tf32(cacc, &sTF[(32 + 16 * mt) * PADF + 32], PADF, &sM[8 * ntile], PADM, 32, lane);
    store_tile(cacc, &sTF[(32 + 16 * mt) * PADF + 8 * ntile], PADF, lane);
  }
  if (tid == 0 && live) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // QK staging read: T1's place
  __syncthreads();
  // the beta and beta e^G factors of the tokens go on T's columns (rather than on V's and K's rows): T1, T2 bf16 in
  // the swizzled K-major layout (B operands of the U, W products)
  {
    const int j = (tid & 31) * 2, i0 = tid >> 5;  // thread: columns j, j+1 of rows i0, i0 + 8, ... (loads in flight together)
    const float b0 = sBeta[j], b1 = sBeta[j + 1], e0 = seG[j], e1 = seG[j + 1];
#pragma unroll
    for (int it = 0; it < CT / 8; ++it) {
      const int i = i0 + 8 * it;
      const float2 t = *reinterpret_cast<const float2*>(&sTF[i * PADF + j]);
      const float v0 = (j <= i) ? t.x * b0 : 0.f, v1 = (j + 1 <= i) ? t.y * b1 : 0.f;
      *reinterpret_cast<uint32_t*>(base + kOffT1 + swz(i, j)) = tcx::pack_bf16(v0, v1);
      *reinterpret_cast<uint32_t*>(base + kOffT2 + swz(i, j)) = tcx::pack_bf16(v0 * e0, v1 * e1);
    }
  }
  tcx::fence_async_smem();
  tcx::fence_before();
  __syncthreads();
  tcx::fence_after();
  if (tid == 0 && live) {  // T is consumed: the chunk's V goes into its place (the U product needs it)
    tcx::bar_expect_tx(bar_load, 2 * CT * 64 * 2);
    tcx::tma_load3(sbase + kOffNV, &p.vmap, 0, h, (int)t0, bar_load);
    tcx::tma_load3(sbase + kOffNV + 8192, &p.vmap, 64, h, (int)t0, bar_load);
  }
  // P2: U^T = V^T (T diag(beta))^T and W^T = K^T (T diag(beta e^G))^T (M = 128 value / key columns, N = 64 tokens i,
  // K = 64 tokens j): A = the V / K tile read MN-major (its two 64-column atoms LBO apart), B = T1 / T2 K-major; the
  // accumulators reuse P1's TMEM columns (read out long ago)
  bool p2 = false;  // (thread 0) the U, W products were issued
  if (tid == 0 && live) {
    if (tcx::wait_bar(bar_load, 1, p.err)) {
      p2 = true;
      tcx::fence_after();
#pragma unroll
      for (int s = 0; s < CT / 16; ++s) {
        tcx::mma(tm, tcx::sdesc(sbase + kOffNV + s * 16 * 128, 8192, 1024), tcx::sdesc(sbase + kOffT1 + s * 32, 16, 1024),
                 tcx::idesc(128, 64, 1, 0), s > 0);
        tcx::mma(tm + 64, tcx::sdesc(sbase + kOffKQ + s * 16 * 128, 16384, 1024),
                 tcx::sdesc(sbase + kOffT2 + s * 32, 16, 1024), tcx::idesc(128, 64, 1, 0), s > 0);
      }
      tcx::commit(bar_mma);
    } else {
      s_ok = 0;
      tcx::wait_bar_quiet(bar_load, 1, p.err);  // the V load lands before the CTA may leave
    }
  }
  // P2 epilogue: warps 0-3 U^T (lane = value column d), warps 4-7 W^T (lane = key column d), bf16, staged in the
  // [K; Q] region (every operand there has been read by P2) in the swizzled layouts of the workspace's tensor maps
  // and written by TMA stores. U is kept transposed ([value column][64 tokens], the row the state pass's value thread
  // reads): a lane writes its column's row. W is [token][128]: lanes d and d^1 swap one token of each pair, so every
  // lane writes two columns of one token.
  if (live) {
    const bool done = __all_sync(0xffffffffu, tcx::wait_bar(bar_mma, 1, p.err));
    if (!done) s_ok = 0;
    tcx::fence_after();
    const int qw = warp & 3, isw = warp >> 2;
    const int dcol = 32 * qw + lane, odd = lane & 1;
    unsigned char* wst = base + kOffWst + (dcol >> 6) * 8192;  // the W box of this lane's column
#pragma unroll 1
    for (int tb = 0; tb < CT; tb += 32) {
      float d[32];
      const uint32_t la = tm + ((uint32_t)(32 * qw) << 16) + 64 * isw + tb;
      tcx::tld16f(la, d);
      tcx::tld16f(la + 16, d + 16);
      if (done && !isw) {
#pragma unroll
        for (int t = 0; t < 32; t += 8)
          *reinterpret_cast<uint4*>(base + kOffUst + swz(dcol, tb + t)) =
              make_uint4(tcx::pack_bf16(d[t], d[t + 1]), tcx::pack_bf16(d[t + 2], d[t + 3]),
                         tcx::pack_bf16(d[t + 4], d[t + 5]), tcx::pack_bf16(d[t + 6], d[t + 7]));
      } else if (done) {
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          const float mine = odd ? d[t + 1] : d[t];  // this lane's column at the token it stores
          const float give = odd ? d[t] : d[t + 1];  // the partner's token
          const float got = __shfl_xor_sync(0xffffffffu, give, 1);
          const uint32_t w2 = odd ? tcx::pack_bf16(got, mine) : tcx::pack_bf16(mine, got);
          *reinterpret_cast<uint32_t*>(wst + swz(tb + t + odd, (dcol & 63) & ~1)) = w2;
        }
      }
    }
  }
  tcx::fence_async_smem();  // the staged tiles are read by the TMA stores
  __syncthreads();
  if (tid == 0 && live && s_ok) {
    tma_store2(&p.umap, sbase + kOffUst, 0, 2 * rb);
    tma_store2(&p.wmap, sbase + kOffWst, 0, rb);
    tma_store2(&p.wmap, sbase + kOffWst + 8192, 64, rb);
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    // the staging has been read before the CTA leaves; the writes themselves complete with the grid, before the
    // state pass (the next launch in the stream) reads them
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  }
  if (p2) tcx::wait_bar_quiet(bar_mma, 1, p.err);  // no MMA in flight at the dealloc (the epilogue waited already)
  tcx::fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(kPrepTmemCols));
}

size_t align_up(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace
}  // namespace jb

using namespace jb;

extern "C" size_t janus_b200_gdn_chunk_scan_workspace(int64_t T, int64_t n_chunks, int64_t Hv) {
  (void)T;
  const size_t rows = (size_t)n_chunks * Hv * CT;  // chunk-major: [chunk][head][64 tokens]
  return 2 * align_up(rows * DH * sizeof(__nv_bfloat16)) + align_up(rows * CT * 2) + align_up(rows * sizeof(float));
}

namespace jb {
int map2d(CUtensorMap* m, const void* ptr, uint64_t cols, uint64_t rows, uint32_t box_rows);
int map3d(CUtensorMap* m, const void* ptr, uint64_t T, uint64_t H);
int gdn_state_tc(const void* q, const void* k, int64_t T, int64_t B, const int32_t* row_start,
                 const int32_t* chunk_start, int64_t n_chunks, const float* state_in, const int32_t* state_row,
                 float* state_out, int64_t Hk, int64_t Hv, float scale, const void* W, const void* U, const void* QK,
                 const float* G, int32_t* err, void* o, cudaStream_t stream);
}

extern "C" int janus_b200_gdn_chunk_scan(const void* q, const void* k, const void* v, const float* g,
                                         const float* beta, int64_t T, int64_t B, const int32_t* row_start,
                                         const int32_t* chunk_start, int64_t n_chunks, const float* state_in,
                                         const int32_t* state_row, const int32_t* segment, float* state_out,
                                         int64_t Hk, int64_t Hv,
                                         int64_t Dk, int64_t Dv, float scale, void* workspace, size_t workspace_bytes,
                                         void* o, int32_t* status, void* stream) {
  JB_REQUIRE(q && k && v && g && beta && row_start && chunk_start && o, JANUS_ERR_INVALID,
             "gdn_chunk_scan: null pointer");
  JB_REQUIRE(Dk == DH && Dv == DH, JANUS_ERR_UNSUPPORTED, "gdn_chunk_scan: Dk = Dv = 128 only (got %lld, %lld)",
             (long long)Dk, (long long)Dv);
  JB_REQUIRE(T >= 0 && T <= 0x7fffffff && B >= 0 && B <= 65535 && n_chunks >= 0 && n_chunks <= 65535 && Hk > 0 &&
                 Hv > 0 && Hv % Hk == 0 && Hv <= 65535 && n_chunks * Hv * 2 * CT <= 0x7fffffff,
             JANUS_ERR_INVALID, "gdn_chunk_scan: sizes");
  JB_REQUIRE(JB_ALIGNED(q, 16) && JB_ALIGNED(k, 16) && JB_ALIGNED(v, 16) && JB_ALIGNED(o, 16), JANUS_ERR_ALIGNMENT,
             "gdn_chunk_scan: q, k, v, o must be 16-byte aligned");
  JB_REQUIRE(!segment || !state_out, JANUS_ERR_INVALID,
             "gdn_chunk_scan: a segmented scan has no final state (its segments each end their own)");
  const size_t need = janus_b200_gdn_chunk_scan_workspace(T, n_chunks, Hv);
  JB_REQUIRE(workspace && workspace_bytes >= need && JB_ALIGNED(workspace, 256), JANUS_ERR_WORKSPACE,
             "gdn_chunk_scan: workspace %zu bytes (256-aligned) < %zu", workspace_bytes, need);
  if (B == 0 || T == 0) return JANUS_OK;
  const size_t rows = (size_t)n_chunks * Hv * CT;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  __nv_bfloat16* Wg = reinterpret_cast<__nv_bfloat16*>(ws);
  __nv_bfloat16* Ug = reinterpret_cast<__nv_bfloat16*>(ws + align_up(rows * DH * 2));
  __nv_bfloat16* QKg = reinterpret_cast<__nv_bfloat16*>(ws + 2 * align_up(rows * DH * 2));
  float* Gg = reinterpret_cast<float*>(ws + 2 * align_up(rows * DH * 2) + align_up(rows * CT * 2));
  cudaStream_t s = (cudaStream_t)stream;
  if (n_chunks > 0) {
    PrepParams pp{};
    const uint64_t wrows = (uint64_t)n_chunks * Hv * CT;
    int st = map3d(&pp.qmap, q, (uint64_t)T, (uint64_t)Hk);
    if (!st) st = map3d(&pp.kmap, k, (uint64_t)T, (uint64_t)Hk);
    if (!st) st = map3d(&pp.vmap, v, (uint64_t)T, (uint64_t)Hv);
    if (!st) st = map2d(&pp.qkmap, QKg, CT, wrows, 64);
    if (!st) st = map2d(&pp.wmap, Wg, DH, wrows, 64);
    if (!st) st = map2d(&pp.umap, Ug, CT, 2 * wrows, 128);
    if (st) return st;
    pp.g = g;
    pp.beta = beta;
    pp.row_start = row_start;
    pp.chunk_start = chunk_start;
    pp.segment = segment;
    pp.Gg = Gg;
    pp.err = status;
    pp.B = (int)B;
    pp.Hk = (int)Hk;
    pp.Hv = (int)Hv;
    pp.scale = scale;
    cudaError_t e = cudaFuncSetAttribute(gdn_chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kPrepSmem);
    if (e != cudaSuccess) {
      set_error("gdn_chunk_scan: smem attribute: %s", cudaGetErrorString(e));
      return JANUS_ERR_CUDA;
    }
    gdn_chunk_prep_kernel<<<dim3((unsigned)Hv, (unsigned)n_chunks), 256, kPrepSmem, s>>>(pp);
    st = launch_status("gdn_chunk_scan/prep");
    if (st) return st;
  }
  return gdn_state_tc(q, k, T, B, row_start, chunk_start, n_chunks, state_in, state_row, state_out, Hk, Hv, scale,
                      Wg, Ug, QKg, Gg, status, o, s);
}
