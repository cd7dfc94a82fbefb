// Gated delta rule over long rows in 64-token chunks (the state level), in two launches.
//
// 1. gdn_chunk_prep: one CTA per (chunk, value head), all chunks of all rows in parallel. With G the in-chunk
//    cumulative g (every exponential is of a difference of G, so nothing overflows):
//      N  = -tril_strict(diag(beta) K K^T * e^(G_i - G_j))          tensor cores, fp32 accumulate
//      T  = (I - N)^-1                                               fp32: 16x16 diagonal blocks by substitution,
//                                                                    then doubling stages 16 -> 32 -> 64 (tf32 MMAs)
//      U  = (T diag(beta)) V,  W = (T diag(beta e^G)) K              bf16 operands, fp32 accumulate, stored bf16
//      QK = tril(scale Q K^T * e^(G_i - G_j))                        stored bf16, plus G itself
// 2. the sequential pass (gdn_state_tc.cu, tcgen05): one CTA per (row, value head) walking the row's chunks in
//    order with the fp32 state in TMEM:
//      V' = U - W S;   O = scale e^G (Q S) + QK V';   S = e^(G_last) S + K^T (V' * e^(G_last - G))
//    (S rounded to bf16 for the products, as fla's chunk kernels do; the e^G factors scale rows of fp32 results
//    instead of the bf16 operands, so q and k are used as loaded). The WY form of transformers'
//    torch_chunk_gated_delta_rule (the reference's CPU rule) and of fla's chunk kernels (its GPU rule). A row's last
//    chunk is ragged: the missing tokens are zeros with g = beta = 0, which leaves the state untouched.
// The prep writes W, U, QK and G chunk-major ([chunk][value head][64 tokens], zeros past a row's end) for the
// sequential pass's TMA loads; it uses mma.sync m16n8k16 (bf16, fp32 accumulate) on XOR-swizzled shared tiles.
#include "common.cuh"

namespace jb {
namespace {

constexpr int CT = 64;   // chunk tokens
constexpr int DH = 128;  // Dk = Dv
constexpr int PADF = 68;  // fp32 [64][68] tiles: row stride = 4 banks, tf32 A fragments hit 32 distinct banks
constexpr int PADM = 40;  // fp32 [32][40]: stride = 8 banks, the B fragments read from it hit 32 distinct banks

__device__ __forceinline__ uint32_t s32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void cpa16(void* dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s32(dst)), "l"(src), "r"(ok ? 16 : 0));
}
__device__ __forceinline__ void cp_commit_wait() {
  asm volatile("cp.async.commit_group;\n" ::);
  asm volatile("cp.async.wait_group 0;\n" ::);
}
__device__ __forceinline__ void ldx4(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(s32(p)));
}
__device__ __forceinline__ void ldx4t(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(s32(p)));
}
__device__ __forceinline__ void mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

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

// swizzled bf16 tiles [rows][COLS]: COLS >= 64 XOR the 16-byte chunk with row & 7; COLS == 32 (64-byte rows) with
// (row >> 1) & 3, so the 8 rows of an ldmatrix hit 8 distinct bank groups either way
template <int COLS>
__device__ __forceinline__ int sw(int r, int c) {
  if constexpr (COLS == 32) return r * 32 + (((c >> 3) ^ ((r >> 1) & 3)) << 3) + (c & 7);
  else return r * COLS + (((c >> 3) ^ (r & 7)) << 3) + (c & 7);
}
// A fragment (16x16) at (m0, k0) of a row-major tile [m][k]
template <int COLS>
__device__ __forceinline__ void lda(uint32_t* a, const __nv_bfloat16* t, int m0, int k0, int lane) {
  ldx4(a, t + sw<COLS>(m0 + (lane & 15), k0 + ((lane >> 4) << 3)));
}
// A fragment (16x16) at (m0, k0) of A = X^T, X row-major [k][m]
template <int COLS>
__device__ __forceinline__ void lda_t(uint32_t* a, const __nv_bfloat16* t, int m0, int k0, int lane) {
  ldx4t(a, t + sw<COLS>(k0 + (lane & 7) + ((lane >> 4) << 3), m0 + (((lane >> 3) & 1) << 3)));
}
// B fragments of n-tiles n0, n0+8 at k0 with B[k][n] = X[n][k], X row-major [n][k]
template <int COLS>
__device__ __forceinline__ void ldb_nk(uint32_t* b, const __nv_bfloat16* t, int n0, int k0, int lane) {
  ldx4(b, t + sw<COLS>(n0 + (lane & 7) + ((lane >> 4) << 3), k0 + (((lane >> 3) & 1) << 3)));
}
// B fragments of n-tiles n0, n0+8 at k0 with B[k][n] = X[k][n], X row-major [k][n]
template <int COLS>
__device__ __forceinline__ void ldb_kn(uint32_t* b, const __nv_bfloat16* t, int n0, int k0, int lane) {
  ldx4t(b, t + sw<COLS>(k0 + (lane & 7) + (((lane >> 3) & 1) << 3), n0 + ((lane >> 4) << 3)));
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

struct PrepSmem {
  __nv_bfloat16 q[CT * DH];
  __nv_bfloat16 k[CT * DH];
  __nv_bfloat16 v[CT * DH];
  __nv_bfloat16 t[CT * CT];   // T diag(beta) (bf16): U = T diag(beta) V
  __nv_bfloat16 t2[CT * CT];  // T diag(beta e^G) (bf16): W = T diag(beta e^G) K
  float n[CT * PADF];
  float tf[CT * PADF];
  float m[32 * PADM];
  float G[CT], eG[CT], beta[CT], graw[CT];
  int32_t seg[CT];  // segment of each token (tokens of different segments do not interact); 0 when unsegmented
};

__global__ void __launch_bounds__(256, 2) gdn_chunk_prep_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    const float* __restrict__ g, const float* __restrict__ beta, const int32_t* __restrict__ row_start,
    const int32_t* __restrict__ chunk_start, const int32_t* __restrict__ segment, int B, int Hk, int Hv, float scale,
    __nv_bfloat16* __restrict__ Wg,
    __nv_bfloat16* __restrict__ Ug, __nv_bfloat16* __restrict__ QKg, float* __restrict__ Gg) {
  extern __shared__ __align__(16) unsigned char raw[];
  PrepSmem& sm = *reinterpret_cast<PrepSmem*>(raw);
  const int h = blockIdx.x, c = blockIdx.y;  // heads fastest: the Hv/Hk heads sharing q and k run together
  const int hk = h / (Hv / Hk);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = chunk_row(chunk_start, B, c);
  const int64_t t0 = row_start[row] + (int64_t)(c - chunk_start[row]) * CT;
  const int64_t rend = row_start[row + 1];
  const int nt = (rend - t0) < CT ? (int)(rend - t0) : CT;
  for (int x = tid; x < CT * (DH / 8); x += 256) {
    const int r = x / (DH / 8), ch = (x % (DH / 8)) * 8;
    const bool ok = r < nt;
    const int64_t t = ok ? t0 + r : t0;
    cpa16(&sm.q[sw<DH>(r, ch)], q + (t * Hk + hk) * DH + ch, ok);
    cpa16(&sm.k[sw<DH>(r, ch)], k + (t * Hk + hk) * DH + ch, ok);
    cpa16(&sm.v[sw<DH>(r, ch)], v + (t * Hv + h) * DH + ch, ok);
  }
  if (tid < CT) {
    const bool ok = tid < nt;
    sm.graw[tid] = ok ? g[(t0 + tid) * Hv + h] : 0.f;
    sm.beta[tid] = ok ? beta[(t0 + tid) * Hv + h] : 0.f;
    sm.seg[tid] = segment ? (ok ? segment[t0 + tid] : -1) : 0;
  }
  cp_commit_wait();
  __syncthreads();
  if (warp == 0 && segment) {  // cumulative sum of g within each segment (a segmented scan, two tokens per lane)
    const float ga = sm.graw[2 * lane], gb = sm.graw[2 * lane + 1];
    const int sa = sm.seg[2 * lane], sb = sm.seg[2 * lane + 1], sp = lane > 0 ? sm.seg[2 * lane - 1] : -2;
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
    sm.G[2 * lane] = Ga;
    sm.G[2 * lane + 1] = hb ? gb : Ga + gb;
  } else if (warp == 0) {  // in-chunk cumulative sum of g (two values per lane)
    const float a = sm.graw[2 * lane], b = a + sm.graw[2 * lane + 1];
    float inc = b;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, inc, off);
      if (lane >= off) inc += y;
    }
    const float excl = inc - b;
    sm.G[2 * lane] = excl + a;
    sm.G[2 * lane + 1] = excl + b;
  }
  __syncthreads();
  if (tid < CT) {
    sm.eG[tid] = expf(sm.G[tid]);
    Gg[((int64_t)c * Hv + h) * CT + tid] = sm.G[tid];  // chunk-major; past the row's end G stays at G[nt - 1]
  }
  // K K^T -> N (fp32, smem), Q K^T -> QK (bf16, global); warp: m-tile w>>1, n-tiles (w&1)*4 .. +3
  {
    const int mt = warp >> 1, nb = (warp & 1) * 32;
    float kk[4][4] = {}, qk[4][4] = {};
#pragma unroll
    for (int ks = 0; ks < DH; ks += 16) {
      uint32_t ak[4], aq[4], b[4];
      lda<DH>(ak, sm.k, mt * 16, ks, lane);
      lda<DH>(aq, sm.q, mt * 16, ks, lane);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        ldb_nk<DH>(b, sm.k, nb + np * 16, ks, lane);
        mma(kk[2 * np], ak, b[0], b[1]);
        mma(kk[2 * np + 1], ak, b[2], b[3]);
        mma(qk[2 * np], aq, b[0], b[1]);
        mma(qk[2 * np + 1], aq, b[2], b[3]);
      }
    }
    __nv_bfloat16* qkc = QKg + ((int64_t)c * Hv + h) * CT * CT;
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int i = mt * 16 + (lane >> 2) + (e >> 1) * 8, j = nb + n * 8 + (lane & 3) * 2;
        float qv[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const float dec = (j + u <= i && sm.seg[i] == sm.seg[j + u]) ? __expf(sm.G[i] - sm.G[j + u]) : 0.f;
          sm.n[i * PADF + j + u] = (j + u < i) ? -sm.beta[i] * kk[n][e + u] * dec : 0.f;
          qv[u] = (j + u <= i) ? qk[n][e + u] * dec * scale : 0.f;
        }
        *reinterpret_cast<__nv_bfloat162*>(qkc + i * CT + j) = __floats2bfloat162_rn(qv[0], qv[1]);
      }
  }
  __syncthreads();  // N complete
  // T = (I - N)^-1: diagonal 16x16 blocks (warps 0-3, lane c < 16 owns column c)
  if (warp < 4) {
    const int base = warp * 16;
    const int cc = lane & 15;
    float col[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) col[r] = (r == cc) ? 1.f : 0.f;
#pragma unroll
    for (int r = 1; r < 16; ++r) {
      float acc = 0.f;
#pragma unroll
      for (int m = 0; m < 16; ++m)
        if (m < r && m >= cc) acc += sm.n[(base + r) * PADF + base + m] * col[m];
      if (cc < r) col[r] = acc;
    }
    if (lane < 16) {
#pragma unroll
      for (int r = 0; r < 16; ++r) sm.tf[(base + r) * PADF + base + cc] = col[r];
    }
  } else {  // zeros above the block diagonal that the full-length sums below read: T[0:16, 16:32], T[32:48, 48:64]
    for (int x = tid - 128; x < 512; x += 128) {
      const int blk = x >> 8, r = (x >> 4) & 15, cc = x & 15;
      sm.tf[(blk * 32 + r) * PADF + blk * 32 + 16 + cc] = 0.f;
    }
  }
  __syncthreads();
  // stage 1: T[2h+1, 2h] = T[2h+1, 2h+1] N[2h+1, 2h] T[2h, 2h] (16x16 blocks), h = 0, 1, on the tensor cores in
  // tf32 (warps 0-3: block h = w >> 1, 8 columns (w & 1) * 8). The triangular zeros of N and T make full-length
  // products exact.
  if (warp < 4) {
    const int hb = warp >> 1, nt = warp & 1;
    const int bi = (2 * hb + 1) * 16, bj = 2 * hb * 16;
    float c[4] = {0.f, 0.f, 0.f, 0.f};
    tile_mma_tf32(c, &sm.n[bi * PADF + bj], PADF, &sm.tf[bj * PADF + bj + 8 * nt], PADF, 16, lane);
    store_tile(c, &sm.m[(hb * 16) * PADM + 8 * nt], PADM, lane);
  }
  __syncthreads();
  if (warp < 4) {
    const int hb = warp >> 1, nt = warp & 1;
    const int bi = (2 * hb + 1) * 16, bj = 2 * hb * 16;
    float c[4] = {0.f, 0.f, 0.f, 0.f};
    tile_mma_tf32(c, &sm.tf[bi * PADF + bi], PADF, &sm.m[(hb * 16) * PADM + 8 * nt], PADM, 16, lane);
    store_tile(c, &sm.tf[bi * PADF + bj + 8 * nt], PADF, lane);
  }
  __syncthreads();
  // stage 2: T[32:, :32] = T[32:, 32:] N[32:, :32] T[:32, :32] (32x32 blocks, tf32; warp: rows 16 (w >> 2), 8 columns
  // (w & 3) * 8)
  {
    const int mt = warp >> 2, nt = warp & 3;
    float c[4] = {0.f, 0.f, 0.f, 0.f};
    tile_mma_tf32(c, &sm.n[(32 + 16 * mt) * PADF], PADF, &sm.tf[8 * nt], PADF, 32, lane);
    store_tile(c, &sm.m[(16 * mt) * PADM + 8 * nt], PADM, lane);
    __syncthreads();
    c[0] = c[1] = c[2] = c[3] = 0.f;
    tile_mma_tf32(c, &sm.tf[(32 + 16 * mt) * PADF + 32], PADF, &sm.m[8 * nt], PADM, 32, lane);
    store_tile(c, &sm.tf[(32 + 16 * mt) * PADF + 8 * nt], PADF, lane);
  }
  __syncthreads();
  // the beta and beta e^G factors of the tokens go on T's columns (rather than on V's and K's rows)
  for (int x = tid; x < CT * CT; x += 256) {
    const int i = x >> 6, j = x & 63;
    const float tv = j <= i ? sm.tf[i * PADF + j] * sm.beta[j] : 0.f;
    sm.t[sw<CT>(i, j)] = __float2bfloat16_rn(tv);
    sm.t2[sw<CT>(i, j)] = __float2bfloat16_rn(tv * sm.eG[j]);
  }
  __syncthreads();
  // U = T diag(beta) V, W = T diag(beta e^G) K (64 x 128; warp: m-tile w>>1, columns (w&1)*64 .. +63)
  const int mt = warp >> 1, cb = (warp & 1) * 64;
  float U[8][4] = {}, Wacc[8][4] = {};
#pragma unroll
  for (int ks = 0; ks < CT; ks += 16) {
    uint32_t a[4], a2[4], b[4];
    lda<CT>(a, sm.t, mt * 16, ks, lane);
    lda<CT>(a2, sm.t2, mt * 16, ks, lane);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      ldb_kn<DH>(b, sm.v, cb + np * 16, ks, lane);
      mma(U[2 * np], a, b[0], b[1]);
      mma(U[2 * np + 1], a, b[2], b[3]);
      ldb_kn<DH>(b, sm.k, cb + np * 16, ks, lane);
      mma(Wacc[2 * np], a2, b[0], b[1]);
      mma(Wacc[2 * np + 1], a2, b[2], b[3]);
    }
  }
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int i = mt * 16 + (lane >> 2) + (e >> 1) * 8, j = cb + n * 8 + (lane & 3) * 2;
      // chunk-major [chunk][head][64 tokens][128], zeros past the row's end (the tokens there have no V, K)
      const int64_t off = (((int64_t)c * Hv + h) * CT + i) * DH + j;
      const bool in = i < nt;
      *reinterpret_cast<__nv_bfloat162*>(Ug + off) = __floats2bfloat162_rn(in ? U[n][e] : 0.f, in ? U[n][e + 1] : 0.f);
      *reinterpret_cast<__nv_bfloat162*>(Wg + off) =
          __floats2bfloat162_rn(in ? Wacc[n][e] : 0.f, in ? Wacc[n][e + 1] : 0.f);
    }
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
                 Hv > 0 && Hv % Hk == 0 && Hv <= 65535 && n_chunks * Hv * CT <= 0x7fffffff,
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
  cudaError_t e = cudaFuncSetAttribute(gdn_chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)sizeof(PrepSmem));
  if (e != cudaSuccess) {
    set_error("gdn_chunk_scan: smem attribute: %s", cudaGetErrorString(e));
    return JANUS_ERR_CUDA;
  }
  if (n_chunks > 0) {
    gdn_chunk_prep_kernel<<<dim3((unsigned)Hv, (unsigned)n_chunks), 256, sizeof(PrepSmem), s>>>(
        (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, g, beta, row_start, chunk_start,
        segment, (int)B, (int)Hk, (int)Hv, scale, Wg, Ug, QKg, Gg);
    int st = launch_status("gdn_chunk_scan/prep");
    if (st) return st;
  }
  return gdn_state_tc(q, k, T, B, row_start, chunk_start, n_chunks, state_in, state_row, state_out, Hk, Hv, scale,
                      Wg, Ug, QKg, Gg, status, o, s);
}
