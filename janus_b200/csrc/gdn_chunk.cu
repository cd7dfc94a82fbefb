// Gated delta rule over long rows in 64-token chunks (the state level), one CTA per (row, value head).
//
// Per chunk (G = in-chunk cumulative g, all exponentials of differences of G, so nothing overflows):
//   N = -tril_strict(diag(beta) K K^T * e^(G_i - G_j))          (tensor cores, fp32 accumulate)
//   T = (I - N)^-1                                               (fp32: 16x16 diagonal blocks by substitution, then
//                                                                 two doubling stages 16 -> 32 -> 64)
//   U = T (V * beta),  W = T (K * beta * e^G)                    (bf16 operands, fp32 accumulate)
//   V' = U - W S                                                 (S rounded to bf16 for the product)
//   O = scale (Q * e^G) S + tril(scale Q K^T * e^(G_i - G_j)) V'
//   S = e^(G_last) S + (K * e^(G_last - G))^T V'                 (S kept in fp32 registers across chunks)
// the WY form of transformers' torch_chunk_gated_delta_rule (the reference's CPU rule) and of fla's chunk kernels
// (its GPU rule), with fla's rounding points (bf16 operands for every product, fp32 state). Rows end in a ragged
// chunk: the missing tokens are loaded as zeros with g = beta = 0, which leaves the state untouched.
//
// Warp tiling (8 warps, mma.sync m16n8k16 bf16): 64x64 products as 4 m-tiles x 2 column halves; 64x128 products
// likewise with 64-column halves; the 128x128 state update with one 16-row slice of S per warp.
#include "common.cuh"

namespace jb {
namespace {

constexpr int CT = 64;   // chunk tokens
constexpr int DH = 128;  // Dk = Dv
constexpr int NT = 256;
constexpr int PADF = 65; // fp32 [64][65] tiles

__device__ __forceinline__ uint32_t s32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void cpa16(void* dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s32(dst)), "l"(src), "r"(ok ? 16 : 0));
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

// swizzled bf16 tile [rows][COLS]: 16-byte chunk c of row r at chunk c ^ (r & 7)
template <int COLS>
__device__ __forceinline__ int sw(int r, int c) { return r * COLS + (((c >> 3) ^ (r & 7)) << 3) + (c & 7); }

// A fragment (16x16) at (m0, k0) of a row-major swizzled tile [m][k]
template <int COLS>
__device__ __forceinline__ void lda(uint32_t* a, const __nv_bfloat16* t, int m0, int k0, int lane) {
  ldx4(a, t + sw<COLS>(m0 + (lane & 15), k0 + ((lane >> 4) << 3)));
}
// A fragment (16x16) at (m0, k0) of A = X^T where X is a row-major swizzled tile [k][m]
template <int COLS>
__device__ __forceinline__ void lda_t(uint32_t* a, const __nv_bfloat16* t, int m0, int k0, int lane) {
  ldx4t(a, t + sw<COLS>(k0 + (lane & 7) + ((lane >> 4) << 3), m0 + (((lane >> 3) & 1) << 3)));
}
// B fragments of two n-tiles (n0, n0+8) x k16 at k0, B[k][n] = X[n][k] with X row-major [n][k]
template <int COLS>
__device__ __forceinline__ void ldb_nk(uint32_t* b, const __nv_bfloat16* t, int n0, int k0, int lane) {
  ldx4(b, t + sw<COLS>(n0 + (lane & 7) + ((lane >> 4) << 3), k0 + (((lane >> 3) & 1) << 3)));
}
// B fragments of two n-tiles (n0, n0+8) x k16 at k0, B[k][n] = X[k][n] with X row-major [k][n]
template <int COLS>
__device__ __forceinline__ void ldb_kn(uint32_t* b, const __nv_bfloat16* t, int n0, int k0, int lane) {
  ldx4t(b, t + sw<COLS>(k0 + (lane & 7) + (((lane >> 3) & 1) << 3), n0 + ((lane >> 4) << 3)));
}

struct Smem {
  __nv_bfloat16 q[CT * DH];    // Q, then Q * e^G * scale
  __nv_bfloat16 k[CT * DH];    // K, then K * e^(G_last - G)
  __nv_bfloat16 v[CT * DH];    // V, then V * beta
  __nv_bfloat16 kb[CT * DH];   // K * beta * e^G, then W
  __nv_bfloat16 vn[CT * DH];   // V'
  __nv_bfloat16 s[DH * DH];    // S (bf16 copy)
  __nv_bfloat16 qk[CT * CT];   // masked decayed scale * Q K^T
  __nv_bfloat16 t[CT * CT];    // T (bf16)
  float n[CT * PADF];          // N
  float tf[CT * PADF];         // T (fp32)
  float m[32 * 33];            // stage-2 product
  float G[CT], eG[CT], eGl[CT], beta[CT], graw[CT];
};

__global__ void __launch_bounds__(NT, 1) gdn_chunk_kernel(const __nv_bfloat16* __restrict__ q,
                                                          const __nv_bfloat16* __restrict__ k,
                                                          const __nv_bfloat16* __restrict__ v,
                                                          const float* __restrict__ g, const float* __restrict__ beta,
                                                          const int32_t* __restrict__ row_start,
                                                          const float* __restrict__ state_in,
                                                          const int32_t* __restrict__ state_row,
                                                          float* __restrict__ state_out, int Hk, int Hv, float scale,
                                                          __nv_bfloat16* __restrict__ o) {
  extern __shared__ __align__(16) unsigned char raw[];
  Smem& sm = *reinterpret_cast<Smem*>(raw);
  const int row = blockIdx.x, h = blockIdx.y;
  const int hk = h / (Hv / Hk);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t r0 = row_start[row], r1 = row_start[row + 1];

  // S accumulator: warp w owns key rows 16w..16w+15, all 128 value columns (16 n-tiles)
  float S[16][4];
  {
    const int64_t sb = ((int64_t)(state_row ? state_row[row] : row) * Hv + h) * DH * DH;
#pragma unroll
    for (int n = 0; n < 16; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rr = warp * 16 + (lane >> 2) + (e >> 1) * 8, cc = n * 8 + (lane & 3) * 2 + (e & 1);
        S[n][e] = state_in ? state_in[sb + rr * DH + cc] : 0.f;
      }
  }

  for (int64_t c0 = r0; c0 < r1; c0 += CT) {
    const int nt = (r1 - c0) < CT ? (int)(r1 - c0) : CT;
    // ---- bf16 copy of S for this chunk's products
#pragma unroll
    for (int n = 0; n < 16; ++n)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int rr = warp * 16 + (lane >> 2) + (e >> 1) * 8, cc = n * 8 + (lane & 3) * 2;
        *reinterpret_cast<__nv_bfloat162*>(&sm.s[sw<DH>(rr, cc)]) = __floats2bfloat162_rn(S[n][e], S[n][e + 1]);
      }
    // ---- load the chunk
    for (int x = tid; x < CT * (DH / 8); x += NT) {
      const int r = x / (DH / 8), ch = (x % (DH / 8)) * 8;
      const bool ok = r < nt;
      const int64_t t = ok ? c0 + r : r0;
      cpa16(&sm.q[sw<DH>(r, ch)], q + (t * Hk + hk) * DH + ch, ok);
      cpa16(&sm.k[sw<DH>(r, ch)], k + (t * Hk + hk) * DH + ch, ok);
      cpa16(&sm.v[sw<DH>(r, ch)], v + (t * Hv + h) * DH + ch, ok);
    }
    asm volatile("cp.async.commit_group;\n" ::);
    if (tid < CT) {
      const bool ok = tid < nt;
      sm.graw[tid] = ok ? g[(c0 + tid) * Hv + h] : 0.f;
      sm.beta[tid] = ok ? beta[(c0 + tid) * Hv + h] : 0.f;
    }
    asm volatile("cp.async.wait_group 0;\n" ::);
    __syncthreads();
    if (warp == 0) {  // in-chunk cumulative sum of g (two values per lane)
      float a = sm.graw[2 * lane], b = a + sm.graw[2 * lane + 1];
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
    const float Gl = sm.G[CT - 1];
    if (tid < CT) {
      sm.eG[tid] = expf(sm.G[tid]);
      sm.eGl[tid] = expf(Gl - sm.G[tid]);
    }
    // ---- phase A: K K^T -> N (fp32), Q K^T -> qk (bf16); warp: m-tile w>>1, n-tiles (w&1)*4 .. +3
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
      __syncthreads();  // eG / eGl visible (written above by threads < 64)
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = mt * 16 + (lane >> 2) + (e >> 1) * 8, j = nb + n * 8 + (lane & 3) * 2 + (e & 1);
          const float dec = (j <= i) ? expf(sm.G[i] - sm.G[j]) : 0.f;
          sm.n[i * PADF + j] = (j < i) ? -sm.beta[i] * kk[n][e] * dec : 0.f;
          sm.qk[sw<CT>(i, j)] = __float2bfloat16_rn((j <= i) ? qk[n][e] * dec * scale : 0.f);
        }
    }
    __syncthreads();
    // ---- elementwise: kb = K beta e^G, k <- K e^(Gl - G), v <- V beta, q <- Q e^G scale
    for (int x = tid; x < CT * DH / 2; x += NT) {
      const int r = x / (DH / 2), cc = (x % (DH / 2)) * 2;
      const int off = sw<DH>(r, cc);
      const float2 kf = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&sm.k[off]));
      const float2 vf = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&sm.v[off]));
      const float2 qf = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&sm.q[off]));
      const float b = sm.beta[r], eg = sm.eG[r], egl = sm.eGl[r];
      *reinterpret_cast<__nv_bfloat162*>(&sm.kb[off]) = __floats2bfloat162_rn(kf.x * b * eg, kf.y * b * eg);
      *reinterpret_cast<__nv_bfloat162*>(&sm.k[off]) = __floats2bfloat162_rn(kf.x * egl, kf.y * egl);
      *reinterpret_cast<__nv_bfloat162*>(&sm.v[off]) = __floats2bfloat162_rn(vf.x * b, vf.y * b);
      *reinterpret_cast<__nv_bfloat162*>(&sm.q[off]) = __floats2bfloat162_rn(qf.x * eg * scale, qf.y * eg * scale);
    }
    // ---- T = (I - N)^-1: diagonal 16x16 blocks (warps 0-3, lane c < 16 owns column c)
    if (warp < 4) {
      const int base = warp * 16;
      const int c = lane & 15;
      float col[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) col[r] = (r == c) ? 1.f : 0.f;
#pragma unroll
      for (int r = 1; r < 16; ++r) {
        float acc = 0.f;
#pragma unroll
        for (int m = 0; m < 16; ++m)
          if (m < r && m >= c) acc += sm.n[(base + r) * PADF + base + m] * col[m];
        if (c < r) col[r] = acc;
      }
      if (lane < 16) {
#pragma unroll
        for (int r = 0; r < 16; ++r) sm.tf[(base + r) * PADF + base + c] = col[r];
      }
    }
    __syncthreads();
    // stage 1: T[2h+1, 2h] = T[2h+1,2h+1] N[2h+1,2h] T[2h,2h] (16x16 blocks), h = 0, 1
    {
      // M = N[2h+1,2h] T[2h,2h]: 2 x 256 outputs
      for (int x = tid; x < 512; x += NT) {
        const int hb = x >> 8, i = (x >> 4) & 15, j = x & 15;
        const int bi = (2 * hb + 1) * 16, bj = 2 * hb * 16;
        float acc = 0.f;
        for (int m = j; m < 16; ++m) acc += sm.n[(bi + i) * PADF + bj + m] * sm.tf[(bj + m) * PADF + bj + j];
        sm.m[(hb * 16 + i) * 33 + j] = acc;
      }
      __syncthreads();
      for (int x = tid; x < 512; x += NT) {
        const int hb = x >> 8, i = (x >> 4) & 15, j = x & 15;
        const int bi = (2 * hb + 1) * 16, bj = 2 * hb * 16;
        float acc = 0.f;
        for (int m = 0; m <= i; ++m) acc += sm.tf[(bi + i) * PADF + bi + m] * sm.m[(hb * 16 + m) * 33 + j];
        sm.tf[(bi + i) * PADF + bj + j] = acc;
      }
    }
    __syncthreads();
    // stage 2: T[32:, :32] = T[32:,32:] N[32:, :32] T[:32, :32]
    for (int x = tid; x < 1024; x += NT) {
      const int i = x >> 5, j = x & 31;
      float acc = 0.f;
      for (int m = j; m < 32; ++m) acc += sm.n[(32 + i) * PADF + m] * sm.tf[m * PADF + j];
      sm.m[i * 33 + j] = acc;
    }
    __syncthreads();
    for (int x = tid; x < 1024; x += NT) {
      const int i = x >> 5, j = x & 31;
      float acc = 0.f;
      for (int m = 0; m <= i; ++m) acc += sm.tf[(32 + i) * PADF + 32 + m] * sm.m[m * 33 + j];
      sm.tf[(32 + i) * PADF + j] = acc;
    }
    __syncthreads();
    // T to bf16 (lower triangle incl. diagonal; zeros above)
    for (int x = tid; x < CT * CT; x += NT) {
      const int i = x >> 6, j = x & 63;
      sm.t[sw<CT>(i, j)] = __float2bfloat16_rn(j <= i ? sm.tf[i * PADF + j] : 0.f);
    }
    __syncthreads();
    // ---- phase B: U = T vb, W = T kb  (64 x 128; warp: m-tile w>>1, columns (w&1)*64 .. +63)
    const int mt = warp >> 1, cb = (warp & 1) * 64;
    float U[8][4] = {}, Wacc[8][4] = {};
#pragma unroll
    for (int ks = 0; ks < CT; ks += 16) {
      uint32_t a[4], b[4];
      lda<CT>(a, sm.t, mt * 16, ks, lane);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        ldb_kn<DH>(b, sm.v, cb + np * 16, ks, lane);
        mma(U[2 * np], a, b[0], b[1]);
        mma(U[2 * np + 1], a, b[2], b[3]);
        ldb_kn<DH>(b, sm.kb, cb + np * 16, ks, lane);
        mma(Wacc[2 * np], a, b[0], b[1]);
        mma(Wacc[2 * np + 1], a, b[2], b[3]);
      }
    }
    __syncthreads();  // every warp is done reading kb
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int i = mt * 16 + (lane >> 2) + (e >> 1) * 8, j = cb + n * 8 + (lane & 3) * 2;
        *reinterpret_cast<__nv_bfloat162*>(&sm.kb[sw<DH>(i, j)]) = __floats2bfloat162_rn(Wacc[n][e], Wacc[n][e + 1]);
      }
    __syncthreads();
    // ---- phase C: V' = U - W S
    {
      float P[8][4] = {};
#pragma unroll
      for (int ks = 0; ks < DH; ks += 16) {
        uint32_t a[4], b[4];
        lda<DH>(a, sm.kb, mt * 16, ks, lane);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          ldb_kn<DH>(b, sm.s, cb + np * 16, ks, lane);
          mma(P[2 * np], a, b[0], b[1]);
          mma(P[2 * np + 1], a, b[2], b[3]);
        }
      }
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int i = mt * 16 + (lane >> 2) + (e >> 1) * 8, j = cb + n * 8 + (lane & 3) * 2;
          *reinterpret_cast<__nv_bfloat162*>(&sm.vn[sw<DH>(i, j)]) =
              __floats2bfloat162_rn(U[n][e] - P[n][e], U[n][e + 1] - P[n][e + 1]);
        }
    }
    __syncthreads();
    // ---- phase D: O = q S + qk V'
    {
      float O[8][4] = {};
#pragma unroll
      for (int ks = 0; ks < DH; ks += 16) {
        uint32_t a[4], b[4];
        lda<DH>(a, sm.q, mt * 16, ks, lane);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          ldb_kn<DH>(b, sm.s, cb + np * 16, ks, lane);
          mma(O[2 * np], a, b[0], b[1]);
          mma(O[2 * np + 1], a, b[2], b[3]);
        }
      }
#pragma unroll
      for (int ks = 0; ks < CT; ks += 16) {
        uint32_t a[4], b[4];
        lda<CT>(a, sm.qk, mt * 16, ks, lane);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          ldb_kn<DH>(b, sm.vn, cb + np * 16, ks, lane);
          mma(O[2 * np], a, b[0], b[1]);
          mma(O[2 * np + 1], a, b[2], b[3]);
        }
      }
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int i = mt * 16 + (lane >> 2) + (e >> 1) * 8, j = cb + n * 8 + (lane & 3) * 2;
          if (i < nt)
            *reinterpret_cast<__nv_bfloat162*>(o + ((c0 + i) * Hv + h) * DH + j) =
                __floats2bfloat162_rn(O[n][e], O[n][e + 1]);
        }
    }
    // ---- phase E: S = e^(G_last) S + (K e^(Gl - G))^T V'   (warp: key rows 16w..16w+15)
    {
      const float dl = expf(Gl);
#pragma unroll
      for (int n = 0; n < 16; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) S[n][e] *= dl;
#pragma unroll
      for (int ks = 0; ks < CT; ks += 16) {
        uint32_t a[4], b[4];
        lda_t<DH>(a, sm.k, warp * 16, ks, lane);
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          ldb_kn<DH>(b, sm.vn, np * 16, ks, lane);
          mma(S[2 * np], a, b[0], b[1]);
          mma(S[2 * np + 1], a, b[2], b[3]);
        }
      }
    }
    __syncthreads();  // all reads of this chunk's tiles (and of sm.s) are done before the next chunk overwrites them
  }
  if (state_out) {
    const int64_t sb = ((int64_t)row * Hv + h) * DH * DH;
#pragma unroll
    for (int n = 0; n < 16; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rr = warp * 16 + (lane >> 2) + (e >> 1) * 8, cc = n * 8 + (lane & 3) * 2 + (e & 1);
        state_out[sb + rr * DH + cc] = S[n][e];
      }
  }
}

}  // namespace
}  // namespace jb

using namespace jb;

extern "C" int janus_b200_gdn_chunk_scan(const void* q, const void* k, const void* v, const float* g,
                                         const float* beta, int64_t T, int64_t B, const int32_t* row_start,
                                         const float* state_in, const int32_t* state_row, float* state_out, int64_t Hk, int64_t Hv, int64_t Dk,
                                         int64_t Dv, float scale, void* o, void* stream) {
  JB_REQUIRE(q && k && v && g && beta && row_start && o, JANUS_ERR_INVALID, "gdn_chunk_scan: null pointer");
  JB_REQUIRE(Dk == DH && Dv == DH, JANUS_ERR_UNSUPPORTED, "gdn_chunk_scan: Dk = Dv = 128 only (got %lld, %lld)",
             (long long)Dk, (long long)Dv);
  JB_REQUIRE(T >= 0 && B >= 0 && Hk > 0 && Hv > 0 && Hv % Hk == 0 && Hv <= 65535, JANUS_ERR_INVALID,
             "gdn_chunk_scan: sizes");
  JB_REQUIRE(JB_ALIGNED(q, 16) && JB_ALIGNED(k, 16) && JB_ALIGNED(v, 16) && JB_ALIGNED(o, 4), JANUS_ERR_ALIGNMENT,
             "gdn_chunk_scan: alignment");
  if (B == 0 || T == 0) return JANUS_OK;
  const size_t smem = sizeof(Smem);
  cudaError_t e = cudaFuncSetAttribute(gdn_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    set_error("gdn_chunk_scan: smem attribute (%zu bytes): %s", smem, cudaGetErrorString(e));
    return JANUS_ERR_CUDA;
  }
  dim3 grid((unsigned)B, (unsigned)Hv);
  gdn_chunk_kernel<<<grid, NT, smem, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, g, beta, row_start, state_in,
      state_row, state_out, (int)Hk, (int)Hv, scale, (__nv_bfloat16*)o);
  return launch_status("gdn_chunk_scan");
}
