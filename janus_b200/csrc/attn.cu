// Attention of the hybrid's gated full-attention layers on the packed tree levels.
//
// attn_qk_prep: one CTA per token, one warp per head: RMSNorm (1 + w) of q and k heads, rotary on the first `rot`
// dims in fp32 (the partner of dim d is d +- rot/2, read from shared memory), one rounding to bf16.
//
// tree_attention: a flash-attention forward (online softmax, fp32 accumulators, bf16 P) on mma.sync m16n8k16 over
// the key segments a query may see under the tree rule (janus/attention.py:10-23): the ancestor rows at every
// earlier level (no order constraint) and its own row causally, merged in one softmax instead of one piece per
// ancestor plus a log-sum-exp merge. GQA is folded into the M dimension: a CTA owns one kv head and 64 query rows
// = (64 / G) tokens x G query heads, so every K/V tile is loaded once for all G heads. The CTA's key range per
// ancestor level is the union of its tokens' ranges (the caller keeps tiles inside one request, so the union is one
// ancestor row or a few adjacent short ones); keys outside a token's own range are masked. K/V tiles of 64 keys are
// double-buffered with cp.async in XOR-swizzled shared memory; the sigmoid output gate is applied in the epilogue.
#include <stdlib.h>
#include <string.h>

#include "common.cuh"

namespace jb {

// ------------------------------------------------------------------------------------------------- q/k preparation

// CTA per token: each warp computes the rotary cos / sin of the token's position once (for all its heads), then a
// warp per head: 16-byte loads of 8 consecutive dims per lane, RMSNorm(1 + w) over the head with a warp reduction, the
// rotation of the first `rot` dims from the normalised row kept in shared memory, 16-byte stores.
__global__ void attn_qk_prep_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t stride,
                                    const int32_t* __restrict__ positions, const float* __restrict__ inv_freq, int rot,
                                    const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw,
                                    float eps, int Hq, int Hkv, int D, __nv_bfloat16* __restrict__ q,
                                    __nv_bfloat16* __restrict__ k, __nv_bfloat16* __restrict__ v) {
  extern __shared__ float sh[];  // per warp: [D] row, [rot / 2] cos, [rot / 2] sin
  const int64_t t = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int half = rot >> 1;
  float* buf = sh + warp * ((D + rot + 3) & ~3);  // 16-byte aligned rows
  float* cs = buf + D;
  float* sn = cs + half;
  const __nv_bfloat16* row = qkv + t * stride;
  const int nvec = D >> 3;
  auto head_src = [&](int h) {
    return h < Hq ? row + (int64_t)h * 2 * D : row + (int64_t)Hq * 2 * D + (int64_t)(h - Hq) * D;
  };
  // the first 8 dims per lane of the warp's next head are loaded one head ahead (issued before the cos / sin)
  bf16x8 xnext;
  if (warp < Hq + Hkv && lane < nvec) xnext = *reinterpret_cast<const bf16x8*>(head_src(warp) + lane * 8);
  {  // v: a plain copy of the Hkv*D columns after k, issued first so it overlaps the heads
    const __nv_bfloat16* vs = row + (int64_t)Hq * 2 * D + (int64_t)Hkv * D;
    for (int c = threadIdx.x * 8; c < Hkv * D; c += blockDim.x * 8)
      *reinterpret_cast<bf16x8*>(v + t * Hkv * D + c) = *reinterpret_cast<const bf16x8*>(vs + c);
  }
  const float pos = (float)positions[t];
  for (int f = lane; f < half; f += 32) {  // each warp its own table: no block-wide barrier
    const float ang = pos * inv_freq[f];
    cs[f] = cosf(ang);
    sn[f] = sinf(ang);
  }
  __syncwarp();
  for (int head = warp; head < Hq + Hkv; head += nw) {
    const bool isq = head < Hq;
    const __nv_bfloat16* src = head_src(head);
    const __nv_bfloat16* w = isq ? qw : kw;
    const bf16x8 xcur = xnext;
    if (head + nw < Hq + Hkv && lane < nvec)
      xnext = *reinterpret_cast<const bf16x8*>(head_src(head + nw) + lane * 8);
    float x[8], ss = 0.f;
    if (lane < nvec) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float2 f = __bfloat1622float2(xcur.h[u]);
        x[2 * u] = f.x;
        x[2 * u + 1] = f.y;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
    }
    for (int c = lane + 32; c < nvec; c += 32) {  // heads wider than 256 dims
      float y[8];
      load8(src + c * 8, y);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += y[i] * y[i];
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)D + eps);
    __nv_bfloat16* dst = isq ? q + (t * Hq + head) * D : k + (t * Hkv + (head - Hq)) * D;
    if (nvec <= 32 && half % 8 == 0) {
      // one vector of 8 dims per lane: the rotary partner of dim d (d +/- half) sits in lane ^ half/8, so it comes
      // by a shuffle; cos and sin as float4 reads of the warp's table
      float y[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, wv[8], pv[8];
      if (lane < nvec) {
        load8(w + lane * 8, wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = x[i] * r * (1.f + wv[i]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) pv[i] = __shfl_xor_sync(0xffffffffu, y[i], half >> 3);
      if (lane * 8 < rot) {
        const int f0 = lane * 8 < half ? lane * 8 : lane * 8 - half;
        const float4 c0 = reinterpret_cast<const float4*>(cs + f0)[0], c1 = reinterpret_cast<const float4*>(cs + f0)[1];
        const float4 s0 = reinterpret_cast<const float4*>(sn + f0)[0], s1 = reinterpret_cast<const float4*>(sn + f0)[1];
        const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = lane * 8 < half ? y[i] * cv[i] - pv[i] * sv[i] : y[i] * cv[i] + pv[i] * sv[i];
      }
      if (lane < nvec) store8(dst + lane * 8, y);
      continue;
    }
    float nx[8];  // this lane's normalised dims (first 256)
    for (int c = lane; c < nvec; c += 32) {
      float y[8], wv[8];
      if (c == lane) {
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = x[i];
      } else {
        load8(src + c * 8, y);
      }
      load8(w + c * 8, wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = y[i] * r * (1.f + wv[i]);
      if (c == lane) {
#pragma unroll
        for (int i = 0; i < 8; ++i) nx[i] = y[i];
      }
      // 32 contiguous bytes per lane: whole 128-byte wavefronts, no bank conflicts
      reinterpret_cast<float4*>(buf + c * 8)[0] = make_float4(y[0], y[1], y[2], y[3]);
      reinterpret_cast<float4*>(buf + c * 8)[1] = make_float4(y[4], y[5], y[6], y[7]);
    }
    __syncwarp();
    for (int c = lane; c < nvec; c += 32) {
      float o[8];
      if (c != lane) {
        const float4 a = reinterpret_cast<const float4*>(buf + c * 8)[0], b = reinterpret_cast<const float4*>(buf + c * 8)[1];
        o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = nx[i];
      }
      if (c * 8 < rot) {  // the rotated dims: the partner of d is d -/+ half, from the shared row
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int d = c * 8 + i;
          if (d < rot) {
            const int fi = d < half ? d : d - half;
            o[i] = d < half ? o[i] * cs[fi] - buf[d + half] * sn[fi] : o[i] * cs[fi] + buf[d - half] * sn[fi];
          }
        }
      }
      store8(dst + c * 8, o);
    }
    __syncwarp();
  }
}

// ------------------------------------------------------------------------------------------------ tree attention

constexpr int kMaxLevels = 4;
constexpr int kBM = 64;  // query rows per CTA (tokens x folded heads)
constexpr int kBN = 64;  // keys per tile
constexpr int kAttnThreads = 128;

struct TreeAttnParams {
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
  int64_t gate_stride, gate_head_stride;
  int Hq, Hkv, G, n_levels;
  float scale_log2;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(dst)), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Element offset of (row, 16-byte chunk) in a swizzled [rows][D] bf16 tile.
template <int D>
__device__ __forceinline__ int swz(int row, int chunk) {
  constexpr int CH = D / 8;
  constexpr int MASK = (CH >= 8 ? 8 : CH) - 1;
  return row * D + ((chunk ^ (row & MASK)) << 3);
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads, 1) tree_attention_kernel(TreeAttnParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* sK = sQ + kBM * D;          // [2][kBN][D]
  __nv_bfloat16* sV = sK + 2 * kBN * D;      // [2][kBN][D]
  __shared__ int s_tok[kBM], s_own[kBM];
  __shared__ int s_lo[kMaxLevels][kBM], s_hi[kMaxLevels][kBM];
  __shared__ int s_klo[kMaxLevels], s_khi[kMaxLevels];

  constexpr int CH = D / 8;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hkv = blockIdx.y;
  const int G = p.G, TQ = kBM / G;
  const int q0 = p.tiles[2 * blockIdx.x];
  const int ntok = min(p.tiles[2 * blockIdx.x + 1] - q0, TQ);  // longer tiles are truncated (the host never makes them)
  const int q1 = q0 + ntok;
  const int L = p.n_levels;

  // per-token metadata and the CTA's key range per level
  if (tid < TQ) {
    const int tq = tid;
    const bool live = tq < ntok;
    const int t = live ? q0 + tq : q0;
    const int row = p.row_of_token[t];
    s_tok[tq] = live ? t : -1;
    s_own[tq] = p.row_start[row];
    for (int l = 0; l < L - 1; ++l) {
      s_lo[l][tq] = live ? p.lo[l][row] : 0x7fffffff;
      s_hi[l][tq] = live ? p.hi[l][row] : -1;
    }
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
  }
  __syncthreads();

  // Q tile: row r = tq * G + g -> q[(q0 + tq) * Hq + hkv * G + g]
  for (int c = tid; c < kBM * CH; c += kAttnThreads) {
    const int r = c / CH, ch = c % CH;
    const int tq = r / G, g = r % G;
    const bool ok = tq < ntok;
    const __nv_bfloat16* src = p.q + ((int64_t)(ok ? q0 + tq : q0) * p.Hq + hkv * G + g) * D + ch * 8;
    cp_async16(sQ + swz<D>(r, ch), src, ok);
  }
  cp_async_commit();

  // flattened key blocks over the levels
  int nblk[kMaxLevels], total = 0;
  for (int l = 0; l < L; ++l) {
    nblk[l] = (s_khi[l] - s_klo[l] + kBN - 1) / kBN;
    total += nblk[l];
  }
  auto block_of = [&](int b, int& lvl, int& kstart) {
    int l = 0;
    while (b >= nblk[l]) {
      b -= nblk[l];
      ++l;
    }
    lvl = l;
    kstart = s_klo[l] + b * kBN;
  };
  auto load_block = [&](int b, int stage) {
    int lvl, ks;
    block_of(b, lvl, ks);
    const int kend = s_khi[lvl];
    const __nv_bfloat16* K = p.k[lvl];
    const __nv_bfloat16* V = p.v[lvl];
    __nv_bfloat16* dk = sK + stage * kBN * D;
    __nv_bfloat16* dv = sV + stage * kBN * D;
    for (int c = tid; c < kBN * CH; c += kAttnThreads) {
      const int r = c / CH, ch = c % CH;
      const int kk = ks + r;
      const bool ok = kk < kend;
      const int64_t off = ((int64_t)(ok ? kk : ks) * p.Hkv + hkv) * D + ch * 8;
      cp_async16(dk + swz<D>(r, ch), K + off, ok);
      cp_async16(dv + swz<D>(r, ch), V + off, ok);
    }
  };

  float o_acc[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o_acc[n][0] = o_acc[n][1] = o_acc[n][2] = o_acc[n][3] = 0.f;
  float m_i[2] = {-INFINITY, -INFINITY}, l_i[2] = {0.f, 0.f};
  const int rA = warp * 16 + (lane >> 2);  // rows rA and rA + 8 of this thread's C fragments
  const int tqA = rA / G, tqB = (rA + 8) / G;

  if (total > 0) {
    load_block(0, 0);
    cp_async_commit();
  }
  for (int b = 0; b < total; ++b) {
    const int stage = b & 1;
    if (b + 1 < total) {
      load_block(b + 1, stage ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    int lvl, ks;
    block_of(b, lvl, ks);
    const __nv_bfloat16* tK = sK + stage * kBN * D;
    const __nv_bfloat16* tV = sV + stage * kBN * D;

    // S = Q K^T : 16 x 64 per warp
    float s[kBN / 8][4];
#pragma unroll
    for (int n = 0; n < kBN / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kc = 0; kc < D / 16; ++kc) {
      uint32_t a0, a1, a2, a3;
      {
        const int r = warp * 16 + (lane & 15);
        const int ch = kc * 2 + (lane >> 4);
        ldsm_x4(a0, a1, a2, a3, sQ + swz<D>(r, ch));
      }
#pragma unroll
      for (int np = 0; np < kBN / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int ch = kc * 2 + ((lane >> 3) & 1);
        ldsm_x4(b0, b1, b2, b3, tK + swz<D>(r, ch));
        mma16816(s[2 * np], a0, a1, a2, a3, b0, b1);
        mma16816(s[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }

    // mask and online softmax (rows rA: s[..][0..1], rA+8: s[..][2..3])
    const bool own = (lvl == L - 1);
    int loA, hiA, loB, hiB;
    if (own) {
      loA = s_own[min(tqA, TQ - 1)];
      hiA = s_tok[min(tqA, TQ - 1)] + 1;
      loB = s_own[min(tqB, TQ - 1)];
      hiB = s_tok[min(tqB, TQ - 1)] + 1;
    } else {
      loA = s_lo[lvl][min(tqA, TQ - 1)];
      hiA = s_hi[lvl][min(tqA, TQ - 1)];
      loB = s_lo[lvl][min(tqB, TQ - 1)];
      hiB = s_hi[lvl][min(tqB, TQ - 1)];
    }
    if (tqA >= ntok) hiA = -1;  // padded rows see nothing
    if (tqB >= ntok) hiB = -1;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < kBN / 8; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kk = ks + n * 8 + (lane & 3) * 2 + e;
        float va = s[n][e] * p.scale_log2, vb = s[n][2 + e] * p.scale_log2;
        va = (kk >= loA && kk < hiA) ? va : -INFINITY;
        vb = (kk >= loB && kk < hiB) ? vb : -INFINITY;
        s[n][e] = va;
        s[n][2 + e] = vb;
        mx[0] = fmaxf(mx[0], va);
        mx[1] = fmaxf(mx[1], vb);
      }
    }
    float alpha[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
      const float mnew = fmaxf(m_i[i], mx[i]);
      alpha[i] = (mnew == -INFINITY) ? 1.f : exp2f(m_i[i] - mnew);
      m_i[i] = mnew;
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pa[kBN / 8][2];
#pragma unroll
    for (int n = 0; n < kBN / 8; ++n) {
      const float m0 = m_i[0] == -INFINITY ? 0.f : m_i[0];
      const float m1 = m_i[1] == -INFINITY ? 0.f : m_i[1];
      const float p0 = exp2f(s[n][0] - m0), p1 = exp2f(s[n][1] - m0);
      const float p2 = exp2f(s[n][2] - m1), p3 = exp2f(s[n][3] - m1);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      pa[n][0] = pack_bf16(p0, p1);
      pa[n][1] = pack_bf16(p2, p3);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 1);
      rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 2);
      l_i[i] = l_i[i] * alpha[i] + rs[i];
    }
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      o_acc[n][0] *= alpha[0];
      o_acc[n][1] *= alpha[0];
      o_acc[n][2] *= alpha[1];
      o_acc[n][3] *= alpha[1];
    }
    // O += P V
#pragma unroll
    for (int kc = 0; kc < kBN / 16; ++kc) {
      const uint32_t a0 = pa[2 * kc][0], a1 = pa[2 * kc][1], a2 = pa[2 * kc + 1][0], a3 = pa[2 * kc + 1][1];
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t b0, b1, b2, b3;
        const int r = kc * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int ch = dp * 2 + (lane >> 4);
        ldsm_x4_t(b0, b1, b2, b3, tV + swz<D>(r, ch));
        mma16816(o_acc[2 * dp], a0, a1, a2, a3, b0, b1);
        mma16816(o_acc[2 * dp + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // stage is free for the load of block b + 2
  }

  // epilogue: normalise, gate, store
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = rA + i * 8;
    const int tq = r / G, g = r % G;
    if (tq >= ntok) continue;
    const int64_t t = q0 + tq;
    const int h = hkv * G + g;
    const float inv = l_i[i] > 0.f ? 1.f / l_i[i] : 0.f;
    const __nv_bfloat16* gr = p.gate + t * p.gate_stride + (int64_t)h * p.gate_head_stride;
    __nv_bfloat16* orow = p.out + (t * p.Hq + h) * D;
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      const int d = n * 8 + (lane & 3) * 2;
      const __nv_bfloat162 gv = *reinterpret_cast<const __nv_bfloat162*>(gr + d);
      const float2 gf = __bfloat1622float2(gv);
      const float v0 = o_acc[n][2 * i] * inv * sigmoidf_(gf.x);
      const float v1 = o_acc[n][2 * i + 1] * inv * sigmoidf_(gf.y);
      *reinterpret_cast<__nv_bfloat162*>(orow + d) = __floats2bfloat162_rn(v0, v1);
    }
  }
}

template <int D>
static int launch_tree(const TreeAttnParams& p, int64_t n_tiles, cudaStream_t s) {
  const size_t smem = (size_t)(kBM + 4 * kBN) * D * sizeof(__nv_bfloat16);
  cudaError_t e = cudaFuncSetAttribute(tree_attention_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    set_error("tree_attention: smem attribute %s", cudaGetErrorString(e));
    return JANUS_ERR_CUDA;
  }
  dim3 grid((unsigned)n_tiles, (unsigned)p.Hkv);
  tree_attention_kernel<D><<<grid, kAttnThreads, smem, s>>>(p);
  return launch_status("tree_attention");
}

int tree_attention_tc(const void* q, int64_t Hq, int64_t Hkv, int64_t D, int32_t n_levels, const void* const* k_levels,
                      const void* const* v_levels, const int64_t* level_tokens, const int32_t* const* anc_lo,
                      const int32_t* const* anc_hi,
                      const int32_t* row_start, const int32_t* row_of_token, const int32_t* tiles, int64_t n_tiles,
                      const void* gate, int64_t gate_stride, int64_t gate_head_stride, float scale, void* out,
                      int32_t* err, cudaStream_t stream);

int tree_attention_pair(const void* q, int64_t Hq, int64_t Hkv, int64_t D, int32_t n_levels,
                        const void* const* k_levels, const void* const* v_levels, const int64_t* level_tokens,
                        const int32_t* const* anc_lo, const int32_t* const* anc_hi, const int32_t* row_start,
                        const int32_t* row_of_token, const int32_t* tiles, int64_t n_tiles, const void* gate,
                        int64_t gate_stride, int64_t gate_head_stride, float scale, void* out, int32_t* err,
                        cudaStream_t stream);

int wait_timeout_selftest(int32_t* status, cudaStream_t stream);

// Which tcgen05 form runs head dims 128 and 256: single CTAs (the default, the faster one on B200) or CTA pairs
// (JANUS_B200_ATTN=pairs in the environment at the call; for comparisons of the two)
static bool attn_pairs() {
  const char* v = getenv("JANUS_B200_ATTN");
  return v && strcmp(v, "pairs") == 0;
}

}  // namespace jb

using namespace jb;

extern "C" int janus_b200_selftest_wait_timeout(int32_t* status, void* stream) {
  JB_REQUIRE(status, JANUS_ERR_INVALID, "selftest_wait_timeout: null status");
  return wait_timeout_selftest(status, (cudaStream_t)stream);
}

extern "C" int janus_b200_tree_attention_tile_tokens(int64_t D, int64_t Hq, int64_t Hkv) {
  if (Hq <= 0 || Hkv <= 0 || Hq % Hkv) return 0;
  const int64_t G = Hq / Hkv;
  const int64_t rows = (D == 128 || D == 256) ? 128 : kBM;
  return G <= rows && rows % G == 0 ? (int)(rows / G) : 0;
}

extern "C" int janus_b200_attn_qk_prep(const void* qkv, int64_t qkv_stride, int64_t T, const int32_t* positions,
                                       const float* inv_freq, int64_t rot, const void* q_norm_w, const void* k_norm_w,
                                       float eps, int64_t Hq, int64_t Hkv, int64_t D, void* q, void* k, void* v,
                                       void* stream) {
  JB_REQUIRE(qkv && positions && inv_freq && q_norm_w && k_norm_w && q && k && v, JANUS_ERR_INVALID,
             "attn_qk_prep: null pointer");
  JB_REQUIRE(T >= 0 && Hq > 0 && Hkv > 0 && D > 0 && D % 8 == 0 && rot >= 0 && rot <= D && rot % 2 == 0,
             JANUS_ERR_INVALID, "attn_qk_prep: sizes");
  JB_REQUIRE(qkv_stride >= Hq * 2 * D + 2 * Hkv * D && qkv_stride % 8 == 0, JANUS_ERR_INVALID,
             "attn_qk_prep: qkv stride");
  JB_REQUIRE(JB_ALIGNED(qkv, 16) && JB_ALIGNED(v, 16) && JB_ALIGNED(q, 16) && JB_ALIGNED(k, 16) &&
                 JB_ALIGNED(q_norm_w, 16) && JB_ALIGNED(k_norm_w, 16),
             JANUS_ERR_ALIGNMENT, "attn_qk_prep: 16-byte alignment of qkv, q, k, v and the norm weights");
  JB_REQUIRE((128 / 32) * ((D + rot + 3) & ~3) * 4 <= 48 * 1024, JANUS_ERR_UNSUPPORTED, "attn_qk_prep: head dim %lld",
             (long long)D);
  if (T == 0) return JANUS_OK;
  const int th = 128;
  attn_qk_prep_kernel<<<(unsigned)T, th, (th / 32) * ((D + rot + 3) & ~3) * sizeof(float), (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)qkv, qkv_stride, positions, inv_freq, (int)rot, (const __nv_bfloat16*)q_norm_w,
      (const __nv_bfloat16*)k_norm_w, eps, (int)Hq, (int)Hkv, (int)D, (__nv_bfloat16*)q, (__nv_bfloat16*)k,
      (__nv_bfloat16*)v);
  return launch_status("attn_qk_prep");
}

extern "C" int janus_b200_tree_attention(const void* q, int64_t T, int64_t Hq, int64_t Hkv, int64_t D,
                                         int32_t n_levels, const void* const* k_levels, const void* const* v_levels,
                                         const int64_t* level_tokens, const int32_t* const* anc_lo,
                                         const int32_t* const* anc_hi, const int32_t* row_start, const int32_t* row_of_token, const int32_t* tiles,
                                         int64_t n_tiles, const void* gate, int64_t gate_stride,
                                         int64_t gate_head_stride, float scale, void* out, int32_t* status,
                                         void* stream) {
  JB_REQUIRE(q && k_levels && v_levels && level_tokens && row_start && row_of_token && tiles && gate && out,
             JANUS_ERR_INVALID, "tree_attention: null pointer");
  JB_REQUIRE(n_levels >= 1 && n_levels <= kMaxLevels, JANUS_ERR_UNSUPPORTED, "tree_attention: %d levels (1..%d)",
             n_levels, kMaxLevels);
  JB_REQUIRE(Hq > 0 && Hkv > 0 && Hq % Hkv == 0, JANUS_ERR_INVALID, "tree_attention: heads %lld/%lld",
             (long long)Hq, (long long)Hkv);
  const int64_t G = Hq / Hkv;
  JB_REQUIRE(G <= kBM && kBM % G == 0, JANUS_ERR_UNSUPPORTED, "tree_attention: GQA group %lld must divide %d",
             (long long)G, kBM);
  JB_REQUIRE(n_tiles >= 0 && n_tiles <= 0x7fffffff && Hkv <= 65535, JANUS_ERR_INVALID, "tree_attention: grid");
  JB_REQUIRE(level_tokens[n_levels - 1] == T, JANUS_ERR_INVALID, "tree_attention: own level has %lld tokens, T=%lld",
             (long long)level_tokens[n_levels - 1], (long long)T);
  JB_REQUIRE(JB_ALIGNED(q, 16) && JB_ALIGNED(out, 4) && JB_ALIGNED(gate, 4) && gate_stride % 2 == 0 &&
                 gate_head_stride % 2 == 0,
             JANUS_ERR_ALIGNMENT, "tree_attention: alignment");
  TreeAttnParams p{};
  p.q = (const __nv_bfloat16*)q;
  for (int l = 0; l < n_levels; ++l) {
    JB_REQUIRE(level_tokens[l] >= 0 && level_tokens[l] <= 0x7fffffff, JANUS_ERR_INVALID,
               "tree_attention: level %d token count", l);
    JB_REQUIRE(level_tokens[l] == 0 || (k_levels[l] && v_levels[l] && JB_ALIGNED(k_levels[l], 16) &&
                                        JB_ALIGNED(v_levels[l], 16)),
               JANUS_ERR_ALIGNMENT, "tree_attention: level %d keys/values null or unaligned", l);
    p.k[l] = (const __nv_bfloat16*)k_levels[l];
    p.v[l] = (const __nv_bfloat16*)v_levels[l];
    if (l < n_levels - 1) {
      JB_REQUIRE(anc_lo && anc_hi && anc_lo[l] && anc_hi[l], JANUS_ERR_INVALID, "tree_attention: ancestor ranges");
      p.lo[l] = anc_lo[l];
      p.hi[l] = anc_hi[l];
    }
  }
  p.row_start = row_start;
  p.row_of_token = row_of_token;
  p.tiles = tiles;
  p.gate = (const __nv_bfloat16*)gate;
  p.out = (__nv_bfloat16*)out;
  p.gate_stride = gate_stride;
  p.gate_head_stride = gate_head_stride;
  p.Hq = (int)Hq;
  p.Hkv = (int)Hkv;
  p.G = (int)G;
  p.n_levels = n_levels;
  p.scale_log2 = scale * 1.4426950408889634f;
  if (n_tiles == 0 || T == 0) return JANUS_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if ((D == 128 || D == 256) && 128 % G == 0 && attn_pairs())
    return tree_attention_pair(q, Hq, Hkv, D, n_levels, k_levels, v_levels, level_tokens, anc_lo, anc_hi, row_start,
                               row_of_token, tiles, n_tiles, gate, gate_stride, gate_head_stride, scale, out, status,
                               s);
  if ((D == 128 || D == 256) && 128 % G == 0)
    return tree_attention_tc(q, Hq, Hkv, D, n_levels, k_levels, v_levels, level_tokens, anc_lo, anc_hi, row_start,
                             row_of_token, tiles, n_tiles, gate, gate_stride, gate_head_stride, scale, out, status, s);
  switch (D) {
    case 32: return launch_tree<32>(p, n_tiles, s);
    case 64: return launch_tree<64>(p, n_tiles, s);
    case 128: return launch_tree<128>(p, n_tiles, s);
    case 256: return launch_tree<256>(p, n_tiles, s);
    default:
      set_error("tree_attention: head dim %lld not compiled (32, 64, 128, 256)", (long long)D);
      return JANUS_ERR_UNSUPPORTED;
  }
}
