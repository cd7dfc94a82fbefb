// Row-wise glue between the GEMMs: embedding + RMSNorm, residual add + RMSNorm, SwiGLU gate, gated RMSNorm.
// All HBM-bound: one CTA (or warp) per token row, 16- or 32-byte vector accesses, one pass over the inputs, fp32
// math and a single rounding to bf16 at each output.
#include "common.cuh"

namespace jb {

// 32-byte global accesses (ld/st .v8.b32, sm_100): half the instructions per byte of 16-byte vectors, which
// matters where a kernel's rate is set by its load queue. The .nc form only for data no thread writes.
__device__ __forceinline__ void ldg32(const void* p, uint32_t (&r)[8]) {
  asm volatile("ld.global.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "l"(p));
}
__device__ __forceinline__ void ldg_nc32(const void* p, uint32_t (&r)[8]) {
  asm volatile("ld.global.nc.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "l"(p));
}
__device__ __forceinline__ void stg32(void* p, const uint32_t (&r)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(r[0]), "r"(r[1]), "r"(r[2]),
               "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t v) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
}
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

constexpr int kNormThreads = 128;
constexpr int kNormVec = 4;  // vectors of 8 per thread kept in registers: hidden <= 8 * 4 * threads

// y = x * rsqrt(mean(x^2) + eps) * (1 + w); x fp32 [H] already in registers as vals.
template <bool kEmbed>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_rows_kernel(const __nv_bfloat16* __restrict__ table,
                                                                     const int32_t* __restrict__ ids,
                                                                     const __nv_bfloat16* __restrict__ delta,
                                                                     int64_t delta_stride, float* __restrict__ x,
                                                                     int H, const __nv_bfloat16* __restrict__ w,
                                                                     float eps, __nv_bfloat16* __restrict__ y) {
  __shared__ float red[32];
  const int64_t t = blockIdx.x;
  const int nv = H >> 3;
  float vals[kNormVec][8];
  float ss = 0.f;
  float* xr = x + t * (int64_t)H;
  const bool wide = JB_ALIGNED(x, 32);  // rows of H % 8 == 0 floats keep 32-byte alignment
#pragma unroll
  for (int j = 0; j < kNormVec; ++j) {
    const int v = threadIdx.x + j * blockDim.x;
    if (v < nv) {
      if (kEmbed) {
        load8(table + (int64_t)ids[t] * H + v * 8, vals[j]);
      } else {
        if (wide) {  // one 32-byte load
          uint32_t raw[8];
          ldg32(xr + 8 * v, raw);
#pragma unroll
          for (int i = 0; i < 8; ++i) vals[j][i] = __uint_as_float(raw[i]);
        } else {
          float4 a = reinterpret_cast<const float4*>(xr)[2 * v];
          float4 b = reinterpret_cast<const float4*>(xr)[2 * v + 1];
          vals[j][0] = a.x; vals[j][1] = a.y; vals[j][2] = a.z; vals[j][3] = a.w;
          vals[j][4] = b.x; vals[j][5] = b.y; vals[j][6] = b.z; vals[j][7] = b.w;
        }
        if (delta) {
          float d[8];
          load8(delta + t * delta_stride + v * 8, d);
#pragma unroll
          for (int i = 0; i < 8; ++i) vals[j][i] += d[i];
        }
      }
      if (kEmbed || delta) {
        if (wide) {
          uint32_t raw[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) raw[i] = __float_as_uint(vals[j][i]);
          stg32(xr + 8 * v, raw);
        } else {
          reinterpret_cast<float4*>(xr)[2 * v] = make_float4(vals[j][0], vals[j][1], vals[j][2], vals[j][3]);
          reinterpret_cast<float4*>(xr)[2 * v + 1] = make_float4(vals[j][4], vals[j][5], vals[j][6], vals[j][7]);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += vals[j][i] * vals[j][i];
    }
  }
  ss = block_sum(ss, red);
  const float r = rsqrtf(ss / (float)H + eps);
#pragma unroll
  for (int j = 0; j < kNormVec; ++j) {
    const int v = threadIdx.x + j * blockDim.x;
    if (v < nv) {
      float wv[8], o[8];
      load8(w + v * 8, wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = vals[j][i] * r * (1.f + wv[i]);
      store8(y + t * (int64_t)H + v * 8, o);
    }
  }
}

// CTA per token (grid-stride over tokens), thread per 8 columns; kSiluUnroll column vectors in flight per thread.
constexpr int kSiluThreads = 128, kSiluUnroll = 4;
__global__ void __launch_bounds__(kSiluThreads) silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, int64_t T, int I,
                                                                __nv_bfloat16* __restrict__ out) {
  const int nv = I >> 3;
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    const __nv_bfloat16* gr = gu + t * 2 * I;
    __nv_bfloat16* orow = out + t * I;
    for (int c0 = threadIdx.x; c0 < nv; c0 += kSiluThreads * kSiluUnroll) {
      bf16x8 g[kSiluUnroll], u[kSiluUnroll];
#pragma unroll
      for (int j = 0; j < kSiluUnroll; ++j) {
        const int c = c0 + j * kSiluThreads;
        if (c < nv) {
          g[j] = *reinterpret_cast<const bf16x8*>(gr + c * 8);
          u[j] = *reinterpret_cast<const bf16x8*>(gr + I + c * 8);
        }
      }
#pragma unroll
      for (int j = 0; j < kSiluUnroll; ++j) {
        const int c = c0 + j * kSiluThreads;
        if (c < nv) {
          bf16x8 o;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 a = __bfloat1622float2(g[j].h[i]), b = __bfloat1622float2(u[j].h[i]);
            o.h[i] = __floats2bfloat162_rn(silu_fast(a.x) * b.x, silu_fast(a.y) * b.y);
          }
          *reinterpret_cast<bf16x8*>(orow + c * 8) = o;
        }
      }
    }
  }
}

// silu_mul with 32-byte accesses: half the load instructions per byte of the 16-byte version above, whose rate is
// set by its load queue. Thread per 16 columns, 192 threads x 3 vectors cover a 9216-wide row in one round. Needs
// I % 16 == 0 and 32-byte aligned rows; the results are bit-identical.
constexpr int kSilu32Threads = 192, kSilu32Unroll = 3;
__global__ void __launch_bounds__(kSilu32Threads, 4) silu_mul32_kernel(const __nv_bfloat16* __restrict__ gu, int64_t T,
                                                                    int I, __nv_bfloat16* __restrict__ out) {
  const int nv = I >> 4;
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    const __nv_bfloat16* gr = gu + t * 2 * I;
    __nv_bfloat16* orow = out + t * I;
    for (int c0 = threadIdx.x; c0 < nv; c0 += kSilu32Threads * kSilu32Unroll) {
      uint32_t g[kSilu32Unroll][8], u[kSilu32Unroll][8];
#pragma unroll
      for (int j = 0; j < kSilu32Unroll; ++j) {
        const int c = c0 + j * kSilu32Threads;
        if (c < nv) {
          ldg_nc32(gr + c * 16, g[j]);
          ldg_nc32(gr + I + c * 16, u[j]);
        }
      }
#pragma unroll
      for (int j = 0; j < kSilu32Unroll; ++j) {
        const int c = c0 + j * kSilu32Threads;
        if (c < nv) {
          uint32_t o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float2 a = unpack_bf16x2(g[j][i]), b = unpack_bf16x2(u[j][i]);
            o[i] = pack_bf16x2(silu_fast(a.x) * b.x, silu_fast(a.y) * b.y);
          }
          stg32(orow + c * 16, o);
        }
      }
    }
  }
}

// Thread per 8 consecutive elements of one (token, value head); the DV / 8 threads of a head are consecutive lanes
// of one warp and reduce the sum of squares with shuffles.
template <int DV>
__global__ void gated_rmsnorm_kernel(const __nv_bfloat16* __restrict__ core, const __nv_bfloat16* __restrict__ z,
                                     int64_t z_stride, int64_t T, int Hv, const __nv_bfloat16* __restrict__ w,
                                     float eps, __nv_bfloat16* __restrict__ out) {
  constexpr int LPH = DV / 8;
  static_assert(LPH >= 1 && LPH <= 32 && (32 % LPH) == 0, "head must span a power-of-two lane group");
  const int64_t gi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const bool live = gi < T * Hv * LPH;
  const int64_t head = live ? gi / LPH : 0;
  const int sub = (int)(gi % LPH);
  const int64_t t = head / Hv;
  const int h = (int)(head - t * Hv);
  float cv[8], zv[8], wv[8], ss = 0.f;
  if (live) {
    load8(core + head * DV + sub * 8, cv);
    load8(z + t * z_stride + (int64_t)h * DV + sub * 8, zv);
    load8(w + sub * 8, wv);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += cv[i] * cv[i];
  }
#pragma unroll
  for (int o = LPH >> 1; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (live) {
    const float r = rsqrtf(ss / (float)DV + eps);
    float res[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) res[i] = wv[i] * (cv[i] * r) * silu_fast(zv[i]);
    store8(out + head * DV + sub * 8, res);
  }
}

// The same op with 32-byte accesses: thread per 16 elements (DV / 16 lanes per head), the lane's 16 weights loaded
// once, warps striding over the (token, head) units. The sum of squares is taken in a different order from the
// kernel above (16 per thread, then DV / 16 lanes), so results may differ from it in the last bit.
template <int DV>
__global__ void __launch_bounds__(256, 4) gated_rmsnorm32_kernel(const __nv_bfloat16* __restrict__ core,
                                                                 const __nv_bfloat16* __restrict__ z, int64_t z_stride,
                                                                 uint32_t n_heads, uint32_t Hv,
                                                                 const __nv_bfloat16* __restrict__ w, float eps,
                                                                 __nv_bfloat16* __restrict__ out) {
  constexpr int LPH = DV / 16;
  static_assert(LPH >= 1 && LPH <= 32 && (32 % LPH) == 0, "head must span a power-of-two lane group");
  const uint32_t lane = threadIdx.x & 31, sub = lane % LPH;
  const uint32_t total = n_heads * LPH, stride = gridDim.x * blockDim.x;
  float wv[16];
  {
    uint32_t raw[8];
    ldg_nc32(w + sub * 16, raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 f = unpack_bf16x2(raw[i]);
      wv[2 * i] = f.x;
      wv[2 * i + 1] = f.y;
    }
  }
  // the loop bound is uniform over a warp (base is the warp's first unit), so every lane reaches the shuffles
  for (uint32_t base = blockIdx.x * blockDim.x + (threadIdx.x & ~31u); base < total; base += stride) {
    const uint32_t gi = base + lane;
    const bool live = gi < total;
    const uint32_t head = live ? gi / LPH : 0;
    uint32_t c[8], zz[8];
    float ss = 0.f;
    if (live) {
      const uint32_t t = head / Hv, h = head - t * Hv;
      ldg_nc32(core + (int64_t)head * DV + sub * 16, c);
      ldg_nc32(z + (int64_t)t * z_stride + h * DV + sub * 16, zz);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 f = unpack_bf16x2(c[i]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
#pragma unroll
    for (int o = LPH >> 1; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (live) {
      const float r = rsqrtf(ss / (float)DV + eps);
      uint32_t res[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 f = unpack_bf16x2(c[i]), zf = unpack_bf16x2(zz[i]);
        res[i] = pack_bf16x2(wv[2 * i] * (f.x * r) * silu_fast(zf.x), wv[2 * i + 1] * (f.y * r) * silu_fast(zf.y));
      }
      stg32(out + (int64_t)head * DV + sub * 16, res);
    }
  }
}

static int check_norm_args(int64_t T, int64_t H, const void* y, const void* w) {
  JB_REQUIRE(T >= 0 && H > 0 && H % 8 == 0 && H <= 8 * kNormVec * kNormThreads, JANUS_ERR_INVALID,
             "rmsnorm: hidden %lld must be a positive multiple of 8 up to %d", (long long)H, 8 * kNormVec * kNormThreads);
  JB_REQUIRE(y && w, JANUS_ERR_INVALID, "rmsnorm: null output or weight");
  JB_REQUIRE(JB_ALIGNED(y, 16) && JB_ALIGNED(w, 16), JANUS_ERR_ALIGNMENT, "rmsnorm: output/weight not 16-byte aligned");
  return JANUS_OK;
}

}  // namespace jb

using namespace jb;

extern "C" int janus_b200_embed_rmsnorm(const void* table, int64_t vocab, int64_t hidden, const int32_t* ids,
                                        int64_t T, const void* norm_w, float eps, float* x, void* y, void* stream) {
  int st = check_norm_args(T, hidden, y, norm_w);
  if (st) return st;
  JB_REQUIRE(table && ids && x && vocab > 0, JANUS_ERR_INVALID, "embed_rmsnorm: null table/ids/x");
  JB_REQUIRE(JB_ALIGNED(table, 16) && JB_ALIGNED(x, 16), JANUS_ERR_ALIGNMENT, "embed_rmsnorm: table/x alignment");
  if (T == 0) return JANUS_OK;
  JB_REQUIRE((hidden / 8 + kNormThreads - 1) / kNormThreads <= kNormVec, JANUS_ERR_UNSUPPORTED,
             "embed_rmsnorm: hidden %lld too large", (long long)hidden);
  rmsnorm_rows_kernel<true><<<(unsigned)T, kNormThreads, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)table, ids, nullptr, 0, x, (int)hidden, (const __nv_bfloat16*)norm_w, eps,
      (__nv_bfloat16*)y);
  return launch_status("embed_rmsnorm");
}

extern "C" int janus_b200_add_rmsnorm(float* x, const void* delta, int64_t delta_stride, int64_t T, int64_t hidden,
                                      const void* norm_w, float eps, void* y, void* stream) {
  int st = check_norm_args(T, hidden, y, norm_w);
  if (st) return st;
  JB_REQUIRE(x, JANUS_ERR_INVALID, "add_rmsnorm: null x");
  JB_REQUIRE(JB_ALIGNED(x, 16), JANUS_ERR_ALIGNMENT, "add_rmsnorm: x alignment");
  if (delta) {
    JB_REQUIRE(delta_stride >= hidden && delta_stride % 8 == 0 && JB_ALIGNED(delta, 16), JANUS_ERR_ALIGNMENT,
               "add_rmsnorm: delta stride %lld / alignment", (long long)delta_stride);
  }
  if (T == 0) return JANUS_OK;
  JB_REQUIRE((hidden / 8 + kNormThreads - 1) / kNormThreads <= kNormVec, JANUS_ERR_UNSUPPORTED,
             "add_rmsnorm: hidden %lld too large", (long long)hidden);
  rmsnorm_rows_kernel<false><<<(unsigned)T, kNormThreads, 0, (cudaStream_t)stream>>>(
      nullptr, nullptr, (const __nv_bfloat16*)delta, delta_stride, x, (int)hidden, (const __nv_bfloat16*)norm_w,
      eps, (__nv_bfloat16*)y);
  return launch_status("add_rmsnorm");
}

extern "C" int janus_b200_silu_mul(const void* gu, int64_t T, int64_t inter, void* out, void* stream) {
  JB_REQUIRE(gu && out && T >= 0 && inter > 0 && inter % 8 == 0, JANUS_ERR_INVALID,
             "silu_mul: bad arguments (inter %lld must be a multiple of 8)", (long long)inter);
  JB_REQUIRE(JB_ALIGNED(gu, 16) && JB_ALIGNED(out, 16), JANUS_ERR_ALIGNMENT, "silu_mul: alignment");
  if (T == 0) return JANUS_OK;
  if (inter % 16 == 0 && JB_ALIGNED(gu, 32) && JB_ALIGNED(out, 32)) {
    const int64_t blocks = T < 148 * 4 ? T : 148 * 4;  // 4 CTAs of 192 threads per SM (80 registers)
    silu_mul32_kernel<<<(unsigned)blocks, kSilu32Threads, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16*)gu, T, (int)inter, (__nv_bfloat16*)out);
    return launch_status("silu_mul");
  }
  const int64_t blocks = T < 148 * 16 ? T : 148 * 16;
  silu_mul_kernel<<<(unsigned)blocks, kSiluThreads, 0, (cudaStream_t)stream>>>((const __nv_bfloat16*)gu, T,
                                                                                (int)inter, (__nv_bfloat16*)out);
  return launch_status("silu_mul");
}

extern "C" int janus_b200_gated_rmsnorm(const void* core, const void* z, int64_t z_stride, int64_t T, int64_t Hv,
                                        int64_t Dv, const void* w, float eps, void* out, void* stream) {
  JB_REQUIRE(core && z && w && out && T >= 0 && Hv > 0 && z_stride >= Hv * Dv, JANUS_ERR_INVALID,
             "gated_rmsnorm: bad arguments");
  JB_REQUIRE(JB_ALIGNED(core, 16) && JB_ALIGNED(z, 16) && JB_ALIGNED(w, 16) && JB_ALIGNED(out, 16) && z_stride % 8 == 0,
             JANUS_ERR_ALIGNMENT, "gated_rmsnorm: 16-byte alignment of core/z/w/out and z_stride % 8");
  if (T == 0) return JANUS_OK;
  const int th = 256;
  cudaStream_t s = (cudaStream_t)stream;
  if ((Dv == 64 || Dv == 128) && T * Hv * (Dv / 16) < (int64_t(1) << 31) && z_stride % 16 == 0 &&
      JB_ALIGNED(core, 32) && JB_ALIGNED(z, 32) && JB_ALIGNED(w, 32) && JB_ALIGNED(out, 32)) {
    const int64_t units = T * Hv * (Dv / 16);
    const int64_t want = (units + th - 1) / th;
    const unsigned blocks32 = (unsigned)(want < 148 * 4 ? want : 148 * 4);  // 4 CTAs of 256 threads per SM
    if (Dv == 128)
      gated_rmsnorm32_kernel<128><<<blocks32, th, 0, s>>>((const __nv_bfloat16*)core, (const __nv_bfloat16*)z,
                                                          z_stride, (uint32_t)(T * Hv), (uint32_t)Hv,
                                                          (const __nv_bfloat16*)w, eps, (__nv_bfloat16*)out);
    else
      gated_rmsnorm32_kernel<64><<<blocks32, th, 0, s>>>((const __nv_bfloat16*)core, (const __nv_bfloat16*)z, z_stride,
                                                         (uint32_t)(T * Hv), (uint32_t)Hv, (const __nv_bfloat16*)w,
                                                         eps, (__nv_bfloat16*)out);
    return launch_status("gated_rmsnorm");
  }
  const unsigned blocks = (unsigned)((T * Hv * (Dv / 8) + th - 1) / th);
  switch (Dv) {
    case 32:
      gated_rmsnorm_kernel<32><<<blocks, th, 0, s>>>((const __nv_bfloat16*)core, (const __nv_bfloat16*)z, z_stride, T,
                                                     (int)Hv, (const __nv_bfloat16*)w, eps, (__nv_bfloat16*)out);
      break;
    case 64:
      gated_rmsnorm_kernel<64><<<blocks, th, 0, s>>>((const __nv_bfloat16*)core, (const __nv_bfloat16*)z, z_stride, T,
                                                     (int)Hv, (const __nv_bfloat16*)w, eps, (__nv_bfloat16*)out);
      break;
    case 128:
      gated_rmsnorm_kernel<128><<<blocks, th, 0, s>>>((const __nv_bfloat16*)core, (const __nv_bfloat16*)z, z_stride,
                                                      T, (int)Hv, (const __nv_bfloat16*)w, eps, (__nv_bfloat16*)out);
      break;
    default:
      set_error("gated_rmsnorm: Dv %lld not compiled (32, 64, 128)", (long long)Dv);
      return JANUS_ERR_UNSUPPORTED;
  }
  return launch_status("gated_rmsnorm");
}
