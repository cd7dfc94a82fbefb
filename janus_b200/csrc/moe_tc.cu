// The permuted grouped W4A16 GEMMs of the MoE on the 5th-generation tensor cores (the two GEMMs of
// janus/moe_w4a16.py:37-86): one CTA per (tile of 128 expert-sorted rows, block of output columns).
//
//   GEMM 1 (gated):  h[sorted row] = silu(x[token] Wg^T) * (x[token] Wu^T)   B rows: 128 gate + 128 up rows
//   GEMM 2 (down):   y[assignment] = w_assignment * (h[sorted row] Wd^T)       B rows: 128 or 256 output rows
//
// Weights stay int4 in HBM (two codes per byte, k = 2j in the low nibble, one bf16 scale per 128 inputs); the B
// operand is decoded on the fly: TMA brings the packed codes of a 64-deep k-block into a ring, four converter
// warps turn them into bf16 in registers (code * scale, rounded once to bf16: the value the reference's
// dequantise path feeds its GEMM) and write the 128B-swizzled K-major tile the MMA reads. The activation rows are
// gathered with cp.async (GEMM 1 reads the token of each assignment; GEMM 2 the sorted rows), and one thread issues
// M=128 MMAs into an fp32 accumulator in TMEM, so decode, gather and the tensor core overlap across a 4-stage ring.
//
// Warps: 0 TMA producer (codes), 1 TMEM owner and MMA issuer, 2-3 activation gather, 4-7 converters; all eight
// read the accumulator in the epilogue (warp w reads TMEM lanes 32 (w % 4) .. +31, columns half w / 4).
// Every hand-off is an mbarrier with a bounded wait: a wait that runs out sets the status word and the CTA
// winds down (loads in flight are waited for, MMAs drained, TMEM released) without storing.
#include "tcgen05.cuh"

namespace jb {
namespace mtc {
using namespace tcx;

constexpr int BM = 128;    // rows per tile (the routing plan's tile height)
constexpr int BK = 64;     // one 128-byte swizzle atom of bf16 along k
constexpr int GROUP = 128;  // inputs per scale
constexpr int NT = 256;
constexpr int S = 4;  // activation + decoded-weight stages
constexpr int C = 4;  // packed-code slots
constexpr uint32_t kA = BM * BK * 2;  // 16 KB

template <int BN>
struct Layout {
  static constexpr uint32_t kB = BN * BK * 2;    // decoded weights of a stage
  static constexpr uint32_t kCode = BN * BK / 2;  // packed codes of a k-block
  __host__ __device__ static constexpr uint32_t a(int s) { return s * kA; }
  __host__ __device__ static constexpr uint32_t b(int s) { return S * kA + s * kB; }
  __host__ __device__ static constexpr uint32_t code(int c) { return S * (kA + kB) + c * kCode; }
  static constexpr uint32_t bytes = S * (kA + kB) + C * kCode;
};

struct Params {
  CUtensorMap cmap;  // codes [E * NW rows][K / 2 bytes], boxes of 128 rows x 32 bytes
  const __nv_bfloat16* A;
  int64_t lda;
  const __nv_bfloat16* scales;  // [E * NW][K / 128]
  const int32_t* sorted_ids;
  const int32_t* tile_expert;
  const int32_t* n_tiles;
  const float* topk_w;
  __nv_bfloat16* out;
  int64_t ldo;
  int32_t* err;
  int N, K, topk, nblk;
};

struct Bars {
  uint64_t full[S], empty[S], cfull[C], cempty[C], drain;
};

// 8 int4 codes (k = 0..7 of a 32-bit word, k even in the low nibble) -> 8 bf16 (code * scale, one rounding).
// 128 + (code ^ 8) is exact in bf16 (exponent of 128, code in the low mantissa bits); subtracting 136 gives the
// signed code exactly, and the bf16 product with the scale is the fp32 product rounded once to nearest even.
__device__ __forceinline__ uint4 decode8(uint32_t x, __nv_bfloat162 s2) {
  const uint32_t t = x >> 4;
  const __nv_bfloat162 c136 = __floats2bfloat162_rn(136.f, 136.f);
  uint32_t w[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    // byte p of x to byte 0 (k = 2p in bits 0-3), byte p of x >> 4 to byte 2 (k = 2p + 1 in bits 16-19)
    const uint32_t pr = __byte_perm(x, t, 0x0400u | (uint32_t)p | ((uint32_t)p << 8));
    const uint32_t m = (pr & 0x000F000Fu) ^ 0x43084308u;
    __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&m);
    v = __hmul2(__hsub2(v, c136), s2);
    w[p] = *reinterpret_cast<uint32_t*>(&v);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ void cpa16(uint32_t dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0) : "memory");
}

// BN = MMA width: 256 for the gated GEMM (128 output columns: 128 gate + 128 up rows of B), 128 or 256 otherwise
template <bool GATED, int BN>
__global__ void __launch_bounds__(NT, 1) moe_w4a16_tc_kernel(const __grid_constant__ Params p) {
  using L = Layout<BN>;
  extern __shared__ unsigned char raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = s32(base);
  __shared__ Bars bars;
  __shared__ uint32_t tmem_base;
  __shared__ int32_t s_rows[BM];
  __shared__ int s_ok;

  const int tile = blockIdx.x / p.nblk, nb = blockIdx.x % p.nblk;
  if (tile >= p.n_tiles[0]) return;  // worst-case grid: tiles past the plan's count have no rows
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int e = p.tile_expert[tile];
  const int NW = GATED ? 2 * p.N : p.N;
  const int n0 = nb * (GATED ? BN / 2 : BN);  // first output column of the block
  const int nkb = p.K / BK;

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(&tmem_base)),
                 "r"(BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  if (tid < BM) {
    const int id = p.sorted_ids[(int64_t)tile * BM + tid];
    // GEMM 1 gathers the token (or received row) of the assignment; GEMM 2 reads its own sorted row
    s_rows[tid] = id < 0 ? -1 : (GATED ? id / p.topk : tile * BM + tid);
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      bar_init(&bars.full[s], 64 + 128);  // the gather threads and the converter threads
      bar_init(&bars.empty[s], 1);        // the stage's MMAs (commit)
    }
    for (int c = 0; c < C; ++c) {
      bar_init(&bars.cfull[c], 1);   // the producer's expect_tx, then the TMA bytes
      bar_init(&bars.cempty[c], 4);  // one arrival per converter warp
    }
    bar_init(&bars.drain, 1);
    s_ok = 1;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tm = tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------------------------ TMA producer (codes)
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      const int wrow = e * NW + n0;  // first weight row of box 0
      for (int kb = 0; kb < nkb && ok; ++kb) {
        const int c = kb % C;
        if (kb >= C) ok = wait_bar(&bars.cempty[c], ((kb / C) - 1) & 1, p.err);
        if (!ok) break;
        bar_expect_tx(&bars.cfull[c], L::kCode);
#pragma unroll
        for (int bx = 0; bx < BN / 128; ++bx) {
          const int r = GATED ? (bx == 0 ? wrow : wrow + p.N) : wrow + bx * 128;
          tma_load2(sbase + L::code(c) + bx * 128 * 32, &p.cmap, kb * (BK / 2), r, &bars.cfull[c]);
        }
        issued = kb + 1;
      }
      if (!ok) s_ok = 0;
      // every issued load has landed before the CTA may leave (on the normal path the converters consume them all)
      for (int kb = issued - C < 0 ? 0 : issued - C; kb < issued; ++kb)
        wait_bar_quiet(&bars.cfull[kb % C], (kb / C) & 1, p.err);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID = idesc(BM, BN, 0, 0);
      bool ok = true;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % S;
        ok = wait_bar(&bars.full[s], (kb / S) & 1, p.err);
        if (!ok) break;
        fence_after();
#pragma unroll
        for (int ks = 0; ks < BK / 16; ++ks)
          mma(tm, sdesc(sbase + L::a(s) + ks * 32, 16, 1024), sdesc(sbase + L::b(s) + ks * 32, 16, 1024), ID,
              (kb | ks) != 0);
        commit(&bars.empty[s]);
      }
      if (!ok) s_ok = 0;
      commit(&bars.drain);  // completes once every MMA issued above has finished
    }
  } else if (warp < 4) {
    // ---------------------------------------------------------------------------------- activation gather
    const int gt = tid - 64;
    bool ok = true;
    int pending = -1;  // k-block whose loads are in flight and not yet signalled
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % S;
      if (kb >= S) ok = wait_bar(&bars.empty[s], ((kb / S) - 1) & 1, p.err);
      if (!ok) break;
      const uint32_t dst = sbase + L::a(s);
#pragma unroll
      for (int i = 0; i < BM * (BK / 8) / 64; ++i) {
        const int x = gt + 64 * i, r = x >> 3, c = x & 7;
        const int row = s_rows[r];
        cpa16(dst + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4),
              p.A + (int64_t)(row < 0 ? 0 : row) * p.lda + kb * BK + c * 8, row >= 0);
      }
      asm volatile("cp.async.commit_group;\n" ::: "memory");
      if (pending >= 0) {
        asm volatile("cp.async.wait_group 1;\n" ::: "memory");
        fence_async_smem();  // the generic-proxy writes are visible to the tensor core's reads
        bar_arrive(&bars.full[pending % S]);
      }
      pending = kb;
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    if (ok && pending >= 0) {
      fence_async_smem();
      bar_arrive(&bars.full[pending % S]);
    }
    if (!ok) s_ok = 0;
  } else {
    // ----------------------------------------------------------------------------------------- converters
    constexpr int U = BN / 64;  // units (one row, 32 codes) per thread and k-block
    const int ct = tid - 128, hf = ct & 1;
    const __nv_bfloat16* sc[U];
    int rr[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int r = (ct >> 1) + 64 * j;  // row of the B tile
      rr[j] = r;
      const int wr = GATED ? (r < 128 ? n0 + r : p.N + n0 + r - 128) : n0 + r;
      sc[j] = p.scales + ((int64_t)e * NW + wr) * (p.K / GROUP);
    }
    __nv_bfloat16 s_cur[U], s_nxt[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      s_cur[j] = sc[j][0];
      s_nxt[j] = p.K / GROUP > 1 ? sc[j][1] : s_cur[j];
    }
    bool ok = true;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % S, c = kb % C;
      if (kb > 0 && (kb & 1) == 0) {  // a new scale group; prefetch the one after it
        const int g = kb >> 1;
#pragma unroll
        for (int j = 0; j < U; ++j) {
          s_cur[j] = s_nxt[j];
          if (g + 1 < p.K / GROUP) s_nxt[j] = sc[j][g + 1];
        }
      }
      ok = wait_bar(&bars.cfull[c], (kb / C) & 1, p.err);
      if (!ok) break;
      uint4 q[U];
#pragma unroll
      for (int j = 0; j < U; ++j)
        q[j] = *reinterpret_cast<const uint4*>(base + L::code(c) + rr[j] * 32 + hf * 16);
      __syncwarp();
      if (lane == 0) bar_arrive(&bars.cempty[c]);
      if (kb >= S) ok = wait_bar(&bars.empty[s], ((kb / S) - 1) & 1, p.err);
      if (!ok) break;
      unsigned char* bt = base + L::b(s);
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const __nv_bfloat162 s2 = __halves2bfloat162(s_cur[j], s_cur[j]);
        const uint32_t wv[4] = {q[j].x, q[j].y, q[j].z, q[j].w};
        const int r = rr[j];
#pragma unroll
        for (int w = 0; w < 4; ++w)
          *reinterpret_cast<uint4*>(bt + (r >> 3) * 1024 + (r & 7) * 128 + (((hf * 4 + w) ^ (r & 7)) << 4)) =
              decode8(wv[w], s2);
      }
      fence_async_smem();
      bar_arrive(&bars.full[s]);
    }
    if (!ok) s_ok = 0;
  }

  // ------------------------------------------------------------------------------------------------ epilogue
  fence_before();
  __syncthreads();
  fence_after();
  wait_bar_quiet(&bars.drain, 0, p.err);
  fence_after();
  if (s_ok) {
    const int q = warp & 3, hc = warp >> 2;
    const int r = 32 * q + lane;
    const int id = p.sorted_ids[(int64_t)tile * BM + r];
    const uint32_t la = tm + ((uint32_t)(32 * q) << 16);
    if (GATED) {
      // 64 output columns per warp: gate columns hc*64 .. +63 of the accumulator, up columns 128 + the same
      __nv_bfloat16* dst = p.out + ((int64_t)tile * BM + r) * p.ldo + n0 + hc * 64;
#pragma unroll
      for (int cc = 0; cc < 64; cc += 16) {
        float g[16], u[16];
        tld16f(la + hc * 64 + cc, g);
        tld16f(la + 128 + hc * 64 + cc, u);
        uint32_t o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = pack_bf16(silu(g[2 * i]) * u[2 * i], silu(g[2 * i + 1]) * u[2 * i + 1]);
        if (id >= 0) {
          reinterpret_cast<uint4*>(dst + cc)[0] = make_uint4(o[0], o[1], o[2], o[3]);
          reinterpret_cast<uint4*>(dst + cc)[1] = make_uint4(o[4], o[5], o[6], o[7]);
        }
      }
    } else {
      constexpr int CW = BN / 2;  // columns per warp
      const float wgt = id >= 0 ? p.topk_w[id] : 0.f;
      __nv_bfloat16* dst = p.out + (int64_t)(id < 0 ? 0 : id) * p.ldo + n0 + hc * CW;
#pragma unroll
      for (int cc = 0; cc < CW; cc += 16) {
        float a[16];
        tld16f(la + hc * CW + cc, a);
        uint32_t o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = pack_bf16(a[2 * i] * wgt, a[2 * i + 1] * wgt);
        if (id >= 0) {
          reinterpret_cast<uint4*>(dst + cc)[0] = make_uint4(o[0], o[1], o[2], o[3]);
          reinterpret_cast<uint4*>(dst + cc)[1] = make_uint4(o[4], o[5], o[6], o[7]);
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(BN));
}

}  // namespace mtc
}  // namespace jb

// ------------------------------------------------------------------------------------------------ host side

using namespace jb;

namespace {

// packed codes [rows][K / 2] bytes, boxes of 128 rows x 32 bytes (one 64-deep k-block), no swizzle
int code_map(CUtensorMap* m, const void* codes, uint64_t rows, uint64_t K) {
  tcx::EncodeTiled enc = tcx::encode_tiled_fn();
  if (!enc) {
    set_error("moe_grouped_w4a16: cuTensorMapEncodeTiled unavailable");
    return JANUS_ERR_CUDA;
  }
  const cuuint64_t dims[2] = {K / 2, rows};
  const cuuint64_t strides[1] = {K / 2};
  const cuuint32_t box[2] = {mtc::BK / 2, 128};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(codes), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("moe_grouped_w4a16: tensor map encode failed (%d)", (int)r);
    return JANUS_ERR_INVALID;
  }
  return JANUS_OK;
}

template <bool GATED, int BN>
int launch(const mtc::Params& p, int64_t max_tiles, cudaStream_t s) {
  const size_t smem = mtc::Layout<BN>::bytes + 1024;
  auto kern = mtc::moe_w4a16_tc_kernel<GATED, BN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    set_error("moe_grouped_w4a16: smem attribute: %s", cudaGetErrorString(e));
    return JANUS_ERR_CUDA;
  }
  kern<<<(unsigned)(max_tiles * p.nblk), mtc::NT, smem, s>>>(p);
  return launch_status("moe_grouped_w4a16");
}

}  // namespace

extern "C" int janus_b200_moe_grouped_w4a16(const void* x, int64_t ldx, const uint8_t* codes, const void* scales,
                                            int64_t E, int64_t N, int64_t K, int32_t gated, const int32_t* sorted_ids,
                                            const int32_t* tile_expert, const int32_t* n_tiles, int64_t max_tiles,
                                            int64_t topk, const float* topk_w, void* out, int64_t ldo,
                                            int32_t* status, void* stream) {
  JB_REQUIRE(x && codes && scales && sorted_ids && tile_expert && n_tiles && out, JANUS_ERR_INVALID,
             "moe_grouped_w4a16: null pointer");
  JB_REQUIRE(E > 0 && N > 0 && N % 128 == 0 && K > 0 && K % mtc::GROUP == 0 && topk > 0 && max_tiles >= 0,
             JANUS_ERR_UNSUPPORTED, "moe_grouped_w4a16: N %lld and K %lld must be multiples of 128", (long long)N,
             (long long)K);
  JB_REQUIRE(gated || topk_w, JANUS_ERR_INVALID, "moe_grouped_w4a16: the down projection needs routing weights");
  JB_REQUIRE(ldx % 8 == 0 && ldo % 8 == 0 && JB_ALIGNED(x, 16) && JB_ALIGNED(codes, 16) && JB_ALIGNED(out, 16),
             JANUS_ERR_ALIGNMENT, "moe_grouped_w4a16: x, codes and out 16-byte aligned, ldx and ldo multiples of 8");
  const int64_t NW = gated ? 2 * N : N;
  JB_REQUIRE(E * NW < (1ll << 31) && K < (1 << 30), JANUS_ERR_UNSUPPORTED, "moe_grouped_w4a16: sizes");
  const int64_t nblk = gated ? N / 128 : (N % 256 == 0 ? N / 256 : N / 128);
  JB_REQUIRE(max_tiles * nblk < (1ll << 31), JANUS_ERR_UNSUPPORTED, "moe_grouped_w4a16: grid");
  if (max_tiles == 0) return JANUS_OK;
  mtc::Params p{};
  int st = code_map(&p.cmap, codes, (uint64_t)(E * NW), (uint64_t)K);
  if (st) return st;
  p.A = (const __nv_bfloat16*)x;
  p.lda = ldx;
  p.scales = (const __nv_bfloat16*)scales;
  p.sorted_ids = sorted_ids;
  p.tile_expert = tile_expert;
  p.n_tiles = n_tiles;
  p.topk_w = topk_w;
  p.out = (__nv_bfloat16*)out;
  p.ldo = ldo;
  p.err = status;
  p.N = (int)N;
  p.K = (int)K;
  p.topk = (int)topk;
  p.nblk = (int)nblk;
  cudaStream_t s = (cudaStream_t)stream;
  if (gated) return launch<true, 256>(p, max_tiles, s);
  if (N % 256 == 0) return launch<false, 256>(p, max_tiles, s);
  return launch<false, 128>(p, max_tiles, s);
}
