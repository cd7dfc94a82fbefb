// The permuted grouped W4A16 GEMMs of the MoE on the 5th-generation tensor cores (the two GEMMs of
// janus/moe_w4a16.py:37-86): one CTA per (tile of 128 expert-sorted rows, block of output columns).
//
//   GEMM 1 (gated):  h[sorted row] = silu(x[token] Wg^T) * (x[token] Wu^T)   B rows: 128 gate + 128 up rows
//   GEMM 2 (down):   y[assignment] = w_assignment * (h[sorted row] Wd^T)       B rows: 128 or 256 output rows
//
// Weights stay 4-bit in HBM, two codes per byte (k = 2j in the low nibble), in one of two formats: int4 with one bf16
// scale per 128 inputs (code * scale), or the reference's NVFP4 (e2m1 codes, one e4m3 scale per 16 inputs and an
// fp32 global scale per weight row: e2m1 * (scale * global), janus/hybrid.py:400-425). The B operand is decoded on
// the fly: TMA brings the packed codes of a 64-deep k-block into a ring, converter warps turn them into bf16 in
// registers (the exact fp32 value rounded once to bf16: the value the reference's dequantise path feeds its GEMM)
// and write the 128B-swizzled K-major tile the MMA reads. The activation rows are
// gathered with cp.async (GEMM 1 reads the token of each assignment; GEMM 2 the sorted rows), and one thread issues
// M=128 MMAs into an fp32 accumulator in TMEM, so decode, gather and the tensor core overlap across a 3-stage ring.
//
// Persistent CTAs (one per SM) walk the work items; the fp32 accumulator is double-buffered in TMEM so an item's
// epilogue overlaps the next item's main loop. Warps: 0 TMA producer (codes), 1 TMEM owner and MMA issuer, 2-3
// activation gather, 4-11 converters (two groups of four: even and odd k-blocks, so the decode of two k-blocks is
// in flight at once), 12-15 epilogue (warp w reads TMEM lanes 32 (w % 4) .. +31). Every hand-off is an mbarrier
// with a bounded wait: a wait that runs out sets the status word and the CTA winds down (loads in flight are
// waited for, MMAs drained, TMEM released).
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "tcgen05.cuh"

namespace jb {
namespace mtc {
using namespace tcx;

constexpr int BM = 128;    // rows per tile (the routing plan's tile height)
constexpr int BK = 64;     // one 128-byte swizzle atom of bf16 along k
constexpr int GROUP = 128;  // inputs per scale
constexpr int NT = 512;  // producer, MMA, 2 gather, 8 converter (two groups), 4 epilogue warps
constexpr int S = 3;  // activation + decoded-weight stages
constexpr int C = 4;  // packed-code slots
constexpr uint32_t kA = BM * BK * 2;  // 16 KB

template <int BN>
struct Layout {
  static constexpr uint32_t kB = BN * BK * 2;    // decoded weights of a stage
  static constexpr uint32_t kCode = BN * BK / 2;  // packed codes of a k-block
  __host__ __device__ static constexpr uint32_t a(int s) { return s * kA; }
  __host__ __device__ static constexpr uint32_t b(int s) { return S * kA + s * kB; }
  __host__ __device__ static constexpr uint32_t code(int c) { return S * (kA + kB) + c * kCode; }
  static constexpr uint32_t out_stage = S * (kA + kB) + C * kCode;  // 4 epilogue warps x 32 rows x 64 bytes
  static constexpr uint32_t bytes = out_stage + 4 * 32 * 64;
};

struct Params {
  CUtensorMap cmap;  // codes [E * NW rows][K / 2 bytes], boxes of 128 rows x 32 bytes
  const __nv_bfloat16* A;
  int64_t lda;
  const __nv_bfloat16* scales;  // int4: [E * NW][K / 128]
  const uint8_t* bscales;       // NVFP4: e4m3 [E * NW][K / 16]
  const float* gscales;         // NVFP4: fp32 [E * NW]
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
  uint64_t full[S], empty[S], cfull[C], cempty[C], acc_full[2], acc_empty[2], drain;
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

// 8 e2m1 codes (k = 0..7 of a 32-bit word, k even in the low nibble) -> 8 bf16 of e2m1 * s, s the fp32 block scale
// times the global scale passed in as s * 2^14. The code's bits e1 e0 m placed as an fp16 exponent and top mantissa
// bit give e2m1 * 2^-14 exactly (code 1, 0.5, as a denormal); times s * 2^14 that is the fp32 product e2m1 * s of the
// reference, rounded once to bf16.
__device__ __forceinline__ uint4 decode8_fp4(uint32_t x, float s14) {
  const uint32_t t = x >> 4;
  uint32_t w[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t n = __byte_perm(x, t, 0x0400u | (uint32_t)p | ((uint32_t)p << 8)) & 0x000F000Fu;
    const uint32_t hb = ((n & 0x00070007u) << 9) | ((n & 0x00080008u) << 12);
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hb));
    w[p] = pack_bf16(f.x * s14, f.y * s14);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// block scale (e4m3) times the row's global scale, in fp32 as the reference forms it, times 2^14 (exact)
__device__ __forceinline__ float fp4_scale14(uint8_t e4m3, float global) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)e4m3, __NV_E4M3);
  return (__half2float(*reinterpret_cast<const __half*>(&h)) * global) * 16384.f;
}

__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
__device__ __forceinline__ void cpa16(uint32_t dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0) : "memory");
}

// BN = MMA width: 256 for the gated GEMM (128 output columns: 128 gate + 128 up rows of B), 128 or 256 otherwise.
// Persistent: CTA b takes the work items (tile, column block) b, b + grid, ...; the accumulator is double-buffered
// in TMEM so the epilogue of one item overlaps the main loop of the next.
template <bool GATED, int BN, bool FP4>
__global__ void __launch_bounds__(NT, 1) moe_w4a16_tc_kernel(const __grid_constant__ Params p) {
  using L = Layout<BN>;
  extern __shared__ unsigned char raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = s32(base);
  __shared__ Bars bars;
  __shared__ uint32_t tmem_base;

  const int n_items = p.n_tiles[0] * p.nblk;
  if ((int)blockIdx.x >= n_items) return;  // worst-case grid: nothing for this CTA
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x;
  const int NW = GATED ? 2 * p.N : p.N;
  const int nkb = p.K / BK;  // even: K is a multiple of the scale group
  // item -> (tile, first output column); B-tile row r -> weight row of expert e
  auto tile_of = [&](int it) { return it / p.nblk; };
  auto n0_of = [&](int it) { return (it % p.nblk) * (GATED ? BN / 2 : BN); };
  auto wrow = [&](int e, int n0, int r) {
    return e * NW + (GATED ? (r < 128 ? n0 + r : p.N + n0 + r - 128) : n0 + r);
  };

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(&tmem_base)),
                 "r"(2 * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      bar_init(&bars.full[s], 64 + 128);  // the gather threads and one converter group
      bar_init(&bars.empty[s], 1);        // the stage's MMAs (commit)
    }
    for (int c = 0; c < C; ++c) {
      bar_init(&bars.cfull[c], 1);   // the producer's expect_tx, then the TMA bytes
      bar_init(&bars.cempty[c], 4);  // one arrival per warp of the converter group
    }
    for (int a = 0; a < 2; ++a) {
      bar_init(&bars.acc_full[a], 1);   // the item's last MMAs (commit)
      bar_init(&bars.acc_empty[a], 4);  // one arrival per epilogue warp
    }
    bar_init(&bars.drain, 1);
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
      int q = 0, issued = 0;
      int e_next = p.tile_expert[tile_of(blockIdx.x)];
      for (int it = blockIdx.x; it < n_items && ok; it += G) {
        const int e = e_next, n0 = n0_of(it);
        if (it + G < n_items) e_next = p.tile_expert[tile_of(it + G)];
        for (int kb = 0; kb < nkb; ++kb, ++q) {
          const int c = q % C;
          if (q >= C) ok = wait_bar(&bars.cempty[c], ((q / C) - 1) & 1, p.err);
          if (!ok) break;
          bar_expect_tx(&bars.cfull[c], L::kCode);
#pragma unroll
          for (int bx = 0; bx < BN / 128; ++bx)
            tma_load2(sbase + L::code(c) + bx * 128 * 32, &p.cmap, kb * (BK / 2), wrow(e, n0, bx * 128),
                      &bars.cfull[c]);
          issued = q + 1;
        }
      }
      // every issued load has landed before the CTA may leave (on the normal path the converters consume them all)
      for (int j = issued - C < 0 ? 0 : issued - C; j < issued; ++j)
        wait_bar_quiet(&bars.cfull[j % C], (j / C) & 1, p.err);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID = idesc(BM, BN, 0, 0);
      bool ok = true;
      int q = 0, i = 0;
      for (int it = blockIdx.x; it < n_items && ok; it += G, ++i) {
        const int ab = i & 1;
        if (i >= 2) ok = wait_bar(&bars.acc_empty[ab], ((i >> 1) - 1) & 1, p.err);
        if (!ok) break;
        fence_after();
        const uint32_t acc = tm + ab * BN;
        for (int kb = 0; kb < nkb; ++kb, ++q) {
          const int s = q % S;
          ok = wait_bar(&bars.full[s], (q / S) & 1, p.err);
          if (!ok) break;
          fence_after();
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks)
            mma(acc, sdesc(sbase + L::a(s) + ks * 32, 16, 1024), sdesc(sbase + L::b(s) + ks * 32, 16, 1024), ID,
                (kb | ks) != 0);
          commit(&bars.empty[s]);
        }
        if (ok) commit(&bars.acc_full[ab]);
      }
      commit(&bars.drain);  // completes once every MMA issued above has finished
    }
  } else if (warp < 4) {
    // ---------------------------------------------------------------------------------- activation gather
    // thread: 16-byte chunk c8 of rows rb + 8 i (i = 0..15) of the tile; smem row rb + 8 i of the swizzled stage
    const int gt = tid - 64, c8 = gt & 7, rb = gt >> 3;
    const uint32_t doff = rb * 128 + ((c8 ^ rb) << 4);
    bool ok = true;
    int q = 0, pending = -1;
    int id_next[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) id_next[i] = p.sorted_ids[(int64_t)tile_of(blockIdx.x) * BM + rb + 8 * i];
    for (int it = blockIdx.x; it < n_items && ok; it += G) {
      const int tile = tile_of(it);
      const __nv_bfloat16* src[16];  // the row's 16-byte chunk at k = 0 (row 0 for a padding row, zero-filled)
      uint32_t live = 0;             // bit i: row rb + 8 i is an assignment
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int id = id_next[i];
        // GEMM 1 gathers the token (or received row) of the assignment; GEMM 2 reads its own sorted row
        const int64_t row = id < 0 ? 0 : (GATED ? id / p.topk : (int64_t)tile * BM + rb + 8 * i);
        src[i] = p.A + row * p.lda + c8 * 8;
        live |= (id >= 0 ? 1u : 0u) << i;
      }
      if (it + G < n_items) {
#pragma unroll
        for (int i = 0; i < 16; ++i) id_next[i] = p.sorted_ids[(int64_t)tile_of(it + G) * BM + rb + 8 * i];
      }
      for (int kb = 0; kb < nkb; ++kb, ++q) {
        const int s = q % S;
        if (q >= S) ok = wait_bar(&bars.empty[s], ((q / S) - 1) & 1, p.err);
        if (!ok) break;
        const uint32_t dst = sbase + L::a(s) + doff;
#pragma unroll
        for (int i = 0; i < 16; ++i) cpa16(dst + i * 1024, src[i] + kb * BK, (live >> i) & 1u);
        asm volatile("cp.async.commit_group;\n" ::: "memory");
        if (pending >= 0) {
          asm volatile("cp.async.wait_group 1;\n" ::: "memory");
          fence_async_smem();  // the generic-proxy writes are visible to the tensor core's reads
          bar_arrive(&bars.full[pending % S]);
        }
        pending = q;
      }
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    if (ok && pending >= 0) {
      fence_async_smem();
      bar_arrive(&bars.full[pending % S]);
    }
  } else if (warp < 12) {
    // ----------------------------------------------------------------------------------------- converters
    // two groups of four warps take the even and the odd k-blocks; thread: half hf of rows rr0 + 64 j of B
    constexpr int U = BN / 64;
    const int grp = (warp - 4) >> 2, ct = ((warp - 4) & 3) * 32 + lane, hf = ct & 1, rr0 = ct >> 1;
    const int gk = p.K / GROUP;
    const int fk = p.K / 16;  // NVFP4 block scales per row
    // 32-bit shared addresses: the codes of row rr0 (+ 64 j rows), and row rr0 of the B stage: row r of a 128B-swizzled
    // K-major tile starts at r * 128, its 16-byte unit u sits at (u ^ (r & 7)) * 16; r & 7 is the same for every j
    const uint32_t code0 = sbase + L::code(0) + rr0 * 32 + hf * 16;
    const uint32_t b0 = sbase + L::b(0) + rr0 * 128;
    uint32_t xo[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) xo[w] = (uint32_t)(((hf * 4 + w) ^ (rr0 & 7)) << 4);
    bool ok = true;
    int q = 0;
    // int4: this thread's rows' bf16 scales; NVFP4: their e4m3 block scales (the two blocks of this thread's half of
    // a k-block are one 16-bit load) and fp32 global scales
    const __nv_bfloat16* sp[U];
    const uint8_t* bp[U];
    float gs[U];
    __nv_bfloat16 s_nxt[U];  // int4: the scales of the next k-block this group decodes
    uint16_t b_nxt[U];       // NVFP4: the two block scales of the next k-block
    auto rows_of = [&](int it) {
      const int e = p.tile_expert[tile_of(it)], n0 = n0_of(it);
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const int64_t wr = wrow(e, n0, rr0 + 64 * j);
        if (FP4) {
          bp[j] = p.bscales + wr * fk + hf * 2;
          gs[j] = p.gscales[wr];
        } else {
          sp[j] = p.scales + wr * gk;
        }
      }
    };
    auto fetch = [&](int kb) {  // the scales of k-block kb of the current rows
#pragma unroll
      for (int j = 0; j < U; ++j) {
        if (FP4)
          b_nxt[j] = *reinterpret_cast<const uint16_t*>(bp[j] + kb * (BK / 16));
        else
          s_nxt[j] = sp[j][kb / (GROUP / BK)];
      }
    };
    rows_of(blockIdx.x);
    float g_cur[U];
#pragma unroll
    for (int j = 0; j < U; ++j) g_cur[j] = FP4 ? gs[j] : 0.f;
    fetch(grp);
    for (int it = blockIdx.x; it < n_items && ok; it += G) {
      const int nit = it + G;
      for (int kb = grp; kb < nkb; kb += 2) {
        const int qq = q + kb;
        __nv_bfloat16 s_cur[U];
        uint16_t b_cur[U];
#pragma unroll
        for (int j = 0; j < U; ++j) {
          s_cur[j] = s_nxt[j];
          b_cur[j] = b_nxt[j];
        }
        float g_use[U];
#pragma unroll
        for (int j = 0; j < U; ++j) g_use[j] = g_cur[j];
        if (kb + 2 < nkb) {  // prefetch the scales of this group's next k-block, in this item or the next
          fetch(kb + 2);
        } else if (nit < n_items) {
          rows_of(nit);
          fetch(grp);
#pragma unroll
          for (int j = 0; j < U; ++j) g_cur[j] = FP4 ? gs[j] : 0.f;
        }
        const int c = qq % C, s = qq % S;
        ok = wait_bar(&bars.cfull[c], (qq / C) & 1, p.err);
        if (!ok) break;
        // the codes are decoded into registers while the stage may still be in use; the slot is released only after
        // the stores that consume them: a release right after the loads let the TMA refilling the slot overwrite
        // codes whose loads had not returned yet
        uint4 dv[U][4];
#pragma unroll
        for (int j = 0; j < U; ++j) {
          const uint4 cw = lds128(code0 + c * L::kCode + j * (64 * 32));
          if (FP4) {  // words 0-1: the first 16-element block of this half, words 2-3 the second
            const float s0 = fp4_scale14((uint8_t)(b_cur[j] & 0xff), g_use[j]);
            const float s1 = fp4_scale14((uint8_t)(b_cur[j] >> 8), g_use[j]);
            dv[j][0] = decode8_fp4(cw.x, s0);
            dv[j][1] = decode8_fp4(cw.y, s0);
            dv[j][2] = decode8_fp4(cw.z, s1);
            dv[j][3] = decode8_fp4(cw.w, s1);
          } else {
            const __nv_bfloat162 s2 = __halves2bfloat162(s_cur[j], s_cur[j]);
            dv[j][0] = decode8(cw.x, s2);
            dv[j][1] = decode8(cw.y, s2);
            dv[j][2] = decode8(cw.z, s2);
            dv[j][3] = decode8(cw.w, s2);
          }
        }
        if (qq >= S) ok = wait_bar(&bars.empty[s], ((qq / S) - 1) & 1, p.err);
        if (!ok) break;
        const uint32_t bt = b0 + s * L::kB;
#pragma unroll
        for (int j = 0; j < U; ++j)
#pragma unroll
          for (int w = 0; w < 4; ++w) sts128(bt + j * (64 * 128) + xo[w], dv[j][w]);
        fence_async_smem();
        bar_arrive(&bars.full[s]);
        __syncwarp();
        if (lane == 0) bar_arrive(&bars.cempty[c]);
      }
      q += nkb;
    }
  } else {
    // ------------------------------------------------------------------------------------------- epilogue
    // thread = accumulator row (TMEM lane 32 (warp % 4) + lane). Each 32-column slice of the warp's rows goes through
    // a small shared-memory buffer so the global stores cover 8 rows x 64 bytes per instruction instead of 32 rows x
    // 16 bytes; the assignment ids and routing weights are loaded an item ahead of their use.
    const int eq = warp & 3, r = 32 * eq + lane;
    unsigned char* stg = base + L::out_stage + eq * (32 * 64);  // [32 rows][64 bytes], 16-byte units swizzled by row
    bool ok = true;
    int i = 0;
    int id_a = p.sorted_ids[(int64_t)tile_of(blockIdx.x) * BM + r];
    float w_a = (!GATED && id_a >= 0) ? p.topk_w[id_a] : 0.f;
    int id_b = (int)blockIdx.x + G < n_items ? p.sorted_ids[(int64_t)tile_of(blockIdx.x + G) * BM + r] : -1;
    for (int it = blockIdx.x; it < n_items && ok; it += G, ++i) {
      const int ab = i & 1, tile = tile_of(it), n0 = n0_of(it);
      const int id = id_a;
      const float wgt = w_a;
      w_a = (!GATED && id_b >= 0) ? p.topk_w[id_b] : 0.f;  // the next item's ids arrived an item ago
      id_a = id_b;
      id_b = it + 2 * G < n_items ? p.sorted_ids[(int64_t)tile_of(it + 2 * G) * BM + r] : -1;
      int64_t orow[4];  // output row of the rows k * 8 + lane / 4 this lane stores; -1: padding, not stored
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int src = k * 8 + (lane >> 2);
        const int sid = __shfl_sync(kFull, id, src);
        orow[k] = sid < 0 ? -1 : (GATED ? (int64_t)tile * BM + 32 * eq + src : (int64_t)sid);
      }
      ok = __all_sync(kFull, wait_bar_sleep(&bars.acc_full[ab], (i >> 1) & 1, p.err));
      if (!ok) break;
      fence_after();
      const uint32_t la = tm + ((uint32_t)(32 * eq) << 16) + ab * BN;
      constexpr int OUTC = GATED ? BN / 2 : BN;  // output columns of an item
#pragma unroll 1
      for (int cc = 0; cc < OUTC; cc += 32) {
        uint32_t o[16];
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          float a[16];
          tld16f(la + cc + 16 * h2, a);
          if (GATED) {  // silu(gate) * up: gate in accumulator columns 0..127, up in 128..255
            float u[16];
            tld16f(la + 128 + cc + 16 * h2, u);
#pragma unroll
            for (int k = 0; k < 8; ++k)
              o[8 * h2 + k] = pack_bf16(silu(a[2 * k]) * u[2 * k], silu(a[2 * k + 1]) * u[2 * k + 1]);
          } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) o[8 * h2 + k] = pack_bf16(a[2 * k] * wgt, a[2 * k + 1] * wgt);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
          *reinterpret_cast<uint4*>(stg + lane * 64 + ((u ^ ((lane >> 1) & 3)) << 4)) =
              make_uint4(o[4 * u], o[4 * u + 1], o[4 * u + 2], o[4 * u + 3]);
        __syncwarp();
        uint4 v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int rr = k * 8 + (lane >> 2);
          v[k] = *reinterpret_cast<const uint4*>(stg + rr * 64 + (((lane & 3) ^ ((rr >> 1) & 3)) << 4));
        }
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (orow[k] >= 0) *reinterpret_cast<uint4*>(p.out + orow[k] * p.ldo + n0 + cc + (lane & 3) * 8) = v[k];
        __syncwarp();  // the buffer is read before the next slice overwrites it
      }
      fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&bars.acc_empty[ab]);  // this warp's lanes of the buffer are read
    }
  }

  // wind down: every MMA issued has completed before TMEM is released
  fence_before();
  __syncthreads();
  fence_after();
  wait_bar_quiet(&bars.drain, 0, p.err);
  fence_before();
  __syncthreads();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(2 * BN));
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

template <bool GATED, int BN, bool FP4>
int launch(const mtc::Params& p, int64_t max_tiles, cudaStream_t s) {
  const size_t smem = mtc::Layout<BN>::bytes + 1024;
  auto kern = mtc::moe_w4a16_tc_kernel<GATED, BN, FP4>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    set_error("moe_grouped_w4a16: smem attribute: %s", cudaGetErrorString(e));
    return JANUS_ERR_CUDA;
  }
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                 cudaSuccess || sms <= 0) {
    set_error("moe_grouped_w4a16: device query failed");
    return JANUS_ERR_CUDA;
  }
  const int64_t items = max_tiles * p.nblk;  // worst case; the CTAs read the plan's count on the device
  kern<<<(unsigned)(items < sms ? items : sms), mtc::NT, smem, s>>>(p);
  return launch_status("moe_grouped_w4a16");
}

}  // namespace

// the checks and parameters shared by both weight formats; scales / bscales + gscales select the format
static int moe_grouped(const void* x, int64_t ldx, const uint8_t* codes, const void* scales, const uint8_t* bscales,
                       const float* gscales, int64_t E, int64_t N, int64_t K, int32_t gated, const int32_t* sorted_ids,
                       const int32_t* tile_expert, const int32_t* n_tiles, int64_t max_tiles, int64_t topk,
                       const float* topk_w, void* out, int64_t ldo, int32_t* status, void* stream, const char* name) {
  const bool fp4 = bscales != nullptr;
  JB_REQUIRE(x && codes && (fp4 ? (gscales != nullptr) : (scales != nullptr)) && sorted_ids && tile_expert && n_tiles &&
                 out,
             JANUS_ERR_INVALID, "%s: null pointer", name);
  JB_REQUIRE(E > 0 && N > 0 && N % 128 == 0 && K > 0 && K % mtc::GROUP == 0 && topk > 0 && max_tiles >= 0,
             JANUS_ERR_UNSUPPORTED, "%s: N %lld and K %lld must be multiples of 128", name, (long long)N, (long long)K);
  JB_REQUIRE(gated || topk_w, JANUS_ERR_INVALID, "%s: the down projection needs routing weights", name);
  JB_REQUIRE(ldx % 8 == 0 && ldo % 8 == 0 && JB_ALIGNED(x, 16) && JB_ALIGNED(codes, 16) && JB_ALIGNED(out, 16) &&
                 (!fp4 || JB_ALIGNED(bscales, 2)),
             JANUS_ERR_ALIGNMENT, "%s: x, codes and out 16-byte aligned, ldx and ldo multiples of 8", name);
  const int64_t NW = gated ? 2 * N : N;
  JB_REQUIRE(E * NW < (1ll << 31) && K < (1 << 30), JANUS_ERR_UNSUPPORTED, "%s: sizes", name);
  const int64_t nblk = gated ? N / 128 : (N % 256 == 0 ? N / 256 : N / 128);
  JB_REQUIRE(max_tiles * nblk < (1ll << 31), JANUS_ERR_UNSUPPORTED, "%s: grid", name);
  if (max_tiles == 0) return JANUS_OK;
  mtc::Params p{};
  int st = code_map(&p.cmap, codes, (uint64_t)(E * NW), (uint64_t)K);
  if (st) return st;
  p.A = (const __nv_bfloat16*)x;
  p.lda = ldx;
  p.scales = (const __nv_bfloat16*)scales;
  p.bscales = bscales;
  p.gscales = gscales;
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
  if (fp4) {
    if (gated) return launch<true, 256, true>(p, max_tiles, s);
    if (N % 256 == 0) return launch<false, 256, true>(p, max_tiles, s);
    return launch<false, 128, true>(p, max_tiles, s);
  }
  if (gated) return launch<true, 256, false>(p, max_tiles, s);
  if (N % 256 == 0) return launch<false, 256, false>(p, max_tiles, s);
  return launch<false, 128, false>(p, max_tiles, s);
}

extern "C" int janus_b200_moe_grouped_w4a16(const void* x, int64_t ldx, const uint8_t* codes, const void* scales,
                                            int64_t E, int64_t N, int64_t K, int32_t gated, const int32_t* sorted_ids,
                                            const int32_t* tile_expert, const int32_t* n_tiles, int64_t max_tiles,
                                            int64_t topk, const float* topk_w, void* out, int64_t ldo,
                                            int32_t* status, void* stream) {
  return moe_grouped(x, ldx, codes, scales, nullptr, nullptr, E, N, K, gated, sorted_ids, tile_expert, n_tiles,
                     max_tiles, topk, topk_w, out, ldo, status, stream, "moe_grouped_w4a16");
}

extern "C" int janus_b200_moe_grouped_nvfp4(const void* x, int64_t ldx, const uint8_t* codes,
                                            const uint8_t* block_scales, const float* global_scales, int64_t E,
                                            int64_t N, int64_t K, int32_t gated, const int32_t* sorted_ids,
                                            const int32_t* tile_expert, const int32_t* n_tiles, int64_t max_tiles,
                                            int64_t topk, const float* topk_w, void* out, int64_t ldo,
                                            int32_t* status, void* stream) {
  JB_REQUIRE(block_scales && global_scales, JANUS_ERR_INVALID, "moe_grouped_nvfp4: null scale pointer");
  return moe_grouped(x, ldx, codes, nullptr, block_scales, global_scales, E, N, K, gated, sorted_ids, tile_expert,
                     n_tiles, max_tiles, topk, topk_w, out, ldo, status, stream, "moe_grouped_nvfp4");
}
