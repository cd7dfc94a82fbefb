// Pieces of the chunk prep of the gated delta rule shared by the two-launch prep (gdn_chunk.cu) and the one-launch
// scan (gdn_scan_tc.cu), so that both round identically: the masked, decayed entries of N and QK from the [K; Q] K^T
// product, and the diagonal 16x16 blocks of T = (I - N)^-1.
#pragma once

namespace jb {

// e^(G_i - G_j) = 2^(Gl_i - Gl_j) with Gl = G log2(e) precomputed per token: one MUFU exponential per entry
constexpr float kLog2e = 1.4426950408889634f;
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// N_ij = -beta_i (K K^T)_ij e^(G_i - G_j) where the mask holds (j < i, same segment), else 0; nb = -beta_i. Masked
// entries may have a positive exponent (an infinite factor): the select drops them.
__device__ __forceinline__ float n_entry(float kk, float nb, float gli, float glj, bool m) {
  const float v = nb * kk * ex2_approx(gli - glj);
  return m ? v : 0.f;
}
// QK_ij = scale (Q K^T)_ij e^(G_i - G_j) where the mask holds (j <= i, same segment, token i live), else 0
__device__ __forceinline__ float qk_entry(float qk, float scale, float gli, float glj, bool m) {
  const float v = scale * qk * ex2_approx(gli - glj);
  return m ? v : 0.f;
}

// One warp inverts the block at rows / columns [bs, bs + 16): lane c < 16 owns column c of the block's T and solves
// (I - N) t = e_c by column-oriented forward substitution: once t[m] is final it is pushed into every later row,
// t[r] += N[r][m] t[m] for r > m. The 15 steps each issue independent FMAs, so the dependent chain is 15 FMAs long
// (a row-by-row dot product would chain all 120). Entries of t above the lane's column stay exactly zero and its
// diagonal entry exactly one. Lanes 16-31 compute a copy and store nothing. T may be N itself (the block is inverted
// in place: every lane's reads of N are done before the first write).
template <int LD>
__device__ __forceinline__ void diag_inverse16(const float* N, float* T, int bs, int lane) {
  const int cc = lane & 15;
  float col[16];
#pragma unroll
  for (int r = 0; r < 16; ++r) col[r] = (r == cc) ? 1.f : 0.f;
#pragma unroll
  for (int m = 0; m < 15; ++m) {
    const float tm = col[m];
#pragma unroll
    for (int r = m + 1; r < 16; ++r) col[r] = fmaf(N[(bs + r) * LD + bs + m], tm, col[r]);
  }
  __syncwarp();
  if (lane < 16) {
#pragma unroll
    for (int r = 0; r < 16; ++r) T[(bs + r) * LD + bs + cc] = col[r];
  }
}

}  // namespace jb
