// The diagonal 16x16 blocks of T = (I - N)^-1 for the chunked gated delta rule (N strictly lower triangular, fp32 in
// shared memory with row stride LD), shared by the two-launch prep (gdn_chunk.cu) and the one-launch scan
// (gdn_scan_tc.cu) so that both round identically.
#pragma once

namespace jb {

// One warp inverts the block at rows / columns [bs, bs + 16): lane c < 16 owns column c of the block's T and solves
// (I - N) t = e_c by column-oriented forward substitution: once t[m] is final it is pushed into every later row,
// t[r] += N[r][m] t[m] for r > m. The 15 steps each issue independent FMAs, so the dependent chain is 15 FMAs long
// (a row-by-row dot product would chain all 120). Entries of t above the lane's column stay exactly zero and its
// diagonal entry exactly one. Lanes 16-31 compute a copy and store nothing.
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
  if (lane < 16) {
#pragma unroll
    for (int r = 0; r < 16; ++r) T[(bs + r) * LD + bs + cc] = col[r];
  }
}

}  // namespace jb
