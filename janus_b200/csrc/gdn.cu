// Gated DeltaNet: the prologue (conv + silu + l2 + gates) and the recurrent rule with the in-place state fork.
//
// Prologue: a CTA covers 32 consecutive tokens x 2048 channels; each thread owns 8 channels and slides the causal
// conv window over the tokens (registers), restarting it at a row boundary from the row's earlier tokens or the
// parent row's conv tail, so the projection output is read once. q and k are l2-normalised per head with a shuffle
// reduction over the lanes that hold the head. Every output is rounded to bf16 once: the conv activation stays fp32
// through the l2 norm (the reference's fp32 arithmetic, janus/hybrid.py:220-238, 276-301; its bf16 serving glue
// rounds the activation before the norm as well, one rounding more than here).
//
// Fork recurrent: grid (parent row, value head). A parent's fp32 state [Dk, Dv] is read in place by every child row
// (no per-row copy); each thread holds Dk*Dv/256 state entries (one value column, a slice of the key rows), so the
// two reductions over the key dimension per token are a register loop plus one shared-memory exchange.
#include "common.cuh"

namespace jb {

constexpr int kProThreads = 256;
constexpr int kMaxTaps = 8;
constexpr int kProTokens = 96;  // tokens per CTA: each thread slides its conv window over them
constexpr int kProBatch = 2;    // tokens per step (the l2 norms of a step share their shuffle rounds)
constexpr int kProRing = 8;     // tokens staged ahead per thread in the shared-memory ring (power of two)

__device__ __forceinline__ void cp_async(void* dst, const void* src, int bytes) {
  if (bytes == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src));
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src));
}

// grid (token tiles of kProTokens, channel blocks of 8 * kProThreads). Thread = 8 consecutive channels; it keeps the
// last K-1 conv inputs of its channels in registers while it walks the tile's tokens, so every projection element is
// read once (plus K-1 halo rows at a tile or row start, from the previous tokens or the parent's conv tail).
template <int K>
__global__ void __launch_bounds__(kProThreads, 2) gdn_prologue_kernel(
    const __nv_bfloat16* __restrict__ proj, int64_t proj_stride, int64_t T, const int32_t* __restrict__ row_start,
    const int32_t* __restrict__ row_of_token, const int32_t* __restrict__ parent,
    const __nv_bfloat16* __restrict__ tail_in, __nv_bfloat16* __restrict__ tail_out,
    const __nv_bfloat16* __restrict__ conv_w, const __nv_bfloat16* __restrict__ A_log,
    const __nv_bfloat16* __restrict__ dt_bias, int Hk, int Dk, int Hv, int Dv, __nv_bfloat16* __restrict__ q,
    __nv_bfloat16* __restrict__ k, __nv_bfloat16* __restrict__ v, float* __restrict__ g, float* __restrict__ beta) {
  __shared__ uint4 ring[kProRing][kProThreads];
  const int64_t t0 = (int64_t)blockIdx.x * kProTokens;
  const int64_t t1 = t0 + kProTokens < T ? t0 + kProTokens : T;
  const int key_dim = Hk * Dk;
  const int C = 2 * key_dim + Hv * Dv;
  const int vec = blockIdx.y * kProThreads + threadIdx.x;
  const bool live = vec * 8 < C;
  const int c0 = live ? vec * 8 : 0;
  const int lanes_per_head = Dk >> 3;
  // q and k channels get an l2 norm over their head (a shuffle reduction); v channels skip it. Uniform over a warp
  // whenever 2 * Hk * Dk is a multiple of 256 channels; otherwise the warp reduces for all its lanes.
  const bool warp_qk = __any_sync(0xffffffffu, live && c0 < 2 * key_dim);
  float wf[8][K];  // conv taps, fp32
#pragma unroll
  for (int u = 0; u < 8; ++u)
#pragma unroll
    for (int j = 0; j < K; ++j) wf[u][j] = live ? bf2f(conv_w[(int64_t)(c0 + u) * K + j]) : 0.f;
  float hist[K - 1][8];  // hist[j]: conv input at relative position j - (K-1) before the current token
  int cur_row = -1;
  int64_t r0 = 0, L = 0;
  const __nv_bfloat16* tail = nullptr;
  // the thread's 8 channels of the next kProRing tokens stream through its own column of a shared-memory ring
  // (cp.async: the loads in flight hold no registers); a slot is refilled only after the stores that depend on
  // the value read from it, so the refill cannot overtake that read
  // (threads past the last channel read channel 0 and store nothing: no per-token checks for them)
  uint4* my = &ring[0][threadIdx.x];
  const __nv_bfloat16* src = proj + t0 * proj_stride + c0;  // the next token to stage
  auto issue = [&](int64_t t) {  // one commit group per token; an empty group past the tile keeps the count
    if (t < t1) cp_async(my + ((int)(t - t0) & (kProRing - 1)) * kProThreads, src, 16);
    src += proj_stride;
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };
  // this thread's output: q, k (l2-normalised) or v channels, advanced by one row per token
  const bool is_qk = c0 < 2 * key_dim;
  const int64_t dst_stride = is_qk ? key_dim : (int64_t)Hv * Dv;
  __nv_bfloat16* dst = (c0 < key_dim ? q + c0 : is_qk ? k + (c0 - key_dim) : v + (c0 - 2 * key_dim)) + t0 * dst_stride;
#pragma unroll
  for (int i = 0; i < kProRing; ++i) issue(t0 + i);
  int rows_n[kProBatch];
#pragma unroll
  for (int b = 0; b < kProBatch; ++b) rows_n[b] = row_of_token[t0 + b < t1 ? t0 + b : t1 - 1];
  // K = 4: the window rotates through its 3 registers instead of sliding (the slot of the oldest input takes the
  // newest), so a pass of 3 batches (6 tokens, a multiple of both) fixes every register index at compile time and
  // the per-token moves of the slide are gone; other K slide
  constexpr int W = K - 1;
  constexpr int kRot = (K == 4) ? 3 : 1;  // batches per pass
  static_assert(kRot == 1 || (kProTokens % (kRot * kProBatch) == 0 && (kRot * kProBatch) % W == 0), "rotation");
  for (int64_t tp = t0; tp < t1; tp += kRot * kProBatch) {
#pragma unroll
  for (int bb = 0; bb < kRot; ++bb) {
    const int64_t tb = tp + bb * kProBatch;
    if (tb >= t1) break;
    int rows[kProBatch];
#pragma unroll
    for (int b = 0; b < kProBatch; ++b) rows[b] = rows_n[b];
    if (tb + kProBatch < t1) {
#pragma unroll
      for (int b = 0; b < kProBatch; ++b)
        rows_n[b] = row_of_token[tb + kProBatch + b < t1 ? tb + kProBatch + b : t1 - 1];
    }
    // kProRing groups are outstanding (tokens tb .. tb + kProRing - 1): the oldest kProBatch are complete after
    asm volatile("cp.async.wait_group %0;\n" ::"n"(kProRing - kProBatch) : "memory");
    bf16x8 xr[kProBatch];
#pragma unroll
    for (int b = 0; b < kProBatch; ++b)
      xr[b] = *reinterpret_cast<const bf16x8*>(my + ((int)(tb + b - t0) & (kProRing - 1)) * kProThreads);
    float act[kProBatch][8];  // conv + silu in fp32 (q/k normalised before their one rounding, v rounded once)
#pragma unroll
    for (int b = 0; b < kProBatch; ++b) {
      const int64_t t = tb + b;
      if (t >= t1) {
#pragma unroll
        for (int u = 0; u < 8; ++u) act[b][u] = 0.f;
        continue;
      }
      const int row = rows[b];
      if (row != cur_row) {  // (re)fill the window from the row's earlier tokens or the parent's conv tail
        cur_row = row;
        r0 = row_start[row];
        L = row_start[row + 1] - r0;
        tail = (tail_in && parent) ? tail_in + (int64_t)parent[row] * (K - 1) * C : nullptr;
        const int64_t i = t - r0;
#pragma unroll
        for (int j = 0; j < K - 1; ++j) {
          const int64_t e = i + j;  // ext index of relative position j - (K-1)
          float* hj = hist[kRot > 1 ? (bb * kProBatch + b + j) % W : j];
          if (e >= K - 1) {
            load8(proj + (r0 + e - (K - 1)) * proj_stride + c0, hj);
          } else if (tail) {
            load8(tail + e * C + c0, hj);
          } else {
#pragma unroll
            for (int u = 0; u < 8; ++u) hj[u] = 0.f;
          }
        }
      }
      float x[8];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float2 f = __bfloat1622float2(xr[b].h[u]);
        x[2 * u] = f.x;
        x[2 * u + 1] = f.y;
      }
      float a[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        a[u] = x[u] * wf[u][K - 1];
#pragma unroll
        for (int j = 0; j < K - 1; ++j) a[u] += hist[kRot > 1 ? (bb * kProBatch + b + j) % W : j][u] * wf[u][j];
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) act[b][u] = silu_fast(a[u]);
      if (kRot > 1) {  // the oldest input's slot takes the newest
#pragma unroll
        for (int u = 0; u < 8; ++u) hist[(bb * kProBatch + b) % W][u] = x[u];
      } else {  // slide the window
#pragma unroll
        for (int j = 0; j < K - 2; ++j)
#pragma unroll
          for (int u = 0; u < 8; ++u) hist[j][u] = hist[j + 1][u];
#pragma unroll
        for (int u = 0; u < 8; ++u) hist[K - 2][u] = x[u];
      }
      if (live && tail_out && t == r0 + L - 1) {  // the row's last K-1 conv inputs are the window now
#pragma unroll
        for (int j = 0; j < K - 1; ++j)
          store8(tail_out + ((int64_t)row * (K - 1) + j) * C + c0,
                 hist[kRot > 1 ? (bb * kProBatch + b + 1 + j) % W : j]);
      }
    }
    float rn[kProBatch];  // 1 / l2 norm of the token's head (q, k channels)
    if (warp_qk) {
#pragma unroll
      for (int b = 0; b < kProBatch; ++b) {
        rn[b] = 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u) rn[b] += act[b][u] * act[b][u];
      }
      for (int o = lanes_per_head >> 1; o > 0; o >>= 1)
#pragma unroll
        for (int b = 0; b < kProBatch; ++b) rn[b] += __shfl_xor_sync(0xffffffffu, rn[b], o);
#pragma unroll
      for (int b = 0; b < kProBatch; ++b) rn[b] = rsqrtf(rn[b] + 1e-6f);
    }
    if (live) {
#pragma unroll
      for (int b = 0; b < kProBatch; ++b) {
        if (tb + b >= t1) break;
        if (is_qk) {
          float o8[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) o8[u] = act[b][u] * rn[b];
          store8(dst + b * dst_stride, o8);
        } else {
          store8(dst + b * dst_stride, act[b]);
        }
      }
    }
    dst += kProBatch * dst_stride;
    asm volatile("" ::: "memory");  // the slots' reads and the stores above stay before their refill
#pragma unroll
    for (int b = 0; b < kProBatch; ++b) issue(tb + kProRing + b);  // into the slots just read
  }
  }
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");  // no copy outlives the CTA
  // gates, by the first channel block: b at column C + Hv*Dv + h, a at C + Hv*Dv + Hv + h
  if (blockIdx.y == 0) {
    for (int x = threadIdx.x; x < (int)(t1 - t0) * Hv; x += blockDim.x) {
      const int64_t t = t0 + x / Hv;
      const int h = x % Hv;
      const float b = bf2f(proj[t * proj_stride + C + Hv * Dv + h]);
      const float a = bf2f(proj[t * proj_stride + C + Hv * Dv + Hv + h]);
      beta[t * Hv + h] = sigmoidf_(b);
      g[t * Hv + h] = -expf(bf2f(A_log[h])) * softplus(a + bf2f(dt_bias[h]));
    }
  }
}

// ------------------------------------------------------------------------------------------- fork recurrent rule

// One CTA per (parent row, value head), kForkSplit threads per value column j (consecutive lanes of a warp, each
// with a slice of the key rows): they keep column j of the state in registers, so the recurrence needs a few
// shuffles per reduction and no barrier: per token kv_j = sum_k S[k][j] k[k] (after the decay), delta_j =
// (v_j - kv_j) beta, S[:, j] += k delta_j, o_j = scale sum_k S[k][j] q[k]. The parent's state is read from global
// memory once into shared memory and every child starts from that copy. The tokens' k, q, v (bf16), g and beta
// stream through a ring of kForkRing shared buffers with cp.async, kForkRing - 1 tokens ahead, so no thread waits
// for a load of the token it computes; one barrier per token.
constexpr int kForkSplit = 4;  // threads per value column
constexpr int kForkRing = 8;   // token buffers


template <int DK, int DV>
__global__ void __launch_bounds__(kForkSplit * DV) gdn_fork_recurrent_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    const float* __restrict__ g, const float* __restrict__ beta, const int32_t* __restrict__ row_start,
    const int32_t* __restrict__ child_start, const float* __restrict__ state_in, float* __restrict__ state_out,
    int Hk, int Hv, float scale, __nv_bfloat16* __restrict__ o) {
  constexpr int NT = kForkSplit * DV, ROWS = DK / kForkSplit;
  constexpr int CK = DK / 8, CV = DV / 8;  // 16-byte chunks of a k (q) row and of a v row
  static_assert(2 * CK + CV + 2 <= NT && ROWS % 4 == 0, "staging threads and row split");
  extern __shared__ float s0[];  // [DK][DV]: the parent's state
  __shared__ __align__(16) __nv_bfloat16 s_k[kForkRing][DK], s_q[kForkRing][DK], s_v[kForkRing][DV];
  __shared__ float s_g[kForkRing], s_b[kForkRing];
  const int p = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int j = tid / kForkSplit, r0 = (tid % kForkSplit) * ROWS;  // value column, first key row of this thread
  const int hk = h / (Hv / Hk);
  const int c0 = child_start[p], c1 = child_start[p + 1];
  if (c0 >= c1) return;
  if (state_in) {
    const float* src = state_in + ((int64_t)p * Hv + h) * DK * DV;
#pragma unroll 8
    for (int r = r0; r < r0 + ROWS; ++r) s0[r * DV + j] = src[(int64_t)r * DV + j];  // this thread's own entries
  }
  const int64_t tbeg = row_start[c0], tend = row_start[c1];
  auto stage = [&](int64_t t, int buf) {  // one commit group per call on every thread (empty ones included)
    if (t < tend) {
      if (tid < CK) {
        cp_async(&s_k[buf][tid * 8], k + (t * Hk + hk) * DK + tid * 8, 16);
      } else if (tid < 2 * CK) {
        cp_async(&s_q[buf][(tid - CK) * 8], q + (t * Hk + hk) * DK + (tid - CK) * 8, 16);
      } else if (tid < 2 * CK + CV) {
        cp_async(&s_v[buf][(tid - 2 * CK) * 8], v + (t * Hv + h) * DV + (tid - 2 * CK) * 8, 16);
      } else if (tid == 2 * CK + CV) {
        cp_async(&s_g[buf], g + t * Hv + h, 4);
      } else if (tid == 2 * CK + CV + 1) {
        cp_async(&s_b[buf], beta + t * Hv + h, 4);
      }
    }
    asm volatile("cp.async.commit_group;\n" ::);
  };
  for (int d = 0; d < kForkRing - 1; ++d) stage(tbeg + d, d);
  int64_t step = 0;  // tokens processed by this CTA: the buffer of token t is step % kForkRing
  for (int c = c0; c < c1; ++c) {
    float S[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) S[r] = state_in ? s0[(r0 + r) * DV + j] : 0.f;
    for (int64_t t = row_start[c]; t < row_start[c + 1]; ++t, ++step) {
      const int buf = (int)(step % kForkRing);
      asm volatile("cp.async.wait_group %0;\n" ::"n"(kForkRing - 2) : "memory");  // this token's copies landed
      __syncthreads();  // ... for every thread's copies; every reader of the buffer staged next is done
      stage(t + kForkRing - 1, (int)((step + kForkRing - 1) % kForkRing));
      const float decay = expf(s_g[buf]);
      const __nv_bfloat162* kb = reinterpret_cast<const __nv_bfloat162*>(&s_k[buf][r0]);
      const __nv_bfloat162* qb = reinterpret_cast<const __nv_bfloat162*>(&s_q[buf][r0]);
      float k4[4] = {0.f, 0.f, 0.f, 0.f};  // four independent partial sums (short dependency chains)
#pragma unroll
      for (int r = 0; r < ROWS; r += 4) {
        const float2 ka = __bfloat1622float2(kb[r / 2]), kc = __bfloat1622float2(kb[r / 2 + 1]);
        S[r] *= decay;
        S[r + 1] *= decay;
        S[r + 2] *= decay;
        S[r + 3] *= decay;
        k4[0] += S[r] * ka.x;
        k4[1] += S[r + 1] * ka.y;
        k4[2] += S[r + 2] * kc.x;
        k4[3] += S[r + 3] * kc.y;
      }
      float kv = (k4[0] + k4[1]) + (k4[2] + k4[3]);
#pragma unroll
      for (int x = 1; x < kForkSplit; x <<= 1) kv += __shfl_xor_sync(0xffffffffu, kv, x);
      const float delta = (__bfloat162float(s_v[buf][j]) - kv) * s_b[buf];
      float o4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int r = 0; r < ROWS; r += 4) {
        const float2 ka = __bfloat1622float2(kb[r / 2]), kc = __bfloat1622float2(kb[r / 2 + 1]);
        const float2 qa = __bfloat1622float2(qb[r / 2]), qc = __bfloat1622float2(qb[r / 2 + 1]);
        S[r] += ka.x * delta;
        S[r + 1] += ka.y * delta;
        S[r + 2] += kc.x * delta;
        S[r + 3] += kc.y * delta;
        o4[0] += S[r] * qa.x;
        o4[1] += S[r + 1] * qa.y;
        o4[2] += S[r + 2] * qc.x;
        o4[3] += S[r + 3] * qc.y;
      }
      float ov = (o4[0] + o4[1]) + (o4[2] + o4[3]);
#pragma unroll
      for (int x = 1; x < kForkSplit; x <<= 1) ov += __shfl_xor_sync(0xffffffffu, ov, x);
      if (tid % kForkSplit == 0) o[(t * Hv + h) * DV + j] = f2bf(ov * scale);
    }
    if (state_out) {
      float* dst = state_out + ((int64_t)c * Hv + h) * DK * DV;
#pragma unroll
      for (int r = 0; r < ROWS; ++r) dst[(int64_t)(r0 + r) * DV + j] = S[r];
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");  // no copy outlives the CTA
}

}  // namespace jb

using namespace jb;

extern "C" int janus_b200_gdn_prologue(const void* proj, int64_t proj_stride, int64_t T, int64_t B,
                                       const int32_t* row_start, const int32_t* row_of_token, const int32_t* parent,
                                       const void* tail_in, void* tail_out, const void* conv_w, const void* A_log,
                                       const void* dt_bias, int64_t Hk, int64_t Dk, int64_t Hv, int64_t Dv, int64_t K,
                                       void* q, void* k, void* v, float* g, float* beta, void* stream) {
  JB_REQUIRE(proj && row_start && row_of_token && conv_w && A_log && dt_bias && q && k && v && g && beta,
             JANUS_ERR_INVALID, "gdn_prologue: null pointer");
  JB_REQUIRE(T >= 0 && B >= 0 && Hk > 0 && Hv > 0 && Hv % Hk == 0 && K >= 2 && K <= kMaxTaps, JANUS_ERR_INVALID,
             "gdn_prologue: bad head counts or K");
  JB_REQUIRE(Dk == 32 || Dk == 64 || Dk == 128 || Dk == 256, JANUS_ERR_UNSUPPORTED, "gdn_prologue: Dk %lld",
             (long long)Dk);
  JB_REQUIRE(Dv % 8 == 0, JANUS_ERR_UNSUPPORTED, "gdn_prologue: Dv %lld", (long long)Dv);
  const int64_t C = 2 * Hk * Dk + Hv * Dv;
  JB_REQUIRE(proj_stride >= C + Hv * Dv + 2 * Hv && proj_stride % 8 == 0, JANUS_ERR_INVALID,
             "gdn_prologue: proj stride %lld < %lld", (long long)proj_stride, (long long)(C + Hv * Dv + 2 * Hv));
  JB_REQUIRE(JB_ALIGNED(proj, 16) && JB_ALIGNED(q, 16) && JB_ALIGNED(k, 16) && JB_ALIGNED(v, 16) &&
                 (!tail_in || JB_ALIGNED(tail_in, 16)) && (!tail_out || JB_ALIGNED(tail_out, 16)),
             JANUS_ERR_ALIGNMENT, "gdn_prologue: 16-byte alignment");
  JB_REQUIRE(!tail_in || parent, JANUS_ERR_INVALID, "gdn_prologue: tail_in needs parent");
  if (T == 0) return JANUS_OK;
  dim3 grid((unsigned)((T + kProTokens - 1) / kProTokens), (unsigned)((C / 8 + kProThreads - 1) / kProThreads));
  cudaStream_t s = (cudaStream_t)stream;
#define JB_PRO(K_)                                                                                                  \
  gdn_prologue_kernel<K_><<<grid, kProThreads, 0, s>>>(                                                             \
      (const __nv_bfloat16*)proj, proj_stride, T, row_start, row_of_token, parent, (const __nv_bfloat16*)tail_in,   \
      (__nv_bfloat16*)tail_out, (const __nv_bfloat16*)conv_w, (const __nv_bfloat16*)A_log,                          \
      (const __nv_bfloat16*)dt_bias, (int)Hk, (int)Dk, (int)Hv, (int)Dv, (__nv_bfloat16*)q, (__nv_bfloat16*)k,      \
      (__nv_bfloat16*)v, g, beta)
  switch (K) {
    case 2: JB_PRO(2); break;
    case 3: JB_PRO(3); break;
    case 4: JB_PRO(4); break;
    case 5: JB_PRO(5); break;
    default:
      set_error("gdn_prologue: conv kernel size %lld not compiled (2..5)", (long long)K);
      return JANUS_ERR_UNSUPPORTED;
  }
#undef JB_PRO
  return launch_status("gdn_prologue");
}

extern "C" int janus_b200_gdn_fork_recurrent(const void* q, const void* k, const void* v, const float* g,
                                             const float* beta, int64_t T, int64_t B, const int32_t* row_start,
                                             const int32_t* child_start, int64_t P, const float* state_in,
                                             float* state_out, int64_t Hk, int64_t Hv, int64_t Dk, int64_t Dv,
                                             float scale, void* o, void* stream) {
  JB_REQUIRE(q && k && v && g && beta && row_start && child_start && o, JANUS_ERR_INVALID,
             "gdn_fork_recurrent: null pointer");
  JB_REQUIRE(T >= 0 && B >= 0 && P >= 0 && Hk > 0 && Hv > 0 && Hv % Hk == 0, JANUS_ERR_INVALID,
             "gdn_fork_recurrent: sizes");
  JB_REQUIRE(JB_ALIGNED(q, 16) && JB_ALIGNED(k, 16) && JB_ALIGNED(v, 16) && JB_ALIGNED(g, 4) && JB_ALIGNED(beta, 4),
             JANUS_ERR_ALIGNMENT, "gdn_fork_recurrent: q, k, v must be 16-byte aligned");
  if (P == 0 || T == 0) return JANUS_OK;
  JB_REQUIRE(P <= 0x7fffffff && Hv <= 65535, JANUS_ERR_INVALID, "gdn_fork_recurrent: grid too large");
  dim3 grid((unsigned)P, (unsigned)Hv);
  cudaStream_t s = (cudaStream_t)stream;
#define JB_FORK(DK_, DV_)                                                                                     \
  do {                                                                                                        \
    const int smem = (DK_) * (DV_) * (int)sizeof(float);                                                      \
    cudaError_t e = cudaFuncSetAttribute(gdn_fork_recurrent_kernel<DK_, DV_>,                                 \
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);                  \
    if (e != cudaSuccess) {                                                                                   \
      set_error("gdn_fork_recurrent: smem attribute %s", cudaGetErrorString(e));                              \
      return JANUS_ERR_CUDA;                                                                                  \
    }                                                                                                         \
    gdn_fork_recurrent_kernel<DK_, DV_><<<grid, kForkSplit * (DV_), smem, s>>>(                                              \
        (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, g, beta, row_start,       \
        child_start, state_in, state_out, (int)Hk, (int)Hv, scale, (__nv_bfloat16*)o);                        \
  } while (0)
  if (Dk == 128 && Dv == 128) {
    JB_FORK(128, 128);
  } else if (Dk == 64 && Dv == 64) {
    JB_FORK(64, 64);
  } else if (Dk == 32 && Dv == 32) {
    JB_FORK(32, 32);
  } else {
    set_error("gdn_fork_recurrent: (Dk, Dv) = (%lld, %lld) not compiled", (long long)Dk, (long long)Dv);
    return JANUS_ERR_UNSUPPORTED;
  }
#undef JB_FORK
  return launch_status("gdn_fork_recurrent");
}
