/*
 * janus_b200 — C ABI of the B200 (sm_100a) kernels of the Janus decision readout.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t passed as `void*`, launches asynchronously
 * on that stream and returns 0 on success or a negative JANUS_* status (the text of the last error of the calling
 * thread is available from janus_b200_last_error). No entry point allocates, frees, synchronises or keeps a pointer
 * past the call; the caller owns every buffer, including workspaces. Kernels never trap: bad arguments are rejected
 * on the host before any launch.
 *
 * Layouts: a "level" is a batch of rows (tree segments) packed back to back without padding: T tokens, B rows,
 * row_start[B+1] the first token of each row (row_start[B] == T), row_of_token[T] the row of each token. Rows are
 * ordered so that the children of one parent row are consecutive (tree order). bf16 is __nv_bfloat16.
 *
 * Each entry point names the reference interface it replaces (IcarusAICo/janus paths; transformers 5.5.0 for the
 * modules the reference reuses).
 */
#ifndef JANUS_B200_H
#define JANUS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define JANUS_OK 0
#define JANUS_ERR_INVALID (-1)     /* null pointer, size or shape out of range */
#define JANUS_ERR_ALIGNMENT (-2)   /* a pointer or stride breaks the kernel's vector alignment */
#define JANUS_ERR_UNSUPPORTED (-3) /* a head dimension / configuration no kernel is compiled for */
#define JANUS_ERR_WORKSPACE (-4)   /* workspace too small */
#define JANUS_ERR_CUDA (-5)        /* a CUDA launch or runtime error */
#define JANUS_ERR_TIMEOUT (-6)     /* a bounded device-side wait ran out */

/* Library version (major * 10000 + minor * 100 + patch). */
int janus_b200_version(void);

/* Copies the calling thread's last error text into buf (always NUL-terminated); returns its full length. */
int janus_b200_last_error(char* buf, size_t len);

/* Token embedding gather and the first Qwen3_5RMSNorm of the decoder:
 * x[t] = table[ids[t]] (fp32 residual stream), y[t] = x[t] * rsqrt(mean(x^2) + eps) * (1 + norm_w) in bf16.
 * Replaces embed_tokens + layers[0].input_layernorm (janus/hybrid.py:1665-1676, 1081-1087). */
int janus_b200_embed_rmsnorm(const void* table, int64_t vocab, int64_t hidden, const int32_t* ids, int64_t T,
                             const void* norm_w, float eps, float* x, void* y, void* stream);

/* Residual add and the next RMSNorm in one pass: x += delta (bf16 [T, hidden] rows of stride delta_stride, or
 * NULL for no add), y = rmsnorm(x) * (1 + norm_w) in bf16. x is the fp32 residual stream.
 * Replaces `_add_norm` / `_add_rmsnorm` (janus/hybrid.py:257-273) and Qwen3_5RMSNorm. */
int janus_b200_add_rmsnorm(float* x, const void* delta, int64_t delta_stride, int64_t T, int64_t hidden,
                           const void* norm_w, float eps, void* y, void* stream);

/* SwiGLU gate: out[t, i] = silu(gu[t, i]) * gu[t, I + i] (gu bf16 [T, 2I], out bf16 [T, I]).
 * Replaces `_silu_mul` (janus/hybrid.py:263-264) on the merged gate/up projection (janus/hybrid.py:1108-1133). */
int janus_b200_silu_mul(const void* gu, int64_t T, int64_t inter, void* out, void* stream);

/* Gated RMSNorm over each value head: out = rmsnorm(core) * w * silu(z) (core bf16 [T, Hv, Dv]; z bf16 rows of
 * stride z_stride, head h at column h*Dv; out bf16 [T, Hv*Dv]; Dv in {32, 64, 128}; core, z, w, out 16-byte aligned
 * and z_stride a multiple of 8).
 * Replaces `_gate_norm` / Qwen3_5RMSNormGated (janus/hybrid.py:241-247). */
int janus_b200_gated_rmsnorm(const void* core, const void* z, int64_t z_stride, int64_t T, int64_t Hv, int64_t Dv,
                             const void* w, float eps, void* out, void* stream);

/* DeltaNet prologue of one level: causal depthwise conv (K taps) over [parent tail || projections] in fp32,
 * silu, l2-normalised q and k (eps 1e-6), v, beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias).
 * proj: bf16 rows of stride proj_stride with columns [q Hk*Dk | k Hk*Dk | v Hv*Dv | z Hv*Dv | b Hv | a Hv].
 * tail_in: bf16 [B_parent, K-1, C] conv inputs before each parent row's end, row parent[b] (NULL: zeros);
 * tail_out: bf16 [B, K-1, C] the last K-1 conv inputs of each row (NULL: not kept).
 * Outputs q, k bf16 [T, Hk, Dk], v bf16 [T, Hv, Dv], g, beta fp32 [T, Hv].
 * Replaces `_delta_serve` / `_delta_mix` (janus/hybrid.py:220-238, 276-301). */
int janus_b200_gdn_prologue(const void* proj, int64_t proj_stride, int64_t T, int64_t B, const int32_t* row_start,
                            const int32_t* row_of_token, const int32_t* parent, const void* tail_in, void* tail_out,
                            const void* conv_w, const void* A_log, const void* dt_bias, int64_t Hk, int64_t Dk,
                            int64_t Hv, int64_t Dv, int64_t K, void* q, void* k, void* v, float* g, float* beta,
                            void* stream);

/* Gated delta rule, token by token, with the per-branch state fork read in place: the rows of a level are grouped
 * under P parents (children of parent p are rows child_start[p] .. child_start[p+1]-1); every child starts from
 * its parent's fp32 state state_in[p] ([P, Hv, Dk, Dv], NULL: zeros) without copying it, and runs
 * S <- S*exp(g); S <- S + k (beta (v - S^T k))^T; o = scale * S^T q over its tokens (value head h reads qk head
 * h / (Hv/Hk)). state_out [B, Hv, Dk, Dv] receives each row's final state (NULL: not kept). o bf16 [T, Hv, Dv].
 * Replaces the `index_select` fork + fla fused_recurrent_gated_delta_rule (janus/hybrid.py:1082-1083,
 * 1064-1065; transformers torch_recurrent_gated_delta_rule). */
int janus_b200_gdn_fork_recurrent(const void* q, const void* k, const void* v, const float* g, const float* beta,
                                  int64_t T, int64_t B, const int32_t* row_start, const int32_t* child_start,
                                  int64_t P, const float* state_in, float* state_out, int64_t Hk, int64_t Hv,
                                  int64_t Dk, int64_t Dv, float scale, void* o, void* stream);

/* Gated delta rule in 64-token chunks for long rows (the state level), two launches: a fully parallel pass per
 * (chunk, value head) computes the intra-chunk WY form (K K^T, the triangular inverse, U = T V beta,
 * W = T K beta e^G, the decayed Q K^T) on the tensor cores into `workspace` (chunk-major); a second pass per
 * (row, value head) carries the fp32 state across the row's chunks in TMEM (tcgen05) and writes o bf16
 * [T, Hv, Dv]. chunk_start [B+1]: the first chunk of each row (prefix sum of ceil(rows' lengths / 64)),
 * n_chunks = chunk_start[B]. Row b starts from state_in[state_row[b]] ([*, Hv, Dk, Dv] fp32, read in place;
 * state_row NULL: row b; state_in NULL: zeros); state_out [B, Hv, Dk, Dv] (NULL: not kept). Dk = Dv = 128; q, k,
 * v, o 16-byte aligned. workspace: 256-byte aligned, at least janus_b200_gdn_chunk_scan_workspace(T, n_chunks, Hv)
 * bytes. status: optional device int32, zero on entry, set to 1 if a bounded device-side wait ran out (after 1 s;
 * the output is then invalid); NULL: not reported. Same results as janus_b200_gdn_fork_recurrent up to fp32/bf16
 * accumulation order.
 * segment: NULL, or int32 [T] ids of consecutive token segments (the state fork packed into chunks): tokens of
 * different segments do not interact and every segment of row b starts from state_in[state_row[b]] (the parent
 * state of sibling rows whose tokens were packed into one row of at most 64 tokens). Every row must then be a
 * single chunk and state_out NULL.
 * Replaces fla chunk_gated_delta_rule (janus/hybrid.py:100-125, 1064-1069; transformers
 * torch_chunk_gated_delta_rule). */
int janus_b200_gdn_chunk_scan(const void* q, const void* k, const void* v, const float* g, const float* beta,
                              int64_t T, int64_t B, const int32_t* row_start, const int32_t* chunk_start,
                              int64_t n_chunks, const float* state_in, const int32_t* state_row,
                              const int32_t* segment, float* state_out, int64_t Hk, int64_t Hv, int64_t Dk,
                              int64_t Dv, float scale, void* workspace, size_t workspace_bytes, void* o,
                              int32_t* status, void* stream);

/* Workspace bytes janus_b200_gdn_chunk_scan needs for T tokens, n_chunks chunks and Hv value heads. */
size_t janus_b200_gdn_chunk_scan_workspace(int64_t T, int64_t n_chunks, int64_t Hv);

/* The same chunked rule in one launch, for rows without segments: one CTA per (row, value head) computes chunk
 * c+1's WY products (the prep above) while the state pass runs chunk c, handing W, U, QK and G over in shared memory
 * (no workspace, nothing of the prep through HBM). Arguments as janus_b200_gdn_chunk_scan without segment and
 * workspace; outputs and states bit-identical to it.
 * Replaces fla chunk_gated_delta_rule (janus/hybrid.py:100-125, 1064-1069) on the state level's long rows. */
int janus_b200_gdn_chunk_scan_fused(const void* q, const void* k, const void* v, const float* g, const float* beta,
                                    int64_t T, int64_t B, const int32_t* row_start, const int32_t* chunk_start,
                                    int64_t n_chunks, const float* state_in, const int32_t* state_row,
                                    float* state_out, int64_t Hk, int64_t Hv, int64_t Dk, int64_t Dv, float scale,
                                    void* o, int32_t* status, void* stream);

/* Attention q/k preparation: per head RMSNorm (1 + w) of q and k, rotary on the first `rot` dims (cos/sin of
 * positions[t] * inv_freq[i], fp32), v copied. qkv: bf16 rows of stride qkv_stride with columns
 * [per q head: query D | gate D] (Hq*2D) | k Hkv*D | v Hkv*D]. Outputs q bf16 [T, Hq, D], k, v bf16 [T, Hkv, D].
 * Replaces `_attn_serve` / `_attn_qk` (janus/hybrid.py:304-329) and apply_rotary_pos_emb. */
int janus_b200_attn_qk_prep(const void* qkv, int64_t qkv_stride, int64_t T, const int32_t* positions,
                            const float* inv_freq, int64_t rot, const void* q_norm_w, const void* k_norm_w, float eps,
                            int64_t Hq, int64_t Hkv, int64_t D, void* q, void* k, void* v, void* stream);

/* Tree attention of one level with the output gate: every query token attends, in one online softmax, to the
 * tokens of its row's ancestor at each earlier level (key range [anc_lo[l][row], anc_hi[l][row]) of level l's
 * keys) and to its own row's tokens causally; out = softmax(q k^T * scale) v * sigmoid(gate). GQA folded: the
 * Hq/Hkv query heads of a kv head share every K/V tile. n_levels = ancestors + 1; k_levels[l], v_levels[l] are
 * contiguous [level_tokens[l], Hkv, D] (host array of n_levels counts); k_levels[n_levels-1] is the level's own keys
 * (level_tokens[n_levels-1] == T). tiles: [n_tiles, 2] query token ranges [start, end) of at most
 * janus_b200_tree_attention_tile_tokens(D, Hq, Hkv) tokens, each within one request (janus_b200 python builds them).
 * gate: bf16, token t head h at gate[t*gate_stride + h*gate_head_stride + d]. out bf16 [T, Hq*D]. D in
 * {32, 64, 128, 256}; 128 and 256 run on tcgen05 with TMEM accumulators (one CTA per query tile; with
 * JANUS_B200_ATTN=pairs in the environment, on CTA pairs sharing each K/V block, the slower form on B200), 32 and 64
 * on mma.sync. status: optional
 * device int32, zero on entry, set to 1 if a bounded device-side wait ran out (after 1 s; the output is then invalid;
 * the other CTAs see the word and give up at once); NULL: not reported.
 * Replaces branch_attention / state_attention / _piece / _merge_gate (janus/hybrid.py:806-855, 943-989) and the
 * tree rule of janus/attention.py:10-23. */
int janus_b200_tree_attention(const void* q, int64_t T, int64_t Hq, int64_t Hkv, int64_t D, int32_t n_levels,
                              const void* const* k_levels, const void* const* v_levels, const int64_t* level_tokens,
                              const int32_t* const* anc_lo, const int32_t* const* anc_hi, const int32_t* row_start,
                              const int32_t* row_of_token, const int32_t* tiles, int64_t n_tiles, const void* gate,
                              int64_t gate_stride, int64_t gate_head_stride, float scale, void* out, int32_t* status,
                              void* stream);

/* Self-test of the device-side failure detection (no counterpart in the reference): launches one thread that waits
 * on a barrier phase nothing completes, with the same bounded wait as janus_b200_tree_attention; after about 1 s the
 * wait gives up and sets *status (device int32, zero on entry) to 1. Nothing faults or traps, so the context stays
 * usable; tests use it to check that a wait that runs out is reported instead of hanging. */
int janus_b200_selftest_wait_timeout(int32_t* status, void* stream);

/* The largest number of query tokens per tile janus_b200_tree_attention accepts for this head dim and GQA layout
 * (128 rows of the tensor-core tile, or 64, divided by Hq/Hkv); 0 for an unsupported layout.
 * The tiling of the query axis that `_piece` bounds by PIECE_BYTES (janus/hybrid.py:407-420). */
int janus_b200_tree_attention_tile_tokens(int64_t D, int64_t Hq, int64_t Hkv);

/* ScalarHead readout fused with the final norm: for each of n rows r = rows[i] of the fp32 residual x [*, H]:
 * h = rmsnorm(x[r]) * (1 + final_w) (eps rms_eps), logits[i] = LayerNorm(h; ln_w, ln_b, ln_eps) . w_out + b_out[0].
 * final_w NULL: h = x[r] (rows that are already final-normed, ScalarHead.forward alone; same for the pointer heads).
 * Replaces lm.norm + ScalarHead.forward (janus/model.py:85-92, 342-350). */
int janus_b200_head_scalar(const float* x, int64_t H, const int32_t* rows, int64_t n, const void* final_w,
                           float rms_eps, const float* ln_w, const float* ln_b, float ln_eps, const float* w_out,
                           const float* b_out, float* logits, void* stream);

/* PointerHead readout fused with the final norm: option i (row option_rows[i], question option_question[i])
 * scores logits[i] = (LN(h_opt) Wk^T) . (LN(h_dec) Wq^T) / sqrt(R), h the final-normed rows, h_dec the row
 * decision_rows[option_question[i]]. wq, wk fp32 [R, H]. workspace: fp32, at least (n + Q) * R floats.
 * R <= 4096, n + Q <= 2^24, Q > 0 when n > 0. The caller guarantees 0 <= option_question[i] < Q; an option outside
 * that range reads nothing and gets a NaN logit.
 * Replaces lm.norm + PointerHead.forward (janus/model.py:71-82, 361-365). */
int janus_b200_head_pointer(const float* x, int64_t H, const int32_t* option_rows, const int32_t* option_question,
                            int64_t n, const int32_t* decision_rows, int64_t Q, const void* final_w, float rms_eps,
                            const float* ln_w, const float* ln_b, float ln_eps, const float* wq, const float* wk,
                            int64_t R, float* workspace, size_t workspace_bytes, float* logits, void* stream);

/* Dense bf16 GEMM on the tcgen05 tensor cores: out[M, n] = sum_k a[M, k] w[n, k] (y = x W^T, torch F.linear), fp32
 * accumulation, one rounding to bf16. a [M, K] (row stride lda), w [N, K] (row stride ldw), both bf16, 16-byte
 * aligned, strides multiples of 8 elements; N a multiple of 16, K of 8. epilogue 0: out [M, N] (row stride ldo);
 * epilogue 1 (SwiGLU): w's rows come in 256-row blocks of 128 gate rows then the 128 matching up rows (N a multiple
 * of 256), out [M, N/2] = silu(gate) * up of the fp32 accumulators. status: optional device int32 word set to 1 if a
 * bounded device-side wait ran out. Runs 512 x 256 tiles per CTA pair; the environment variable JANUS_B200_GEMM=pair
 * selects 256 x 256 tiles instead (bit-identical results).
 * Replaces the F.linear of the merged projections (`_merge_projections`, janus/hybrid.py:1108-1133) and, with
 * epilogue 1, the MLP's gate/up GEMM plus `_silu_mul` (janus/hybrid.py:263, 1093-1096). */
int janus_b200_gemm_bf16(const void* a, int64_t lda, const void* w, int64_t ldw, int64_t M, int64_t N, int64_t K,
                         int32_t epilogue, void* out, int64_t ldo, int32_t* status, void* stream);

/* MoE routing and tile plan, sync-free: softmax over fp32 router logits [S, E] (E <= 512), top-k (k <= 16),
 * renormalised weights (topk_idx int32 / topk_w fp32 [S, k]); assignments a = t*k + j sorted by expert into
 * sorted_ids [max_tiles * tile_rows] (-1 pads each expert to a multiple of tile_rows, which must be 128),
 * tile_expert [max_tiles], the tile count in n_tiles[0] on the device. max_tiles >= ceil((S*k + E*127) / 128).
 * workspace: int32, at least 3*E.
 * Replaces Qwen3_5MoeTopKRouter.forward (transformers qwen3_5_moe :754-770) and `align`
 * (janus/moe_w4a16.py:89-106). */
int janus_b200_moe_route(const float* logits, int64_t S, int64_t E, int64_t k, int64_t tile_rows, int32_t* topk_idx,
                         float* topk_w, int32_t* sorted_ids, int32_t* tile_expert, int64_t max_tiles,
                         int32_t* n_tiles, int32_t* workspace, size_t workspace_bytes, void* stream);

/* The router GEMM fused with the routing: logits = x w_router^T (x bf16 [S, H] with row stride x_stride, w_router
 * bf16 [E, H], E <= 256) on the tensor cores, kept in TMEM (never written), then the softmax / top-k / renormalised
 * weights of janus_b200_moe_route with the same arithmetic (k in {1, 2, 4, 6, 8}), and the same tile plan into
 * sorted_ids / tile_expert / n_tiles. w_gate: optional bf16 [1, H], the shared expert's gate row: gate_logit fp32 [S]
 * = x w_gate^T from the same pass. status: optional device int32 word, set to 1 if a bounded device-side wait ran
 * out. Same workspace and max_tiles rules as janus_b200_moe_route.
 * Replaces the router GEMM plus Qwen3_5MoeTopKRouter.forward (transformers qwen3_5_moe :754-770), the shared expert
 * gate's GEMV (:789-790) and `align` (janus/moe_w4a16.py:89-106). */
int janus_b200_moe_route_fused(const void* x, int64_t x_stride, int64_t S, int64_t H, const void* w_router, int64_t E,
                               const void* w_gate, int64_t k, int64_t tile_rows, int32_t* topk_idx, float* topk_w,
                               float* gate_logit, int32_t* sorted_ids, int32_t* tile_expert, int64_t max_tiles,
                               int32_t* n_tiles, int32_t* workspace, size_t workspace_bytes, int32_t* status,
                               void* stream);

/* W4A16 grouped GEMM over the expert-sorted 128-row tiles of janus_b200_moe_route / janus_b200_moe_plan, on the
 * tcgen05 tensor cores. Weights: codes uint8 [E, rows, K/2] (two int4 per byte, even element in the low nibble,
 * two's complement) and bf16 scales [E, rows, K/128]; the value fed to the tensor cores is code * scale rounded
 * once to bf16 (the fp32 product's rounding).
 * gated = 1 (gate_up, rows = 2N): x rows are tokens (assignment / topk), out[sorted row, n] =
 * silu(x W_gate^T) * (x W_up^T) in bf16, out rows = max_tiles*128 sorted rows.
 * gated = 0 (down, rows = N): x rows are the sorted rows of the first GEMM's output, out[assignment, n] =
 * topk_w[assignment] * x W^T in bf16. N % 128 == 0, K % 128 == 0; x, codes, out 16-byte aligned, ldx and ldo
 * multiples of 8. status: NULL or an int32 that is 0 on entry; a device-side wait that ran out sets it to 1 (the
 * affected tiles are not stored).
 * Replaces _w4a16_moe_kernel / fused_moe (janus/moe_w4a16.py:37-86, 122-140) for the int4-g128 format. */
int janus_b200_moe_grouped_w4a16(const void* x, int64_t ldx, const uint8_t* codes, const void* scales, int64_t E,
                                 int64_t N, int64_t K, int32_t gated, const int32_t* sorted_ids,
                                 const int32_t* tile_expert, const int32_t* n_tiles, int64_t max_tiles, int64_t topk,
                                 const float* topk_w, void* out, int64_t ldo, int32_t* status, void* stream);

/* MoE output: out[t] = sum_j y[t*k + j] (fp32 sum of the weighted expert rows) + sigmoid(shared_gate_logit[t]) *
 * shared[t] (shared NULL: none), bf16 [S, H].
 * Replaces the per-token sum and the gated shared expert of Qwen3_5MoeSparseMoeBlock.forward
 * (transformers qwen3_5_moe :778-791, janus/moe_w4a16.py:140). */
int janus_b200_moe_combine(const void* y, int64_t k, const void* shared, const float* shared_gate_logit, int64_t S,
                           int64_t H, void* out, void* stream);

/* Expert-parallel MoE (no counterpart in the reference, which runs on one device): the tile plan of
 * janus_b200_moe_route built from explicit slot -> expert ids instead of router logits. expert_ids int32 [n]
 * (slot a = row * k + j; an id < 0 or >= E means the slot has no expert here and is skipped); outputs as
 * janus_b200_moe_route (sorted_ids hold slot indices, -1 padding; the tile count stays on the device).
 * Used by the receiving rank of an expert-parallel dispatch, whose rows carry their local expert ids. */
int janus_b200_moe_plan(const int32_t* expert_ids, int64_t n, int64_t E, int64_t tile_rows, int32_t* sorted_ids,
                        int32_t* tile_expert, int64_t max_tiles, int32_t* n_tiles, int32_t* workspace,
                        size_t workspace_bytes, void* stream);

/* out[r] = sum over the slots j of row r with slot_expert[r*k + j] >= 0 (all slots when slot_expert is NULL) of
 * y[r*k + j], in fp32 and slot order (y bf16 [R*k, H], out fp32 [R, H]): the per-rank partial of the expert sum
 * that an expert-parallel combine sends back. No counterpart in the reference. */
int janus_b200_moe_reduce_slots(const void* y, int64_t k, const int32_t* slot_expert, int64_t R, int64_t H, float* out,
                                void* stream);

/* out[t] = sum over ranks w = 0..W-1 with row_index[t*W + w] >= 0 of partials[row_index[t*W + w]] (fp32, rank order)
 * + sigmoid(shared_gate_logit[t]) * shared[t], rounded once to bf16 [S, H]: the owner's side of the
 * expert-parallel combine (janus_b200_moe_combine with the k expert rows replaced by per-rank partial sums). */
int janus_b200_moe_combine_ep(const float* partials, const int32_t* row_index, int64_t W, const void* shared,
                              const float* shared_gate_logit, int64_t S, int64_t H, void* out, void* stream);

/* The grouped GEMMs of janus_b200_moe_grouped_w4a16 on the reference's own NVFP4 expert format: codes uint8
 * [E, rows, K/2] (two e2m1 codes per byte, even element in the low nibble), block_scales e4m3 bytes [E, rows, K/16]
 * (one per 16 inputs), global_scales fp32 [E, rows]; the value fed to the tensor cores is e2m1 * (scale * global)
 * formed in fp32 and rounded once to bf16, the reference's dequantised weight bit for bit. Everything else (plan,
 * gated / down semantics, layouts, status) as janus_b200_moe_grouped_w4a16.
 * Replaces `_w4a16_moe_kernel` / `fused_moe` (janus/moe_w4a16.py:37-140) with its NVFP4 codec
 * (janus/hybrid.py:400-425). */
int janus_b200_moe_grouped_nvfp4(const void* x, int64_t ldx, const uint8_t* codes, const uint8_t* block_scales,
                                 const float* global_scales, int64_t E, int64_t N, int64_t K, int32_t gated,
                                 const int32_t* sorted_ids, const int32_t* tile_expert, const int32_t* n_tiles,
                                 int64_t max_tiles, int64_t topk, const float* topk_w, void* out, int64_t ldo,
                                 int32_t* status, void* stream);

/* The PointerHead readout of janus_b200_head_pointer for callers that cannot allocate device memory: it takes no
 * workspace and allocates nothing; the projected rows go to a static 1 MiB device array inside this library
 * (kept by every GPU that loads the library until the process exits). Limit: (n + Q) * R <= 262144 floats (2048
 * rows at rank 128); larger calls return JANUS_ERR_WORKSPACE without launching. The first call on a device looks
 * up the array's device address (cudaGetSymbolAddress) with that device current; make that first call before any
 * stream capture. All calls on a device share the array, so calls that overlap on the GPU race: serialise them.
 * This entry point has no counterpart in the reference (its heads run in torch with the caching allocator). */
int janus_b200_head_pointer_noalloc(const float* x, int64_t H, const int32_t* option_rows,
                                    const int32_t* option_question, int64_t n, const int32_t* decision_rows, int64_t Q,
                                    const void* final_w, float rms_eps, const float* ln_w, const float* ln_b,
                                    float ln_eps, const float* wq, const float* wk, int64_t R, float* logits,
                                    void* stream);

#ifdef __cplusplus
}
#endif

#endif /* JANUS_B200_H */
