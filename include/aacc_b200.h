/*
 * aacc_b200.h — C ABI of the B200-native (sm_100a) Qwen3 per-step hot path.
 *
 * Every entry point takes raw device pointers, 64-bit sizes and a CUDA
 * stream; none allocates memory (KV pools, workspaces and outputs are owned
 * by the caller).  All tensors are contiguous row-major, bf16 unless stated.
 * Return value: AACC_OK (0) or an AACC_ERR_* code; aacc_last_error() then
 * describes the failure (thread-local).  Kernels never trap: an out-of-range
 * block id, cache slot, position or token id, or a device wait that ran out
 * of iterations, skips the access and ORs a code into the device error word
 * read by aacc_get_device_error().
 *
 * Each declaration cites the reference code it replaces
 * (yijichar/AWesome_ACceleration, path:line).
 *
 * Paged KV cache layout (per layer, K and V separately):
 *   cache[num_blocks][num_kv_heads][block_size][128]   (bf16)
 * A sequence owns a row of `block_tables` (int32 [rows][max_blocks]); token
 * `pos` lives at flat slot block_tables[row][pos / block_size] * block_size
 * + pos % block_size.  This replaces the reference's slot-contiguous cache
 * K[num_slots][max_seq_len][Hkv][D] with flat index slot*max_seq_len + pos
 * (model/model.py:324-336, llm.py:139-140).  block_size must be a multiple
 * of 64; head_dim is 128 (all Qwen3 models).
 */
#ifndef AACC_B200_H
#define AACC_B200_H

#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AACC_OK 0
#define AACC_ERR_INVALID 1     /* bad shape, alignment or argument */
#define AACC_ERR_CUDA 2        /* a CUDA runtime call or launch failed */
#define AACC_ERR_UNSUPPORTED 3 /* configuration outside the compiled kernels */

/* ---- library / error plumbing ------------------------------------------ */
int aacc_version(void);
const char* aacc_last_error(void);
/* Kernels this library has launched (or recorded into a graph capture) in
 * this process; used for launch accounting by the benchmark. */
unsigned long long aacc_launch_count(void);
/* Copy the device error word of the current device into *out (synchronous). */
int aacc_get_device_error(unsigned* out);
/* The same read queued on `stream` behind its work (out: pinned host memory,
 * valid once the stream reaches the copy), so an engine can check every step
 * without waiting for the step queued after it. */
int aacc_get_device_error_async(unsigned* out, cudaStream_t stream);
int aacc_clear_device_error(void);

/* ---- KV cache ------------------------------------------------------------ */

/* Scatter new K/V rows into the paged cache: row t of k/v (Hkv*128 values,
 * row strides in elements) goes to flat slot slot_mapping[t]; -1 skips.
 * Replaces the KV write inside flash_attn_with_kvcache (model/model.py:233-241)
 * and the prefill index_copy_ scatter (llm.py:171-175; llm_tp.py:454-468). */
int aacc_kv_store(const void* k, const void* v, int64_t num_tokens, int64_t k_row_stride,
                  int64_t v_row_stride, const int64_t* slot_mapping, void* k_cache, void* v_cache,
                  int64_t num_blocks, int num_kv_heads, int block_size, cudaStream_t stream);

/* Flat cache slot of the next token of each decode row:
 * out[b] = block_tables[row][n / bs] * bs + n % bs, n = seqlens[row],
 * row = slot_indices[b]; a negative row is padding and gets -1 (no store).
 * (The position the reference writes at, cache_seqlens[slot],
 * model/model.py:233-238.) */
int aacc_decode_slot_mapping(const int64_t* slot_indices, const int32_t* seqlens,
                             const int32_t* block_tables, int64_t max_blocks, int block_size,
                             int64_t num_blocks, int64_t* slot_mapping_out, int64_t batch,
                             cudaStream_t stream);

/* seqlens[slot_indices[b]] += 1 for b < batch
 * (model/model.py:241 `_cache_seqlens[slot_indices] += 1`); when positions
 * is not NULL also positions[b] += 1 (the scheduler's `pos += 1`,
 * llm.py:419), so a decode step can be replayed on device.  Padding rows
 * (negative slot index) are left alone. */
int aacc_advance_seqlens(const int64_t* slot_indices, int32_t* seqlens, int64_t* positions, int64_t batch,
                         cudaStream_t stream);

/* dst[i] = src[idx[i]] for i < n, rows of row_bytes bytes (multiple of 16):
 * the last-token gather of the packed prefill (llm.py:199-201
 * `hidden[cu_seqlens[1:] - 1]`). */
int aacc_gather_rows(const void* src, int64_t n_src, int64_t row_bytes, const int64_t* idx, int64_t n, void* dst,
                     cudaStream_t stream);

/* ---- attention ----------------------------------------------------------- */

/* Workspace bytes aacc_paged_decode_attention needs for `batch` rows with at
 * most `max_context` tokens each.  The workspace must be zero-filled before
 * its first use (it holds merge counters that every call leaves at zero). */
int64_t aacc_paged_decode_workspace_bytes(int64_t batch, int num_q_heads, int64_t max_context,
                                          int split_tokens);

/* Decode attention of one query token per row over its paged context of
 * seqlens[row] + ctx_add tokens (GQA, softmax scale `scale`, non-causal);
 * a padding row (negative slot index) reads nothing and outputs zeros.
 * q, out: [batch][num_q_heads][128].  split_tokens (multiple of 64, 0 =
 * default) is the context length one CTA streams; longer contexts are split
 * and merged.  Replaces flash_attn_with_kvcache (model/model.py:233-240,
 * model/model_tp.py:204-211). */
int aacc_paged_decode_attention(const void* q, void* out, const void* k_cache, const void* v_cache,
                                int64_t num_blocks, const int32_t* block_tables, int64_t max_blocks,
                                const int64_t* slot_indices, const int32_t* seqlens, int ctx_add,
                                int64_t batch, int num_q_heads, int num_kv_heads, int block_size,
                                float scale, int split_tokens, int64_t max_context, void* workspace,
                                int64_t workspace_bytes, cudaStream_t stream);

/* Allocation-free variant of aacc_paged_decode_attention (same arguments
 * minus the workspace), for callers that cannot allocate device memory, such
 * as plugins under a host runtime that owns all device allocations, or
 * services that keep a fixed device footprint after start-up.  Its scratch
 * (split partials + merge counters) is a static 16 MiB array inside this
 * library, held by every GPU that loads it; calls whose split plan needs more
 * (aacc_paged_decode_noalloc_capacity_bytes) fail with AACC_ERR_INVALID.
 * The first call on a device, with that device current, looks up the array's
 * address; make it before any stream capture.  All calls on a device share the
 * array (the counters are cleared on the caller's stream each call), so calls
 * that overlap on the GPU race.  No counterpart in the reference. */
int aacc_paged_decode_attention_noalloc(const void* q, void* out, const void* k_cache, const void* v_cache,
                                        int64_t num_blocks, const int32_t* block_tables, int64_t max_blocks,
                                        const int64_t* slot_indices, const int32_t* seqlens, int ctx_add,
                                        int64_t batch, int num_q_heads, int num_kv_heads, int block_size,
                                        float scale, int split_tokens, int64_t max_context, cudaStream_t stream);

/* Bytes of static scratch aacc_paged_decode_attention_noalloc can use. */
int64_t aacc_paged_decode_noalloc_capacity_bytes(void);

/* Causal (chunked) prefill attention over the paged cache.  Sequence s owns
 * query rows [cu_q[s], cu_q[s+1]) of q/out ([num_tokens][num_q_heads][128],
 * cu_q[num_seqs] <= num_tokens) at positions ctx_start[s] + i; its K/V
 * (earlier chunks and this chunk) are already in the cache under
 * block-table row seq_rows[s].  max_q_len bounds cu_q[s+1]-cu_q[s].
 * Replaces flash_attn_varlen_func (llm.py:178-184, llm_tp.py:471-477) and
 * flash_attn_func (model/model.py:253-254). */
int aacc_prefill_attention(const void* q, void* out, int64_t num_tokens, const void* k_cache,
                           const void* v_cache, int64_t num_blocks, const int32_t* block_tables,
                           int64_t max_blocks, const int64_t* seq_rows, const int32_t* cu_q,
                           const int32_t* ctx_start, int64_t num_seqs, int64_t max_q_len, int num_q_heads,
                           int num_kv_heads, int block_size, float scale, cudaStream_t stream);

/* The same computation on mma.sync m16n8k16 with one CTA per query head
 * (block_size % 64 == 0).  aacc_prefill_attention runs it for block sizes
 * that are not multiples of 128; kept for A/B timing against the tcgen05
 * kernel.  Replaces the same call (llm.py:178-184). */
int aacc_prefill_attention_mma(const void* q, void* out, const void* k_cache, const void* v_cache,
                               int64_t num_blocks, const int32_t* block_tables, int64_t max_blocks,
                               const int64_t* seq_rows, const int32_t* cu_q, const int32_t* ctx_start,
                               int64_t num_seqs, int64_t max_q_len, int num_q_heads, int num_kv_heads,
                               int block_size, float scale, cudaStream_t stream);

/* ---- RMSNorm ------------------------------------------------------------- */

/* y = w * bf16(x * rsqrt(mean(x^2) + eps)), rows of `hidden` (multiple of
 * 1024).  RMSNorm.forward, model/model.py:47-52. */
int aacc_rmsnorm(const void* x, const void* w, void* y, int64_t rows, int64_t hidden, float eps,
                 cudaStream_t stream);

/* residual = bf16(residual + delta); y = rmsnorm(residual).  The residual add
 * and the next pre-norm of TransformerBlock.forward (model/model.py:259-263,
 * :265 + next layer :213 / final norm :285). */
int aacc_add_rmsnorm(const void* delta, void* residual, const void* w, void* y, int64_t rows,
                     int64_t hidden, float eps, cudaStream_t stream);

/* delta = bf16(sum_s partial[s]) (split order), then as aacc_add_rmsnorm:
 * residual = bf16(residual + delta); y = rmsnorm(residual).  The split-K
 * o_proj / down_proj output feeding the residual add and the next norm
 * (model/model.py:258-263, :190 + :265). */
int aacc_splitk_add_rmsnorm(const float* partial, int splits, void* residual, const void* w, void* y,
                            int64_t rows, int64_t hidden, float eps, cudaStream_t stream);

/* out = bf16(sum_s partial[s]) for partial [splits][rows][cols] (TP: the
 * bf16 RowParallel output that the all-reduce then sums). */
int aacc_splitk_reduce(const float* partial, int splits, void* out, int64_t rows, int64_t cols,
                       cudaStream_t stream);

/* residual = table[ids]; y = rmsnorm(residual).  embed_tokens + first
 * input_layernorm (model/model.py:280, :213). */
int aacc_embed_rmsnorm(const int64_t* ids, const void* table, int64_t vocab, void* residual,
                       const void* w, void* y, int64_t rows, int64_t hidden, float eps,
                       cudaStream_t stream);

/* ---- GEMMs (tcgen05 / TMEM, TMA-fed) --------------------------------------
 * x: [M][K] activations, w: [N][K] weights (nn.Linear layout); K multiple
 * of 64; fp32 accumulation, bf16 outputs.
 *
 * All kernels of this library use programmatic dependent launch: a kernel
 * may start while the previous kernel on the stream drains, and waits for
 * it before touching its data.  The GEMMs start streaming `w` before that
 * wait, so `w` must be a weight, i.e. not written by the kernel launched
 * immediately before on the same stream.  AACC_PDL=0 disables the overlap. */

/* out[M][N] = x @ w^T.  nn.Linear / F.linear (o_proj model/model.py:258,
 * down_proj :190, RowParallelLinear parallel_layers.py:190). */
int aacc_gemm(const void* x, const void* w, void* out, int64_t M, int64_t N, int64_t K,
              cudaStream_t stream);

/* ---- decode projections: cluster split-K with the epilogue fused ----------
 * For decode-sized batches (1 <= M <= 256 rows; N % 128 == 0, K % 64 == 0).
 * The K dimension of every 128-column output tile is split over the `splits`
 * CTAs of one thread-block cluster; the fp32 partials are summed in split
 * order through distributed shared memory (bit-identical to aacc_gemm_splitk
 * + the split-K epilogue at the same split count) and the epilogue runs in
 * the same kernel.  splits = 0 picks the split count (and 128- or 256-row
 * tiles) so that all CTAs are resident at once.  One launch per projection,
 * no workspace. */

/* out[M][N] = bf16(x @ w^T): o_proj / down_proj of a decode step
 * (model/model.py:237-238, :189-190), before the residual add + RMSNorm. */
int aacc_gemm_cluster(const void* x, const void* w, void* out, int64_t M, int64_t N, int64_t K, int splits,
                      cudaStream_t stream);

/* out[M][I] = bf16(silu(bf16(gate))) * bf16(up) over gate/up rows
 * interleaved by 64 (model/model.py:189-190), as aacc_gemm_silu_mul. */
int aacc_gemm_silu_mul_cluster(const void* x, const void* w_gate_up, void* out, int64_t M, int64_t I, int64_t K,
                               int splits, cudaStream_t stream);

/* Fused QKV projection + q/k RMSNorm + RoPE + paged KV store of a decode
 * step, as aacc_qkv_norm_rope_store (model/model.py:219-226, :233-240). */
int aacc_qkv_norm_rope_store_cluster(const void* x, const void* w_qkv, const void* q_norm_w, const void* k_norm_w,
                                     float eps, const int64_t* positions, const void* rope_cos_sin, int64_t max_pos,
                                     const int64_t* slot_mapping, void* q_out, void* k_cache, void* v_cache,
                                     int64_t num_blocks, int num_q_heads, int num_kv_heads, int block_size, int64_t M,
                                     int64_t K, int splits, cudaStream_t stream);

/* The plan splits = 0 selects for an M x N x K cluster GEMM on the current
 * device: tile rows / 128 (1 or 2), tiles over M, and the split count. */
int aacc_gemm_cluster_plan(int64_t M, int64_t N, int64_t K, int* mt, int* m_tiles, int* splits);

/* CTAs of the cluster GEMM (tile rows / 128 = 1 or 2, clusters of `splits`)
 * that fit on the current device at once (0 when none). */
int64_t aacc_gemm_cluster_capacity(int tile_rows_128, int splits);

/* ---- decode projections of small batches: weights as the 128-row operand -
 * For 1 <= M <= 64 rows; N % 128 == 0, K % 64 == 0, `splits` divides K / 64.
 * Each CTA holds four 16 KB weight slabs plus the matching slabs of x, so
 * two or three CTAs share an SM and a projection streams its weights while
 * the kernel before it is still running.  The fp32 partials go to
 * partial[splits][M][N] (as aacc_gemm_splitk).  The _qkv / _silu forms also
 * finish each 128-row weight tile in the same launch: the tile's last CTA
 * sums the partials in split order and applies the epilogue of
 * aacc_splitk_qkv_norm_rope_store / aacc_splitk_silu_mul (same rounding).
 * `counters` is caller-owned, one int per 128-row tile, zero before the
 * first call; each launch leaves it zero again unless it reported an error
 * (then zero it before the next call).  Launches sharing `counters` must be
 * ordered on one stream. */

/* partial[s][M][N] = x[:, Ks] @ w[:, Ks]^T: o_proj / down_proj of a decode
 * step (model/model.py:237-238, :189-190), summed by aacc_splitk_add_rmsnorm
 * or the tensor-parallel exchange. */
int aacc_gemm_skinny_splitk(const void* x, const void* w, float* partial, int64_t M, int64_t N, int64_t K,
                            int splits, cudaStream_t stream);

/* QKV projection + q/k RMSNorm + RoPE + paged KV store of a decode step
 * (model/model.py:219-226, :233-240), as aacc_qkv_norm_rope_store. */
int aacc_skinny_qkv_norm_rope_store(const void* x, const void* w_qkv, float* partial, int splits, int* counters,
                                    const void* q_norm_w, const void* k_norm_w, float eps, const int64_t* positions,
                                    const void* rope_cos_sin, int64_t max_pos, const int64_t* slot_mapping,
                                    void* q_out, void* k_cache, void* v_cache, int64_t num_blocks, int num_q_heads,
                                    int num_kv_heads, int block_size, int64_t M, int64_t K, cudaStream_t stream);

/* out[M][I] = bf16(silu(bf16(gate))) * bf16(up) over gate/up rows
 * interleaved by 64 (model/model.py:189-190), as aacc_gemm_silu_mul. */
int aacc_skinny_silu_mul(const void* x, const void* w_gate_up, float* partial, int splits, int* counters, void* out,
                         int64_t M, int64_t I, int64_t K, cudaStream_t stream);

/* out[M][N] = bf16(x[M][K] @ w[N][K]^T + bias[N]): the bias added in fp32
 * before the rounding, as a fused-bias F.linear does.  Column-parallel and
 * QKV-parallel layers built with bias=True (model/parallel_layers.py:72-89,
 * :299-342: F.linear(x, weight, bias)). */
int aacc_gemm_bias(const void* x, const void* w, const void* bias, void* out, int64_t M, int64_t N, int64_t K,
                   cudaStream_t stream);

/* x[rows][cols] <- bf16(x + bias[cols]): the RowParallel bias, added after
 * the all-reduce on TP rank 0 only (model/parallel_layers.py:197-199). */
int aacc_bias_add(void* x, const void* bias, int64_t rows, int64_t cols, cudaStream_t stream);

/* Split-K GEMM: partial[s][M][N] (fp32) = x[:, Ks] @ w[:, Ks]^T for the s-th
 * of `splits` equal K ranges (splits must divide K/64).  Spreads a small
 * decode GEMM (N = hidden, e.g. o_proj / down_proj) over every SM; the
 * partials are summed in split order by aacc_splitk_add_rmsnorm or
 * aacc_splitk_reduce.  Same reference call sites as aacc_gemm. */
int aacc_gemm_splitk(const void* x, const void* w, float* partial, int64_t M, int64_t N, int64_t K, int splits,
                     cudaStream_t stream);

/* out[M][I] = bf16(silu(bf16(x@Wg^T))) * bf16(x@Wu^T), rounded per op as the
 * eager reference.  w_gate_up rows interleave gate/up in groups of 64:
 * rows [128j, 128j+64) = gate rows [64j, 64j+64), the next 64 = up rows.
 * MLP.forward, model/model.py:189-190 (MLPTP.forward model/model_tp.py:294-299). */
int aacc_gemm_silu_mul(const void* x, const void* w_gate_up, void* out, int64_t M, int64_t I,
                       int64_t K, cudaStream_t stream);

/* Fused QKV projection + per-head q/k RMSNorm + RoPE + KV-cache store.
 * w_qkv: [(Hq + 2*Hkv) * 128][K] rows [Q | K | V] (Attention.fuse_qkv,
 * model/model.py:132-154).  q_out: [M][Hq][128].  K/V rows go to
 * k_cache/v_cache at slot_mapping[m] (-1 skips).  rope_cos_sin:
 * [max_pos][128] bf16 = cos[64] | sin[64] of the reference's cached table.
 * Replaces model/model.py:219-226 (+ RotaryEmbedding :80-92) and the KV
 * writes of :233-250 / llm.py:153-175. */
int aacc_qkv_norm_rope_store(const void* x, const void* w_qkv, const void* q_norm_w,
                             const void* k_norm_w, float eps, const int64_t* positions,
                             const void* rope_cos_sin, int64_t max_pos, const int64_t* slot_mapping,
                             void* q_out, void* k_cache, void* v_cache, int64_t num_blocks,
                             int num_q_heads, int num_kv_heads, int block_size, int64_t M,
                             int64_t K, cudaStream_t stream);

/* The QKV epilogue of aacc_qkv_norm_rope_store applied to split-K partials
 * partial [splits][M][(Hq+2Hkv)*128] (from aacc_gemm_splitk): sum in split
 * order, q/k RMSNorm, RoPE, Q to q_out, K/V into the paged cache.  Lets the
 * decode QKV projection use every SM.  Same reference lines as
 * aacc_qkv_norm_rope_store. */
int aacc_splitk_qkv_norm_rope_store(const float* partial, int splits, const void* q_norm_w,
                                    const void* k_norm_w, float eps, const int64_t* positions,
                                    const void* rope_cos_sin, int64_t max_pos, const int64_t* slot_mapping,
                                    void* q_out, void* k_cache, void* v_cache, int64_t num_blocks,
                                    int num_q_heads, int num_kv_heads, int block_size, int64_t M,
                                    cudaStream_t stream);

/* The SiLU-mul epilogue of aacc_gemm_silu_mul applied to split-K partials
 * partial [splits][M][2I] of the interleaved gate/up GEMM -> out [M][I]
 * (MLP.forward, model/model.py:189-190). */
int aacc_splitk_silu_mul(const float* partial, int splits, void* out, int64_t M, int64_t I,
                         cudaStream_t stream);

/* Workspace bytes for aacc_lm_head_argmax. */
int64_t aacc_lm_head_workspace_bytes(int64_t M, int64_t vocab);

/* Greedy next token: tokens[m] = argmax_n bf16(x[m] @ w[n]^T) (first index
 * on ties) without materialising logits.  Optionally also writes bf16
 * logits [M][vocab] (logits may be NULL).  vocab_offset is added to the
 * returned ids (vocab-parallel shards); best_val (may be NULL) receives the
 * winning logit as fp32.  Tied lm_head + greedy sampling
 * (model/model.py:316-318, llm.py:215-219). */
int aacc_lm_head_argmax(const void* x, const void* w, int64_t M, int64_t vocab, int64_t K,
                        int64_t vocab_offset, int64_t* tokens, float* best_val, void* logits,
                        void* workspace, int64_t workspace_bytes, cudaStream_t stream);

/* aacc_lm_head_argmax with temperature sampling: row m with
 * temperature[m] > 0 draws token ~ softmax(bf16(logits / T)) as
 * argmax_v bf16(logit_v / T) + Gumbel(seeds[m], counters[m], global id v)
 * (counter-based noise, the same on every TP rank; `counters` is the
 * position of the token whose logits are sampled); best_val then holds the
 * perturbed score, which the vocab-parallel merge compares.  Rows with
 * temperature <= 0, or all rows when temperature is NULL, stay greedy.
 * Replaces torch.multinomial(F.softmax(logits / temperature)) (llm.py:219,
 * llm_tp.py:609-616). */
int aacc_lm_head_sample(const void* x, const void* w, int64_t M, int64_t vocab, int64_t K, int64_t vocab_offset,
                        const float* temperature, const int64_t* seeds, const int64_t* counters, int64_t* tokens,
                        float* best_val, void* logits, void* workspace, int64_t workspace_bytes, cudaStream_t stream);

/* Temperature sampling from materialised bf16 logits [M][vocab]: the draw of
 * aacc_lm_head_sample (same noise for the same seed, counter and column) for
 * rows with temperature > 0, argmax otherwise (llm.py:215-219). */
int aacc_sample_rows(const void* logits, int64_t M, int64_t vocab, const float* temperature, const int64_t* seeds,
                     const int64_t* counters, int64_t* tokens, cudaStream_t stream);

/* Greedy sample from materialised bf16 logits [M][vocab] (llm.py:218). */
int aacc_argmax_rows(const void* logits, int64_t M, int64_t vocab, int64_t* tokens,
                     cudaStream_t stream);

/* Vocab-parallel argmax merge: candidates [shards][M] (value, global id),
 * as all-gathered from every rank's aacc_lm_head_argmax -> tokens[M];
 * highest value wins, lowest id on ties (the global argmax the reference's
 * rank-0 lm_head computes, model/model_tp.py:369-373 + llm_tp.py:612-614). */
int aacc_argmax_merge(const float* cand_val, const int64_t* cand_idx, int64_t M, int shards,
                      int64_t* tokens, cudaStream_t stream);

/* The same merge over candidates laid out with a per-shard stride (in
 * elements): shard s's value of row m is cand_val[s * val_shard_stride + m],
 * its id cand_idx[s * idx_shard_stride + m].  Lets a TP group all-gather each
 * rank's (ids, values) as ONE packed buffer and merge in place (the
 * reference gathers full logits to rank 0 instead, model/model_tp.py:369-381). */
int aacc_argmax_merge_strided(const float* cand_val, const int64_t* cand_idx, int64_t M, int shards,
                              int64_t val_shard_stride, int64_t idx_shard_stride, int64_t* tokens,
                              cudaStream_t stream);

/* ---- tensor-parallel exchange over NVLink peer memory -------------------- */

/* Bytes of the exchange buffer each rank of a TP group allocates for
 * aacc_tp_allreduce_add_rmsnorm (flags + double-buffered receive areas). */
int64_t aacc_tp_exchange_bytes(int world, int64_t max_rows, int64_t hidden);

/* Set-up only (the one place this library allocates device memory): a
 * zero-filled cudaMalloc of `bytes` on the current device and its CUDA IPC
 * handle (64 bytes written to ipc_handle).  A dedicated allocation, so that
 * the handle maps exactly this buffer in the peers.  Replaces the NCCL
 * communicator set-up of the reference's TP groups (model/distributed.py:39-95)
 * for this one collective. */
int aacc_peer_buffer_alloc(int64_t bytes, void** ptr, void* ipc_handle);
/* Map a peer's buffer (its ipc_handle) into this process (P2P over NVLink). */
int aacc_peer_buffer_open(const void* ipc_handle, void** ptr);
int aacc_peer_buffer_close(void* peer_ptr);
int aacc_peer_buffer_free(void* ptr);

/* Limit, in ms (default 20000), after which a wait for a peer in
 * aacc_tp_allreduce_add_rmsnorm gives up (applies to later launches and
 * graph captures).  No counterpart in the reference (NCCL waits for its
 * watchdog). */
int aacc_tp_set_peer_wait_ms(int64_t ms);

/* RowParallel all-reduce fused with the residual add and the next RMSNorm,
 * over the group's exchange buffers (buffers[p] = rank p's buffer as mapped in
 * this process, buffers[rank] = this rank's own):
 *   delta_r  = bf16(sum_s partial[s])        (splits >= 1, fp32 [splits][M][hidden])
 *            | src                            (splits == 0, bf16 [M][hidden])
 *   delta    = bf16(sum over ranks of delta_r, fp32 in rank order)
 *   residual = bf16(residual + delta); y = RMSNorm(residual) * w
 * Every rank of the group must make the same sequence of calls with the same
 * M (<= max_rows), world and two_shot, in stream order.  one-shot
 * (two_shot = 0) pushes the whole output to every rank; two-shot
 * reduce-scatters by columns and all-gathers the reduced slices.  A peer that
 * does not arrive within 20 s sets the device error word (bit 64), poisons
 * this rank's exchange buffer (every later call skips its waits) and the
 * output is invalid; the caller reads the error word and gives up on the
 * group.  Replaces RowParallelLinear's dist.all_reduce
 * (parallel_layers.py:190-195) plus the residual add and RMSNorm after it
 * (model/model.py:259-265; model/model_tp.py:311-322). */
int aacc_tp_allreduce_add_rmsnorm(const void* src, int splits, void* const* buffers, int world, int rank,
                                  int two_shot, int64_t max_rows, void* residual, const void* w, void* y, int64_t M,
                                  int64_t hidden, float eps, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* AACC_B200_H */
