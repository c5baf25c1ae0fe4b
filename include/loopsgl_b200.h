/*
 * loopsgl_b200.h -- C ABI of the B200 (sm_100a) looped-decoder hot path.
 *
 * Plain pointers, sizes and a CUDA stream (passed as void*); no framework
 * types. Every entry point returns LSB_OK (0) or an LSB_ERR_* code and, on
 * failure, leaves a message for lsb_last_error() on the calling thread.
 * Tensors are device pointers in the layouts stated per function; "bf16" is
 * IEEE bfloat16. Launches are asynchronous on `stream`, never synchronise the
 * host, and can be captured into CUDA graphs unless stated otherwise.
 *
 * Each declaration names the reference interface (Loop-SGLang,
 * python/loopsgl/...) whose work it replaces.
 */
#ifndef LOOPSGL_B200_H_
#define LOOPSGL_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LSB_OK 0
#define LSB_ERR_INVALID 1     /* an argument is out of range, misaligned or null */
#define LSB_ERR_CUDA 2        /* the CUDA runtime reported an error */
#define LSB_ERR_TIMEOUT 3     /* a bounded cross-GPU wait gave up */
#define LSB_ERR_UNSUPPORTED 4 /* shape or mode this build does not implement */

/* Message of the last failing call on this thread ("" if none). */
const char* lsb_last_error(void);
/* ABI version, bumped on any signature change. */
int lsb_abi_version(void);
/* Kernels this library has enqueued in this process so far, over every entry point and
 * thread (an entry point may enqueue one or several, e.g. paged attention's merge). */
int64_t lsb_kernel_launch_count(void);

/* Reads the sticky device error word that kernels set, instead of faulting,
 * when they meet an out-of-range index: LSB_DEVERR_* bits. reset != 0 clears it.
 * Synchronises `stream` (not capturable). */
#define LSB_DEVERR_POSITION 1 /* a RoPE position outside the cos/sin table */
#define LSB_DEVERR_SLOT 2     /* a KV slot outside the pool */
#define LSB_DEVERR_SEQLEN 4   /* a sequence longer than the max_seqlen bound */
#define LSB_DEVERR_TIMEOUT 8  /* a bounded in-kernel wait gave up */
#define LSB_DEVERR_COMM_TIMEOUT 16 /* a bounded wait for a peer GPU's data gave up */
int lsb_device_error_word(int32_t* out, int32_t reset, void* stream);

/* ---------------------------------------------------------------- norms --
 * Row-wise RMSNorm over `dim` bf16 elements: fp32 sum of squares, output
 * dtype(x * rsqrt(mean(x^2) + eps) * w). dim % 8 == 0, rows 16-byte aligned.
 */

/* out[r] = rmsnorm(x[r]) * w.  Replaces layers/norm.py:16-17 (RMSNorm.forward,
 * flashinfer.rmsnorm). */
int lsb_rmsnorm(void* out, int64_t out_stride, const void* x, int64_t x_stride,
                const void* weight, int64_t rows, int64_t dim, float eps, void* stream);

/* residual <- x + residual; x <- rmsnorm(residual) * w, with the norm taken on
 * the fp32 sum.  Replaces layers/norm.py:32-38 (RMSNormFused.forward with a
 * residual, flashinfer.fused_add_rmsnorm). In place on x and residual. */
int lsb_fused_add_rmsnorm(void* x, void* residual, const void* weight, int64_t rows, int64_t dim,
                          float eps, void* stream);

/* The sandwich step of the Ouro layer: y = rmsnorm(x) * w_a (rounded), then
 * residual <- y + residual and out = rmsnorm(residual) * w_b.  Replaces the
 * pair models/looped/ouro.py:49-50 (input_layernorm_2 then
 * post_attention_layernorm) and :52 + :45 (post_attention_layernorm_2 then the
 * next layer's input_layernorm). out may alias x. */
int lsb_sandwich_norm(void* out, const void* x, void* residual, const void* w_a,
                      const void* w_b, int64_t rows, int64_t dim, float eps, void* stream);

/* ------------------------------------------------------ RoPE + KV store --
 * qkv: [T, (hq + 2*hkv) * head_dim] bf16 rows of stride qkv_stride elements.
 * Applies neox RoPE in place to the q and k heads at positions[T] using the
 * fp32 table cos_sin[max_pos, head_dim] = cat(cos, sin), then stores the
 * rotated k heads and the v heads of row t into slot out_loc[t] of k_cache /
 * v_cache ([slots, hkv, head_dim] bf16, slot stride slot_stride elements),
 * skipping slot 0 (the padding slot). With hkv == 0 (and no caches) it only
 * rotates the hq heads of each row.  Replaces layers/attention.py:88-90
 * (rotary.py:40-55, flashinfer apply_rope_with_cos_sin_cache_inplace) and the
 * backend's store_kv (kvcache/mha_pool.py:54-66, kernel/store.py:89-152,
 * kernel/csrc/jit/store.cu:127-156). */
int lsb_rope_store_kv(void* qkv, int64_t qkv_stride, const int32_t* positions,
                      const float* cos_sin, int64_t max_pos, void* k_cache, void* v_cache,
                      int64_t slot_stride, int64_t num_slots, const int32_t* out_loc,
                      int64_t tokens, int32_t hq, int32_t hkv, int32_t head_dim, void* stream);

/* Scatter k[t] and v[t] (rows of row_elems bf16, row strides k_stride /
 * v_stride) into slot out_loc[t] of k_cache / v_cache, skipping slot 0.
 * Replaces kvcache/mha_pool.py:54-66 / last_exited.py:298-311 store_kv
 * (kernel/store.py:89-152, kernel/csrc/jit/store.cu:127-156). */
int lsb_store_kv(void* k_cache, void* v_cache, int64_t slot_stride, int64_t num_slots,
                 const void* k, int64_t k_stride, const void* v, int64_t v_stride,
                 const int32_t* out_loc, int64_t tokens, int64_t row_elems, void* stream);

/* ------------------------------------------------------ paged attention --
 * Causal attention of query rows over one paged KV layer.
 *   q:        [rows, hq, head_dim] bf16, row stride q_stride elements
 *   out:      [rows, hq, head_dim] bf16, row stride out_stride elements
 *   k_cache/v_cache: slots of hkv*head_dim bf16 (slot = page*page_size + offset),
 *             slot stride slot_stride elements
 *   page_table: [num_reqs, pt_stride] int32 page ids (page_size 1: slots)
 *   cache_seqlens: [num_reqs] keys of each request (its last query row sees all)
 *   cu_seqlens_q: [num_reqs + 1] query-row offsets per request
 * Row i of the n rows of a request attends to keys 0 .. seqlen - n + i; a
 * context longer than max_seqlen is cut at max_seqlen and flagged.
 * Up to 64 query heads (and a stage of 8-32 tokens of every KV head within
 * 64 KB) run on persistent CTAs, one per SM, that take (row, key split) items
 * from a queue and stream the keys into shared memory with bulk copies (a
 * second, small kernel chained by programmatic dependent launch then merges the
 * rows whose keys ended in several partials, so a call enqueues one or two
 * kernels, both capturable); larger head counts run one CTA per (row, 4 heads,
 * split). Either way the keys of long rows are split; the partial results and
 * the queue go to the caller's workspace (required:
 * lsb_paged_attention_workspace_size bytes, zeroed once before first use; its
 * head holds counters that every call leaves zeroed, so one workspace serves
 * calls of any shape). head_dim 32, 64, 96 or 128.
 * Slots outside [0, num_slots) are skipped and flagged in the device error
 * word instead of being read.  Replaces the backends'
 * attention call (attention/trtllm.py:80-91 decode, :62-78 prefill;
 * attention/fa.py:82-93; attention/fi.py:161-199). */
int64_t lsb_paged_attention_workspace_size(int64_t rows, int32_t hq, int32_t head_dim,
                                           int64_t max_seqlen);
int lsb_paged_attention(void* out, int64_t out_stride, const void* q, int64_t q_stride,
                        const void* k_cache, const void* v_cache, int64_t slot_stride,
                        int64_t num_slots, const int32_t* page_table, int64_t pt_stride,
                        const int32_t* cache_seqlens, const int32_t* cu_seqlens_q,
                        int64_t num_reqs, int64_t rows, int32_t hq, int32_t hkv,
                        int32_t head_dim, int32_t page_size, int64_t max_seqlen, float scale,
                        void* workspace, int64_t workspace_bytes, void* stream);

/* The launch plan lsb_paged_attention picks for a decode call (one query row per
 * request) of this shape on the current device (diagnostics, host only, nothing
 * launched): out[0] 1 for the streaming kernel, 0 for the per-CTA kernel; out[1]
 * keys per work item (split); out[2] splits of a max_seqlen row; streaming only
 * (else 0): out[3] pipeline stages, out[4] keys per stage, out[5] 1 when the
 * producer issues a stage's page runs one per lane. No counterpart in the reference. */
int lsb_paged_attention_plan(int64_t rows, int32_t hq, int32_t hkv, int32_t head_dim,
                             int32_t page_size, int64_t max_seqlen, int64_t slot_stride,
                             int32_t* out);

/* Kernel selection of later lsb_paged_attention calls of this process, for
 * benchmarks and tuning: 0 automatic (calls with several query rows per request
 * take the tensor-core kernel, decode calls the streaming or per-CTA kernel),
 * 1 the tensor-core kernel for every call, 2 never. No counterpart in the
 * reference. */
int lsb_attention_force_kernel(int32_t mode);

/* Decode attention (one query row per request) where groups of rows share
 * leading KV pages -- a radix-cache prefix: the reference's cache manager points
 * every request that matched a prefix at one copy of its pages
 * (kvcache/radix_cache.py:92-99, 133-147, attention/fa.py:82-93 reads them per
 * row). Each group's shared keys are read once for all of its rows (QK^T and PV
 * on the tensor cores, split into partials), each row's own keys by the decode
 * kernel, which merges both parts by their softmax statistics; the result equals
 * lsb_paged_attention on the same arguments. Groups in CSR form, int32 device
 * arrays: group_ptr [num_groups + 1] into group_rows (member row indices; a row
 * in at most one group), group_prefix [num_groups] (shared keys of the group:
 * the first group_prefix keys of every member's page table are the same pages,
 * and no member's context is shorter), row_prefix [rows] (group_prefix of the
 * row's group, 0 for rows in none; must agree with the groups).
 * max_group_rows / max_group_prefix bound the groups' sizes. Needs the
 * streaming decode kernel's layouts (a packed pool, at most 64 query heads):
 * otherwise LSB_ERR_UNSUPPORTED. Workspace:
 * lsb_paged_attention_shared_prefix_workspace_size bytes, zeroed once. A call
 * with no groups is lsb_paged_attention. No counterpart in the reference. */
int64_t lsb_paged_attention_shared_prefix_workspace_size(int64_t rows, int32_t hq,
                                                         int32_t head_dim, int64_t max_seqlen,
                                                         int64_t max_group_prefix);
int lsb_paged_attention_shared_prefix(
    void* out, int64_t out_stride, const void* q, int64_t q_stride, const void* k_cache,
    const void* v_cache, int64_t slot_stride, int64_t num_slots, const int32_t* page_table,
    int64_t pt_stride, const int32_t* cache_seqlens, const int32_t* cu_seqlens_q,
    int64_t num_reqs, int64_t rows, int32_t hq, int32_t hkv, int32_t head_dim,
    int32_t page_size, int64_t max_seqlen, float scale, const int32_t* group_ptr,
    const int32_t* group_rows, const int32_t* group_prefix, const int32_t* row_prefix,
    int64_t num_groups, int64_t max_group_rows, int64_t max_group_prefix, void* workspace,
    int64_t workspace_bytes, void* stream);

/* lsb_paged_attention for callers that cannot allocate device memory (a plugin
 * whose host framework owns all device memory and passes only inputs and
 * outputs, or a loop that must not pay cudaMalloc's device-wide
 * synchronisation). No counterpart in the reference. The split-KV scratch is a
 * static device array of LSB_NOALLOC_ATTENTION_SCRATCH_BYTES per GPU, held
 * until the process exits; calls needing more (see
 * lsb_paged_attention_workspace_size) fail with LSB_ERR_INVALID. All calls on a
 * device share the array: calls that overlap on the GPU race. Every call looks
 * up the array's device address and clears its arrival counters (an async
 * memset on `stream`) before the kernel, so a call whose bounded wait gave up
 * leaves nothing stale for the next; the first call on a device may load the
 * module, so make it before any stream capture. Allocates nothing. */
#define LSB_NOALLOC_ATTENTION_SCRATCH_BYTES (16 * 1024 * 1024)
int lsb_paged_attention_noalloc(void* out, int64_t out_stride, const void* q, int64_t q_stride,
                                const void* k_cache, const void* v_cache, int64_t slot_stride,
                                int64_t num_slots, const int32_t* page_table, int64_t pt_stride,
                                const int32_t* cache_seqlens, const int32_t* cu_seqlens_q,
                                int64_t num_reqs, int64_t rows, int32_t hq, int32_t hkv,
                                int32_t head_dim, int32_t page_size, int64_t max_seqlen,
                                float scale, void* stream);

/* ------------------------------------------------------------ GEMM --------
 * y[M, N] = x[M, K] . w[N, K]^T (+ bias[N]) in bf16 with fp32 accumulation on
 * the sm_100a tensor cores (tcgen05.mma, TMEM accumulators, TMA-fed).
 * x, w row-major with leading dimensions ldx, ldw (elements); y row stride ldy.
 * epilogue: LSB_EPI_NONE, LSB_EPI_BIAS (fp32 bias add before rounding),
 * LSB_EPI_BIAS_AFTER_ROUND (round, then add bias and round again),
 * LSB_EPI_SWIGLU (w rows interleaved in blocks of 64 gate / 64 up rows by
 * lsb_swiglu_interleave; y[M, N/2] = silu(g) * u of the rounded g, u).
 * Any M, N, K (ragged tails are zero-filled by TMA); SwiGLU needs N % 128 == 0;
 * ldx/ldw multiples of 8 and x, w 16-byte aligned (TMA); y any row stride.
 * Split-K (when the tiles alone cannot fill the SMs) runs in thread-block
 * clusters reduced through distributed shared memory, so no workspace is used:
 * lsb_gemm_workspace_size returns 0 and `workspace` may be NULL. Launched with
 * programmatic stream serialisation: the weight stream starts before the
 * previous kernel on `stream` has finished; `x` is read only after it has.
 * Replaces layers/linear.py:32-33 (F.linear, cuBLAS) for the QKV, o_proj,
 * gate_up, down, adapter and LM-head projections, and models/utils.py:46-48
 * (gate_up + silu_and_mul) with LSB_EPI_SWIGLU. */
#define LSB_EPI_NONE 0
#define LSB_EPI_BIAS 1
#define LSB_EPI_BIAS_AFTER_ROUND 2
#define LSB_EPI_SWIGLU 3
int64_t lsb_gemm_workspace_size(int64_t M, int64_t N, int64_t K);
int lsb_gemm(void* y, int64_t ldy, const void* x, int64_t ldx, const void* w, int64_t ldw,
             const void* bias, int64_t M, int64_t N, int64_t K, int32_t epilogue,
             void* workspace, int64_t workspace_bytes, void* stream);

/* Tile plan used by later lsb_gemm* calls of this process, for benchmarks and
 * tuning: 0 automatic (the default), 1 one wide tile of all tokens for
 * 257..384 tokens (two MMAs of up to 192 tokens per K step, one CTA per SM;
 * never chosen automatically), 2 tiles of at most 96 tokens for 257..512
 * tokens, 3 one CTA per SM for every tile size, 4 tiles of 256 weight rows on
 * CTA pairs (tcgen05 cta_group::2; calls without the fused all-reduce). No
 * counterpart in the reference (its cuBLAS heuristics). */
int lsb_gemm_force_plan(int32_t mode);
/* Largest token-tile width later lsb_gemm* calls may use (0 automatic; else a
 * multiple of 16 in 16..256), for the same benchmarks and tuning. */
int lsb_gemm_force_tile_tokens(int32_t tokens);

/* The attention's QKV projection with its RoPE and KV store fused into the GEMM
 * epilogue: qkv[M, N] = x . w^T (N = (hq + 2 hkv) x head_dim, bf16, rounded as
 * lsb_gemm rounds), then neox RoPE on the q and k heads exactly as
 * lsb_rope_store_kv applies it to that output, the rotated k heads and the v
 * heads also stored into slot out_loc[t] of k_cache / v_cache (slot 0 skipped,
 * slots outside [0, num_slots) and positions outside [0, max_pos) flagged). qkv
 * ends with the same contents as lsb_gemm followed by lsb_rope_store_kv. One
 * launch instead of two. head_dim 128 only (one head per 128-row weight tile;
 * otherwise LSB_ERR_UNSUPPORTED); no bias.  Replaces models/utils.py:119-131 (the
 * qkv F.linear) with layers/attention.py:88-90 (RoPE, store_kv). */
int lsb_gemm_rope_store(void* qkv, int64_t ldq, const void* x, int64_t ldx, const void* w,
                        int64_t ldw, int64_t M, int64_t N, int64_t K, const int32_t* positions,
                        const float* cos_sin, int64_t max_pos, void* k_cache, void* v_cache,
                        int64_t slot_stride, int64_t num_slots, const int32_t* out_loc,
                        int32_t hq, int32_t hkv, int32_t head_dim, void* stream);

/* y[M, N] = [x1 | x2] . w^T (+ bias) with w [N, K1 + K2]: the product over the
 * concatenation of two activation tensors along K without materialising it (the
 * K loop reads x1 and w's first K1 columns, then x2 and the last K2). Replaces
 * Huginn's adapter, models/looped/huginn.py:162-167 (F.linear over
 * torch.cat([hidden, injection], -1)). K1 a multiple of 8; epilogue LSB_EPI_NONE,
 * LSB_EPI_BIAS or LSB_EPI_BIAS_AFTER_ROUND. */
int lsb_gemm_concat(void* y, int64_t ldy, const void* x1, int64_t ldx1, const void* x2,
                    int64_t ldx2, const void* w, int64_t ldw, const void* bias, int64_t M,
                    int64_t N, int64_t K1, int64_t K2, int32_t epilogue, void* stream);

/* Greedy sampling fused into the LM-head GEMM (layers/embedding.py:89-111 +
 * model_executor/sample.py:108-112): for every row m of x and every 128-entry
 * vocabulary tile t of w [N, K], pairs[m * ld_pairs + t] = {float value, int32
 * index} of the largest bf16-rounded logit in the tile (first index on ties), so
 * the [M, N] logits are never written. ld_pairs >= lsb_gemm_argmax_tiles(N)
 * (the tile count rounded up to even, so a row of pairs is a multiple of 16
 * bytes); pairs 8-byte aligned. Tensor-parallel ranks pass their own vocabulary
 * range's valid row count as N (padding rows are never scored) and all-gather
 * the pairs instead of the logits. */
int64_t lsb_gemm_argmax_tiles(int64_t N);
int lsb_gemm_argmax(void* pairs, int64_t ld_pairs, const void* x, int64_t ldx, const void* w,
                    int64_t ldw, int64_t M, int64_t N, int64_t K, void* stream);

/* out[m] = the global index of the best pair of row m over `shards` blocks of
 * pairs [shards][rows][ld_pairs] (the first `tiles` of each row scored), shard
 * s covering global indices s*shard_cols ..: the argmax of the gathered,
 * permuted logits of layers/embedding.py:99-111 with torch.argmax's first-index
 * rule. Unscored tiles must hold value -inf. */
int lsb_argmax_pairs(int32_t* out, const void* pairs, int64_t shards, int64_t rows,
                     int64_t tiles, int64_t ld_pairs, int64_t shard_cols, void* stream);

/* The launch plan lsb_gemm picks for an M x N x K product on the current device
 * (diagnostics): out[0] tokens per tile, out[1] output tiles, out[2] split-K
 * factor (CTAs per cluster), out[3] pipeline stages, out[4] dynamic shared
 * memory bytes per CTA. */
int lsb_gemm_plan(int64_t M, int64_t N, int64_t K, int32_t* out);

/* Reorders a [2*I, K] gate_up weight ([gate; up], models/weight.py:136-141)
 * into 128-row tiles of 64 gate rows followed by the matching 64 up rows, the
 * layout LSB_EPI_SWIGLU reads. I % 64 == 0. out must not alias w. */
int lsb_swiglu_interleave(void* out, const void* w, int64_t inter, int64_t K, void* stream);

/* ---------------------------------------------- loop-step exit kernels ---
 * Ouro step end fused with the exit gate and the CDB state scatter:
 *   y = rmsnorm(x) * w_post2 (rounded); residual <- y + residual;
 *   h = rmsnorm(residual) * w_final                      (ouro.py:52, :136)
 *   logit = bf16(h . gate_w + gate_b)                     (ouro.py:149)
 *   p' = p + (1 - p) * sigmoid(logit)                     (exit_gates.py:6-15)
 *   signal = p' >= threshold && depth + 1 + lookahead >= min_loop_steps
 * Row r writes h to hidden_out[slot[r]] (slot == NULL: row r), reads and writes
 * exit_state[slot[r]] (fp32), writes signal[r] (uint8 0/1). depth: per-row int32
 * array, or NULL to use depth_scalar. gate_w/gate_b may be NULL (no gate: only
 * h is written).  Replaces ouro.py:136 + :142-155 and
 * model_executor/cdb_model_runner.py:102-108. */
int lsb_ouro_step_exit(void* hidden_out, int64_t hidden_stride, const void* x, void* residual,
                       const void* w_post2, const void* w_final, const void* gate_w,
                       const void* gate_b, const int64_t* slot, float* exit_state,
                       uint8_t* signal, const int32_t* depth, int32_t depth_scalar,
                       int32_t lookahead, int32_t min_loop_steps, float threshold,
                       int64_t rows, int64_t dim, float eps, void* stream);

/* Huginn exit: signal[r] = ||h - prev|| / max(||h||, 1e-9) < threshold in fp32,
 * prev = exit_state[slot[r]] (bf16 rows), then exit_state[slot[r]] = h and
 * hidden_out[slot[r]] = h.  Replaces huginn.py:184-194, exit_gates.py:18-24 and
 * cdb_model_runner.py:102-108. */
int lsb_huginn_step_exit(void* hidden_out, void* exit_state, const void* h, const int64_t* slot,
                         uint8_t* signal, float threshold, int64_t rows, int64_t dim,
                         void* stream);

/* ------------------------------------------------ gathers and sampling ---
 * out[t] = dtype(weight[ids[t] - vocab_start] * scale), zero rows for ids outside
 * [vocab_start, vocab_start + vocab_len).  Replaces layers/embedding.py:34-43
 * (VocabParallelEmbedding.forward before its all-reduce) and huginn.py:147-148. */
int lsb_embedding(void* out, const int32_t* ids, const void* weight, int64_t tokens, int64_t dim,
                  int64_t vocab_start, int64_t vocab_len, float scale, void* stream);

/* out[r] = src[index[r]] over rows of `dim` bf16 (index_select).
 * Replaces cdb_model_runner.py:94-101 (state-pool gathers). */
int lsb_gather_rows(void* out, const void* src, const int64_t* index, int64_t rows, int64_t dim,
                    void* stream);

/* out[r] = argmax_j logits[r, j] (first index on ties), logits bf16 [rows, vocab]
 * with row stride ld.  Replaces model_executor/sample.py:108-112. */
int lsb_argmax(int32_t* out, const void* logits, int64_t rows, int64_t vocab, int64_t ld,
               void* stream);

/* Greedy token over tensor-parallel LM-head logits gathered rank by rank:
 * logits [shards][rows][cols] bf16 (rank r holds vocabulary entries
 * r*cols .. r*cols+cols-1, layers/embedding.py:89-111); entries at or beyond
 * `vocab` are padding. Same tie rule as lsb_argmax (smallest global index), so
 * the result equals the argmax of the reference's all-gathered, permuted row. */
int lsb_argmax_sharded(int32_t* out, const void* logits, int64_t shards, int64_t rows,
                       int64_t cols, int64_t vocab, void* stream);

/* silu(x[:, :I]) * x[:, I:] -> out[:, :I].  Replaces layers/activation.py:9-12. */
int lsb_silu_and_mul(void* out, const void* x, int64_t rows, int64_t inter, void* stream);

/* ------------------------------------------------- last-exited metadata --
 * Resolve logical token handles to physical KV slots at each row's depth:
 * physical_table[g, r, c] = version_map[depth_r, g, logical_table[r, c]] for
 * c < cache_seqlens[r]; physical_out[g, i] = version_map[depth_r, g,
 * logical_out[i]] for the query rows i of request r. version_map is
 * [steps, groups, num_handles] int32 (group stride vm_group_stride, depth stride
 * vm_depth_stride); depth = depths[r] or depth_scalar when depths is NULL.
 * Replaces attention/metadata.py:220-291 (prepare_last_exited_metadata). */
int lsb_last_exited_resolve(int32_t* physical_table, int64_t pt_group_stride, int64_t pt_stride,
                            int32_t* physical_out, int64_t out_group_stride,
                            const int32_t* logical_table, int64_t lt_stride,
                            const int32_t* version_map, int64_t vm_depth_stride,
                            int64_t vm_group_stride, const int32_t* cache_seqlens,
                            const int32_t* cu_seqlens_q, const int32_t* logical_out,
                            const int32_t* depths, int32_t depth_scalar, int64_t num_reqs,
                            int64_t cols, int32_t groups, void* stream);

/* Reserve the KV versions of n new token handles (one per loop depth and
 * layer group) from the shared free-slot stack, exactly as the reference's
 * _reserve_versions does when its programs run in handle order:
 * token t pops fixed_groups + d_t * core_groups slots (d_t = steps, or
 * restore_depths[t] when not NULL) and depths it did not compute alias the
 * last computed version. slot_map [fixed + steps*core, width] int32,
 * completed_depth [width], free_slots stack, free_count [1] (device). A
 * negative handle reserves nothing (rows of a fixed-shape batch that have
 * nothing to reserve). Replaces kvcache/last_exited.py:15-47 and :181-202,
 * :269-290. */
int lsb_last_exited_reserve(int32_t* slot_map, int32_t* completed_depth, int64_t width,
                            int32_t* free_slots, int32_t* free_count, const int32_t* handles,
                            const int32_t* restore_depths, int64_t n, int32_t steps,
                            int32_t fixed_groups, int32_t core_groups, void* stream);

/* Release versions back to the stack in handle order (the reference's
 * _release_versions): with exits (alias) the versions at depths >= exits[t]
 * are freed and alias the final computed version; with exits == NULL every
 * version of the token is freed; a negative handle releases nothing.
 * Replaces kvcache/last_exited.py:50-84, :204-248. */
int lsb_last_exited_release(int32_t* slot_map, int32_t* completed_depth, int64_t width,
                            int32_t* free_slots, int32_t* free_count, const int32_t* handles,
                            const int32_t* exits, int64_t n, int32_t steps, int32_t fixed_groups,
                            int32_t core_groups, void* stream);

/* --------------------------------------------------- batch metadata ----
 * Per-token batch inputs from the token-granular request table req_to_token
 * [rows, r2t_stride] int32 (locations page*page_size + offset): for request r,
 * query token j sits at seq_lens[r] - extend_lens[r] + j (decode: extend 1,
 * token r) and reads its KV location from req_to_token[req_pool_indices[r], pos].
 * Writes positions, req_mapping (may be NULL) and out_loc, flattened over
 * requests.  Replaces kernel/batch.py:72-129 (_prepare_batch_inputs). */
int lsb_prepare_batch_inputs(int32_t* positions, int32_t* req_mapping, int32_t* out_loc,
                             const int32_t* seq_lens, const int32_t* extend_lens,
                             const int32_t* req_pool_indices, const int32_t* req_to_token,
                             int64_t r2t_stride, int64_t bs, int32_t is_decode, void* stream);

/* Attention metadata: cache_seqlens = seq_lens + seq_len_delta; prefix sums
 * cu_seqlens_k / cu_seqlens_q (decode: one query per request); page-table row r
 * = req_to_token[req_pool_indices[r], c * page_size] / page_size for the
 * min(ceil(seq/page), max_seq_pages) live columns (others untouched).
 * Replaces attention/metadata.py:59-216 (_fused_metadata_kernel_general via
 * normal_decode_set_metadata / extend_set_metadata). */
int lsb_set_metadata(int32_t* cache_seqlens, int32_t* cu_seqlens_k, int32_t* cu_seqlens_q,
                     int32_t* page_table, int64_t pt_stride, const int32_t* req_to_token,
                     int64_t r2t_stride, const int32_t* req_pool_indices,
                     const int32_t* seq_lens, const int32_t* extend_lens, int64_t bs,
                     int64_t max_seq_pages, int32_t page_size, int32_t seq_len_delta,
                     int32_t is_decode, void* stream);

/* ------------------------------------------- device-side CDB routing -------
 * One core step of continuous-depth batching routed on the device
 * (CDBScheduler._run_core / _consume_gate / _run_coda, managers/cdb_scheduler.py:
 * 189-267, with disable_lookahead_exit timing), so a decode iteration needs no
 * host round trip. Per row r, after the step at depth[r]: d = depth[r] + 1; the
 * row exits when d >= max_depth or its gate fired (signal[r] != 0) -- or, when
 * replay_depths [rows, out_stride] is given, when d reaches the prescribed exit
 * depth of its next output (the reference's replay_exit_depths). An exiting row
 * takes its greedy token sampled[r] (or forced_ids[r, k] when given: teacher
 * forcing) as the next input, records sampled[r] and d in out_tokens / out_depths
 * [rows, out_stride] at k = out_count[r] (optional), advances seq_lens[r] and sets
 * depth[r] = 0; alias_handle[r] /
 * alias_depth[r] then name its KV versions to alias (else -1) and reserve_handle[r]
 * the successor position to reserve (else -1), ready for lsb_last_exited_release /
 * lsb_last_exited_reserve, which skip negative handles. *produced (optional)
 * counts the outputs. No counterpart kernel in the reference (host logic there). */
int lsb_cdb_route(int32_t* depth, int32_t* seq_lens, int32_t* ids, const int32_t* sampled,
                  const uint8_t* signal, const int32_t* replay_depths, const int32_t* forced_ids,
                  int64_t out_stride, int32_t* out_count, int32_t* out_tokens, int32_t* out_depths,
                  int32_t* alias_handle, int32_t* alias_depth, int32_t* reserve_handle,
                  uint8_t* exited, const int32_t* req_to_token, int64_t r2t_stride,
                  const int32_t* req_pool_indices, int64_t rows, int32_t max_depth,
                  int32_t max_seq_len, int32_t* produced, void* stream);

/* Re-admission of the rows that exited: hidden[slots[r]] = emb[r] (the successor's
 * prelude output) and exit_state[slots[r]] = 0 (optional) where exited[r]; the
 * prelude phase's state writes (cdb_model_runner.py:84-91). */
int lsb_cdb_admit(void* hidden, int64_t ld, float* exit_state, const int64_t* slots,
                  const uint8_t* exited, const void* emb, int64_t rows, int64_t dim, void* stream);

/* ------------------------------------------------- TP communicator --------
 * Tensor parallelism over the GPUs of one node, one process per GPU, without
 * NCCL on the data path. Every rank allocates one symmetric buffer of
 * lsb_comm_buffer_bytes(max_elems) with lsb_comm_alloc (zeroed), exports it with
 * lsb_ipc_handle, maps every peer's with lsb_ipc_open (the handles travel over
 * the host process group), and builds a communicator from the world's mapped
 * addresses (buffers[rank] = its own). max_elems bounds the bf16 elements of one
 * all-reduce (rows x cols) and the bytes/2 of one all-gather contribution.
 * Data moves with stores into peer memory over NVLink: each output region is
 * owned by one rank, which sums every rank's bf16 partial in rank order (fp32,
 * one rounding: all ranks receive identical bits) and writes the sum back to
 * every rank. Flags carry per-call epochs, so no reset is needed between calls;
 * every wait is bounded (LSB_DEVERR_COMM_TIMEOUT in the device error word). All ranks
 * must make the same calls, with the same shapes, in the same order. Calls are
 * stream-ordered and capturable in CUDA graphs. Replaces the PyNCCL communicator
 * (python/loopsgl/distributed/impl.py:44-60, kernel/csrc/src/pynccl.cu:72-161,
 * python/loopsgl/kernel/pynccl.py:59-92). */
#define LSB_IPC_HANDLE_BYTES 64
typedef struct lsb_comm lsb_comm;
int64_t lsb_comm_buffer_bytes(int64_t max_elems);
int lsb_comm_alloc(int64_t bytes, void** ptr);
int lsb_comm_free(void* ptr);
int lsb_ipc_handle(void* ptr, void* handle);
int lsb_ipc_open(const void* handle, void** ptr);
int lsb_ipc_close(void* ptr);
int lsb_comm_create(int32_t rank, int32_t world, void* const* buffers, int64_t max_elems,
                    lsb_comm** comm);
int lsb_comm_destroy(lsb_comm* comm);
/* All-reduce protocol of later calls on this communicator (every rank must choose the
 * same): 0 automatic (per call: one hop for two ranks, and for three or four while a
 * rank's one-hop sends stay within 1 MB; else two), 1 one hop -- every rank stores its
 * partial into every rank's buffer and sums all of them itself (at most 4 ranks; the
 * same bits on every rank), 2 two hops -- partials to the owner of each region, sums
 * back from it ((world - 1) / world of the bytes each way). The two use separate parts
 * of the buffers, so consecutive calls may use different ones. No counterpart in the
 * reference (its NCCL picks the algorithm). */
int lsb_comm_set_protocol(lsb_comm* comm, int32_t mode);

/* In-place sum of x[rows, cols] (row stride ld) over the ranks: the reference's
 * DistributedCommunicator.all_reduce (distributed/impl.py:63-67), used for the
 * vocab-parallel embedding and by callers that keep their own GEMM. */
int lsb_allreduce(lsb_comm* comm, void* x, int64_t rows, int64_t cols, int64_t ld, void* stream);

/* out[world][bytes] = every rank's `in` (bytes a multiple of 16), the reference's
 * all_gather along dim 0 (distributed/impl.py:68-70; LM-head logits,
 * layers/embedding.py:99-111). */
int lsb_allgather(lsb_comm* comm, void* out, const void* in, int64_t bytes, void* stream);

/* Row-parallel linear fused with its all-reduce: y[M, N] = sum over ranks of
 * x_r[M, K_r] . w_r[N, K_r]^T (+ bias on every rank, as the reference adds it
 * before reducing), in ONE kernel: the tcgen05 GEMM's epilogue pushes each
 * rank's bf16 tile to the tile's owner over NVLink, the owner reduces and
 * broadcasts, and the kernel ends when y is complete on this rank. epilogue
 * LSB_EPI_NONE or LSB_EPI_BIAS; M x N <= the communicator's max_elems. With one
 * rank it is lsb_gemm. Replaces LinearOProj.forward / LinearRowParallel.forward
 * (layers/linear.py:103-107, 124-128: F.linear then all_reduce). */
int lsb_gemm_allreduce(lsb_comm* comm, void* y, int64_t ldy, const void* x, int64_t ldx,
                       const void* w, int64_t ldw, const void* bias, int64_t M, int64_t N,
                       int64_t K, int32_t epilogue, void* stream);

/* ------------------------------------------------------------------------
 * KV snapshots for retraction: a request's KV rows copied to host memory in
 * the reference's byte layout and restored into newly reserved locations.
 * Host layout: [2][E][n][row_bytes] (K then V; E expanded layers in layer order,
 * each core layer of a versioned pool once per loop depth; tokens in the order
 * of `indices`), then, for a versioned pool, n int32 completed depths.
 * pool is [2][lanes][pool_rows][row_bytes] on the device: a paged pool passes
 * lanes = num_layers, pool_rows = pages * page_size and slot_map = NULL (the row
 * of token j is indices[j]); the last-exited pool passes its slot map
 * [fixed + steps*core groups, width], lanes = layers per slot and the core
 * layer range [core_start, core_end) with `steps` loop depths. row_bytes must be
 * a multiple of 16. Rows move through `staging` (device, >= 2*E*row_bytes) in
 * chunks of tokens: one gather / scatter kernel and one strided 2-D copy per
 * chunk; both calls return after their copies completed. A row outside the
 * pool (or a restore into row 0, the padding row) is skipped and flagged
 * LSB_DEVERR_SLOT. Replaces MHAKVCache.get_cpu_copy / load_cpu_copy
 * (kvcache/mha_pool.py:68-105) and LastExitedKVCache.get_cpu_copy /
 * load_cpu_copy (kvcache/last_exited.py:320-376).
 * ------------------------------------------------------------------------ */

/* Snapshot bytes of n tokens (cpu_copy_size, mha_pool.py:68-69 with versioned
 * = 0; last_exited.py:317-318 with versioned = 1), or -1 for invalid shapes. */
int64_t lsb_kv_snapshot_bytes(int64_t n, int64_t row_bytes, int32_t num_layers,
                              int32_t core_start, int32_t core_end, int32_t steps,
                              int32_t versioned);

int lsb_kv_backup(void* host_out, const void* pool, int64_t lanes, int64_t pool_rows,
                  int64_t row_bytes, const int32_t* indices, int64_t n, const int32_t* slot_map,
                  int64_t width, const int32_t* completed_depth, int32_t num_layers,
                  int32_t core_start, int32_t core_end, int32_t steps, void* staging,
                  int64_t staging_bytes, void* stream);

/* The inverse: host_in's rows into the pool at the (already reserved) rows of
 * `indices`; a versioned snapshot's trailing depths are not read here (the
 * caller reserves the versions with them: lsb_last_exited_reserve with
 * restore_depths). */
int lsb_kv_restore(void* pool, const void* host_in, int64_t lanes, int64_t pool_rows,
                   int64_t row_bytes, const int32_t* indices, int64_t n, const int32_t* slot_map,
                   int64_t width, int32_t num_layers, int32_t core_start, int32_t core_end,
                   int32_t steps, void* staging, int64_t staging_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Radix prefix cache (host runtime; no GPU work). A prefix tree over token ids
 * whose nodes hold the KV token locations of those ids, matched and split at
 * page granularity, with lock counts and oldest-first eviction of unlocked
 * leaves: the reference's RadixPrefixCache (kvcache/radix_cache.py:102-232).
 * Node handles are opaque int64 values that carry a generation: a handle to a
 * node that was evicted since is refused (LSB_ERR_INVALID). One tree may be
 * used from several threads (calls are serialised).
 * ------------------------------------------------------------------------ */
typedef struct lsb_radix lsb_radix;

/* Length of the common prefix of two 1-D int32 (bits 32) or int64 (bits 64)
 * arrays, the reference's fast_compare_key (kernel/csrc/src/radix.cpp:19-40). */
int lsb_fast_compare_key(const void* a, int64_t na, const void* b, int64_t nb, int32_t bits,
                         int64_t* out);

/* A tree matching whole pages of page_size ids (RadixPrefixCache.__init__,
 * radix_cache.py:103-112; the root is permanently locked). */
int lsb_radix_create(int32_t page_size, lsb_radix** out);
int lsb_radix_destroy(lsb_radix* tree);

/* Longest cached page-aligned prefix of ids[n]: its end node and length
 * (match_prefix / _tree_walk, radix_cache.py:133-135, 206-232). A node matched
 * part-way is split at the page boundary, and the walked path is marked used. */
int lsb_radix_match(lsb_radix* tree, const int32_t* ids, int64_t n, int64_t* node,
                    int64_t* prefix_len);

/* Insert the first floor(n / page) pages of ids with their KV locations:
 * prefix_len = the length already cached (those locations stay the tree's; the
 * caller frees its own copies), node/insert_len = the handle of the whole
 * inserted prefix (insert_prefix, radix_cache.py:137-147). */
int lsb_radix_insert(lsb_radix* tree, const int32_t* ids, const int32_t* indices, int64_t n,
                     int64_t* node, int64_t* prefix_len, int64_t* insert_len);

/* Lock (unlock = 0) or unlock a handle's path: locked nodes are never evicted
 * (lock_handle, radix_cache.py:114-131). Unlocking an unlocked path fails and
 * changes nothing. */
int lsb_radix_lock(lsb_radix* tree, int64_t node, int32_t unlock);

/* The KV locations of the prefix ending at `node`, root first, into out[capacity];
 * *n = their number (RadixCacheHandle.get_matched_indices, radix_cache.py:92-99). */
int lsb_radix_indices(lsb_radix* tree, int64_t node, int32_t* out, int64_t capacity, int64_t* n);

/* Evict unlocked leaves, oldest first, until at least `size` locations are freed;
 * writes them to out (capacity >= the evictable size), *n = how many (evict,
 * radix_cache.py:149-176). size above the evictable size fails, changing nothing. */
int lsb_radix_evict(lsb_radix* tree, int64_t size, int32_t* out, int64_t capacity, int64_t* n);

/* Locations held by unlocked / locked nodes (size_info, radix_cache.py:181-186). */
int lsb_radix_size_info(lsb_radix* tree, int64_t* evictable, int64_t* protected_size);

/* Structural check: parent links, child keys, page-aligned runs, lock counts and
 * the two size totals recounted (check_integrity, radix_cache.py:188-189). */
int lsb_radix_check(lsb_radix* tree);

#ifdef __cplusplus
}
#endif

#endif /* LOOPSGL_B200_H_ */
