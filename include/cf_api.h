/*
 * cudaforge_b200 C ABI -- the drop-in boundary of the speculative-decoding
 * verify + accept path on B200 (sm_100a).
 *
 * Conventions (all entry points):
 *   - plain pointers, sizes and POD argument structs; no C++ or torch types;
 *   - every device pointer is caller-owned; the library allocates no device
 *     memory of its own on these paths (scratch comes in through `workspace`
 *     arguments sized by the matching *_workspace_bytes query);
 *   - work is enqueued on the caller's stream (`stream` is a cudaStream_t;
 *     NULL = legacy default stream) and the call returns without
 *     synchronising;
 *   - the return value is CF_OK (0) or a negative cf_status; nothing throws
 *     across this boundary.  Argument errors are detected on the host before
 *     any launch; errors that depend on device data (an out-of-range draft
 *     token, a block id outside the pool) are reported through the outputs
 *     documented per call.
 *
 * The reference (CUDAForge) has no C ABI for this path; each entry point
 * names the reference interface it replaces.
 */
#ifndef CF_API_H_
#define CF_API_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum cf_status {
  CF_OK = 0,
  CF_EINVAL = -1,       /* bad argument (shape, null pointer, alignment)      */
  CF_ERANGE = -2,       /* index out of range (block id, token id, sequence)  */
  CF_ETIMEOUT = -3,     /* a bounded device-side wait gave up                  */
  CF_ECUDA = -4,        /* a CUDA runtime call failed                          */
  CF_ENOMEM = -5,       /* host allocation failed / KV pool exhausted          */
  CF_EUNSUPPORTED = -6  /* configuration not built in this library            */
} cf_status;

typedef enum cf_dtype {
  CF_F32 = 0,
  CF_BF16 = 1,
  CF_F16 = 2
} cf_dtype;

/* Human-readable name of a status code (static storage). */
const char *cf_status_string(int status);

/* Library version string, e.g. "cudaforge_b200 0.1 sm_100a". */
const char *cf_version(void);

/* ------------------------------------------------------------------------
 * Acceptance sampling
 *
 * Replaces: SpeculativeEngine::verify_candidates and
 * SpeculativeEngine::verify_candidates_greedy
 * (csrc/include/cudaforge/scheduler/speculative.h:48-63,
 *  csrc/src/scheduler/speculative.cpp:50-150, bound in
 *  csrc/bindings/pybind_module.cpp:229-236), batched over sequences and fed
 * logits instead of probability lists.  The softmax of
 * cudaforge/speculative.py:118 and :145 (softmax(logits / T)) is fused in.
 *
 * Per sequence b (K = k):
 *   q = softmax(draft_logits[b, i] / T), p = softmax(target_logits[b, i] / T)
 *   for i < K: ratio = q[x_i] > 0 ? min(1, p[x_i] / q[x_i]) : 0,
 *              accept iff uniforms[b, i] <= ratio;
 *              an accepted EOS stops with final token = EOS;
 *              on the first rejection at i the final token is drawn from
 *              norm(max(0, p - q)) (target row i when that sum <= 1e-6) with
 *              uniforms[b, i + 1];
 *   all accepted: the bonus token is drawn from p (target row K) with
 *              uniforms[b, K].
 * Draws are inverse-CDF with a sequential fp32 cumulative sum (first index
 * with u <= cum, else V-1), exactly as the reference computes it.
 * Greedy mode (greedy != 0): accept while x_i == argmax(p_i) (lowest index
 * on ties), final = that argmax, bonus = argmax of row K; uniforms unused.
 *
 * Outputs: out_tokens[b, 0..n-1] = accepted drafts, out_tokens[b, n] = final
 * token, n = out_num_accepted[b]; out_eos[b] = 1 when the sequence ended.
 * A draft token outside [0, vocab) makes that sequence's out_num_accepted
 * -1 (the reference's behaviour there is undefined).
 *
 * Optional parity export: when probs_draft / probs_target are non-NULL the
 * kernel also writes the fp32 probabilities it decided on
 * ([B, K, V] and [B, K+1, V], contiguous).
 * ---------------------------------------------------------------------- */
typedef struct cf_accept_args {
  int32_t batch;            /* B >= 0                                   */
  int32_t k;                /* K >= 0 draft tokens per sequence           */
  int64_t vocab;            /* V >= 1                                   */
  int32_t logits_dtype;     /* cf_dtype of both logits tensors          */
  const void *draft_logits; /* row (b, i) at b*draft_seq_stride + i*draft_row_stride (elements) */
  int64_t draft_seq_stride;
  int64_t draft_row_stride;
  const void *target_logits; /* row (b, i), i <= K                       */
  int64_t target_seq_stride;
  int64_t target_row_stride;
  const int32_t *draft_tokens; /* [B, K] contiguous                      */
  const float *uniforms;       /* [B, K+1] contiguous, U[0,1); NULL if greedy */
  float temperature;           /* > 0 (the Python layer clamps at 1e-5)  */
  int32_t eos_token_id;        /* -1: none                               */
  int32_t greedy;
  int32_t *out_tokens;       /* [B, K+1]                                 */
  int32_t *out_num_accepted; /* [B]                                      */
  uint8_t *out_eos;          /* [B]                                      */
  void *workspace;           /* >= cf_accept_workspace_bytes(B, K) bytes, 16-B aligned */
  float *probs_draft;        /* optional parity export                   */
  float *probs_target;       /* optional parity export                   */
  float top_p;               /* in (0, 1): nucleus filter on the bonus draw (the
                              * reference Python engine's top-p, speculative.py:58-84,
                              * :188-195; not in the reference C++ path, so not
                              * parity-pinned); 0 or >= 1: off */
} cf_accept_args;

size_t cf_accept_workspace_bytes(int32_t batch, int32_t k);
int cf_accept_sample(const cf_accept_args *args, void *stream);

/* Same as cf_accept_sample, for callers that must not allocate device memory
 * (an allocator hook, a runtime that owns all device memory, a plugin limited
 * to the buffers it is given).  No counterpart in the reference.  args->workspace
 * is ignored: the scratch goes to a fixed array compiled into this library
 * (cf_accept_noalloc_max_bytes() = 2 MiB per GPU that loads the library, held
 * until exit).  A call whose cf_accept_workspace_bytes(batch, k) exceeds that
 * returns CF_ERANGE and launches nothing (K = 5: up to 1,833 sequences).  The
 * first call on a device looks up the array's device address
 * (cudaGetSymbolAddress), so make that first call before any stream capture.
 * The address is cached per device ordinal for the life of the process: after
 * cudaDeviceReset (or any teardown of the device's primary context) it is
 * stale, so do not call this entry point again in that process.  All calls
 * share the array: calls that can run at the same time on the GPU (different
 * streams, different host threads) race and must be serialised by the caller.
 * No cudaMalloc / cudaFree. */
int cf_accept_sample_noalloc(const cf_accept_args *args, void *stream);
size_t cf_accept_noalloc_max_bytes(void);

/* ------------------------------------------------------------------------
 * Tree acceptance.  The reference has no tree verifier; this extends
 * verify_candidates (speculative.cpp:50-150) so that a branching-1 tree gives
 * exactly its results.  Nodes 0..N (nodes = N+1): node 0 is the root (the
 * last emitted token), parent[b][i] < i for i > 0, tokens[b][i] the draft
 * token of node i; siblings are tried in increasing node index.  Logits row u
 * of sequence b: target distribution after node u, and the draft
 * distribution node u's children were drawn from (uses the strides of
 * cf_accept_args).  Walking from the root with p = softmax(target[u] / T),
 * q = softmax(draft[u] / T): each child is accepted iff
 * uniforms[b][n] <= min(1, p[x]/q[x]) (q[x] > 0), n counting tests in order;
 * a rejection replaces p with norm(max(0, p - q)) (kept when that sum is
 * <= 1e-6) and tries the next sibling; when all children are rejected the
 * final token is drawn from p, at a leaf from the leaf's target row; an
 * accepted EOS stops.  Greedy: move to the child whose token is the argmax.
 * Outputs: out_path[b][0..n] the accepted node ids (out_path[b][0] = 0),
 * out_tokens[b][0..n] their tokens then the final token, n =
 * out_num_accepted[b].  workspace: cf_accept_tree_workspace_bytes bytes,
 * 256-B aligned (row statistics + one fp32 residual row per sequence).
 * ---------------------------------------------------------------------- */
typedef struct cf_accept_tree_args {
  int32_t batch, nodes;
  int64_t vocab;
  int32_t logits_dtype;
  const void *draft_logits;
  int64_t draft_seq_stride, draft_row_stride;
  const void *target_logits;
  int64_t target_seq_stride, target_row_stride;
  const int32_t *parent;   /* [B][nodes] */
  const int32_t *tokens;   /* [B][nodes] */
  const float *uniforms;   /* [B][nodes] */
  float temperature;
  int32_t eos_token_id;
  int32_t greedy;
  int32_t *out_path;       /* [B][nodes] */
  int32_t *out_tokens;     /* [B][nodes] */
  int32_t *out_num_accepted;
  uint8_t *out_eos;
  void *workspace;
  float *probs_draft;      /* optional parity export [B][nodes][V] */
  float *probs_target;     /* optional parity export [B][nodes][V] */
} cf_accept_tree_args;

size_t cf_accept_tree_workspace_bytes(int32_t batch, int32_t nodes, int64_t vocab);
int cf_accept_tree(const cf_accept_tree_args *args, void *stream);

/* Row-wise top-k of logits for the draft-tree builder (no reference
 * counterpart; the reference drafts chains, cudaforge/speculative.py:113-123).
 * rows x vocab logits (dtype CF_F32/CF_BF16/CF_F16) at row_stride elements;
 * out_idx[rows][k] the k largest in descending order, ties to the lower index,
 * NaN last (-1 when a row has fewer than k non-NaN entries); out_val optional. */
int cf_topk_rows(const void *logits, int64_t row_stride, int32_t rows, int64_t vocab, int32_t dtype, int32_t k,
                 int32_t *out_idx, float *out_val, void *stream);

/* ------------------------------------------------------------------------
 * GEMM on tcgen05 tensor cores (TMEM accumulators, TMA-staged operands)
 *
 * cf_w4a16_gemm replaces the reference INT4 GEMM launcher
 * launch_int4_gemm_dequant(const Int4GemmParams&, cudaStream_t)
 * (csrc/include/cudaforge/kernels/dequantize.cuh:12-31,
 *  csrc/kernels/cuda/int4_gemm_dequant.cu:117-133) and its tested Triton
 * twin int4_gemm_dequant_triton (csrc/kernels/triton/int4_dequant_triton.py:80-131):
 *     y[m, n] = sum_k x[m, k] * (nibble(k, n) - 8) * scales[k / 128, n]
 *               (+ residual[m, n])
 * x: bf16 [m, k] (row pitch ldx elements, 16-B aligned rows);
 * w: packed INT4 [k/8, n] uint32 in the kernel order made by
 *    cf_w4a16_repack from the reference packing (nibble i of word (j, n)
 *    holds k = 8j + i; tests/unit/test_int4_dequant.py:6-15), zero point 8;
 * scales: fp16 [k/128, n]; y: bf16 [m, n] (pitch ldy); residual optional.
 * Requirements: n % 128 == 0, k % 128 == 0 (k % 64 == 0 for cf_dense_gemm).  When the plan splits K
 * (split_k = 0 picks it from the SM count) the fp32 partials go to
 * `workspace` (cf_gemm_workspace_bytes) and a fixed-order reduction kernel
 * produces y.  `status` (optional, device int) receives CF_ETIMEOUT if a
 * bounded pipeline wait expired (timeout_ns, 0 = 2 s).
 *
 * cf_dense_gemm is the same kernel with 16-bit weights w [n, k] (k
 * contiguous, nn.Linear layout) loaded by TMA instead of dequantised; act
 * dtype CF_BF16 or CF_F16 (x, w, y, residual all of that type).
 * ---------------------------------------------------------------------- */
typedef struct cf_gemm_args {
  int32_t m, n, k;
  int32_t act_dtype;     /* cf_dtype of x / y / residual (and w when dense) */
  const void *x;
  int64_t ldx;
  const void *w;
  const void *scales;    /* int4 only */
  void *y;
  int64_t ldy;
  const void *residual;  /* optional */
  int64_t ldr;
  int32_t split_k;       /* 0 = automatic */
  void *workspace;
  size_t workspace_bytes;
  int32_t *status;       /* optional */
  uint64_t timeout_ns;   /* 0 = default */
  uint64_t *trace;       /* optional profiling aid: [11][512] SM-clock stamps of CTA (0,0,0)
                            per 64-k stage and role: 0 W issue, 1 dequant TMEM store start,
                            2 dequant arrive, 3 MMA issue start, 4 X issue, 5 epilogue
                            start/end, 6-7 MMA waits, 8 MMA commits, 9 dequant W ready,
                            10 dequant computed */
} cf_gemm_args;

size_t cf_gemm_workspace_bytes(int32_t m, int32_t n, int32_t k, int32_t split_k, int32_t int4);
int cf_w4a16_gemm(const cf_gemm_args *args, void *stream);
int cf_dense_gemm(const cf_gemm_args *args, void *stream);
/* Split-K without the reduction launch (no reference counterpart: the
 * reference has no split-K).  cf_gemm_splits() = the number of K splits the
 * plan for this shape uses (1 = no split, 0 = unsupported shape).  When it is
 * > 1, the *_partials calls run only the GEMM and leave fp32 partials
 * [splits][m][n] (contiguous) at the start of `workspace`, and `y` /
 * `residual` are not touched; one of the cf_splitk_* consumers below then
 * forms y exactly as the reduction would (fixed order s = 0..splits-1, then
 * + residual, then one rounding) and fuses its own op.  With 1 split they
 * behave as cf_w4a16_gemm / cf_dense_gemm. */
int cf_gemm_splits(int32_t m, int32_t n, int32_t k, int32_t split_k, int32_t int4);
int cf_w4a16_gemm_partials(const cf_gemm_args *args, void *stream);
int cf_dense_gemm_partials(const cf_gemm_args *args, void *stream);
/* Reference [k/8, n] packing -> kernel nibble order (same values). */
int cf_w4a16_repack(const uint32_t *wq_ref, uint32_t *wq_out, int32_t k, int32_t n, void *stream);

/* ------------------------------------------------------------------------
 * Paged KV cache: host page tables (reference semantics) over caller-owned
 * device pools.
 *
 * Replaces cudaforge::memory::PagedKVCache
 * (csrc/include/cudaforge/memory/paged_kv_cache.h:36-178,
 *  csrc/src/memory/paged_kv_cache.cpp, bound in
 *  csrc/bindings/pybind_module.cpp:27-99).  Pool layout (per pool, K and V):
 *  [block][layer][kv_head][slot][head_dim] elements, block stride
 *  bytes_per_block = num_layers * layer_block_bytes, layer_block_bytes =
 *  num_kv_heads * block_size * head_dim * element_size_bytes.
 * Errors: CF_ENOMEM where the reference throws OutOfPagesException,
 * CF_ERANGE for an unknown sequence id (the reference's runtime_error) or a
 * batch beyond max_supported_batch_size / max_blocks_per_sequence.
 * ---------------------------------------------------------------------- */
typedef struct cf_kv_config {      /* KVCacheConfig, paged_kv_cache.h:36-46 */
  uint32_t num_layers;
  uint32_t num_kv_heads;
  uint32_t head_dim;
  uint32_t block_size;
  uint64_t element_size_bytes;
  uint64_t total_gpu_blocks;
  int32_t enable_prefix_caching;
  uint64_t max_supported_batch_size;
  uint64_t max_blocks_per_sequence;
} cf_kv_config;

typedef struct cf_kv_stats {       /* KVCacheStats, paged_kv_cache.h:63-75 */
  uint64_t total_blocks, free_blocks, allocated_blocks, cached_prefix_blocks;
  uint64_t total_memory_bytes, used_memory_bytes;
  double pool_utilization_ratio;
  uint32_t active_sequences_count;
  uint64_t prefix_cache_hits, prefix_cache_misses, lru_evictions_count;
} cf_kv_stats;

typedef struct cf_kvcache cf_kvcache;

/* PagedKVCache(config, allocator) (paged_kv_cache.cpp:9-60); NULL on bad config. */
cf_kvcache *cf_kvcache_create(const cf_kv_config *cfg, void *key_pool, void *val_pool);
void cf_kvcache_destroy(cf_kvcache *h);
/* register_sequence_with_prefix (paged_kv_cache.cpp:167-253) */
int cf_kvcache_register_sequence(cf_kvcache *h, uint64_t seq, const int32_t *tokens, uint32_t n,
                                 uint32_t *matched_out);
/* append_tokens (:255-286) */
int cf_kvcache_append_tokens(cf_kvcache *h, uint64_t seq, uint32_t n);
/* append_tokens for seqs[i] with n[i] tokens (n <= 0 skipped), in index
 * order -- the engine's per-token commit loop (cudaforge/engine.py:222-224)
 * in one call; stops at the first error. */
int cf_kvcache_append_batch(cf_kvcache *h, const uint64_t *seqs, const int32_t *n, uint32_t batch);
/* unregister_sequence (:288-299) */
int cf_kvcache_unregister_sequence(cf_kvcache *h, uint64_t seq);
/* fork_sequence (:301-316) */
int cf_kvcache_fork_sequence(cf_kvcache *h, uint64_t parent, uint64_t child);
/* get_block_table (:398-407): copies up to cap ids, *len = table length */
int cf_kvcache_get_block_table(cf_kvcache *h, uint64_t seq, int32_t *out, uint32_t cap, uint32_t *len);
/* prepare_batch_metadata (:318-396), host half: tables[batch][*max_blocks_out]
 * padded with -1 (tables may be NULL to query the width), context_lens[batch].
 * The caller copies both to the device on its stream. */
int cf_kvcache_prepare_batch(cf_kvcache *h, const uint64_t *seqs, uint32_t batch, int32_t *tables,
                             uint32_t table_cap, int32_t *context_lens, uint32_t *max_blocks_out);
/* get_stats (:423-445) */
int cf_kvcache_get_stats(cf_kvcache *h, cf_kv_stats *s);
/* The free stack, bottom to top (the next block handed out is out[n - 1]),
 * for a device-resident copy (cf_kv_append_device).  *n = its size; at most
 * cap entries are written.  No reference counterpart (the reference's stack
 * is private, paged_kv_cache.cpp:44-53). */
int cf_kvcache_export_free_stack(cf_kvcache *h, int32_t *out, uint32_t cap, uint32_t *n);
/* get_key_block_ptr / get_value_block_ptr (:409-421) */
void *cf_kvcache_key_block_ptr(cf_kvcache *h, int32_t block, uint32_t layer);
void *cf_kvcache_value_block_ptr(cf_kvcache *h, int32_t block, uint32_t layer);

/* ------------------------------------------------------------------------
 * Device view of the paged KV pools (the KVCacheBatchDescriptor contract,
 * csrc/include/cudaforge/memory/paged_kv_cache.h:81-94).
 * ---------------------------------------------------------------------- */
typedef struct cf_kv_layout {
  void *key_pool;        /* [total_blocks][num_layers][num_kv_heads][block_size][head_dim] */
  void *val_pool;
  int64_t total_blocks;
  int32_t num_layers, num_kv_heads, head_dim, block_size;
  int32_t dtype;         /* CF_BF16 or CF_F16 */
} cf_kv_layout;

/* ------------------------------------------------------------------------
 * Paged verify attention over the cached context plus R new rows.
 *
 * Replaces the reference attention launchers launch_flash_attn_v2
 * (csrc/include/cudaforge/kernels/flash_attn_v2.h:12-31,
 *  csrc/kernels/cuda/flash_attn_v2.cu:197-221) and flash_attn_triton
 * (csrc/kernels/triton/flash_attn_triton.py:112-172), which take contiguous
 * [B, H, S, D] tensors and a causal flag; this one reads the paged pool
 * through block tables, handles grouped-query heads and a tree mask.
 * q: row (b*R + r), head hq at q + (b*R + r)*q_row_stride + hq*head_dim;
 * k_new / v_new: this step's new rows [B][R][Hkv][D] for `layer` (or
 *   [L][B][R][Hkv][D] when new_kv_all_layers != 0);
 * block_tables [B][max_blocks] (-1 padded), context_lens [B] = cached tokens
 *   (the new rows follow them); max_context = max over context_lens (host);
 * tree_mask NULL: causal chain (new row r sees new rows j <= r); else
 *   [B][R][mask_words] uint64 bits, bit j of row r = r may see new row j;
 * out: same addressing as q (out_row_stride); scale 0 = head_dim^-1/2.
 * head_dim 64 or 128, block_size 16.  Split-KV partials use `workspace`
 * (cf_attention_workspace_bytes); num_splits 0 = automatic.
 * A block id outside [0, total_blocks) sets *status = CF_ERANGE and that page
 * reads block 0; an expired pipeline wait sets CF_ETIMEOUT.
 * bf16, head_dim 128, rows * (num_q_heads / num_kv_heads) >= 128, rows <= 128,
 * num_splits <= 1 and a 16-byte aligned out: a tcgen05 kernel (S, P and O in
 * TMEM; no workspace); other shapes: the warp-MMA kernel.
 * ---------------------------------------------------------------------- */
typedef struct cf_attn_args {
  cf_kv_layout kv;
  int32_t layer;
  int32_t batch, rows, num_q_heads;
  const void *q;
  int64_t q_row_stride;
  const void *k_new, *v_new;
  int32_t new_kv_all_layers;
  const int32_t *block_tables;
  int32_t max_blocks;
  const int32_t *context_lens;
  int32_t max_context;
  const uint64_t *tree_mask;
  int32_t mask_words;
  void *out;
  int64_t out_row_stride;
  float scale;
  int32_t num_splits;
  void *workspace;
  size_t workspace_bytes;
  int32_t *status;
  uint64_t timeout_ns;
  uint64_t *trace;       /* optional profiling aid: [4][1024] SM-clock stamps of CTA 0 */
} cf_attn_args;

size_t cf_attention_workspace_bytes(const cf_attn_args *args);
int cf_verify_attention(const cf_attn_args *args, void *stream);

/* ------------------------------------------------------------------------
 * Accepted-KV commit: copy the surviving new rows of every layer from the
 * step's scratch into their paged slots.
 *
 * The reference never writes KV (its engine only advances page tables,
 * cudaforge/engine.py:222-224 -> PagedKVCache::append_tokens,
 * paged_kv_cache.cpp:255-286); this is the device half of that commit.
 * For sequence b, committed token j < n_b (n_b = n_commit[b] + n_commit_add)
 * comes from scratch row row_index[b][j] (identity when NULL; tree paths pass
 * the accepted node rows) and lands at position start_pos[b] + j, i.e. slot
 * (pos % block_size) of block block_tables[b][pos / block_size], for every
 * layer in [layer_begin, layer_begin + layer_count) and every kv head.
 * k_new / v_new: [L][B][R][Hkv][D].  Invalid destinations set *status =
 * CF_ERANGE and are skipped.
 * ---------------------------------------------------------------------- */
typedef struct cf_kv_commit_args {
  cf_kv_layout kv;
  int32_t batch, rows;
  int32_t layer_begin, layer_count;
  const void *k_new, *v_new;
  const int32_t *n_commit;
  int32_t n_commit_add;
  const int32_t *row_index;
  const int32_t *start_pos;
  const int32_t *block_tables;
  int32_t max_blocks;
  int32_t *status;
} cf_kv_commit_args;

int cf_kv_commit(const cf_kv_commit_args *args, void *stream);

/* ---------------------------------------------------------------------------
 * Device-resident page-table growth: PagedKVCache::append_tokens
 * (csrc/src/memory/paged_kv_cache.cpp:255-286) for a batch, in batch order,
 * on the GPU (one launch, graph-capturable, no host round trip).  Sequence b
 * grows by max(n_append[b], 0) + n_add tokens; context_lens[b] is its length
 * before the growth, table_len[b] its number of blocks (updated), tables its
 * fixed-width row [batch][max_blocks] (new blocks appended), free_stack /
 * *free_top a device copy of the cache's free stack (cf_kvcache_export_free_stack;
 * blocks are popped from the top, as the host cache pops them).  Identical
 * tables to cf_kvcache_append_batch when no eviction is needed; when the stack
 * runs short or a row would exceed max_blocks nothing changes and *status
 * records CF_ENOMEM / CF_ERANGE.  The host cache is brought up to date by
 * cf_kvcache_append_batch with the same counts (same result).
 * ------------------------------------------------------------------------- */
typedef struct cf_kv_append_args {
  int32_t batch;
  int32_t block_size;
  const int32_t *n_append;    /* [batch] (device; negative counts as 0) */
  int32_t n_add;              /* added to every count (1: num_accepted + 1) */
  const int32_t *context_lens;/* [batch] tokens before the growth (device) */
  int32_t *table_len;         /* [batch] blocks per row (device, updated) */
  int32_t *tables;            /* [batch][max_blocks] (device, -1 past table_len) */
  int32_t max_blocks;
  int32_t *free_stack;        /* device copy, bottom to top */
  int32_t *free_top;          /* [1] entries in use (device, updated) */
  int32_t *status;            /* optional status word */
} cf_kv_append_args;

int cf_kv_append_device(const cf_kv_append_args *args, void *stream);

/* ------------------------------------------------------------------------
 * Fused elementwise pieces of the verify forward (bf16 or fp16 `dtype`).
 * ---------------------------------------------------------------------- */
/* out[m, :] = table[ids[m], :]  (ids outside [0, vocab) give zero rows) */
int cf_embedding(const int32_t *ids, int32_t m, const void *table, int32_t vocab, int32_t dim, void *out,
                 int32_t dtype, void *stream);
/* RMSNorm: out = x * rsqrt(mean(x^2) + eps) * w, fp32 math
 * (csrc/kernels/cuda/fused_rmsnorm.cu:53-144 without the residual add, which
 * the producing GEMM epilogue fuses). Rows of `dim` elements, pitches in
 * elements. */
int cf_rmsnorm(const void *x, int64_t ldx, const void *w, void *out, int64_t ldo, int32_t m, int32_t dim,
               float eps, int32_t dtype, void *stream);
/* Half-split RoPE (csrc/include/cudaforge/kernels/rope.cuh:13-31:
 * o1 = x1 c - x2 s, o2 = x1 s + x2 c; angle = pos * base^(-2i/D)) on the
 * fused QKV rows qkv[m][(Hq + 2 Hkv) * D] (m = b*R + r, position pos[m]):
 * q is rotated in place; rotated k and plain v go to k_new / v_new
 * [B][R][Hkv][D] (this layer's slice).  D a multiple of 16, at most 256;
 * qkv, k_new and v_new 16-byte aligned. */
int cf_rope_qkv(void *qkv, int64_t ld, int32_t m, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                const int32_t *pos, float base, void *k_new, void *v_new, int32_t dtype, void *stream);
/* SwiGLU: out[m, j] = silu(gu[m, j]) * gu[m, ffn + j] */
int cf_silu_mul(const void *gu, int64_t ldg, void *out, int64_t ldo, int32_t m, int32_t ffn, int32_t dtype,
                void *stream);

/* Split-K consumers (partials from *_gemm_partials, m rows, n = row width):
 * cf_splitk_rmsnorm: y = reduce(+ residual) written (in place over the
 *   residual is allowed), out = RMSNorm(y) * w as cf_rmsnorm;
 * cf_splitk_rope_qkv: cf_rope_qkv on the reduced QKV rows (n = (Hq + 2 Hkv)
 *   * head_dim; rotated q is written to qkv, k / v to k_new / v_new);
 * cf_splitk_silu_mul: cf_silu_mul on the reduced gate|up rows (n = 2 ffn).
 * Bit-identical to the reduction followed by the plain op. */
int cf_splitk_rmsnorm(const float *partials, int32_t splits, int32_t m, int32_t n, const void *residual,
                      int64_t ldr, void *y, int64_t ldy, const void *w, void *out, int64_t ldo, float eps,
                      int32_t dtype, void *stream);
int cf_splitk_rope_qkv(const float *partials, int32_t splits, int32_t m, void *qkv, int64_t ld, int32_t num_q_heads,
                       int32_t num_kv_heads, int32_t head_dim, const int32_t *pos, float base, void *k_new,
                       void *v_new, int32_t dtype, void *stream);
int cf_splitk_silu_mul(const float *partials, int32_t splits, int32_t m, int32_t ffn, void *out, int64_t ldo,
                       int32_t dtype, void *stream);

/* ---------------------------------------------------------------------------
 * Host speculative verification engine.  Replaces the reference's native
 * SpeculativeEngine (csrc/include/cudaforge/scheduler/speculative.h:14-85,
 * csrc/src/scheduler/speculative.cpp:8-150, bound at
 * csrc/bindings/pybind_module.cpp:199-239): a configuration plus a
 * std::mt19937 stream seeded with rng_seed, drawn with
 * std::uniform_real_distribution<float>(0, 1) in the reference's order, so a
 * sequence of calls gives the reference engine's outputs.  Per-sequence
 * probability rows (host memory, possibly ragged: row i has lens[i] floats).
 * cf_spec_engine_verify: stochastic (greedy = 0; n_draft must equal k,
 * speculative.cpp:58-62) or greedy (greedy = 1; draft rows unused,
 * speculative.cpp:105-150); n_target >= k + 1 (CF_EINVAL otherwise).
 * out_accepted[0..num_accepted) are the accepted drafts, out_final_token the
 * correction / bonus / EOS token.  A draft token outside its rows returns
 * CF_ERANGE (the reference reads out of bounds).  Calls on one engine are
 * serialised by its mutex.  cf_spec_engine_draw_uniforms: the next n values
 * of the engine's stream (for cf_accept_sample's uniforms).
 * ------------------------------------------------------------------------- */
typedef struct cf_spec_config {
  int64_t gamma;       /* draft tokens per step (K); stored, as in the reference */
  float temperature;   /* stored; the probability rows are already softmaxed */
  float top_p;         /* stored; unused by verification (speculative.h:17) */
  uint64_t rng_seed;   /* seeds the engine's stream once, at creation */
} cf_spec_config;

typedef struct cf_spec_engine cf_spec_engine;

int cf_spec_engine_create(const cf_spec_config *config, cf_spec_engine **out);
void cf_spec_engine_destroy(cf_spec_engine *engine);
int cf_spec_engine_set_config(cf_spec_engine *engine, const cf_spec_config *config);
int cf_spec_engine_get_config(cf_spec_engine *engine, cf_spec_config *out);
int cf_spec_engine_verify(cf_spec_engine *engine, int32_t k, const int32_t *draft_tokens,
                          const float *const *draft_rows, const int64_t *draft_lens, int32_t n_draft,
                          const float *const *target_rows, const int64_t *target_lens, int32_t n_target,
                          int32_t eos_token_id, int32_t greedy, int32_t *out_accepted,
                          int32_t *out_num_accepted, int32_t *out_final_token, int32_t *out_eos);
int cf_spec_engine_draw_uniforms(cf_spec_engine *engine, int64_t n, float *out);

#ifdef __cplusplus
}
#endif
#endif /* CF_API_H_ */
