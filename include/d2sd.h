/*
 * d2sd.h - C ABI of the B200 (sm_100a) tree-verification hot path of D2-SD.
 *
 * Every entry point takes plain device pointers, element strides, sizes and a
 * cudaStream_t (passed as void*), returns an int status (D2SD_OK == 0) and
 * never allocates device memory, never synchronises the host and never frees
 * anything: workspaces are passed in by the caller. All work is enqueued on the
 * caller's stream, so every launch is capturable in a CUDA graph.
 *
 * Reference call sites each entry point replaces (paths inside catnanami/D2-SD):
 *   d2sd_prefix_plan / d2sd_prefix_attention
 *       flashinfer.single_prefill_with_kv_cache(q_all, k_shared, v_shared,
 *       causal=False, return_lse=True)  generation/verification.py:145-148,
 *       model/dflash.py:112-115 (level 1 of the cascade).
 *   d2sd_suffix_merge
 *       CascadeGraphRunner.run (model/cascade_graph.py:76-112, the graph body at
 *       :52-60: per-branch single_prefill + merge_state_in_place), the loop at
 *       generation/verification.py:158-165 and the GPT-OSS sink rescale at
 *       generation/verification.py:173-176.
 *   d2sd_cascade_attention_f32
 *       the same cascade in fp32 (BASELINE config 1's fp32 contract).
 *   d2sd_merge_state
 *       flashinfer.merge_state_in_place(v, s, v_other, s_other)
 *       model/cascade_graph.py:58-60, generation/verification.py:163-165.
 *   d2sd_verify_accept
 *       the greedy acceptance walk generation/d3_generator.py:204-225 with
 *       model/utils.py:28-32 (sample, temperature 0), and its single-branch
 *       form generation/dflash_generator.py:110-125.
 *   d2sd_verify_accept_batch / d2sd_verify_accept_sharded
 *       the same walk for a batch of requests in one launch, and its
 *       vocabulary-sharded multi-GPU form (no reference counterpart: the
 *       reference verifies one request on one GPU).
 *   d2sd_commit_kv / d2sd_commit_kv_batch
 *       the accepted-branch KV append generation/d3_generator.py:227-232 (one
 *       request, or a batch of requests sharing one page pool).
 *   d2sd_qk_norm_rope
 *       the step before the attention, generation/verification.py:113-124:
 *       attn.q_norm / attn.k_norm (transformers' Qwen3RMSNorm; skipped for
 *       GPT-OSS) and rope_apply (_apply_rotary_pos_emb_qwen3 :21-28 or
 *       _apply_rotary_pos_emb_gpt_oss :31-43) on the block's q and k.
 *   d2sd_commit_kv_hidden
 *       the same, fused with the draft's context-feature gather
 *       generation/d3_generator.py:239 (model/utils.py:17-26,
 *       extract_context_feature, indexed [valid_block, :acceptance_length]).
 */
#ifndef D2SD_H_
#define D2SD_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define D2SD_OK 0
#define D2SD_ERR_INVALID_ARGUMENT 1  /* shape, stride, dtype or pointer rejected */
#define D2SD_ERR_UNSUPPORTED 2       /* valid request outside the built kernels */
#define D2SD_ERR_WORKSPACE 3         /* workspace / plan buffer too small */
#define D2SD_ERR_CUDA 4              /* a CUDA runtime/driver call failed */
#define D2SD_ERR_NO_DEVICE 5         /* no sm_100 device current */

/* ---- dtypes ------------------------------------------------------------ */
#define D2SD_DTYPE_F32 0
#define D2SD_DTYPE_BF16 1
#define D2SD_DTYPE_F16 2

/* ---- KV cache formats (d2sd_prefix_attention, d2sd_commit_kv) ---------- */
/* Rows: a key/value row of head_dim elements is contiguous; pages or tokens,
 * slots and heads are addressed through the given strides. */
#define D2SD_KV_ROWS 0
/* UMMA pages: page_size 16; the 16 x head_dim block of one (page, head) is
 * stored in the order [2 row groups][head_dim/8 chunks][8 rows][8 elements]
 * (the tensor core's no-swizzle core-matrix order), so one block is a single
 * contiguous copy that the tensor core reads in place. Element (page, slot r,
 * head h, d) sits at page*stride_page + h*stride_head + ((r/8)*(head_dim/8)
 * + d/8)*64 + (r%8)*8 + d%8. */
#define D2SD_KV_UMMA_PAGES 1

/* ---- suffix mask modes (d2sd_suffix_merge) ----------------------------- */
#define D2SD_MASK_NONE 0    /* every block token sees the whole block (DTA) */
#define D2SD_MASK_CAUSAL 1  /* token t sees tokens 0..t of its block (verify) */
#define D2SD_MASK_CUSTOM 2  /* token t sees the set bits of mask[block][t] */

/* ---- sink modes (d2sd_suffix_merge) ------------------------------------ */
#define D2SD_SINK_NONE 0
/* out *= sigmoid(lse2 - sink): the formula of generation/verification.py:173-176,
 * where lse2 is the base-2 log-sum-exp and sink is a natural-log logit. */
#define D2SD_SINK_REFERENCE 1
/* out *= sigmoid(lse2 * ln2 - sink): the softmax-with-sink of the HF GPT-OSS
 * attention (an extra exp(sink) term in the denominator). */
#define D2SD_SINK_EXACT 2

/* Library version (major*10000 + minor*100 + patch). */
int d2sd_version(void);

/* Human-readable text of the last error raised on the calling host thread. */
const char* d2sd_last_error(void);

/* Number of int32 entries a prefix plan needs (upper bound). */
int64_t d2sd_prefix_plan_capacity(int32_t num_requests, int32_t num_qo_heads,
                                  int32_t num_kv_heads, int32_t num_ctas,
                                  int64_t total_q_tokens);

/* Host-side work partition of the shared-prefix attention.
 *
 * Request r has q_tokens[r] query tokens (rows q_token_offset[r] ..
 * q_token_offset[r]+q_tokens[r]-1 of the Q tensor) and attends the prefix keys
 * kv_start[r] .. kv_end[r]-1 (absolute positions inside its KV sequence; the
 * sliding-window truncation of generation/verification.py:130-135 is
 * kv_start = kv_end - window). num_ctas is the persistent grid (the SM count).
 * The plan is written into plan[0 .. capacity) on the HOST; copy it to device
 * memory before d2sd_prefix_attention. *num_partial_slots receives the number of
 * 128-row partial-state slots the launch writes (workspace sizing).
 * Pure host code: callable without a GPU. */
int d2sd_prefix_plan(const int32_t* q_tokens, const int32_t* q_token_offset,
                     const int32_t* kv_start, const int32_t* kv_end,
                     int32_t num_requests, int32_t num_qo_heads,
                     int32_t num_kv_heads, int32_t num_ctas, int32_t* plan,
                     int64_t capacity, int32_t* num_partial_slots);

/* Bytes of partial state per slot: the normalised O of 128 rows in bf16
 * ([128][head_dim]) followed by their 128 base-2 LSEs in fp32. */
int64_t d2sd_partial_slot_bytes(int32_t head_dim);

/* Shared-prefix (level-1) attention on tcgen05/TMEM.
 *
 * q:        bf16 [tokens, num_qo_heads, head_dim], strides in elements
 *           (q_stride_token, q_stride_head), dim stride 1.
 * kv_format: D2SD_KV_ROWS or D2SD_KV_UMMA_PAGES (then page_table is required,
 *           page_size is 16 and kv_stride_slot is unused).
 * k, v:     bf16 KV of the prefix. Paged (page_table != NULL): element
 *           (page, slot, head, d) at page*kv_stride_page + slot*kv_stride_slot
 *           + head*kv_stride_head + d, page_size slots per page, num_pages pages;
 *           request r's position p lives in page
 *           page_table[page_table_offset[r] + p / page_size].
 *           Contiguous (page_table == NULL): element (token, head, d) at
 *           token*kv_stride_slot + head*kv_stride_head + d with num_pages
 *           tokens in total, and request r's position p is token
 *           page_table_offset[r] + p.
 * plan:     device copy of d2sd_prefix_plan's output.
 * partial:  device workspace of num_partial_slots * d2sd_partial_slot_bytes.
 * Writes, for every query row, the normalised prefix output and its base-2
 * log-sum-exp (the FlashInfer convention) into the partial slots; the rows are
 * combined by d2sd_suffix_merge. head_dim is 64 or 128; the group size
 * num_qo_heads / num_kv_heads divides 128; page_size is a multiple of 8 that
 * divides 128. Pool slots past a request's last position must hold finite
 * values (the pools this library allocates are zero-initialised).
 * status (device int32, may be NULL) receives a nonzero code if a pipeline
 * wait inside the kernel ran out of time; the kernel then returns early. */
int d2sd_prefix_attention(const void* q, int64_t q_stride_token,
                          int64_t q_stride_head, int64_t num_q_tokens,
                          const void* k, const void* v, int64_t kv_stride_page,
                          int64_t kv_stride_slot, int64_t kv_stride_head,
                          int32_t page_size, int32_t kv_format,
                          int64_t num_pages, const int32_t* page_table,
                          const int32_t* page_table_offset,
                          int32_t num_qo_heads, int32_t num_kv_heads,
                          int32_t head_dim, float sm_scale,
                          const int32_t* plan, int32_t num_ctas,
                          void* partial, int64_t partial_bytes,
                          int32_t* status, void* stream);

/* Level-2 (per-block suffix) attention fused with the log-sum-exp merge of
 * both levels and, optionally, the attention-sink rescale.
 *
 * Tokens are grouped in blocks of block_len consecutive tokens (one block per
 * draft branch). q, k_local, v_local: [num_blocks*block_len, heads, head_dim]
 * with (token, head) element strides; k_local/v_local may be NULL for a pure
 * merge (no level 2). q may have its own block stride q_stride_block (0 =
 * block_len * q_stride_token): query (block b, token t, head h) is read at
 * b*q_stride_block + t*q_stride_token + h*q_stride_head, so a per-block view
 * such as [B, Hq, T, D] transposed to [B, T, Hq, D] (model/dflash.py:109,124)
 * is read in place.
 * Prefix state, one of:
 *   - partial != NULL: merged from the slots written by d2sd_prefix_attention;
 *     prefix_token[t] (device, may be NULL = identity) maps block token t to
 *     its row in the prefix-attention Q tensor; plan is the device plan.
 *   - partial == NULL, prefix_out != NULL: a dense state (out [tokens, Hq, D]
 *     in the q dtype, lse [tokens, Hq] fp32 base-2) as produced by
 *     single_prefill_with_kv_cache; the CascadeGraphRunner.run in-place form.
 *   - neither: no prefix (level 2 alone).
 * out/lse receive the merged output (q dtype) and base-2 LSE; they may alias
 * prefix_out/prefix_lse. mask_mode is a D2SD_MASK_*, custom_mask is
 * uint64 [num_blocks*block_len] (bit j = token may see block token j).
 * sinks: fp32 [num_qo_heads] or NULL; sink_mode a D2SD_SINK_*.
 * With k_local, q/k_local/v_local must be 16-byte aligned with token and head
 * strides that are multiples of 8 elements (they are read by TMA), and
 * block_len <= 64. status (device int32, may be NULL) receives a nonzero code
 * if a wait inside the kernel ran out of time. */
int d2sd_suffix_merge(const void* q, int64_t q_stride_token,
                      int64_t q_stride_head, int64_t q_stride_block,
                      const void* k_local,
                      const void* v_local, int64_t kv_stride_token,
                      int64_t kv_stride_head, int32_t num_blocks,
                      int32_t block_len, int32_t mask_mode,
                      const uint64_t* custom_mask, const void* partial,
                      const int32_t* plan, const int32_t* prefix_token,
                      const void* prefix_out, int64_t prefix_out_stride_token,
                      int64_t prefix_out_stride_head, const float* prefix_lse,
                      int64_t prefix_lse_stride_token, void* out,
                      int64_t out_stride_token, int64_t out_stride_head,
                      float* lse, int64_t lse_stride_token,
                      const float* sinks, int32_t sink_mode,
                      int32_t num_qo_heads, int32_t num_kv_heads,
                      int32_t head_dim, int32_t dtype, float sm_scale,
                      int32_t* status, void* stream);

/* d2sd_suffix_merge with the head-sharded output exchange fused into its
 * epilogue (KV-head sharding, one process per GPU). It replaces
 * torch.distributed.all_gather_into_tensor of each rank's attention output
 * (the one collective of the KV-head-sharded verify step); the reference runs
 * on one GPU and has no counterpart.
 *
 * epoch counts this exchange's calls (1, 2, ...), identical on every rank, and
 * all ranks launch the same shapes in the same call. Outputs are double
 * buffered by the epoch's parity: out_ptrs is a device array of 2 * world
 * pointers, [parity][rank] (peer ones mapped with d2sd_ipc_open), and every
 * merged row is stored into the head slice [head_offset, head_offset +
 * num_qo_heads) of the `world` buffers out_ptrs[(epoch & 1) * world + r], with
 * element strides (peer_stride_token, peer_stride_head); `out` is not written.
 * counters: device array of `world` pointers to each rank's control block of 8
 * uint64 words, zero before the first call: [0], [1] arrivals of even / odd
 * epochs, [2] a CTA ticket, [3] total and [5] longest time (ns) this rank's
 * signalling CTA waited for its peers, [4] the number of such waits.
 * The last CTA of the call signals every rank once and waits until every rank
 * has signalled this rank, so the kernel completes only once every rank's rows
 * have landed in this rank's buffer of this parity.
 * Consumption contract: the rows of call e may be read by work enqueued on this
 * rank's stream after call e and before call e + 1 (e.g. o_proj); peers write
 * call e + 2 into the same buffer only after this rank's call e + 1 has begun
 * its epilogue. The wait is bounded (2 s); on time-out *status receives 3 and
 * the exchange must be abandoned. status is required. Rows are stored with
 * 16-byte vectors: the output bases must be 16-byte aligned and the strides
 * multiples of 8. */
int d2sd_suffix_merge_gather(const void* q, int64_t q_stride_token,
                             int64_t q_stride_head, int64_t q_stride_block,
                             const void* k_local,
                             const void* v_local, int64_t kv_stride_token,
                             int64_t kv_stride_head, int32_t num_blocks,
                             int32_t block_len, int32_t mask_mode,
                             const uint64_t* custom_mask, const void* partial,
                             const int32_t* plan, const int32_t* prefix_token,
                             const void* prefix_out, int64_t prefix_out_stride_token,
                             int64_t prefix_out_stride_head, const float* prefix_lse,
                             int64_t prefix_lse_stride_token, void* out,
                             int64_t out_stride_token, int64_t out_stride_head,
                             float* lse, int64_t lse_stride_token,
                             const float* sinks, int32_t sink_mode,
                             int32_t num_qo_heads, int32_t num_kv_heads,
                             int32_t head_dim, int32_t dtype, float sm_scale,
                             void* const* out_ptrs, uint64_t* const* counters,
                             int32_t world, int32_t rank, int32_t head_offset,
                             int64_t peer_stride_token, int64_t peer_stride_head,
                             int64_t epoch, int32_t* status, void* stream);

/* CUDA IPC of a device buffer for the peer exchange: the 64-byte handle of the
 * allocation holding ptr and ptr's byte offset inside it. */
int d2sd_ipc_handle(const void* ptr, void* handle_out, int64_t* offset_out);
/* Maps a peer's handle into this process (peer access enabled on demand);
 * *base_out receives the allocation's base address here. */
int d2sd_ipc_open(const void* handle, void** base_out);
/* Unmaps a base address returned by d2sd_ipc_open. */
int d2sd_ipc_close(void* base);

/* In-place merge of two attention states (v,s) <- merge((v,s),(v_other,s_other))
 * with base-2 LSEs: v [n, heads, head_dim] (dtype), s [n, heads] fp32. */
int d2sd_merge_state(void* v, int64_t v_stride_token, int64_t v_stride_head,
                     float* s, int64_t s_stride_token, const void* v_other,
                     int64_t vo_stride_token, int64_t vo_stride_head,
                     const float* s_other, int64_t so_stride_token, int64_t n,
                     int32_t heads, int32_t head_dim, int32_t dtype,
                     void* stream);

/* Workspace bytes for d2sd_verify_accept; must be zeroed once before its
 * first use (the kernel leaves it zeroed again on exit). */
int64_t d2sd_verify_accept_workspace_size(int32_t num_branches,
                                          int32_t block_len, int64_t vocab);

/* Greedy multi-branch acceptance over target logits in one launch, no host
 * synchronisation.
 * logits: [num_branches, block_len, vocab] (dtype F32/BF16/F16), strides in
 *         elements (branch, pos), vocab stride 1.
 * block_ids: int64 [num_branches, block_len] (branch, pos strides); column 0
 *         is the anchor token.
 * result (device int32[2]): result[0] = acceptance_length in [1, block_len]
 *         (includes the bonus token), result[1] = the winning branch.
 * accepted_ids (device int64[block_len]): the accepted tokens, bonus last;
 *         entries at and after acceptance_length are set to -1.
 * argmax_out (device int64[num_branches*block_len] or NULL): the per-position
 *         argmax of every branch (first maximal index, NaN counts as maximal).
 * num_branches <= 64. */
int d2sd_verify_accept(const void* logits, int32_t dtype,
                       int32_t num_branches, int32_t block_len, int64_t vocab,
                       int64_t stride_branch, int64_t stride_pos,
                       const int64_t* block_ids, int64_t ids_stride_branch,
                       int64_t ids_stride_pos, int32_t* result,
                       int64_t* accepted_ids, int64_t* argmax_out,
                       void* workspace, int64_t workspace_bytes, void* stream);

/* Workspace bytes for d2sd_verify_accept_batch / _sharded (same rules as
 * d2sd_verify_accept_workspace_size). */
int64_t d2sd_verify_accept_batch_workspace_size(int32_t num_requests,
                                                int32_t num_branches,
                                                int32_t block_len, int64_t vocab);

/* Greedy acceptance of num_requests independent requests in one launch
 * (batched serving): the walk of generation/d3_generator.py:204-225 for each
 * request, as d2sd_verify_accept does for one. Request q's logits are
 * [num_branches, block_len, vocab] at q*stride_request elements, its block ids
 * at q*ids_stride_request; result is int32 [num_requests][2] ({acceptance
 * length, branch} per request), accepted_ids int64 [num_requests][block_len],
 * argmax_out (or NULL) int64 [num_requests][num_branches][block_len].
 * num_requests * num_branches * block_len <= 4096. */
int d2sd_verify_accept_batch(const void* logits, int32_t dtype,
                             int32_t num_requests, int32_t num_branches,
                             int32_t block_len, int64_t vocab,
                             int64_t stride_request, int64_t stride_branch,
                             int64_t stride_pos, const int64_t* block_ids,
                             int64_t ids_stride_request,
                             int64_t ids_stride_branch, int64_t ids_stride_pos,
                             int32_t* result, int64_t* accepted_ids,
                             int64_t* argmax_out, void* workspace,
                             int64_t workspace_bytes, void* stream);

/* Vocabulary-sharded form of d2sd_verify_accept_batch for KV-head-sharded
 * verification on several GPUs (one process per GPU): rank `rank` of `world`
 * passes only its slice of every logits row, columns [vocab_offset,
 * vocab_offset + vocab_slice) of the full vocabulary, with the slices of ranks
 * 0..world-1 in ascending order. Each rank scans its slice; the CTA that
 * finishes last stores every row's (max, first index) record into every
 * rank's record buffer over NVLink, signals each rank once, waits (bounded,
 * 2 s) for every rank's records and combines them in rank order, which yields
 * the first maximal index of the whole row (torch.argmax). Every rank then runs
 * the same walks and writes the same results (indices are full-vocabulary).
 * The reference runs acceptance on one GPU and has no counterpart; this
 * replaces a replicated full-vocabulary scan on every rank.
 * record_ptrs: device array of 2 * world pointers, [epoch parity][rank], each a
 * buffer of world * rows 16-byte records (rows = num_requests * num_branches *
 * block_len); control_ptrs: device array of world pointers to each rank's
 * control block (8 uint64, zero before the first call; [0], [1] are the
 * arrival counters of even / odd epochs). epoch counts the calls (1, 2, ...),
 * identical on every rank. status is required and receives 3 if a rank did
 * not arrive in time. */
int d2sd_verify_accept_sharded(const void* logits, int32_t dtype,
                               int32_t num_requests, int32_t num_branches,
                               int32_t block_len, int64_t vocab_slice,
                               int64_t vocab_offset, int64_t stride_request,
                               int64_t stride_branch, int64_t stride_pos,
                               const int64_t* block_ids,
                               int64_t ids_stride_request,
                               int64_t ids_stride_branch, int64_t ids_stride_pos,
                               int32_t* result, int64_t* accepted_ids,
                               int64_t* argmax_out, void* workspace,
                               int64_t workspace_bytes,
                               void* const* record_ptrs,
                               uint64_t* const* control_ptrs, int32_t world,
                               int32_t rank, int64_t epoch, int32_t* status,
                               void* stream);

/* d2sd_verify_accept without a workspace argument and without allocating.
 * No counterpart in the reference: it exists for callers that cannot provide
 * or allocate device memory at call time -- a runtime whose memory planner owns
 * every allocation, or code running inside a CUDA graph capture. The scratch is
 * a static 256 KiB device array in the library (held by every GPU that loads
 * it until exit); shapes needing more are rejected with D2SD_ERR_UNSUPPORTED.
 * Its device address is looked up on the first call per device (and again
 * when the device's context has changed, e.g. after cudaDeviceReset), so make
 * that first call before any stream capture. All calls share the array: calls
 * that overlap on the GPU race. Other arguments and results as
 * d2sd_verify_accept. */
int d2sd_verify_accept_noalloc(const void* logits, int32_t dtype,
                               int32_t num_branches, int32_t block_len,
                               int64_t vocab, int64_t stride_branch,
                               int64_t stride_pos, const int64_t* block_ids,
                               int64_t ids_stride_branch, int64_t ids_stride_pos,
                               int32_t* result, int64_t* accepted_ids,
                               int64_t* argmax_out, void* stream);

/* Accepted-branch KV commit for all layers in one launch.
 * layer_ptrs: device array of num_layers*4 pointers
 *   {new_k, new_v, cache_k, cache_v} per layer.
 * new_k/new_v: [num_branches, heads, block_len, head_dim] with element strides
 *   (new_stride_branch, new_stride_head, new_stride_token), dim stride 1.
 * cache (cache_format D2SD_KV_ROWS): position p of head h at
 *   page_table[p / page_size]*cache_stride_page + (p % page_size)*cache_stride_slot
 *   + h*cache_stride_head (page_table == NULL: page index p / page_size);
 *   (D2SD_KV_UMMA_PAGES): the element order of d2sd_prefix_attention's UMMA
 *   pages, page_size 16, 16-bit values.
 * accept_result: the device int32[2] {acceptance_length, branch} written by
 *   d2sd_verify_accept; block positions 0..acceptance_length-1 of the winning
 *   branch are written to cache positions cache_len .. cache_len+acc-1, where
 *   cache_len = *cache_len_dev if cache_len_dev != NULL else cache_len_host.
 * elem_bytes is 2 or 4; head_dim*elem_bytes a multiple of 16. */
int d2sd_commit_kv(const void* const* layer_ptrs, int32_t num_layers,
                   int32_t num_kv_heads, int32_t head_dim, int32_t elem_bytes,
                   int32_t block_len, int64_t new_stride_branch,
                   int64_t new_stride_head, int64_t new_stride_token,
                   int64_t cache_stride_page, int64_t cache_stride_slot,
                   int64_t cache_stride_head, int32_t page_size,
                   int32_t cache_format, const int32_t* page_table,
                   const int32_t* accept_result,
                   const int32_t* cache_len_dev, int64_t cache_len_host,
                   void* stream);

/* d2sd_commit_kv for num_requests independent requests in one launch
 * (batched serving; the reference's per-request append of
 * generation/d3_generator.py:227-232). All requests' caches share one pool per
 * layer (layer_ptrs as in d2sd_commit_kv); request q's page table starts at
 * page_table[page_table_offset[q]], its new K/V at q*new_stride_request
 * elements of each layer's new_k/new_v, its acceptance result at
 * accept_results[2q] (as written by d2sd_verify_accept_batch) and its cache
 * length at cache_lens[q] (device int32). */
int d2sd_commit_kv_batch(const void* const* layer_ptrs, int32_t num_layers,
                         int32_t num_requests, int32_t num_kv_heads,
                         int32_t head_dim, int32_t elem_bytes,
                         int32_t block_len, int64_t new_stride_request,
                         int64_t new_stride_branch, int64_t new_stride_head,
                         int64_t new_stride_token, int64_t cache_stride_page,
                         int64_t cache_stride_slot, int64_t cache_stride_head,
                         int32_t page_size, int32_t cache_format,
                         const int32_t* page_table,
                         const int32_t* page_table_offset,
                         const int32_t* accept_results,
                         const int32_t* cache_lens, void* stream);

/* The two-level cascade verify attention in fp32 (the
 * reference's fp32 path, generation/verification.py:127-176 with a float32
 * target, and its CPU torch.sdpa form), for rows that need fp32 end to end
 * instead of the bf16 tensor-core kernels. Each query row (token t of block
 * t / block_len, query head h, kv head h / G) attends the prefix keys
 * [kv_start, prefix_len) of k_prefix/v_prefix ([prefix_len, Hk, D], token and
 * head strides; may be NULL when prefix_len is 0) and the tokens of its own
 * block in k_local/v_local ([tokens, Hk, D], or NULL) under mask_mode; the
 * state is merged with a dense prefix state (prefix_out [tokens, Hq, D],
 * prefix_lse [tokens, Hq] base 2; the CascadeGraphRunner.run form) when given,
 * and scaled by the sink factor of sink_mode. out [tokens, Hq, D] fp32 and lse
 * [tokens, Hq] base 2 (or NULL). Exact expf/logf, fp32 accumulation. head_dim
 * 32, 64 or 128; block_len <= 64 with k_local. */
int d2sd_cascade_attention_f32(
    const float* q, int64_t q_stride_token, int64_t q_stride_head,
    const float* k_prefix, const float* v_prefix, int64_t prefix_stride_token,
    int64_t prefix_stride_head, int32_t prefix_len, int32_t kv_start,
    const float* k_local, const float* v_local, int64_t local_stride_token,
    int64_t local_stride_head, int32_t num_blocks, int32_t block_len,
    int32_t mask_mode, const uint64_t* custom_mask, const float* prefix_out,
    int64_t prefix_out_stride_token, int64_t prefix_out_stride_head,
    const float* prefix_lse, int64_t prefix_lse_stride_token,
    const float* sinks, int32_t sink_mode, float* out, int64_t out_stride_token,
    int64_t out_stride_head, float* lse, int64_t lse_stride_token,
    int32_t num_qo_heads, int32_t num_kv_heads, int32_t head_dim,
    float sm_scale, void* stream);

/* Per-head RMSNorm (optional) and rotary embedding of the block's q and k in
 * one launch, with the 16-bit roundings of the reference's eager expressions:
 *   y = rnd(w * rnd(x * rsqrt(mean(x^2) + eps)))   (when q_weight/k_weight given)
 *   out = rnd(rnd(y * cos) + rnd(rotate_half(y) * sin)).
 * q_in/q_out: [num_tokens, num_qo_heads, head_dim], k_in/k_out: [num_tokens,
 * num_kv_heads, head_dim], element strides (token, head), head_dim contiguous;
 * out may alias in. q_weight/k_weight: [head_dim] in the data dtype, both or
 * neither (GPT-OSS). cos_table/sin_table: [positions, >= head_dim/2] with row
 * stride table_stride, read through their first head_dim/2 columns (a
 * full-width Qwen3 table has equal halves; GPT-OSS's is half-width). Token t
 * takes row positions[t % block_len] (positions == NULL: t % block_len), the
 * block position shared by every branch. dtype bf16 or f16, head_dim 64 or 128. */
int d2sd_qk_norm_rope(const void* q_in, int64_t q_in_stride_token,
                      int64_t q_in_stride_head, void* q_out,
                      int64_t q_out_stride_token, int64_t q_out_stride_head,
                      const void* k_in, int64_t k_in_stride_token,
                      int64_t k_in_stride_head, void* k_out,
                      int64_t k_out_stride_token, int64_t k_out_stride_head,
                      int32_t num_tokens, int32_t num_qo_heads,
                      int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                      const void* q_weight, const void* k_weight, float eps,
                      const void* cos_table, const void* sin_table,
                      int64_t table_stride, int32_t block_len,
                      const int32_t* positions, void* stream);

/* d2sd_commit_kv fused with the gather of the draft model's context feature
 * for the same (branch, positions 0..acc-1) index set, in the same launch:
 *   hidden_dst[t, j*hidden_size + c] = hidden_src[j][branch, t, c]
 * for t < acceptance_length, j < num_hidden, c < hidden_size, i.e. the
 * reference's torch.cat of the selected layers' hidden states along the last
 * axis, row-sliced by the winning branch and the accepted length. Rows
 * t >= acceptance_length of hidden_dst are not written.
 * hidden_src: device array of num_hidden pointers, each [num_branches,
 *   block_len, hidden_size] with element strides (hidden_stride_branch,
 *   hidden_stride_token), last axis contiguous; hidden_dst: [block_len,
 *   num_hidden*hidden_size] with row stride hidden_dst_stride_token.
 * hidden_elem_bytes is 2 or 4; hidden_size*hidden_elem_bytes and every stride
 * in bytes must be multiples of 16, the pointers 16-byte aligned. */
int d2sd_commit_kv_hidden(const void* const* layer_ptrs, int32_t num_layers,
                          int32_t num_kv_heads, int32_t head_dim,
                          int32_t elem_bytes, int32_t block_len,
                          int64_t new_stride_branch, int64_t new_stride_head,
                          int64_t new_stride_token, int64_t cache_stride_page,
                          int64_t cache_stride_slot, int64_t cache_stride_head,
                          int32_t page_size, int32_t cache_format,
                          const int32_t* page_table, const int32_t* accept_result,
                          const int32_t* cache_len_dev, int64_t cache_len_host,
                          const void* const* hidden_src, int32_t num_hidden,
                          int32_t hidden_size, int32_t hidden_elem_bytes,
                          int64_t hidden_stride_branch,
                          int64_t hidden_stride_token, void* hidden_dst,
                          int64_t hidden_dst_stride_token, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* D2SD_H_ */
