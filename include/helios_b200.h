/*
 * helios_b200 — C ABI of the B200 (sm_100a) packed-tick hot path.
 *
 * The reference (sidmanale643/helios) runs its packed mixed-batch forward in
 * Python/PyTorch; these entry points replace the op sequences it runs per tick.
 * Every function takes raw device pointers, element counts and a cudaStream_t
 * (a CUstream handle, e.g. torch.cuda.current_stream().cuda_stream), borrows the
 * memory for the launch only, allocates nothing, and returns 0 or a negative
 * HB_ERR_* code with a message from hb_last_error() (per calling thread).
 * Device-side input checks (page indices, KV slots, RoPE positions, token ids)
 * skip the bad element and set a bit in a device status word read back by
 * hb_device_status(). All tensors are bf16 unless stated.
 *
 * Paths below are within the reference project.
 */
#ifndef HELIOS_B200_H_
#define HELIOS_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define HB_API __attribute__((visibility("default")))
#else
#define HB_API
#endif

typedef struct CUstream_st* hb_stream_t; /* same object as cudaStream_t / CUstream */
#if !defined(__CUDACC__) && !defined(__DRIVER_TYPES_H__)
typedef hb_stream_t cudaStream_t;
#endif

#define HB_VERSION 1
#define HB_OK 0
#define HB_ERR_INVALID (-1)     /* bad pointer, size or layout: the reference's ValueError */
#define HB_ERR_UNSUPPORTED (-2) /* shape outside what the kernels are built for */
#define HB_ERR_CUDA (-3)        /* launch or driver failure */
#define HB_MAX_TICK_ROWS 8192

/* Device status bits (hb_device_status). */
#define HB_STATUS_WAIT_TIMEOUT (1u << 0)
#define HB_STATUS_BAD_SLOT (1u << 1)
#define HB_STATUS_BAD_POSITION (1u << 2)
#define HB_STATUS_BAD_PAGE (1u << 3)
#define HB_STATUS_BAD_TOKEN (1u << 4)
#define HB_STATUS_BAD_ROW (1u << 5)
#define HB_STATUS_INDEX_FULL (1u << 6)

HB_API int hb_version(void);
HB_API const char* hb_last_error(void);

/* Synchronise the current device, read the status word, optionally clear it. */
HB_API int hb_device_status(uint32_t* status, int clear);

/*
 * Self-test of the kernels' error path (no counterpart in the reference). One thread of a
 * one-CTA kernel waits, through the same bounded mbarrier wait the attention and GEMM
 * kernels use, for a barrier phase that nothing completes, with a limit of limit_cycles SM
 * clock cycles (1 .. 2^31, a few milliseconds at most). The wait gives up, sets
 * HB_STATUS_WAIT_TIMEOUT and the kernel returns normally; result (device int32[2]) receives
 * whether the wait succeeded (0 expected) and the CTA's abort flag (1 expected).
 */
HB_API int hb_selftest_wait_timeout(int64_t limit_cycles, int32_t* result, cudaStream_t stream);

/*
 * (a) Tick packing. Replaces PackedBatchCache.prepare_packed
 * (src/helios/runtime/qwen3/paged_cache.py:418-494) and PagedBatchCache.prepare
 * (paged_cache.py:221-270), whose Python lists are rebuilt and copied every tick.
 *   rows     device int32 [num_rows][7]: arena slot, committed length, query count,
 *            logit count, pages held (after this tick's acquisitions), shared prefix keys,
 *            group rows. Consecutive single-token decode rows whose block tables start with the
 *            same pages (restored by aliasing) may form a group: every member has shared prefix
 *            keys L (a multiple of the page size, at most its length) and the first member has
 *            group rows = n, the others 0; other rows have 0, 0
 *   updates  device int32 [num_updates][3]: arena slot, page position, page index
 *   arena    device int32 [arena_slots][arena_width]: per-request page lists
 * Outputs (all device): block_table int32 [num_rows][width] (zero-padded),
 * cu_seq_q/cu_seq_k int32 [num_rows+1], seqused_k int32 [num_rows], positions,
 * write_slots int64 [total_tokens], token_row int32 [total_tokens], logit_indices
 * int64 [logit_capacity], decode_items int32 [decode_capacity][6] for rows with count <=
 * decode_max_tokens, split every split_keys keys of the row's own keys (after its shared
 * prefix keys): (row, first key, end key, record base, splits of the row, 0).
 * prefix_items int32 [prefix_capacity][5]: for each group, its shared keys split every
 * prefix_split_keys keys (a multiple of page_size), and its rows taken 2 x prefill_tile_tokens
 * at a time: (first row, rows, first key, end key, split index), each run once for those rows.
 * row_records int32 [num_rows+1] (device, may be null when there are no decode rows) gets
 * each row's first partial record: a decode row's records are its shared-prefix splits, then
 * its own splits, each with one record per query token. prefill_items int32
 * [prefill_capacity][3] (row, start of query
 * tile 2i, start of tile 2i+1 or -1) pairing adjacent tiles of prefill_tile_tokens
 * queries of a row. Entries past a capacity are not written. counts (device int32[4],
 * may be null) receives the number of decode items and prefill pairs written (capped at
 * their capacities), the partial records the decode and prefix items need, and the number
 * of prefix items written (capped).
 */
HB_API int hb_tick_pack(const int32_t* rows, int32_t num_rows, const int32_t* updates, int32_t num_updates,
                        int32_t* arena, int32_t arena_slots, int32_t arena_width, int32_t page_size, int32_t width,
                        int32_t num_pages, int32_t decode_max_tokens, int32_t split_keys, int32_t prefill_tile_tokens,
                        int32_t prefix_split_keys, int32_t total_tokens, int32_t* block_table, int32_t* cu_seq_q,
                        int32_t* cu_seq_k, int32_t* seqused_k, int64_t* positions, int64_t* write_slots,
                        int32_t* token_row, int64_t* logit_indices, int32_t logit_capacity, int32_t* decode_items,
                        int32_t decode_capacity, int32_t* prefill_items, int32_t prefill_capacity,
                        int32_t* prefix_items, int32_t prefix_capacity, int32_t* counts, int32_t* row_records,
                        cudaStream_t stream);

/*
 * (b) Fused per-head q/k RMSNorm + RoPE + paged KV append. Replaces, in
 * GroupedQueryAttention.forward (src/helios/runtime/qwen3/layers.py:147-160),
 * q_norm/k_norm (RMSNorm.forward, layers.py:36-40) and apply_rope with position ids
 * (layers.py:54-72), plus PagedBatchCache._write (paged_cache.py:335-345).
 * q/k/v are addressed by element strides per token and per head; q_out is
 * [tokens][heads][head_dim] (null: q not produced); the pools are
 * [pool_slots][kv_heads][head_dim] (one layer). Null q_scale/k_scale skip the norm,
 * null cos/sin skip the rotation (plain append, as PagedBatchCache.attend needs).
 */
HB_API int hb_qk_norm_rope_append(const void* q, int64_t q_token_stride, int64_t q_head_stride, const void* k,
                                  int64_t k_token_stride, int64_t k_head_stride, const void* v,
                                  int64_t v_token_stride, int64_t v_head_stride, const float* q_scale,
                                  const float* k_scale, float eps, const float* cos, const float* sin,
                                  int64_t rope_rows, const int64_t* positions, const int64_t* write_slots,
                                  void* q_out, void* key_pool, void* value_pool, int64_t pool_slots, int32_t tokens,
                                  int32_t heads, int32_t kv_heads, int32_t head_dim, cudaStream_t stream);

/* Bytes of workspace hb_paged_attention needs: 256 bytes of decode work counters (zero before
 * the first call, left zero by every call) plus the float partials of `partial_records` split
 * records (16-byte aligned; required on every call). */
HB_API size_t hb_attention_workspace_bytes(int32_t partial_records, int32_t heads, int32_t head_dim);

/*
 * (c) Paged varlen GQA attention, bottom-right causal. Replaces the
 * varlen_attn(..., block_table, seqused_k, window_size=(-1, 0), num_splits=1) calls
 * of PackedBatchCache.attend (src/helios/runtime/qwen3/paged_cache.py:501-520) and
 * PagedBatchCache.attend (paged_cache.py:301-333); CPU meaning in
 * paged_cache.py:521-546. q and out are [total_tokens][heads][head_dim]; the
 * pools [num_pages][page_size][kv_heads][head_dim]. Work items come from
 * hb_tick_pack: decode items run split-K (partials in `workspace`, merged by a
 * combine launch), prefill items run on tcgen05 tensor cores, and so do prefix items (rows
 * sharing restored pages: their tokens against each split of the shared keys, once for
 * all of them), whose partials the same combine merges into each row's own splits. With
 * counts null the launch covers exactly num_decode_items / num_prefill_items /
 * num_prefix_items. With counts (device, the array hb_tick_pack filled) those arguments and
 * partial_records are capacities: the grids are sized to them and the kernels read the real
 * numbers from counts, so one launch (for instance inside a CUDA graph) serves every tick
 * within the capacities. Prefix items need decode items in the same call (their rows' own
 * keys). With prefill or prefix items in the same call the decode grid is persistent (at
 * most one CTA per SM) and the tensor-core grids run beside it on the SMs it leaves
 * (hb_attention_set_overlap), all on `stream`.
 * The workspace's first 256 bytes hold a work ticket: they must be zero before the first call
 * with a workspace, and every call leaves them zero.
 */
HB_API int hb_paged_attention(const void* q, const void* key_pool, const void* value_pool, int64_t num_pages,
                              int32_t page_size, const int32_t* block_table, int32_t width, const int32_t* cu_seq_q,
                              const int32_t* seqused_k, int32_t num_rows, const int32_t* row_records,
                              const int32_t* decode_items, int32_t num_decode_items,
                              const int32_t* prefill_items, int32_t num_prefill_items,
                              const int32_t* prefix_items, int32_t num_prefix_items, const int32_t* counts,
                              int32_t partial_records, int32_t split_keys, int32_t total_tokens, int32_t heads,
                              int32_t kv_heads, int32_t head_dim, float scale, void* workspace,
                              size_t workspace_bytes, void* out, cudaStream_t stream);

/*
 * Overlap of decode and prefill attention in one hb_paged_attention call: the decode grid
 * keeps decode_sms SMs (one persistent CTA each) and the prefill grid, launched behind it,
 * starts on the others at once. 0: the decode grid keeps every SM and the prefill tiles start
 * as decode CTAs finish. Process-wide; applies to later calls.
 */
HB_API int hb_attention_set_overlap(int32_t decode_sms);

/*
 * Paged attention with a built-in workspace (no counterpart in the reference).
 * Same arguments and results as hb_paged_attention, minus the workspace: the split-K
 * partials go to a fixed device array inside this library (HB_STATIC_WORKSPACE_BYTES,
 * 8 MiB, held on every GPU that loads the library until the process exits). It is for
 * callers that cannot allocate device memory: hosts that hand the whole GPU to their
 * own pool up front (so a cudaMalloc would fail or break their accounting) and
 * latency-bound callers that must not pay cudaMalloc's implicit synchronisation.
 * It allocates nothing. A call whose partial_records * heads * (head_dim + 1) floats
 * exceed the array is rejected with HB_ERR_INVALID. The first call on a device looks
 * up the array's device address (cudaGetSymbolAddress) with that device current; make
 * that first call before any stream capture. Every call shares the one array and leaves
 * its contents behind. Of those, only the decode work ticket in the first 256 bytes must
 * start at zero: the array is zero when the library loads and every call resets the ticket
 * (the split-K partials are written before they are read; a call that fails after queuing
 * the decode grid queues a 4-byte reset of the ticket). Calls that overlap on the GPU,
 * from different streams or threads, race on the array.
 * The device address is cached per device number for the life of the process: after
 * cudaDeviceReset, or when another context is made current on that device (driver API),
 * the cached address is stale and this entry point must not be called again.
 */
#define HB_STATIC_WORKSPACE_BYTES (8u << 20)
HB_API int hb_paged_attention_static_workspace(const void* q, const void* key_pool, const void* value_pool,
                                               int64_t num_pages, int32_t page_size, const int32_t* block_table,
                                               int32_t width, const int32_t* cu_seq_q, const int32_t* seqused_k,
                                               int32_t num_rows, const int32_t* row_records,
                                               const int32_t* decode_items, int32_t num_decode_items,
                                               const int32_t* prefill_items, int32_t num_prefill_items,
                                               const int32_t* prefix_items, int32_t num_prefix_items,
                                               const int32_t* counts, int32_t partial_records, int32_t split_keys,
                                               int32_t total_tokens, int32_t heads, int32_t kv_heads,
                                               int32_t head_dim, float scale, void* out, cudaStream_t stream);

/*
 * Hidden-size RMSNorm (RMSNorm.forward, src/helios/runtime/qwen3/layers.py:36-40).
 * With row_index (int64 [rows]) the rows are gathered first, as the logit-row
 * index_select before the final norm (src/helios/runtime/qwen3/model.py:108-110).
 */
HB_API int hb_rmsnorm(const void* x, int64_t rows_in, const int64_t* row_index, const float* scale, float eps,
                      void* out, int32_t rows, int32_t hidden, cudaStream_t stream);

/* Residual add rounded to bf16 (TransformerBlock.forward, layers.py:220-232) fused with the next RMSNorm. */
HB_API int hb_add_rmsnorm(const void* x, const void* y, const float* scale, float eps, void* sum_out,
                          void* norm_out, int32_t rows, int32_t hidden, cudaStream_t stream);

/* silu(gate) * up from a [rows][2*inter] gate|up GEMM output (FeedForward.forward, layers.py:26-27). */
HB_API int hb_swiglu(const void* gate_up, void* out, int64_t rows, int64_t inter, cudaStream_t stream);

/*
 * Gate|up projection fused with SwiGLU on tcgen05 tensor cores. Replaces, in FeedForward.forward
 * (src/helios/runtime/qwen3/layers.py:26-27), gate(x), up(x) and silu(gate) * up for
 * x bf16 [m][k] (rows contiguous) and the fused weight w_gate_up bf16 [2*inter][k] (the gate
 * rows, then the up rows): out bf16 [m][inter] = bf16(bf16(silu(bf16(x Wg^T))) * bf16(x Wu^T)).
 * Needs k % 64 == 0 and inter % 128 == 0.
 */
HB_API int hb_gemm_swiglu(const void* x, int32_t m, int32_t k, const void* w_gate_up, int32_t inter, void* out,
                          cudaStream_t stream);

/*
 * Greedy decoding head (replaces the logits GEMM of Qwen3Model._forward_packed,
 * src/helios/runtime/qwen3/model.py:108-110, and the temperature-0 argmax of
 * Decoder._sample, src/helios/runtime/qwen3/decode.py:458-460, as Engine._execute_batch
 * applies it, src/helios/runtime/engine.py:472-473).
 * out_ids[r] = argmax_j bf16(x[r] . weight[j]) for the m rows of x [m, k] (bf16, the final-normed
 * logit rows) against the tied embedding weight [vocab, k] (bf16): ties go to the lowest id and a
 * NaN logit counts as the largest, as torch.argmax over the bf16 logits does. The logits are
 * never written. best [m] (8-byte aligned) must be zero before the first call; every call leaves
 * it zero. k % 64 == 0. Persistent tcgen05 GEMM with the argmax in its epilogue, then one small
 * kernel, both on `stream`. A row with id -1 means the GEMM gave up (hb_device_status).
 */
HB_API int hb_lm_head_argmax(const void* x, int32_t m, int32_t k, const void* weight, int32_t vocab,
                             unsigned long long* best, int64_t* out_ids, cudaStream_t stream);

/*
 * Prefix-cache block keys (replaces hash_token_blocks / build_token_blocks,
 * src/helios/runtime/prefix_cache.py:86-110, as PrefixCache.longest_prefix and
 * store_completed_blocks call them, :208-260). Prompt p is tokens[offsets[p], offsets[p+1])
 * (int32 ids >= 0); it is cut into blocks of block_size tokens, the last one possibly partial,
 * and block i's key is SHA-256(key of block i-1 || "[t0,t1,...]"): the decimal ids joined by
 * commas in brackets, the compact JSON the reference hashes, with no parent bytes for block 0.
 * The 32-byte keys go to digests + 32 * (block_offsets[p] + i). One warp per prompt.
 */
HB_API int hb_hash_token_blocks(const int32_t* tokens, const int64_t* offsets, int32_t prompts, int32_t block_size,
                                const int64_t* block_offsets, uint8_t* digests, cudaStream_t stream);

/*
 * Device-resident prefix index: an open-addressing table of `slots` (a power of two) 48-byte
 * slots, uint32 [slots][12], zeroed before first use. Insert adds n keys (32-byte digests) with
 * int32 values; each key must be absent from the table and appear once in the batch (the
 * caller's host-side map knows), and the caller keeps at most slots / 2 keys live, else
 * HB_STATUS_INDEX_FULL. Remove drops the keys it finds. Lookup replaces the probe loop of
 * PrefixCache.longest_prefix (prefix_cache.py:214-221): for prompt p it probes the keys of its
 * first full_blocks[p] blocks (digests laid out as hb_hash_token_blocks writes them) in order,
 * stops at the first absent one, writes the values of the matched blocks to
 * values[block_offsets[p] + i] and their count to matched[p].
 */
HB_API int hb_prefix_index_insert(uint32_t* table, int32_t slots, const uint8_t* digests, const int32_t* values,
                                  int32_t n, cudaStream_t stream);
HB_API int hb_prefix_index_remove(uint32_t* table, int32_t slots, const uint8_t* digests, int32_t n,
                                  cudaStream_t stream);
HB_API int hb_prefix_index_lookup(const uint32_t* table, int32_t slots, const uint8_t* digests,
                                  const int64_t* block_offsets, const int32_t* full_blocks, int32_t prompts,
                                  int32_t* matched, int32_t* values, cudaStream_t stream);

/* Token-embedding gather (Qwen3Model._forward_packed, src/helios/runtime/qwen3/model.py:97). */
HB_API int hb_embedding(const int64_t* ids, const void* table, int64_t vocab, void* out, int64_t tokens,
                        int32_t hidden, cudaStream_t stream);

/*
 * (d) Page copy: copy page src_pages[i] to dst_pages[i] in each of `tensors` pool
 * tensors spaced tensor_stride_bytes apart (all layers' K and V). The device form of
 * the dense snapshot/restore copies KVCache.snapshot_block / restore_blocks
 * (src/helios/runtime/qwen3/cache.py:109-147) for a paged pool; the paged restore
 * itself (PagedKVCache.restore_blocks, paged_cache.py:142-163) aliases pages and is
 * served by hb_tick_pack's arena updates.
 */
HB_API int hb_page_copy(void* pool_base, int64_t tensor_stride_bytes, int32_t tensors, int64_t page_bytes,
                        int64_t num_pages, const int32_t* src_pages, const int32_t* dst_pages, int32_t pairs,
                        cudaStream_t stream);

/*
 * (d) Fused sampler. Replaces Decoder._sample (src/helios/runtime/qwen3/decode.py:457-473)
 * and the batched sampling in Engine._execute_batch (src/helios/runtime/engine.py:470-492).
 * temperature 0 -> argmax (first index); otherwise temperature softmax with the
 * reference's top-p keep rule, drawn by inverse CDF over kept tokens in index order
 * with the caller's uniforms[rows] in [0, 1). logits bf16 [rows][row_stride].
 */
HB_API int hb_sample(const void* logits, int64_t row_stride, int32_t rows, int32_t vocab, const float* temperature,
                     const float* top_p, const float* uniforms, int64_t* out_ids, cudaStream_t stream);

/*
 * Speculative verification of drafted rows. Replaces the acceptance loop of
 * Engine._execute_batch (src/helios/runtime/engine.py:507-520), which copies every logit
 * row's argmax to the host and compares there. Row r of the tick holds tokens
 * tokens[cu_seq_q[r] .. cu_seq_q[r+1]) and logit rows logit_offsets[r] .. logit_offsets[r+1]
 * (its trailing tokens); predictions holds one id per logit row (the greedy id, e.g. from
 * hb_sample with temperature 0). accepted[r] = the longest prefix of the row's drafted
 * tokens (its tokens after the first logit row) equal to its predictions; emitted receives
 * predictions logit_offsets[r] .. + accepted[r] (the tokens the row produces). A row with
 * one logit row accepts 0 and emits its prediction. All pointers are device memory.
 */
HB_API int hb_verify_drafts(const int64_t* tokens, const int32_t* cu_seq_q, const int32_t* logit_offsets,
                            const int64_t* predictions, int32_t rows, int32_t* accepted, int64_t* emitted,
                            cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* HELIOS_B200_H_ */
