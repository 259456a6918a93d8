/*
 * nvk_paged_kv.h -- C ABI of the B200 paged-KV-cache hot path.
 *
 * Plain pointers, sizes and a CUDA stream; no framework types. Every entry
 * point validates its arguments on the host, returns NVK_OK (0) or a negative
 * NVK_ERR_* code, and only enqueues work on `stream` (no host synchronisation,
 * no allocation), so each call can be captured into a CUDA graph.
 *
 * Memory layout shared by all kernels (the reference pool layout):
 *   key_cache / value_cache of ONE layer: bf16 [num_blocks, block_size,
 *   num_kv_heads, head_dim], contiguous. Token slot s = block_id * block_size
 *   + offset addresses row s of the flattened [num_blocks * block_size,
 *   num_kv_heads, head_dim] view.
 *   The attention kernels stage whole tiles of a block, so the rows of a
 *   sequence's last block past its context are read and weighted by 0: they
 *   must hold finite values (zero-fill the pool once when it is allocated;
 *   appends only ever write real rows).
 *
 * Reference interfaces replaced (paths inside Pla-Yer/nano_vllm_ascend):
 *   nvk_kv_append      <- PagedKVCache.write, src/nanovllm_ascend/npu/paged_kv_cache.py:44-69
 *                         (two Tensor.index_copy_ calls at :68-69)
 *   nvk_paged_decode   <- torch_npu._npu_paged_attention, called from
 *                         src/nanovllm_ascend/layers/npu_paged_attention.py:58,89 and
 *                         src/nanovllm_ascend/npu/acl_graph.py:232
 *   nvk_paged_decode_workspace_size
 *                      <- torch_npu._npu_paged_attention_get_workspace,
 *                         src/nanovllm_ascend/layers/npu_paged_attention.py:42-52
 *   nvk_paged_prefill  <- torch_npu.npu_fused_infer_attention_score, paged mode
 *                         (block_table + absolute actual_seq_lengths_kv, sparse_mode=3),
 *                         src/nanovllm_ascend/layers/npu_prefill_attention.py:82-96
 *   nvk_dense_prefill  <- the same op, dense mode (contiguous k/v, cumulative
 *                         actual_seq_lengths_kv), npu_prefill_attention.py:97-112
 *   nvk_paged_decode_append
 *                      <- PagedKVCache.write + _npu_paged_attention of one decode layer
 *                         (qwen3.py:91-117), fused
 *   nvk_qk_norm_rope_append
 *                      <- q_norm + k_norm + apply_rotary_pos_emb_tnd + PagedKVCache.write,
 *                         src/nanovllm_ascend/models/qwen3.py:83-96, fused
 *   nvk_lm_head_argmax <- lm_head + greedy Sampler.sample + per-sequence .item(),
 *                         src/nanovllm_ascend/model_runner.py:284-286, qwen3.py:221
 *   nvk_prefix_*       <- BlockManager's prefix-cache keys and lookup,
 *                         src/nanovllm_ascend/npu/block_manager.py:57-192 (host code)
 *   nvk_decode_metadata
 *                      <- BlockManager.prepare_decode_metadata's table / length / slot
 *                         building, src/nanovllm_ascend/npu/block_manager.py:207-250,304-328
 *   nvk_paged_decode_gather, nvk_peer_*
 *                      <- no reference counterpart (the reference runs on one
 *                         device, src/nanovllm_ascend/model_runner.py:31): KV-head
 *                         sharded decode whose output all-gather across GPUs
 *                         happens inside the attention kernel
 */
#ifndef NVK_PAGED_KV_H_
#define NVK_PAGED_KV_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define NVK_API __attribute__((visibility("default")))
#else
#define NVK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t / CUstream; NULL is the legacy default stream. */
typedef struct CUstream_st* nvk_stream_t;

enum {
  NVK_OK = 0,
  NVK_ERR_INVALID_ARGUMENT = -1, /* shape, stride, alignment or null-pointer error */
  NVK_ERR_UNSUPPORTED = -2,      /* valid, but outside what the kernels implement   */
  NVK_ERR_WORKSPACE = -3,        /* workspace missing or too small                  */
  NVK_ERR_CUDA = -4              /* a CUDA runtime/driver call failed               */
};

/* Message for the most recent non-zero return on the calling thread. */
NVK_API const char* nvk_last_error(void);

/* ABI version, bumped on any signature change (2: persistent decode, num_ctas;
   3: KV-head-sharded decode with in-kernel gather, peer buffers, fused append,
   device-side decode metadata; 4: per-row lengths and table sizes for
   nvk_decode_metadata; 5: nvk_paged_decode_noalloc_error). */
NVK_API int nvk_abi_version(void);

/*
 * KV append: key_cache[slot_mapping[t]] = key[t]; value_cache[slot_mapping[t]]
 * = value[t] for t < num_tokens, each row num_kv_heads * head_dim bf16 values.
 *
 * key/value: bf16 rows [num_tokens, num_kv_heads, head_dim]; heads and dims are
 *   contiguous, consecutive tokens are key_token_stride / value_token_stride
 *   ELEMENTS apart (lets the caller pass a slice of a fused QKV projection).
 * slot_mapping: int64 [num_tokens], device memory.
 * num_slots: num_blocks * block_size (rows in the flattened pool).
 * error_word: optional device int; a slot outside [0, num_slots) is skipped and
 *   sets bit 4 there (index_copy_ would raise; a device kernel must not write
 *   out of bounds). May be NULL.
 * Bit-exact: rows are moved as raw 16-byte words.
 */
NVK_API int nvk_kv_append(const void* key, const void* value, int64_t key_token_stride, int64_t value_token_stride,
                  void* key_cache, void* value_cache, const int64_t* slot_mapping, int64_t num_tokens,
                  int64_t num_slots, int num_kv_heads, int head_dim, int* error_word, nvk_stream_t stream);

/*
 * Bytes of workspace nvk_paged_decode needs for `batch` sequences with
 * `num_kv_heads` KV heads and `num_heads` query heads on `num_ctas` CTAs
 * (0 = one per SM of the current device): an error word, one arrival ticket
 * per (sequence, KV head) and two partial-result slots per CTA. Zero it once
 * before first use; every call leaves the tickets at zero again for a next
 * call of the same batch, num_heads, num_kv_heads and num_ctas. The tickets'
 * place depends on those four (a call of another shape would find partial
 * results of the previous call there): zero the workspace again before a
 * call whose shape differs from the previous call's. Calls that share one
 * workspace must be ordered on one stream.
 */
NVK_API int nvk_paged_decode_workspace_size(int batch, int num_heads, int num_kv_heads, int head_dim, int num_ctas,
                                            size_t* bytes);

/*
 * Paged GQA decode attention, one query token per sequence:
 *   out[b, h, :] = softmax(scale * q[b, h, :] . K_b[:, g(h), :]^T) V_b[:, g(h), :]
 * over the first context_lens[b] tokens of sequence b, whose token i lives in
 * block block_tables[b * block_table_stride + i / block_size] at offset
 * i % block_size; g(h) = h / (num_heads / num_kv_heads).
 *
 * out, query: bf16 [batch, num_heads, head_dim], contiguous.
 * block_tables: int32, row b at block_tables + b * block_table_stride, the
 *   first max_blocks_per_seq entries meaningful (zero padding is fine: only
 *   entries below ceil(context_lens[b] / block_size) are read).
 * context_lens: int32 [batch] in DEVICE memory (includes the token appended
 *   this step, as in the reference); a length of 0 yields zeros.
 * num_ctas: persistent grid size, 0 = one CTA per SM (the tuned default).
 * workspace: see nvk_paged_decode_workspace_size (same batch/heads/num_ctas).
 * Supported: head_dim 128; num_heads / num_kv_heads in {1, 2, 4, 8};
 *   block_size a power of two in [16, 256].
 */
NVK_API int nvk_paged_decode(void* out, const void* query, const void* key_cache, const void* value_cache, int num_blocks,
                     int block_size, const int32_t* block_tables, int block_table_stride, int max_blocks_per_seq,
                     const int32_t* context_lens, int batch, int num_heads, int num_kv_heads, int head_dim,
                     float scale, int num_ctas, void* workspace, size_t workspace_bytes, nvk_stream_t stream);

/*
 * nvk_paged_decode with this step's KV append fused in: for every sequence b
 * the token row key[b] / value[b] (bf16 [batch, num_kv_heads, head_dim],
 * heads and dims contiguous, key_token_stride / value_token_stride ELEMENTS
 * between tokens, 16-byte aligned) is written to pool slot slot_mapping[b]
 * (int64, device) and then attended over, exactly as nvk_kv_append followed
 * by nvk_paged_decode. Replaces the write + attention pair of one layer
 * (Qwen3Attention.forward, src/nanovllm_ascend/models/qwen3.py:91-117) in
 * decode. slot_mapping[b] must be sequence b's last context position
 * (block_tables[b][(context_lens[b]-1) / block_size] * block_size +
 * (context_lens[b]-1) % block_size), as the reference's decode metadata makes
 * it; a row whose slot is not is skipped and bit 4 of the error word is set.
 */
NVK_API int nvk_paged_decode_append(void* out, const void* query, void* key_cache, void* value_cache,
                                    int num_blocks, int block_size, const int32_t* block_tables,
                                    int block_table_stride, int max_blocks_per_seq, const int32_t* context_lens,
                                    int batch, int num_heads, int num_kv_heads, int head_dim, float scale,
                                    int num_ctas, void* workspace, size_t workspace_bytes, const void* key,
                                    const void* value, int64_t key_token_stride, int64_t value_token_stride,
                                    const int64_t* slot_mapping, nvk_stream_t stream);

/*
 * nvk_paged_decode without a caller workspace. No counterpart in the
 * reference: it exists for callers that cannot allocate device memory where
 * they run attention (a plugin's enqueue callback inside a framework that owns
 * all device buffers, a cgo/JNI/N-API binding with no device allocator, a
 * serving thread that must not take cudaMalloc's implicit synchronisation).
 *
 * Same arguments and outputs as nvk_paged_decode minus the workspace. The
 * scratch is a fixed 16 MiB array in the library's device memory, present on
 * every GPU that loads the library until the process exits; a call whose
 * scratch need (nvk_paged_decode_workspace_size) exceeds 16 MiB returns
 * NVK_ERR_UNSUPPORTED, after the same argument checks as nvk_paged_decode.
 * It calls no allocator. The first call in each CUDA context (the device's
 * primary context, or one a host framework made current) resolves the array's
 * device address there (cudaGetSymbolAddress) and caches it under the
 * context's unique id, so a context created later (after cudaDeviceReset, for
 * one) resolves it afresh; make that first call before any stream capture
 * begins in the context. Every call clears the scratch's error word and
 * counters on `stream` and then uses the same array, so calls whose execution
 * overlaps on the GPU (different streams, or different host threads) race:
 * order them on one stream.
 *
 * The kernel's error word (bits as for nvk_paged_decode: 1 wait timeout, 2
 * block id outside the pool, 8 context longer than the table) lives in the
 * scratch, and the next call clears it: read it with
 * nvk_paged_decode_noalloc_error before the next call.
 */
NVK_API int nvk_paged_decode_noalloc(void* out, const void* query, const void* key_cache, const void* value_cache,
                                     int num_blocks, int block_size, const int32_t* block_tables,
                                     int block_table_stride, int max_blocks_per_seq, const int32_t* context_lens,
                                     int batch, int num_heads, int num_kv_heads, int head_dim, float scale,
                                     int num_ctas, nvk_stream_t stream);

/*
 * Device error word of the last nvk_paged_decode_noalloc call ordered before
 * this one on `stream`, copied to *error_word (host memory). Waits for
 * `stream`, so it must not be called while the stream is capturing (returns
 * NVK_ERR_INVALID_ARGUMENT). Allocates nothing. No counterpart in the
 * reference (the Ascend operator reports bad input by raising).
 */
NVK_API int nvk_paged_decode_noalloc_error(int* error_word, nvk_stream_t stream);

/*
 * Paged causal prefill attention (prefix-cache aware). Sequence b owns query
 * rows [cu_seqlens_q[b], cu_seqlens_q[b+1]) of `query` and attends over the
 * first kv_lens[b] tokens of its paged KV (cached prefix + the rows appended
 * this step), bottom-right aligned: query i of a sequence with q_len Lq and
 * kv_len Lk sees key j iff j <= Lk - Lq + i.
 *
 * out, query: bf16 [total_q, num_heads, head_dim], contiguous.
 * cu_seqlens_q: int32 [batch + 1], kv_lens: int32 [batch], device memory.
 * max_q_len: upper bound of any q_len (sizes the grid).
 * Supported: head_dim 128, block_size 128, num_heads % num_kv_heads == 0.
 */
NVK_API int nvk_paged_prefill(void* out, const void* query, const void* key_cache, const void* value_cache, int num_blocks,
                      int block_size, const int32_t* block_tables, int block_table_stride,
                      const int32_t* cu_seqlens_q, const int32_t* kv_lens, int batch, int total_q, int max_q_len,
                      int num_heads, int num_kv_heads, int head_dim, float scale, int* error_word,
                      nvk_stream_t stream);

/*
 * Dense causal prefill attention over contiguous key/value rows
 * [total_kv, num_kv_heads, head_dim]; sequence b owns key rows
 * [cu_seqlens_kv[b], cu_seqlens_kv[b+1]). Same masking and support as
 * nvk_paged_prefill.
 */
NVK_API int nvk_dense_prefill(void* out, const void* query, const void* key, const void* value,
                      const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_kv, int batch, int total_q,
                      int total_kv, int max_q_len, int num_heads, int num_kv_heads, int head_dim, float scale,
                      int* error_word, nvk_stream_t stream);

/*
 * Fused prologue of one attention layer (Qwen3Attention.forward,
 * src/nanovllm_ascend/models/qwen3.py:83-96): per-head RMSNorm of q and k
 * (q_norm / k_norm, npu_rms_norm over head_dim, layers/layernorm.py:12-17),
 * rotary embedding in "half" mode (apply_rotary_pos_emb_tnd,
 * layers/rotary_embedding.py:58-99; cos/sin rows of the fp32 tables
 * [max_position, head_dim] cast to bf16), and PagedKVCache.write of the
 * rotated k and of v at slot_mapping. query/key/value: bf16 rows of
 * num_heads / num_kv_heads heads, query_stride etc. ELEMENTS between tokens
 * (slices of a fused QKV output work); query_out: bf16 [num_tokens,
 * num_heads, head_dim] contiguous (may alias query when its stride is
 * num_heads * head_dim). Arithmetic in fp32, the norm's output rounded to
 * bf16 before the rotation (as the separate ops do). A bad slot skips that
 * token's k/v rows and sets bit 4 of error_word; a position outside the
 * table is clamped and sets bit 8.
 */
NVK_API int nvk_qk_norm_rope_append(const void* query, const void* key, const void* value, int64_t query_stride,
                                    int64_t key_stride, int64_t value_stride, const void* q_weight,
                                    const void* k_weight, float eps, const float* cos_table, const float* sin_table,
                                    int max_position, const int64_t* positions, void* query_out, void* key_cache,
                                    void* value_cache, const int64_t* slot_mapping, int64_t num_tokens,
                                    int64_t num_slots, int num_heads, int num_kv_heads, int head_dim,
                                    int* error_word, nvk_stream_t stream);

/*
 * Decode-step metadata on the device (replaces the host loops of
 * BlockManager.prepare_decode_metadata, src/nanovllm_ascend/npu/block_manager.py:304-328,
 * with get_block_tables_tensor :207-224, get_context_lens_tensor :226-231 and
 * get_slot_mapping :233-250). table_mirror: int32 [mirror_rows, mirror_stride]
 * device copy of the per-sequence block tables (row = sequence slot), kept
 * by this call: sequence b first gets its new entries
 * table_mirror[seq_slots[b]][update_idx[u]] = update_block[u] for u in
 * [update_offsets[b], update_offsets[b+1]), then
 *   block_tables[b][j] = j < n_b ? table[j] : 0  (j < block_table_width)
 *   context_lens[b]    = ctx_b
 *   slot_mapping[b * q_len + t] = table[p / block_size] * block_size + p % block_size,
 *                        p = start_positions[b] + t
 * where ctx_b = row_context_lens[b] and n_b = row_blocks[b] (the host path's
 * seq_lens[slot] after this step and its whole table length, which is what
 * it returns when a slot is named twice or decoded behind its length), or,
 * when those pointers are NULL, ctx_b = start_positions[b] + q_len and
 * n_b = ceil(ctx_b / block_size). Bit-exact with the host path. All arrays
 * are device memory. A sequence whose table would not fit, whose table does
 * not cover its new tokens, or with a bad slot gets a zero row, length 0,
 * slots -1, and bit 8 in error_word (may be NULL).
 */
NVK_API int nvk_decode_metadata(int32_t* table_mirror, int mirror_stride, int mirror_rows, const int32_t* seq_slots,
                                const int64_t* start_positions, const int32_t* row_context_lens,
                                const int32_t* row_blocks, int batch, int q_len, int block_size,
                                const int32_t* update_offsets, const int32_t* update_idx,
                                const int32_t* update_block, int32_t* block_tables, int block_table_stride,
                                int block_table_width, int32_t* context_lens, int64_t* slot_mapping, int* error_word,
                                nvk_stream_t stream);

/*
 * LM head + greedy argmax for a decode batch: token_ids[b] = argmax_v
 * bf16(hidden[b] . weight[v]) (ties: the smallest v), i.e. Qwen3ForCausalLM's
 * lm_head (src/nanovllm_ascend/models/qwen3.py:196,221) followed by the greedy
 * branch of Sampler.sample (layers/sampler.py:13-14), without the per-sequence
 * .item() of ModelRunner.decode (model_runner.py:284-286). hidden: bf16
 * [batch, hidden_size] rows hidden_stride ELEMENTS apart; weight: bf16
 * [vocab_size, hidden_size] contiguous; token_ids: int64 [batch], device.
 * workspace: nvk_lm_head_argmax_workspace_size bytes, zeroed once (every call
 * leaves it zeroed). batch <= 128, hidden_size a multiple of 128. num_ctas 0 =
 * one CTA per SM. A timed-out wait sets bit 1 of error_word.
 */
NVK_API int nvk_lm_head_argmax_workspace_size(int batch, size_t* bytes);
NVK_API int nvk_lm_head_argmax(const void* hidden, int64_t hidden_stride, const void* weight, int vocab_size,
                               int hidden_size, int batch, int64_t* token_ids, void* workspace,
                               size_t workspace_bytes, int num_ctas, int* error_word, nvk_stream_t stream);

/*
 * ---- Prefix-cache index (host code) ----
 * The chained exact-content block keys and key -> cached-blocks map behind
 * BlockManager's prefix cache (src/nanovllm_ascend/npu/block_manager.py:57-65,
 * :76-81, :89, :136-192). A block's key is (parent block's key, the block's
 * token ids); lookup walks the chain and returns each key's first cached
 * block; a reused physical block forgets its key (nvk_prefix_forget_block).
 * Not thread-safe: one index per BlockManager, driven by one host thread.
 */
typedef struct nvk_prefix_index nvk_prefix_index;

NVK_API int nvk_prefix_create(int num_blocks, int block_size, nvk_prefix_index** out);
NVK_API void nvk_prefix_destroy(nvk_prefix_index* index);
/* Longest chain of cached full blocks of token_ids (at most max_blocks): *count ids into block_ids. */
NVK_API int nvk_prefix_find_longest(nvk_prefix_index* index, const int64_t* token_ids, int64_t num_tokens,
                                    int max_blocks, int32_t* block_ids, int* count);
/* Keys blocks table[num_cached_blocks .. num_full_blocks) by token_ids (blocks already keyed are kept). */
NVK_API int nvk_prefix_cache_blocks(nvk_prefix_index* index, const int32_t* table, int table_len,
                                    int num_cached_blocks, int num_full_blocks, const int64_t* token_ids,
                                    int64_t num_tokens);
NVK_API int nvk_prefix_forget_block(nvk_prefix_index* index, int block_id);
/* The block's key (interned id), -1 when it is not cached. */
NVK_API int64_t nvk_prefix_block_key(const nvk_prefix_index* index, int block_id);
NVK_API int nvk_prefix_clear(nvk_prefix_index* index);
NVK_API int64_t nvk_prefix_num_cached_keys(const nvk_prefix_index* index);
NVK_API int64_t nvk_prefix_num_keys(const nvk_prefix_index* index);

/*
 * ---- KV-head-sharded decode, outputs gathered across GPUs in the kernel ----
 * One process per GPU. Rank r of `world` holds a slice of the KV heads and the
 * query heads of their GQA groups; every rank needs all heads' outputs.
 *
 * Peer buffers: nvk_peer_alloc returns zero-filled device memory of its own
 * allocation, which nvk_peer_export describes in an NVK_PEER_HANDLE_BYTES
 * handle (CUDA IPC); another process on the same node maps it with
 * nvk_peer_import and unmaps it with nvk_peer_close. The exchange of handles
 * between processes is the caller's (e.g. an all-gather over a process group).
 */
#define NVK_MAX_PEERS 8
#define NVK_PEER_HANDLE_BYTES 64
#define NVK_PEER_SIGNAL_BYTES 256 /* per rank: one uint32 flag per source rank and an epoch counter */

NVK_API int nvk_peer_alloc(size_t bytes, void** ptr);
NVK_API int nvk_peer_free(void* ptr);
NVK_API int nvk_peer_export(const void* ptr, void* handle);
NVK_API int nvk_peer_import(const void* handle, void** ptr);
NVK_API int nvk_peer_close(void* ptr);

/*
 * nvk_paged_decode over this rank's heads, with the all-gather of the outputs
 * done by the kernel's own stores. query: this rank's bf16 [batch, num_heads,
 * head_dim] (num_heads query heads over the num_kv_heads KV heads of this
 * rank's pool). The result for (b, h) is written to EVERY rank's gathered
 * output out_peers[p], bf16 [batch, out_heads, head_dim], at head
 * head_offset + h (plain stores over NVLink; out_peers[rank] is this rank's
 * own buffer). signal_peers[p] is rank p's signal area of
 * NVK_PEER_SIGNAL_BYTES (zeroed before first use, used by nothing else).
 *
 * When the call has completed on this rank's stream, out_peers[rank] holds the
 * rows of every rank for this call: the kernel's last CTA posts an epoch flag
 * to every rank and waits for all of theirs (bounded: after 1 s it sets bit 16
 * of the workspace error word and returns). Every rank must make the same
 * sequence of calls with the same batch. A rank can run one call ahead of a
 * slower peer, so consecutive calls must write different output buffers
 * (alternating two is enough when the consumer of a call's output runs on this
 * stream before the next call). world in [1, NVK_MAX_PEERS].
 * key, value, key_token_stride, value_token_stride, slot_mapping: an
 * optional fused append of this rank's KV heads, as in
 * nvk_paged_decode_append (slot_mapping NULL: none).
 */
NVK_API int nvk_paged_decode_gather(const void* query, void* key_cache, void* value_cache, int num_blocks,
                                    int block_size, const int32_t* block_tables, int block_table_stride,
                                    int max_blocks_per_seq, const int32_t* context_lens, int batch, int num_heads,
                                    int num_kv_heads, int head_dim, float scale, int num_ctas, void* workspace,
                                    size_t workspace_bytes, void* const* out_peers, void* const* signal_peers,
                                    int world, int rank, int out_heads, int head_offset, const void* key,
                                    const void* value, int64_t key_token_stride, int64_t value_token_stride,
                                    const int64_t* slot_mapping, nvk_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* NVK_PAGED_KV_H_ */
