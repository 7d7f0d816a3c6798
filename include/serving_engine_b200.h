/*
 * serving_engine_b200.h -- C ABI of the B200 (sm_100a) paged-KV attention backend.
 *
 * This library replaces the hot path of the serving engine's paged attention:
 *   - the Triton paged FlashAttention kernel and its launcher
 *       serving_engine/paged_attention_kernel.py:16-160
 *   - the KV write of the duck-typed cache shim
 *       serving_engine/model_runner.py:21-32 (_PagedKVCache.write, two index_copy_)
 *   - a batched copy-on-write block copy for prefix-cache forks (the reference has
 *     the hook point at serving_engine/block_manager.py:129-132 but no copy).
 *
 * Conventions shared by every entry point:
 *   - All pointers are device pointers unless stated otherwise. No entry point
 *     allocates or frees device memory; callers pass every buffer, including
 *     workspaces whose size the *_workspace_size functions report.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Work is enqueued
 *     asynchronously; no entry point synchronises the host.
 *   - The KV pool of one layer is two contiguous arrays k_cache, v_cache, each
 *     [num_blocks, SEB_BLOCK_SIZE, num_kv_heads, head_dim] (model_runner.py:101-110,
 *     :42-45). Slot s of the flat view is block s / 16, row s % 16.
 *   - Strides are in ELEMENTS; the innermost (head_dim) stride is always 1.
 *   - Return value: SEB_OK, or an SEB_E* status when the host-side validation
 *     rejects the arguments or a launch fails; seb_last_error() then holds a
 *     message for the calling thread.
 *   - `err` (optional, may be NULL) is a device int32 that kernels OR SEB_ERRBIT_*
 *     flags into when they meet an out-of-range index at run time. The offending
 *     access is skipped; kernels never trap. The caller zeroes it and reads it
 *     back whenever it wants to check.
 */
#ifndef SERVING_ENGINE_B200_H
#define SERVING_ENGINE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define SEB_API __attribute__((visibility("default")))
#else
#define SEB_API
#endif

#define SEB_BLOCK_SIZE 16 /* tokens per KV block: serving_engine/block.py:7 */

/* element types of q / k / v / out (the attention computes in fp32) */
enum seb_dtype { SEB_F32 = 0, SEB_F16 = 1, SEB_BF16 = 2 };

/* host-side status codes */
enum seb_status {
  SEB_OK = 0,
  SEB_EINVAL = 1,       /* an argument is out of range, misaligned or NULL */
  SEB_EUNSUPPORTED = 2, /* a valid shape this build has no kernel for */
  SEB_ECUDA = 3,        /* a CUDA launch or attribute call failed */
  SEB_EWORKSPACE = 4    /* the workspace passed is smaller than required */
};

/* device-side error bits ORed into *err */
#define SEB_ERRBIT_BLOCK_ID 1u /* block_table entry outside [0, num_blocks) */
#define SEB_ERRBIT_SLOT 2u     /* slot_mapping entry outside [0, num_blocks*16) */
#define SEB_ERRBIT_TIMEOUT 4u  /* a bounded wait on an mbarrier gave up */
#define SEB_ERRBIT_KLEN 8u     /* k_len larger than the block table row can hold */
#define SEB_ERRBIT_META 16u    /* a row / query index outside the metadata arrays */

SEB_API const char* seb_version(void);
SEB_API const char* seb_status_string(int status);
/* message of the last failing call on this host thread ("" if none) */
SEB_API const char* seb_last_error(void);

/*
 * KV append: k_cache_flat[slot_mapping[t]] = k_new[t], same for V, for t < n_tokens.
 * Replaces _PagedKVCache.write (serving_engine/model_runner.py:21-32), whose two
 * index_copy_ calls scatter [n_tokens, num_kv_heads, head_dim] rows at int64
 * write_index (slot semantics: ModelRunner._flat_slot, model_runner.py:127-129).
 * k_new element (t, h, d) is at k_new + t*k_stride_token + h*k_stride_head + d.
 * One launch writes both K and V. Duplicate slots race (as index_copy_ does on
 * CUDA); out-of-range slots set SEB_ERRBIT_SLOT and are skipped.
 */
SEB_API int seb_kv_append(const void* k_new, int64_t k_stride_token, int64_t k_stride_head,
                  const void* v_new, int64_t v_stride_token, int64_t v_stride_head,
                  int64_t n_tokens, const int64_t* slot_mapping, void* k_cache, void* v_cache,
                  int64_t num_blocks, int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                  int32_t* err, void* stream);

/*
 * Batched block copy for copy-on-write: for every pair i < n_pairs and every
 * layer l < num_layers and K/V plane p, block dst[i] := block src[i], i.e.
 * kv_cache[:, :, dst] = kv_cache[:, :, src] on the engine's pool
 * kv_cache[num_layers, 2, num_blocks, 16, num_kv_heads, head_dim]
 * (model_runner.py:101-110). New: the reference's BlockManager.fork
 * (block_manager.py:129-132) shares whole tables and never copies.
 * `layer_stride_bytes` is the distance between layer l and l+1 in bytes (the
 * full pool passes 2*num_blocks*block_bytes; a per-layer call passes any value
 * with num_layers = 1). All pairs are copied at once by one grid, so the
 * result is defined only when the dst ids are distinct and no dst id appears
 * among the src ids of the same call; otherwise it depends on thread timing.
 * The library does not check this (the ids are device data); the Python
 * wrapper checks host lists. Ids outside [0, num_blocks) set
 * SEB_ERRBIT_BLOCK_ID and are skipped.
 */
SEB_API int seb_copy_blocks(void* kv_cache, int64_t num_layers, int64_t layer_stride_bytes,
                    int64_t num_blocks, int64_t block_bytes, const int64_t* src,
                    const int64_t* dst, int64_t n_pairs, int32_t* err, void* stream);

/*
 * Paged attention over the metadata of build_paged_batch_metadata
 * (paged_attention_kernel.py:163-200), computed exactly as the reference kernel
 * defines it (paged_attention_kernel.py:16-122): for row r, query i < q_lens[r]
 * (token q_starts[r]+i, logical position q_pos_offsets[r]+i) and query head h,
 *   O = softmax_j(scale * q.k_j [causal: k_j <= position]) . v_j,
 *   LSE = m + log(l)   (natural log, fp32),
 * over the keys j < k_lens[r] held at slots block_table[r, j/16]*16 + j%16 of
 * kv head h / (num_q_heads/num_kv_heads). Keys in the last partial block beyond
 * k_lens[r] are zero-padded exactly as the reference's boundary-checked loads
 * make them (they matter only when is_causal = 0). A row with k_lens = 0 and
 * q_lens > 0 yields O = NaN and LSE = -inf, as the reference does.
 *
 * seb_paged_decode is the split-K decode kernel: one warp per
 * (query item, kv head, split of blocks_per_split blocks) with all query heads
 * of the GQA group packed on one tensor-core tile; the last warp to finish a
 * split of an (item, kv head) merges the splits in the same launch.
 * It is correct for any query (decode or prefill rows alike) and is the fast
 * path for q_len = 1 rows.
 *   item_query[i]: token index of item i (NULL: item i is token i); tokens
 *                  index q/out/lse, which hold total_query tokens;
 *   item_row[i]:   its row (NULL: found by binary search over q_starts).
 *   blocks_per_split: at most 64 (larger requests run as 64); <= 0 picks a
 *                  default of 8 to 40 from the batch size and table width.
 * workspace: at least seb_paged_decode_workspace_size(...) bytes, 16-byte aligned.
 *   Nothing in it needs to start at zero: its last bytes hold one arrival
 *   counter per (item, kv head), which the call clears on its stream
 *   (cudaMemsetAsync, capturable in a CUDA graph) before the launch. Calls that
 *   overlap on the GPU must not share a workspace.
 */
SEB_API int64_t seb_paged_decode_workspace_size(int32_t num_items, int32_t num_q_heads,
                                        int32_t num_kv_heads, int32_t head_dim,
                                        int64_t max_blocks, int32_t blocks_per_split);

SEB_API int seb_paged_decode(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                     const void* k_cache, const void* v_cache, int64_t num_blocks,
                     const int32_t* block_table, int64_t block_table_stride, int64_t max_blocks,
                     const int32_t* q_starts, const int32_t* k_lens, const int32_t* q_pos_offsets,
                     int32_t num_rows, int32_t total_query, const int32_t* item_query,
                     const int32_t* item_row, int32_t num_items, int32_t num_q_heads, int32_t num_kv_heads,
                     int32_t head_dim, int32_t dtype, float scale, int32_t is_causal,
                     int32_t blocks_per_split, void* out, int64_t out_stride_token,
                     int64_t out_stride_head, float* lse, int64_t lse_stride_token,
                     void* workspace, int64_t workspace_bytes, int32_t* err, void* stream);

/*
 * Chunked-prefill paged attention on tcgen05 tensor cores (bf16/fp16, head_dim
 * 64 or 128, GQA group 1/2/4/8/16): the prefill / mixed use (q_len > 1) of the
 * reference kernel (paged_attention_kernel.py:16-122), with the semantics stated
 * above for seb_paged_decode. Computes the rows listed in `rows` (NULL: rows
 * 0 .. num_prefill_rows-1); `max_q_len` bounds their q_lens and sizes the grid.
 * q, out: 16-byte aligned, strides multiples of 8 elements. No workspace.
 */
SEB_API int seb_paged_prefill(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                              const void* k_cache, const void* v_cache, int64_t num_blocks,
                              const int32_t* block_table, int64_t block_table_stride, int64_t max_blocks,
                              const int32_t* q_starts, const int32_t* q_lens, const int32_t* k_lens,
                              const int32_t* q_pos_offsets, int32_t num_rows, int32_t total_query,
                              const int32_t* rows, int32_t num_prefill_rows, int32_t max_q_len,
                              int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                              float scale, int32_t is_causal, void* out, int64_t out_stride_token,
                              int64_t out_stride_head, float* lse, int64_t lse_stride_token, int32_t* err,
                              void* stream);

/*
 * Paged attention over a whole mixed batch given only the reference's own step
 * metadata (the dict of build_paged_batch_metadata,
 * serving_engine/paged_attention_kernel.py:163-200, as the engine's
 * ModelRunner.forward builds it at model_runner.py:184 and hands it to the
 * launcher paged_flash_attention, paged_attention_kernel.py:125-160): per-row
 * q_lens, k_lens, q_starts, q_pos_offsets and the zero-padded block table, all
 * device arrays. Semantics as stated above for seb_paged_decode.
 *
 * The host needs to know only num_rows and total_query. When total_query >
 * num_rows and the shape has a tcgen05 prefill kernel (bf16/fp16, head_dim 64
 * or 128, group 1/2/4/8/16, q and out 16-byte aligned with strides that are
 * multiples of 8), a one-CTA routing kernel splits the rows on the device:
 * q_len == 1 rows become split-K decode items and q_len > 1 rows become tcgen05
 * prefill work units, and both kernels read their counts from the device.
 * Otherwise every token runs through the split-K kernel. Three launches at
 * most; no host synchronisation.
 * workspace: at least seb_paged_attention_workspace_size(...) bytes, 256-byte
 *   aligned, not shared by calls that overlap on the GPU; nothing in it needs
 *   to start at zero.
 */
SEB_API int64_t seb_paged_attention_workspace_size(int32_t num_rows, int32_t total_query, int32_t num_q_heads,
                                                   int32_t num_kv_heads, int32_t head_dim, int64_t max_blocks);

SEB_API int seb_paged_attention(const void* q, int64_t q_stride_token, int64_t q_stride_head, const void* k_cache,
                                const void* v_cache, int64_t num_blocks, const int32_t* block_table,
                                int64_t block_table_stride, int64_t max_blocks, const int32_t* q_lens,
                                const int32_t* k_lens, const int32_t* q_starts, const int32_t* q_pos_offsets,
                                int32_t num_rows, int32_t total_query, int32_t num_q_heads, int32_t num_kv_heads,
                                int32_t head_dim, int32_t dtype, float scale, int32_t is_causal, void* out,
                                int64_t out_stride_token, int64_t out_stride_head, float* lse,
                                int64_t lse_stride_token, void* workspace, int64_t workspace_bytes, int32_t* err,
                                void* stream);

/*
 * Allocation-free variant of seb_paged_decode. This entry point has no
 * counterpart in the reference: it exists for callers that cannot hand the
 * library a workspace, such as a host runtime whose allocator already owns all
 * free device memory (the engine sizes its KV pool to most of the free memory
 * at start-up), or an FFI binding with no access to the framework allocator.
 *
 * Arguments and results are those of seb_paged_decode without the workspace.
 * The split-K scratch is a fixed device array built into the library, of
 * SEB_NOALLOC_SCRATCH_BYTES (32 MiB), which every GPU that loads the library
 * holds until the process exits. A call whose scratch need
 * (seb_paged_decode_workspace_size) exceeds it returns SEB_EWORKSPACE with a
 * message and launches nothing. Raising blocks_per_split shrinks the need only
 * up to its cap of 64 blocks per split: the smallest need of a batch is
 *   num_items * num_q_heads * ceil(max_blocks / 64) * (head_dim + 2) * 4 bytes
 *   + num_items * num_kv_heads * 4 bytes (rounded up to 16),
 * and a batch above 32 MiB even there must be split into smaller calls. The
 * call itself never calls cudaMalloc or cudaFree.
 *
 * The first call on each device that needs scratch (num_items > 0 and some row
 * longer than one split) looks up the array's device address
 * (cudaGetSymbolAddress, with that device current) and caches it; make that
 * first call outside any stream capture. Calls that need no scratch never look
 * it up. All calls share the one array and nothing in it needs to start at
 * zero, but calls that overlap on the GPU (for example on two streams at once)
 * race on it and must be serialised.
 */
#define SEB_NOALLOC_SCRATCH_BYTES (32ll << 20)

SEB_API int seb_paged_decode_noalloc(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                                     const void* k_cache, const void* v_cache, int64_t num_blocks,
                                     const int32_t* block_table, int64_t block_table_stride,
                                     int64_t max_blocks, const int32_t* q_starts, const int32_t* k_lens,
                                     const int32_t* q_pos_offsets, int32_t num_rows, int32_t total_query,
                                     const int32_t* item_query, const int32_t* item_row, int32_t num_items,
                                     int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                     int32_t dtype, float scale, int32_t is_causal, int32_t blocks_per_split,
                                     void* out, int64_t out_stride_token, int64_t out_stride_head,
                                     float* lse, int64_t lse_stride_token, int32_t* err, void* stream);

/* ------------------------------------------------------------------------
 * Decode-layer fusions used by the tensor-parallel decode driver (config 5).
 * The reference runs one GPU and leaves these steps to the HF model's eager
 * ops; the first folds HF's rotary embedding (apply_rotary_pos_emb, the
 * rotate-half form) into _PagedKVCache.write (serving_engine/model_runner.py:21-32).
 * All take bf16 or fp16 tensors with unit stride inside a row.
 * ------------------------------------------------------------------------ */

/* qkv: [n_tokens] rows of (num_q_heads + 2 * num_kv_heads) * head_dim elements:
 * q heads, then k heads, then v heads. cos/sin: [n_tokens, head_dim]. Writes
 * q rotated to q_out [n_tokens, num_q_heads, head_dim] (token stride given, heads
 * contiguous) and the rotated k and the v of token t to pool slot
 * slot_mapping[t] of k_cache / v_cache ([num_blocks * 16, num_kv_heads,
 * head_dim]). out = x * cos + rotate_half(x) * sin with each product and the
 * sum rounded to the element type, bit-identical to the eager tensor ops.
 * Out-of-range slots set SEB_ERRBIT_SLOT and skip that token's K/V rows. */
SEB_API int seb_rope_kv_append(const void* qkv, int64_t qkv_stride_token, int64_t n_tokens,
                               int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                               const void* cos, const void* sin, int64_t cos_sin_stride_token,
                               const int64_t* slot_mapping, void* q_out, int64_t q_out_stride_token,
                               void* k_cache, void* v_cache, int64_t num_blocks, int32_t dtype,
                               int32_t* err, void* stream);

/* Per row of [n_rows, hidden]: when residual is not NULL, x <- x + residual
 * (rounded to the element type, in place); then
 * out = x * rsqrt(mean(x^2) + eps) * weight, computed in fp32 and rounded once.
 * hidden <= 32768. */
SEB_API int seb_add_rmsnorm(void* x, int64_t x_stride, const void* residual, int64_t residual_stride,
                            const void* weight, void* out, int64_t out_stride, int64_t n_rows,
                            int32_t hidden, float eps, int32_t dtype, void* stream);

/* out[r, f] = silu(gate_up[r, f]) * gate_up[r, ffn + f] for f < ffn, computed in
 * fp32 and rounded once. */
SEB_API int seb_swiglu(const void* gate_up, int64_t gate_up_stride, void* out, int64_t out_stride,
                       int64_t n_rows, int32_t ffn, int32_t dtype, void* stream);

/* ------------------------------------------------------------------------
 * All-reduce fused with the residual add + RMSNorm that follows it in the
 * tensor-parallel decoder (after o_proj and after down_proj), over CUDA IPC
 * peer memory. New: the reference runs on one GPU; this replaces
 * torch.distributed.all_reduce(SUM) of the [n_tokens, hidden] partial sums
 * followed by seb_add_rmsnorm.
 *
 * Peer memory: seb_peer_alloc returns zeroed device memory (cudaMalloc) whose
 * handle (SEB_PEER_HANDLE_BYTES, from seb_peer_export) another process opens
 * with seb_peer_import (CUDA IPC, peer access enabled). Close imported
 * pointers (seb_peer_close) on every rank before the owner frees them.
 * ------------------------------------------------------------------------ */
#define SEB_MAX_PEERS 8
#define SEB_PEER_HANDLE_BYTES 64
#define SEB_PEER_FLAG_BYTES 1024 /* flag words of one rank, zero before the first call */

SEB_API int seb_peer_alloc(size_t bytes, void** ptr);
SEB_API int seb_peer_free(void* ptr);
SEB_API int seb_peer_export(void* ptr, void* handle);
SEB_API int seb_peer_import(const void* handle, void** ptr);
SEB_API int seb_peer_close(void* ptr);

/* partial, x, out, flags: host arrays of `world` device pointers, rank q's
 * buffers as mapped on this device (this rank's own and the imported ones):
 * partial[q] and x[q], out[q] are contiguous [n_tokens, hidden], flags[q] is
 * SEB_PEER_FLAG_BYTES. For every token row t, with S the sum over ranks of
 * partial[q][t] (fp32 in rank order, rounded once to the element type: the
 * all-reduce result), every rank's x[t] becomes x[t] + S (rounded) and its
 * out[t] the RMSNorm of that row times `weight`, computed as seb_add_rmsnorm
 * computes it. Rank r computes rows [r*n_tokens/world, (r+1)*n_tokens/world)
 * and stores them on every rank. Each rank issues one call per all-reduce, in
 * the same order on every rank (CUDA-graph capturable: the call count is kept
 * in the flag words). all_ranks = 1 (rank 0) runs every rank's part in one
 * cooperative launch on this device, all buffers being on it. `polls` bounds
 * every wait for a peer (0: a default of a few seconds); a wait that gives up
 * sets SEB_ERRBIT_TIMEOUT in *err and the call returns with invalid rows.
 * hidden % 8 == 0, <= 32768; buffers and weight 16-byte aligned. */
SEB_API int seb_allreduce_add_rmsnorm(void* const* partial, void* const* x, void* const* out, void* const* flags,
                                      const void* weight, int64_t n_tokens, int32_t hidden, float eps,
                                      int32_t dtype, int32_t rank, int32_t world, int32_t all_ranks,
                                      uint32_t polls, int32_t* err, void* stream);

/* Self-test of the bounded waits every kernel uses (no counterpart in the
 * reference, which has no device-side waits): one launch waits `polls` times
 * (1 .. 2^20) on an mbarrier that nothing arrives on, gives up, sets
 * SEB_ERRBIT_TIMEOUT in *err and returns; the CUDA context stays usable. It
 * neither faults nor hangs the GPU. */
SEB_API int seb_selftest_bounded_wait(uint32_t polls, int32_t* err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SERVING_ENGINE_B200_H */
