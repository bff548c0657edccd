/*
 * nie_b200.h - C ABI of the B200 (sm_100a) ragged-batch attention path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * passed as `void*` (NULL = legacy default stream).  No torch or C++ types
 * cross this boundary, so the library can be bound from ctypes, cffi, cgo or
 * JNI alike.  All pointers are DEVICE pointers unless stated otherwise.
 *
 * Cache layout (identical to the reference's PagedKVCache storage,
 * nano_infer_engine/paged_cache.py:71-79):
 *     key_cache / value_cache : [num_layers, num_blocks, block_size,
 *                                kv_heads, head_dim], contiguous
 * A "slot" is block_id * block_size + offset_in_block
 * (nano_infer_engine/paged_cache.py:240-262, used by write at :311-322).
 *
 * Return value: NIE_OK (0) or an NIE_ERR_* code; nie_last_error() gives the
 * message of the last failure on the calling thread.  Launches are
 * asynchronous; device-side range violations (a block id outside the pool, a
 * slot outside the cache) never trap: the kernel skips the access and ORs an
 * NIE_DEV_ERR_* bit into the optional `err_flag` word (int32, device).
 */
#ifndef NIE_B200_H
#define NIE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types of q / k / v / caches */
#define NIE_DTYPE_F32 0
#define NIE_DTYPE_BF16 1
#define NIE_DTYPE_F16 2

/* host-side status codes */
#define NIE_OK 0
#define NIE_ERR_INVALID 1     /* bad argument (shape, pointer, range) */
#define NIE_ERR_UNSUPPORTED 2 /* valid but not implemented for this shape */
#define NIE_ERR_CUDA 3        /* a CUDA runtime/driver call failed */

/* device-side error bits (ORed into *err_flag) */
#define NIE_DEV_ERR_BLOCK_RANGE 1 /* block table entry outside [0, num_blocks) */
#define NIE_DEV_ERR_SLOT_RANGE 2  /* slot outside [0, num_blocks*block_size) */
#define NIE_DEV_ERR_TIMEOUT 4     /* a bounded wait on an mbarrier ran out */
#define NIE_DEV_ERR_CAPACITY 8    /* position beyond the block table row */
#define NIE_DEV_ERR_INDEX_RANGE 16 /* token id outside [0, vocab) */

/* Library version (major*10000 + minor*100 + patch). */
int nie_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* nie_last_error(void);

/* Number of SMs of `device` (cached); <0 on error. */
int nie_device_sm_count(int device);

/*
 * (a) Ragged batch packing.
 * Replaces the host-side packing of the reference:
 *   query_start_loc      nano_infer_engine/generation/paged_prefill.py:132-143
 *   position ids         nano_infer_engine/layers/attention.py:363-376
 *   context lengths      nano_infer_engine/models/llama.py:364-369
 *   slot resolution      nano_infer_engine/paged_cache.py:240-262, 306-322
 *   last-token rows      nano_infer_engine/generation/paged_prefill.py:154
 *
 * plan is int32 [3, num_requests] (device): row 0 = block-table row, row 1 =
 * context length (tokens already cached), row 2 = query length, one column
 * per request in ragged order.  block_tables is an int32
 * [num_rows, table_stride] array of physical block ids (logical order).
 * Outputs (device, caller-allocated):
 *   query_start_loc  int64 [R+1]   0, cumsum(query_length)
 *   positions        int64 [T]     context_length + j for the j-th query token
 *   slot_mapping     int64 [T]     table[pos / bs] * bs + pos % bs (-1 if bad)
 *   seq_lens         int32 [R]     context_length + query_length
 *   last_token_index int64 [R]     query_start_loc[r+1] - 1
 *   token_request    int32 [T]     request index of each token
 *   decode_list      int32 [R]     requests with query_length == 1, in order
 *   prefill_list     int32 [R]     requests with query_length > 1, in order
 *   list_counts      int32 [2]     {#decode, #prefill}
 * T = num_tokens must equal sum(query_length).  Any output pointer except
 * query_start_loc/positions/slot_mapping/seq_lens may be NULL.
 */
int nie_pack_ragged(const int32_t* plan, int32_t num_requests, int64_t num_tokens,
                    const int32_t* block_tables, int64_t table_stride,
                    int32_t block_size, int64_t num_blocks,
                    int64_t* query_start_loc, int64_t* positions,
                    int64_t* slot_mapping, int32_t* seq_lens,
                    int64_t* last_token_index, int32_t* token_request,
                    int32_t* decode_list, int32_t* prefill_list,
                    int32_t* list_counts, int32_t* err_flag, void* stream);

/*
 * (b) Paged KV slot write.
 * Replaces PagedKVCache.write (nano_infer_engine/paged_cache.py:264-322):
 * key_cache[layer, slot / bs, slot % bs] = keys[t] (and values) for every t
 * with slot_mapping[t] >= 0.  keys/values are contiguous [T, kv_heads,
 * head_dim] of `dtype`; the copy is bit-exact.
 */
int nie_write_kv(const void* keys, const void* values, int64_t num_tokens,
                 void* key_cache, void* value_cache, int32_t dtype, int32_t layer,
                 int64_t num_layers, int64_t num_blocks, int32_t block_size,
                 int32_t kv_heads, int32_t head_dim, const int64_t* slot_mapping,
                 int32_t* err_flag, void* stream);

/*
 * Paged KV gather into contiguous [T, kv_heads, head_dim] tensors.
 * Replaces PagedKVCache.gather (nano_infer_engine/paged_cache.py:324-362):
 * out[t] = cache[layer, table[t / bs], t % bs] for t in [0, num_tokens).
 * block_table is the sequence's int32 row (logical block order).
 */
int nie_gather_kv(const void* key_cache, const void* value_cache, int32_t dtype,
                  int32_t layer, int64_t num_layers, int64_t num_blocks,
                  int32_t block_size, int32_t kv_heads, int32_t head_dim,
                  const int32_t* block_table, int64_t num_tokens, void* out_keys,
                  void* out_values, int32_t* err_flag, void* stream);

/*
 * (e) Block copy between two paged pools (same or peer device).
 * Replaces PagedKVCache.export_sequence / import_sequence
 * (nano_infer_engine/paged_cache.py:145-238) and the per-block cross-device
 * copy_ of the P/D handoff (nano_infer_engine/generation/pd_scheduler.py:
 * 144-145 into paged_cache.py:228-234).  For every layer l and logical block j < num_copy_blocks:
 *   dst[l, dst_blocks[j]] = src[l, src_blocks[j]]
 * and, when tail_valid_tokens in (0, block_size), token rows
 * [tail_valid_tokens, block_size) of the LAST copied block are written as
 * zeros (the zeroed export tail, paged_cache.py:165-169).  src_blocks or
 * dst_blocks may be NULL meaning the identity (j), which lets a dense
 * [L, n, bs, H, D] transfer tensor act as either side.  The kernel runs on
 * the stream's device; a peer pointer (after nie_enable_peer_access) makes it
 * a direct NVLink copy with 16-byte vector loads/stores.
 */
int nie_copy_blocks(const void* src_keys, const void* src_values,
                    int64_t src_num_blocks, const int32_t* src_blocks,
                    void* dst_keys, void* dst_values, int64_t dst_num_blocks,
                    const int32_t* dst_blocks, int64_t num_copy_blocks,
                    int32_t tail_valid_tokens, int32_t dtype, int64_t num_layers,
                    int32_t block_size, int32_t kv_heads, int32_t head_dim,
                    int32_t* err_flag, void* stream);

/* Enable access from `device` to memory of `peer_device` (idempotent). */
int nie_enable_peer_access(int device, int peer_device);

/*
 * CUDA IPC for prefill/decode processes (one process per GPU).  The
 * reference moves KV between devices inside one process
 * (generation/pd_scheduler.py:144-145, paged_cache.py:228-234); with a process per GPU the decode process maps
 * the prefill process's pool and nie_copy_blocks pulls blocks over NVLink.
 * nie_ipc_export writes the 64-byte handle of the allocation that contains
 * `ptr` and ptr's offset in it; nie_ipc_import (in another process, on the
 * current device) maps it with lazy peer access and returns the pointer and
 * the mapping base, which nie_ipc_close releases.
 */
int nie_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out);
int nie_ipc_import(const void* handle, uint64_t offset, void** ptr_out,
                   void** base_out);
int nie_ipc_close(void* base);

/*
 * (c) Paged decode attention: one query token per request.
 * Replaces batched_paged_attention_reference
 * (nano_infer_engine/layers/paged_attention.py:117-176, per-sequence body
 * :4-114): for request r (= req_list[i] if req_list else i) with query row
 * qr (= q_rows[r] if q_rows else r), block-table row tr (= table_rows[r] if
 * table_rows else r) and n = seq_lens[r] cached tokens:
 *   out[qr, h] = softmax(q[qr, h] . K[0:n, h / G]^T * scale) V[0:n, h / G]
 * with G = q_heads / kv_heads.  q/out rows are [q_heads, head_dim]
 * contiguous with row stride `q_row_stride` / `out_row_stride` elements.
 * Numerics follow the reference: the dot product is rounded to `dtype`,
 * multiplied by `scale`, rounded again, and the softmax runs in fp32.
 *
 * bf16 / head_dim 64 / block_size 16 uses the split-K TMA kernel, which needs
 * `workspace` of nie_paged_decode_workspace_size() bytes (scratch; contents
 * need no initialisation); other shapes use a generic kernel and ignore it.
 */
size_t nie_paged_decode_workspace_size(int device, int32_t num_requests,
                                       int32_t q_heads, int32_t head_dim);

int nie_paged_decode(const void* q, int64_t q_row_stride, void* out,
                     int64_t out_row_stride, const void* key_cache,
                     const void* value_cache, int32_t dtype, int32_t layer,
                     int64_t num_layers, int64_t num_blocks, int32_t block_size,
                     int32_t kv_heads, int32_t head_dim, int32_t q_heads,
                     const int32_t* block_tables, int64_t table_stride,
                     const int32_t* table_rows, const int32_t* seq_lens,
                     const int64_t* q_rows, const int32_t* req_list,
                     int32_t num_requests, float scale, void* workspace,
                     size_t workspace_bytes, int32_t* err_flag, void* stream);

/*
 * nie_paged_decode_overlapped: nie_paged_decode whose split-K kernel may start
 * (block-table walk, barrier setup) while the kernel issued just before it on
 * `stream` is still running; it waits for that kernel before reading q or the
 * caches.  Precondition: the block tables, table rows, seq_lens, q_rows and
 * the request list must be complete before the most recent kernel on `stream`
 * that was launched WITHOUT programmatic stream serialization.  A chain of
 * dependent launches that each trigger at their start (this library's fused
 * kernels and nie_linear do) can run several kernels back at once, so "not
 * written by the kernel just before" is not enough: the metadata must predate
 * the whole chain.  The engine writes it in its packing kernel and launches
 * the q/k/v projection as a plain library GEMM between the two, which ends
 * any chain; q and the new cache rows come from the RoPE + KV write right
 * before.  Same arguments, results and errors as nie_paged_decode.
 */
int nie_paged_decode_overlapped(const void* q, int64_t q_row_stride, void* out,
                                int64_t out_row_stride, const void* key_cache,
                                const void* value_cache, int32_t dtype,
                                int32_t layer, int64_t num_layers,
                                int64_t num_blocks, int32_t block_size,
                                int32_t kv_heads, int32_t head_dim,
                                int32_t q_heads, const int32_t* block_tables,
                                int64_t table_stride, const int32_t* table_rows,
                                const int32_t* seq_lens, const int64_t* q_rows,
                                const int32_t* req_list, int32_t num_requests,
                                float scale, void* workspace,
                                size_t workspace_bytes, int32_t* err_flag,
                                void* stream);

/*
 * Allocation-free paged decode.  This entry point has no counterpart in the
 * reference engine; it exists for callers that cannot allocate device memory:
 * code that binds this C ABI from a host language with no device allocator of
 * its own (a cgo, JNI or plain ctypes binding that only holds the buffers it
 * was handed), or an embedding runtime that owns all device memory through its
 * own pool and must not see extra cudaMalloc/cudaFree calls (which can also
 * stall a serving loop by synchronizing the device).
 *
 * Same arguments and results as nie_paged_decode, minus the workspace: the
 * split-K scratch is a fixed array of NIE_DECODE_NOALLOC_SCRATCH_BYTES inside
 * the library, which every GPU that loads the library holds until the process
 * exits.  The caller still passes q, out, the caches, tables and lengths.
 *  - Limit: the call must fit the array, i.e.
 *    nie_paged_decode_workspace_size(...) <= NIE_DECODE_NOALLOC_SCRATCH_BYTES
 *    (about 840 requests at 32 query heads on a 148-SM B200); larger calls
 *    fail with NIE_ERR_INVALID and a message naming the limit.
 *  - The first call on a device looks up the array's device address with that
 *    device current; make that first call before any stream capture.  An empty
 *    batch (num_requests == 0) only checks its arguments and resolves nothing.
 *  - Devices: ordinals 0 .. NIE_DECODE_NOALLOC_MAX_DEVICES-1 (64 GPUs per
 *    process); a stream on a higher ordinal fails with NIE_ERR_INVALID.
 *  - Every call shares the one array, which keeps the last call's contents
 *    (the kernels need no zeroed scratch).  Calls that overlap on the GPU
 *    (several streams or host threads at once) race on it: serialize them.
 *  - Nothing is allocated: no cudaMalloc, cudaFree or allocating library call.
 */
#define NIE_DECODE_NOALLOC_SCRATCH_BYTES (8 * 1024 * 1024)
#define NIE_DECODE_NOALLOC_MAX_DEVICES 64

/* Size in bytes of the fixed scratch array (NIE_DECODE_NOALLOC_SCRATCH_BYTES). */
size_t nie_paged_decode_noalloc_capacity(void);

int nie_paged_decode_noalloc(const void* q, int64_t q_row_stride, void* out,
                             int64_t out_row_stride, const void* key_cache,
                             const void* value_cache, int32_t dtype,
                             int32_t layer, int64_t num_layers,
                             int64_t num_blocks, int32_t block_size,
                             int32_t kv_heads, int32_t head_dim,
                             int32_t q_heads, const int32_t* block_tables,
                             int64_t table_stride, const int32_t* table_rows,
                             const int32_t* seq_lens, const int64_t* q_rows,
                             const int32_t* req_list, int32_t num_requests,
                             float scale, int32_t* err_flag, void* stream);

/*
 * (d) Varlen causal attention over the paged cache (chunked prefill, and the
 * prefill rows of a mixed step).  Replaces the per-request write/gather/
 * attention loop of GroupedQueryAttention.forward_ragged
 * (nano_infer_engine/layers/attention.py:378-413) and the dense paged
 * prefill (nano_infer_engine/models/llama.py:274-325 with
 * attention.py:275-343).  The new keys/values must already be written into
 * the cache (nie_write_kv).  For request r = req_list[i] (or i), its query
 * tokens are rows [query_start_loc[r], query_start_loc[r+1]) of q/out; the
 * token at offset j has position seq_lens[r] - qlen + j and attends to cached
 * positions [0, position].  q/out hold num_q_rows rows of [q_heads,
 * head_dim] at `row_stride` elements.
 *
 * bf16 / head_dim 64 / block_size 16 runs on the tcgen05 tensor cores (S and
 * O accumulate in TMEM, K/V tiles arrive by TMA); other shapes use the
 * generic kernel.  max_seq_len (host value, >= every seq_lens[r]; 0 =
 * unknown) lets the tensor-core path split long key ranges over several CTAs;
 * the split needs `workspace` of nie_varlen_workspace_size() bytes (scratch,
 * no initialisation needed: the call clears its flags on the stream) and is
 * skipped when it is NULL or too small.  Split ranges are merged inside the
 * one kernel: the call launches a memset and one kernel, and calls sharing a
 * workspace must not overlap on the GPU.
 */
size_t nie_varlen_workspace_size(int32_t num_requests, int32_t max_query_len,
                                 int32_t max_seq_len, int32_t q_heads);

int nie_varlen_attention(const void* q, void* out, int64_t row_stride, int64_t num_q_rows,
                         const void* key_cache, const void* value_cache,
                         int32_t dtype, int32_t layer, int64_t num_layers,
                         int64_t num_blocks, int32_t block_size, int32_t kv_heads,
                         int32_t head_dim, int32_t q_heads,
                         const int32_t* block_tables, int64_t table_stride,
                         const int32_t* table_rows, const int32_t* seq_lens,
                         const int64_t* query_start_loc, const int32_t* req_list,
                         int32_t num_requests, int32_t max_query_len,
                         int32_t max_seq_len, float scale, void* workspace,
                         size_t workspace_bytes, int32_t* err_flag, void* stream);

/*
 * Fused elementwise stages of one ragged step.  Each reproduces the rounding
 * sequence of the torch op chain it replaces (every intermediate that the
 * reference materialises in the activation dtype is rounded to it).
 *
 * nie_add_rmsnorm: sum = x + residual (residual may be NULL), out = weight *
 * (sum / sqrt(mean(sum^2) + eps)), fp32 inside; sum_out (may be NULL)
 * receives the rounded sum.  Rows of `hidden` contiguous elements, hidden <=
 * 4096.  Replaces RmsNorm.forward (nano_infer_engine/layers/rms_norm.py:25-31)
 * together with the residual adds of layers/decoder.py:55-74.
 */
int nie_add_rmsnorm(const void* x, const void* residual, const void* weight,
                    float eps, int64_t rows, int32_t hidden, int32_t dtype,
                    void* sum_out, void* out, void* stream);

/*
 * nie_rope_write_kv: rotary embedding of q and k by per-token sin/cos ([T,
 * head_dim/2], activation dtype) with the half-split pairing, rotated q to
 * q_out [T, q_heads, head_dim], rotated k and v stored into the cache slots
 * (as nie_write_kv).  Replaces the RoPE of layers/rope.py:6-23 applied in
 * layers/attention.py:375-376 plus the slot write of paged_cache.py:264-322.
 */
int nie_rope_write_kv(const void* q, int64_t q_stride, const void* k,
                      int64_t k_stride, const void* v, int64_t v_stride,
                      const void* sin, const void* cos, int64_t num_tokens,
                      int32_t q_heads, int32_t kv_heads, int32_t head_dim,
                      void* q_out, void* key_cache, void* value_cache,
                      int32_t dtype, int32_t layer, int64_t num_layers,
                      int64_t num_blocks, int32_t block_size,
                      const int64_t* slot_mapping, int32_t* err_flag,
                      void* stream);

/*
 * nie_silu_mul: out = silu(gate) * up with silu = x / (1 + exp(-x)) in fp32
 * and both results rounded like torch (layers/mlp.py:18-22).
 */
int nie_silu_mul(const void* gate, int64_t gate_stride, const void* up,
                 int64_t up_stride, void* out, int64_t rows, int32_t cols,
                 int32_t dtype, void* stream);

/*
 * nie_embed_rows: out[t] = table[ids[t]] for t < num_tokens, a bit-exact
 * copy of rows of the [vocab, hidden] embedding table (the nn.Embedding
 * lookup of models/llama.py:269 and :381).  ids are int64 (device); an id
 * outside [0, vocab) gives a zero row and NIE_DEV_ERR_INDEX_RANGE.  Rows
 * must be a multiple of 16 bytes; table and out 16-byte aligned.
 */
int nie_embed_rows(const int64_t* ids, int64_t num_tokens, const void* table,
                   int64_t vocab, int32_t hidden, int32_t dtype, void* out,
                   int32_t* err_flag, void* stream);

/*
 * nie_argmax_rows: out[r] = torch.argmax(logits[r]) for r < rows <= 4096:
 * the first index of the row maximum, NaN ranking above every number (the
 * greedy sampling of generation/scheduler.py:400 and :505).
 * Rows of `cols` elements at `row_stride`.  The workspace
 * (nie_argmax_workspace_size bytes, 256-byte aligned, fixed layout) must be
 * zero before its first use; the kernel leaves its counters at zero.  Calls
 * sharing a workspace must not overlap on the GPU.
 */
size_t nie_argmax_workspace_size(void);

int nie_argmax_rows(const void* logits, int64_t rows, int64_t cols,
                    int64_t row_stride, int32_t dtype, int64_t* out,
                    void* workspace, size_t workspace_bytes, void* stream);

/*
 * nie_linear: y[m, n] = x[m, k] . w[n, k]^T for decode-size batches (the
 * nn.Linear projections of a decode step: layers/attention.py:121-145 q/k/v
 * and o, layers/mlp.py:18-22 gate/up and down).  bf16 in and out, fp32
 * accumulation, one rounding of each output.  Takes m <= 16, n % 128 == 0,
 * k % 64 == 0, x and w 16-byte aligned with row strides ldx (a multiple of 8
 * elements) and k, y rows at ldy (even); anything else returns
 * NIE_ERR_UNSUPPORTED so the caller can use a library GEMM.  The weights are
 * streamed once over all SMs (K split across a thread-block cluster where n
 * is small); no workspace.  Results are deterministic.
 */
int nie_linear(const void* x, int64_t ldx, const void* w, int64_t n, int64_t k,
               int64_t m, void* y, int64_t ldy, int32_t dtype,
               int32_t* err_flag, void* stream);

/*
 * nie_linear_overlapped: nie_linear that starts streaming w while the kernel
 * issued just before it on `stream` is still running (x is read only after
 * that kernel completes).  Precondition: that immediately preceding kernel
 * must NOT write w (weights are normally written long before; the engine calls
 * this right after the attention combine or SiLU * up kernel).  Same
 * arguments, results and errors as nie_linear.
 */
int nie_linear_overlapped(const void* x, int64_t ldx, const void* w, int64_t n,
                          int64_t k, int64_t m, void* y, int64_t ldy,
                          int32_t dtype, int32_t* err_flag, void* stream);

/*
 * nie_linear_timeout_test: failure-path test hook (no reference counterpart).
 * Launches nie_linear's kernel with its producer issuing no copy, so every
 * consumer's bounded mbarrier wait runs out after `wait_probes` probes
 * (1 .. 2^22).  With no copy in flight, the kernel raises NIE_DEV_ERR_TIMEOUT
 * in `err_flag`, joins its cluster barrier, writes zeros to y and returns;
 * the context stays usable.  Checks that a timed-out wait ends the kernel
 * instead of hanging it; never used on the data path.
 */
int nie_linear_timeout_test(const void* x, int64_t ldx, const void* w, int64_t n,
                            int64_t k, int64_t m, void* y, int64_t ldy,
                            int32_t dtype, int32_t* err_flag, void* stream,
                            uint32_t wait_probes);

#ifdef __cplusplus
}
#endif

#endif /* NIE_B200_H */
