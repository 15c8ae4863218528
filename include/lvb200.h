/*
 * lvb200.h -- C ABI of the B200 (sm_100a) hot-path library for light-vllm.
 *
 * The library implements the two GPU pieces of light-vllm's decode/prefill
 * path behind plain C entry points: the AutoAWQ W4A16 linear (the work of the
 * reference's `awq_gemm` / `awq_dequantize` extension) and the paged K/V write
 * plus paged attention (the work of the reference's Triton backend).  Every
 * entry point takes raw device pointers, element counts, strides and a CUDA
 * stream, enqueues work on that stream and returns a status code; none of them
 * synchronises the device or allocates device memory.  No torch types appear
 * here: any FFI (ctypes, cffi, pybind11, a C++ host) can bind it.
 *
 * Reference paths below are relative to the light-vllm repository.
 *
 * Data types: `uint16_t` buffers hold IEEE fp16 or bf16 bit patterns as named
 * by a `dtype` argument (LVB_DTYPE_F16 / LVB_DTYPE_BF16).  AWQ activations,
 * scales, bias and outputs are always fp16 (the reference hard-wires fp16 for
 * AWQ: modeling/quantization/awq.py:673-675, cuda_awq.py:65-66).
 *
 * Errors: a non-zero status means nothing was enqueued.  `lvb_last_error()`
 * returns a thread-local message for the most recent failure on the calling
 * thread.  Kernels never trap: a device-side wait that exceeds its time limit
 * records a code that `lvb_device_error()` returns (and clears).
 */
#ifndef LVB200_H_
#define LVB200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LVB_API __attribute__((visibility("default")))
#else
#define LVB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *lvb_stream_t; /* same handle as cudaStream_t */

enum lvb_status {
  LVB_OK = 0,
  LVB_ERR_INVALID = 1,     /* bad shape, size, alignment or pointer (ValueError) */
  LVB_ERR_UNSUPPORTED = 2, /* valid request outside what the kernels cover   */
  LVB_ERR_CUDA = 3,        /* a CUDA runtime call failed (RuntimeError)      */
  LVB_ERR_WORKSPACE = 4,   /* caller's workspace smaller than required       */
  LVB_ERR_METADATA = 5     /* block tables violate the paged-cache contract (KVCacheError) */
};

enum lvb_dtype { LVB_DTYPE_F16 = 0, LVB_DTYPE_BF16 = 1 };

/* Library identification: ABI version (bumped on any signature change). */
LVB_API int lvb_abi_version(void);

/* Message for the last non-zero status returned on this thread. */
LVB_API const char *lvb_last_error(void);

/* Device-side error word for the current device (0 = none), cleared on read.
 * Bit 0: a pipeline wait timed out; bit 1: an index check failed.
 * Synchronises the current device. */
LVB_API int lvb_device_error(uint32_t *error_out);

/* ------------------------------------------------------------------------ */
/* AWQ W4A16 linear                                                          */
/* ------------------------------------------------------------------------ */

/* Bytes of workspace `lvb_awq_linear` (and `lvb_awq_linear_packed`) needs for
 * an m x k x n call on the current device: split-K reduction semaphores followed by fp32 partial
 * tiles.  A workspace must be zero-filled once before its first use; every
 * call leaves its semaphores zero again, so one buffer serves all later calls
 * of the same or smaller size.  Replaces the fp16 split partial planes that
 * `awq_gemm` allocates per call
 * (modeling/quantization/csrc/awq/gemm_kernels.cu:456-457). */
LVB_API size_t lvb_awq_workspace_bytes(int64_t m, int64_t k, int64_t n, int64_t group_size);

/* y[m, n] = x[m, :k] @ W + bias, W[k, n] = fp16(q - z) * s dequantised on the
 * fly from the AutoAWQ GEMM layout (qweight int32 [k, n/8], qzeros int32
 * [k/group, n/8], scales fp16 [k/group, n]; nibble p of a word holds column
 * 8j + (0,2,4,6,1,3,5,7)[p]).  fp32 accumulation on tcgen05 tensor cores.
 * x and y are row-major with row strides k and n; `bias` may be NULL.
 * Requirements: n % 32 == 0, k % 8 == 0, group_size % 32 == 0,
 * k % group_size == 0, 16-byte aligned x / qweight / scales / workspace.  Replaces `awq_gemm`
 * (csrc/awq/bindings.cpp:10-13, gemm_kernels.cu:444-501) together with the
 * M>255 dequantise + cuBLAS path and the bias add of
 * `CudaAWQOperation.__call__` (cuda_awq.py:96-122). */
LVB_API int lvb_awq_linear(const uint16_t *x, const int32_t *qweight, const int32_t *qzeros,
                   const uint16_t *scales, const uint16_t *bias, uint16_t *y, int64_t m,
                   int64_t k, int64_t n, int64_t group_size, void *workspace,
                   size_t workspace_bytes, lvb_stream_t stream);

/* Same computation as lvb_awq_linear, for callers that cannot allocate
 * device memory: hosts whose device memory is wholly owned by another
 * allocator that they may not grow, or threads on a latency-critical path where
 * the device-wide synchronisation of cudaMalloc is not acceptable.  It takes no
 * workspace; the split-K scratch is a fixed array of 6 MiB + 4 KiB inside the
 * library (every GPU that loads the library holds it until exit), so calls
 * whose plan needs more than that are rejected with LVB_ERR_UNSUPPORTED (no
 * call on a GPU with up to 192 SMs does).  It calls no cudaMalloc/cudaFree.
 * The first call on a device looks up the array's device address (set-up,
 * once per device, on the calling thread's current device); make that first
 * call before any stream capture.  The address is cached for the process and
 * is not valid after cudaDeviceReset.  Every call on a device shares the one
 * array, which keeps the previous call's contents: each call clears the
 * split-K semaphores it will use (cudaMemsetAsync on its stream) before its
 * kernel, so a call that follows one aborted by a wait timeout starts clean.
 * Calls that overlap on the GPU (different streams, no ordering between them)
 * race and may produce wrong results; order them on one stream.  No
 * counterpart in the reference. */
LVB_API int lvb_awq_linear_static(const uint16_t *x, const int32_t *qweight,
                                  const int32_t *qzeros, const uint16_t *scales,
                                  const uint16_t *bias, uint16_t *y, int64_t m, int64_t k,
                                  int64_t n, int64_t group_size, lvb_stream_t stream);

/* w[k, n] = fp16(q - z) * s, the full fp16 weight.  Replaces `awq_dequantize`
 * (csrc/awq/bindings.cpp:10-13, gemm_kernels.cu:391-439). */
LVB_API int lvb_awq_dequantize(const int32_t *qweight, const int32_t *qzeros, const uint16_t *scales,
                       uint16_t *w, int64_t k, int64_t n, int64_t group_size,
                       lvb_stream_t stream);

/* The QKV projection of a decode step with its epilogue: y = x W + bias over
 * the packed layout (lvb_awq_linear_packed), and then, per token, the Qwen2
 * half-rotation RoPE (lvb_rope_kv_write's arithmetic) applied to the query
 * heads in y, the rotated key heads written to the token's paged cache slot
 * and the value heads copied there -- the QKV epilogue of
 * `Qwen2Attention.forward` (modeling/models/qwen2.py:380-411) with the K/V
 * write of the attention step (runtime/execution/triton_paged_attention.py:
 * 31-104, _qwen2_kernels.py:66-133), in the projection's own launch.  y holds
 * merged [q | k | v] rows of (hq + 2 hkv) x head_size values (head size 64 or
 * 128); its key and value heads are left unrotated.  Covers the one-row
 * decode GEMV (m = 1); other shapes return LVB_ERR_UNSUPPORTED and the caller
 * runs lvb_awq_linear_packed + lvb_rope_kv_write.  Positions outside the
 * tables set LVB_DEVERR_INDEX. */
LVB_API int lvb_awq_qkv_rope_packed(const uint16_t *x, const void *codes, const void *groups, const uint16_t *bias,
                                    uint16_t *y, int64_t m, int64_t k, int64_t n, int64_t group_size,
                                    void *workspace, size_t workspace_bytes, const int32_t *positions,
                                    const uint16_t *cos_table, const uint16_t *sin_table, int64_t table_rows,
                                    uint16_t *key_cache, uint16_t *value_cache, const int32_t *block_tables,
                                    int64_t table_stride, const int32_t *num_computed,
                                    const int32_t *query_start_loc, const int32_t *request_indices,
                                    int64_t num_query_heads, int64_t num_kv_heads, int64_t head_size,
                                    int64_t block_size, lvb_stream_t stream);

/* Packed decode layout.  AWQScheme.prepare (modeling/quantization/awq.py:
 * 468-486) hands a backend the checkpoint once, after loading, so that it can
 * convert it (the protocol names Marlin-style backends, which repack); the
 * B200 scheme repacks into a layout the decode kernel streams with one bulk
 * copy per 256-k stage:
 *   codes   [ceil(n/128) column tiles][ceil(k/64)*2 runs][128 columns][16 B]:
 *           the 32 int4 codes of one column for k = 32r .. 32r+31; word w of
 *           the 16 bytes holds k = 4w, 4w+1, 4w+2, 4w+3 in nibbles 0, 4, 2, 6
 *           and k = 16+4w .. 16+4w+3 in nibbles 1, 5, 3, 7 (codes past k or
 *           n are 0);
 *   groups  [ceil(n/128)][k/group_size][128] uint32: fp16 scale bits in the
 *           low half, the int4 zero point in bits 16..19 (0 past n).
 * lvb_awq_pack_bytes reports both sizes; lvb_awq_pack writes them on `stream`
 * from the arrays lvb_awq_linear takes (same requirements). */
LVB_API int lvb_awq_pack_bytes(int64_t k, int64_t n, int64_t group_size, size_t *codes_bytes,
                               size_t *groups_bytes);
LVB_API int lvb_awq_pack(const int32_t *qweight, const int32_t *qzeros, const uint16_t *scales,
                         int64_t k, int64_t n, int64_t group_size, void *codes, void *groups,
                         lvb_stream_t stream);

/* y[m, n] = x[m, :k] @ W + bias from the packed layout, any m.  Same
 * arithmetic and requirements as lvb_awq_linear (the one-row GEMV and the
 * int8 decode path apply the zero point and scale exactly instead of rounding
 * W to fp16).  Decode batches of 2..16 rows run the warp-MMA kernel.  The split-K plan uses at
 * most `workspace_bytes` of workspace (NULL or 0: no split), so a smaller
 * workspace only costs speed; lvb_awq_workspace_bytes gives the size of the
 * fastest plan.  `codes` may be the checkpoint's own qweight buffer
 * after repacking it in place (same byte size when n % 128 == 0 and
 * k % 64 == 0).  Replaces `awq_gemm` and the M>255 dequantise + cuBLAS path
 * (csrc/awq/bindings.cpp:10-13, gemm_kernels.cu:444-501, called from
 * `CudaAWQOperation.__call__`, cuda_awq.py:96-122). */
LVB_API int lvb_awq_linear_packed(const uint16_t *x, const void *codes, const void *groups,
                                  const uint16_t *bias, uint16_t *y, int64_t m, int64_t k,
                                  int64_t n, int64_t group_size, void *workspace,
                                  size_t workspace_bytes, lvb_stream_t stream);

/* y = (silu(gate) * up) @ W (+ bias) on the packed layout, with the SiLU-mul
 * computed inside the activation prologue of the decode kernels (fp32, one
 * fp16 rounding, as lvb_silu_mul): gate_up holds m rows of [gate (k values) |
 * up (k values)], gate_up_stride elements apart.  Replaces `silu_and_mul`
 * followed by the down projection (modeling/models/qwen2.py:237-247,
 * _qwen2_kernels.py:45-64).  Covers the decode batches: one row (the GEMV
 * builds fp16(silu(gate) * up) in its prologue), the shapes of the warp-MMA
 * kernel (the activation goes through the workspace: lvb_silu_mul, then the
 * warp-MMA projection), and the int8 path when the workspace cannot hold
 * the warp-MMA plan (m <= 16, groups of 128 / 256); other shapes return
 * LVB_ERR_UNSUPPORTED and
 * the caller runs lvb_silu_mul + lvb_awq_linear_packed. */
LVB_API int lvb_awq_silu_linear_packed(const uint16_t *gate_up, int64_t gate_up_stride, const void *codes,
                                       const void *groups, const uint16_t *bias, uint16_t *y, int64_t m, int64_t k,
                                       int64_t n, int64_t group_size, void *workspace, size_t workspace_bytes,
                                       lvb_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Paged K/V cache                                                           */
/* ------------------------------------------------------------------------ */
/* Cache layout (runtime/execution/paged_cache.py:328-338): per layer, K and V
 * are separate contiguous tensors [num_blocks, block_size, num_kv_heads,
 * head_size].  Per-step metadata (runtime/execution/paged_attention.py:18-206):
 *   block_tables     int32 [num_seqs, table_stride], row r = request r's
 *                    physical block ids (rows padded with any valid id);
 *   num_computed     int32 [num_seqs], tokens already in the cache;
 *   query_start_loc  int32 [num_seqs + 1], prefix sums of query lengths;
 *   request_indices  int32 [num_tokens], request of each packed token.
 * Token t of request r (offset o = t - query_start_loc[r]) is written to slot
 * block_tables[r][(c + o) / bs] * bs + (c + o) % bs, c = num_computed[r]. */

/* Scatter this step's K/V rows into their slots.  key/value rows: token
 * stride in elements, heads contiguous at stride head_size.  Replaces the
 * Triton `_write_paged_kv_kernel` launch
 * (runtime/execution/triton_paged_attention.py:31-104, 498-517). */
LVB_API int lvb_paged_kv_write(const uint16_t *key, int64_t key_token_stride, const uint16_t *value,
                       int64_t value_token_stride, uint16_t *key_cache, uint16_t *value_cache,
                       const int32_t *block_tables, int64_t table_stride,
                       const int32_t *num_computed, const int32_t *query_start_loc,
                       const int32_t *request_indices, int64_t num_tokens, int64_t num_kv_heads,
                       int64_t head_size, int64_t block_size, int dtype, lvb_stream_t stream);

/* Scatter rows into explicit flat slots (slot = block * block_size + offset).
 * Replaces `PagedKVCache.write_prepared`'s index_copy_
 * (runtime/execution/paged_cache.py:208-248). */
LVB_API int lvb_kv_scatter(const uint16_t *key, int64_t key_token_stride, const uint16_t *value,
                   int64_t value_token_stride, uint16_t *key_cache, uint16_t *value_cache,
                   const int64_t *slots, int64_t num_tokens, int64_t num_kv_heads,
                   int64_t head_size, int64_t num_slots, int dtype, lvb_stream_t stream);

/* Plan of the tree-acceptance compaction `PagedKVCache.compact`
 * (runtime/execution/paged_cache.py:257-326): checks its argument rules in
 * the reference's order (LVB_ERR_INVALID where it raises ValueError,
 * LVB_ERR_METADATA where it raises KVCacheError, same messages) and writes
 * the (source, target) slot of each retained query token; *moved = how many
 * pairs differ (0: nothing to move).  counts = {num_computed_tokens,
 * num_query_tokens, num_reserved_query_tokens, num_readonly_prefix_blocks};
 * callers pass -1 for a value that is not an integer.  Host only. */
LVB_API int lvb_kv_compact_plan(const int64_t *block_ids, int64_t num_table_blocks, const int64_t *counts,
                                const int64_t *retained, int64_t num_retained, int64_t num_blocks,
                                int64_t block_size, int32_t *src_slots, int32_t *dst_slots, int64_t *moved);

/* Move K and V rows of one layer from src_slots[i] to dst_slots[i] (every
 * KV head); every source row is read before any target is written, so the
 * pairs may overlap.  The device half of `PagedKVCache.compact`'s
 * index_select + index_copy_ (paged_cache.py:312-325).  Rows x head_size x 2
 * bytes must fit 96 KiB. */
LVB_API int lvb_kv_move_rows(uint16_t *key_cache, uint16_t *value_cache, const int32_t *src_slots,
                             const int32_t *dst_slots, int64_t num_rows, int64_t num_kv_heads, int64_t head_size,
                             int64_t num_slots, int dtype, lvb_stream_t stream);

/* Host-only (no device work): validate one step's block tables and pack the
 * int32 payload the K/V-write and attention kernels read.  Inputs: the
 * concatenated block ids of every request with table_offsets[num_seqs + 1]
 * row offsets, and per request the computed-token count, the query length,
 * the reserved query slots (>= query length) and the read-only prefix block
 * count.  The rules, their order and the messages are those of
 * PagedAttentionMetadata.validate_block_tables
 * (runtime/execution/paged_attention.py:138-172); a violation returns
 * LVB_ERR_METADATA with the reference's message.  On success `out` holds
 * [block tables padded to *table_stride_out columns | num_computed |
 * query_start_loc (num_seqs + 1) | request_indices (*num_tokens_out) |
 * request_order (2 * num_seqs: the requests by descending num_computed, ties
 * in index order, then their num_computed in that order)], the payload of one
 * host-to-device copy (triton_paged_attention.py:422-440, plus the launch
 * order that lvb_paged_attention takes).  out_capacity (int32 elements) must
 * be at least num_seqs * max_table + 4 * num_seqs + 1 + num_tokens. */
LVB_API int lvb_pack_step_metadata(const int32_t *block_ids, const int64_t *table_offsets,
                                   const int32_t *num_computed, const int32_t *query_lengths,
                                   const int32_t *reserved, const int32_t *readonly,
                                   int64_t num_seqs, int64_t num_blocks, int64_t block_size,
                                   int32_t *out, int64_t out_capacity,
                                   int64_t *table_stride_out, int64_t *num_tokens_out);

/* One step's metadata staged for the device in one call: waits on the host
 * until `slot_event` (NULL: no wait) has passed, i.e. the copy last issued
 * from `pinned_out` finished; packs exactly as lvb_pack_step_metadata into
 * the page-locked `pinned_out`; copies the payload to `device_out`
 * (device_capacity int32 elements) on `stream`; records `slot_event` on
 * `stream` after the copy.  The native form of the reference's
 * SingleStepCudaStagingBuffer.copy_groups (runtime/execution/cuda_staging.py:11-70)
 * for the packed payload; a block-table violation returns LVB_ERR_METADATA
 * before anything is copied. */
LVB_API int lvb_stage_step_metadata(const int32_t *block_ids, const int64_t *table_offsets,
                                    const int32_t *num_computed, const int32_t *query_lengths,
                                    const int32_t *reserved, const int32_t *readonly, int64_t num_seqs,
                                    int64_t num_blocks, int64_t block_size, int32_t *pinned_out,
                                    int64_t out_capacity, int32_t *device_out, int64_t device_capacity,
                                    void *slot_event, lvb_stream_t stream, int64_t *table_stride_out,
                                    int64_t *num_tokens_out);

/* Events for staging slots (cudaEventDisableTiming): create, destroy, record
 * on a stream, and wait on the host (a poll, then a synchronize only if the
 * event is still pending; an event never recorded counts as passed). */
LVB_API int lvb_event_create(void **event);
LVB_API int lvb_event_destroy(void *event);
LVB_API int lvb_event_record(void *event, lvb_stream_t stream);
LVB_API int lvb_event_wait_host(void *event);

/* Stream plumbing for callers that overlap their own host<->device copies
 * with the attention and projection launches (no counterpart in the
 * reference, whose Python callers use torch.cuda streams): make `stream`
 * wait for `event` (cudaStreamWaitEvent), and copy `bytes` bytes between any
 * two addresses on `stream` (cudaMemcpyAsync, direction inferred; host
 * memory should be pinned for the copy to be asynchronous). */
LVB_API int lvb_stream_wait_event(lvb_stream_t stream, void *event);
LVB_API int lvb_copy_async(void *dst, const void *src, size_t bytes, lvb_stream_t stream);

/* Bytes of workspace `lvb_paged_attention` needs: split-context partial
 * outputs and log-sum-exps, then one word per (request, KV head) (the
 * balanced schedule's piece counts).  Zero-fill it once before first use. */
LVB_API size_t lvb_paged_attention_workspace_bytes(int64_t num_seqs, int64_t num_q_heads,
                                           int64_t num_kv_heads, int64_t head_size,
                                           int64_t max_seq_len);

/* out[t, h, :] = softmax(scale * q[t, h] . K_visible^T) V_visible over the
 * pages of token t's request.  Visible positions: every computed position,
 * plus, among this step's queries of the request, the query itself and its
 * ancestors.  visibility == NULL means linear (causal) layouts; otherwise
 * visibility is the packed boolean matrix per request (row-major, qlen x qlen)
 * starting at visibility_start[r].  The query heads of one KV head are
 * num_q_heads / num_kv_heads consecutive heads (GQA).  fp32 accumulation.
 * The K/V of this step must already be in the cache (lvb_paged_kv_write).
 * head_size must be a multiple of 8 and at most 256; query and out rows are
 * 4-byte aligned (even token strides, in elements), the caches 16-byte
 * aligned.  Decode batches (every query length 1, linear) take a
 * split-context path that needs `workspace`; request_order (optional, NULL =
 * index order: 2 * num_seqs int32, a permutation of the requests followed by
 * their num_computed in that order, as lvb_pack_step_metadata writes it) is
 * the order in which that path launches them: longest context first shortens
 * the tail of the launch.  The results do not depend on it.  That path is
 * two launches (the split kernel, then the merge of the splits) and starts
 * reading each request's pages wholly before its newest position before the
 * previous kernel of the stream has finished: rows of those positions must
 * not be written by work still running when the call is made (this
 * library's own K/V writers that let the next launch start early write only
 * the step's new positions; lvb_kv_scatter and lvb_kv_move_rows do not).
 * Other batches (prefill chunks, mixed prefill + decode, tree layouts) with
 * head_size 64 or 128 and 16-token blocks run the tensor-core tile kernel;
 * when request_order is given, its first num_decode_seqs requests are the
 * batch's one-token requests (as lvb_pack_step_metadata orders them) and run
 * the split-context decode path instead (it needs `workspace`), the rest the
 * tile kernel.  With request_order NULL, num_decode_seqs is ignored.  Head
 * sizes 32 / 80 / 256 and other block sizes run a scalar kernel.
 * Replaces the Triton attention launches
 * (runtime/execution/triton_paged_attention.py:106-391, 519-559). */
LVB_API int lvb_paged_attention(const uint16_t *query, int64_t query_token_stride,
                        const uint16_t *key_cache, const uint16_t *value_cache, uint16_t *out,
                        int64_t out_token_stride, const int32_t *block_tables,
                        int64_t table_stride, const int32_t *num_computed,
                        const int32_t *query_start_loc, const int32_t *request_indices,
                        const int32_t *request_order,
                        const uint8_t *visibility, const int32_t *visibility_start,
                        int64_t num_seqs, int64_t num_decode_seqs, int64_t num_tokens, int64_t max_query_len,
                        int64_t max_seq_len, int64_t num_q_heads, int64_t num_kv_heads,
                        int64_t head_size, int64_t block_size, int64_t num_blocks, float scale,
                        int dtype, void *workspace, size_t workspace_bytes,
                        lvb_stream_t stream);

/* lvb_paged_kv_write of this step's key / value rows followed by
 * lvb_paged_attention, in fewer launches: a decode batch on the
 * split-context path stores each request's new row from the warp that loads
 * the page holding it (the rows then need 16-byte aligned starts and token
 * strides that are multiples of 8 elements); other batches run the write
 * first.  The write + attention of the reference's attention step
 * (runtime/execution/triton_paged_attention.py:498-517, 519-559). */
LVB_API int lvb_paged_attention_kv(const uint16_t *key, int64_t key_token_stride, const uint16_t *value,
                                   int64_t value_token_stride, const uint16_t *query, int64_t query_token_stride,
                                   uint16_t *key_cache, uint16_t *value_cache, uint16_t *out,
                                   int64_t out_token_stride, const int32_t *block_tables, int64_t table_stride,
                                   const int32_t *num_computed, const int32_t *query_start_loc,
                                   const int32_t *request_indices, const int32_t *request_order,
                                   const uint8_t *visibility, const int32_t *visibility_start, int64_t num_seqs,
                                   int64_t num_decode_seqs, int64_t num_tokens, int64_t max_query_len,
                                   int64_t max_seq_len, int64_t num_q_heads, int64_t num_kv_heads,
                                   int64_t head_size, int64_t block_size, int64_t num_blocks, float scale,
                                   int dtype, void *workspace, size_t workspace_bytes, lvb_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Tensor-parallel all-reduce + residual add + RMSNorm                        */
/* ------------------------------------------------------------------------ */

/* Peer workspaces (set-up calls; unlike the compute entry points these
 * allocate and map device memory).  lvb_ipc_alloc returns zero-filled device
 * memory on the current device and its 64-byte CUDA IPC handle; every other
 * rank of the node maps it with lvb_ipc_open.  lvb_ipc_close unmaps a peer's
 * workspace, lvb_ipc_free releases one's own (after every peer has closed it).
 * Used by TensorParallelCollectives in place of the NCCL communicator set-up of
 * `CurrentStreamNCCL` (runtime/execution/nccl.py:45-120). */
LVB_API int lvb_ipc_alloc(size_t bytes, void **ptr, void *handle_out);
LVB_API int lvb_ipc_open(const void *handle, void **ptr);
LVB_API int lvb_ipc_close(void *ptr);
LVB_API int lvb_ipc_free(void *ptr);

/* Bytes of one rank's workspace for a group of `world` ranks and up to
 * max_tokens rows of `hidden` fp16: a 64 KiB header (epoch, arrival counter,
 * flags), two parities of `world` staging slots and two gather buffers. */
LVB_API size_t lvb_allreduce_workspace_bytes(int world, int64_t max_tokens, int64_t hidden);

/* Put a freshly allocated workspace in its initial state (header zeroed,
 * sentinel buffers filled with 0xFFFF); synchronises the device.  Every rank
 * initialises its own workspace before the handles are exchanged. */
LVB_API int lvb_allreduce_workspace_init(void *workspace, int world, int64_t max_tokens, int64_t hidden);

/* Row-parallel epilogue of a Qwen2 block in one launch: h = sum over the
 * world ranks of `partial` (fp32, rounded to fp16 once), v = h + residual
 * (fp32), residual <- fp16(v), out <- fp16(v * rsqrt(mean(v^2) + eps) *
 * weight).  Replaces `all_reduce_sum` (modeling/tensor_parallel.py:18-27,
 * runtime/execution/distributed.py:190-197, nccl.py:127-139) followed by
 * `fused_add_rms_norm` (modeling/models/_qwen2_kernels.py:20-43, 145-180).
 * With residual and weight both null it is the plain in-place-capable
 * all-reduce: out <- h (out may equal partial; eps is ignored).
 * workspaces[r] = rank r's workspace as mapped in this process (own for r ==
 * rank), each sized for this world; every rank calls with the same tokens,
 * hidden, max_tokens and mode, in the same order.  The call counter lives in
 * the workspace, so launches may be captured in a CUDA graph.
 * mode: 1 one-shot (push every row to every peer, then flags), 2 two-shot
 * (reduce-scatter + all-gather through peer memory, flags), 3 sentinel
 * one-shot (pushed data carries its own ready marker: no flags, no fences),
 * 4 sentinel two-shot (reduce-scatter + all-gather with sentinel-marked
 * pushes); 0 picks 3 at world <= 2 or while (world - 1) x message bytes <=
 * 4 MiB, else 4 (callers with a library all-reduce at hand do better with it
 * for messages above lvb_allreduce_peer_max_bytes).  An fp16 lane equal to 0xFFFF (a
 * NaN) is pushed as 0xFE00 in mode 3, so NaN payloads are not preserved.  Waits for peers are bounded: on timeout the
 * device error word gets LVB_DEVERR_TIMEOUT, outputs are left unwritten and
 * the workspaces must be rebuilt.  With world == 1 no workspace is touched
 * (the plain sum is a copy, or nothing when out == partial; the norm is one
 * add + RMSNorm launch).  hidden is a multiple of 8 up to 8192;
 * tensors 16-byte aligned; residual must not alias partial or out;
 * world <= 8. */
/* Message bytes per rank up to which the peer-memory kernel beats a ring
 * all-reduce at this world size (larger messages: NCCL in place, then this
 * entry point with world = 1 for the add + RMSNorm). */
LVB_API size_t lvb_allreduce_peer_max_bytes(int world);

LVB_API int lvb_allreduce_add_rmsnorm(void *const *workspaces, int rank, int world, const uint16_t *partial,
                                      uint16_t *residual, const uint16_t *weight, uint16_t *out,
                                      int64_t tokens, int64_t hidden, int64_t max_tokens, float eps,
                                      int mode, lvb_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Qwen2 element-wise layer steps (fp16)                                     */
/* ------------------------------------------------------------------------ */

/* Qwen2 half-rotation RoPE, in place on the query heads (columns [0, hq*D))
 * and key heads (the next hkv*D columns) of each row of the merged QKV
 * projection: x[i] <- x[i]cos[p][i] - x[i+D/2]sin[p][i], x[i+D/2] <-
 * x[i+D/2]cos[p][i+D/2] + x[i]sin[p][i+D/2], fp32 arithmetic, p =
 * positions[t] (int32).  cos/sin are fp16 [table_rows][D] tables.  Replaces
 * `apply_rotary` (modeling/models/_qwen2_kernels.py:66-133, 205-243).  A
 * position outside the table sets LVB_DEVERR_INDEX and leaves its row. */
LVB_API int lvb_rope_qk(uint16_t *qkv, int64_t row_stride, int64_t tokens, int64_t num_query_heads,
                        int64_t num_kv_heads, int64_t head_size, const int32_t *positions,
                        const uint16_t *cos_table, const uint16_t *sin_table, int64_t table_rows,
                        lvb_stream_t stream);

/* lvb_rope_qk and the paged K/V write in one launch (fp16 caches): the
 * query heads of each QKV row are rotated in place, the key heads rotated
 * into the token's cache slot and the value heads copied there (slot of token
 * t as in lvb_paged_kv_write; RoPE position positions[t]).  Replaces
 * `apply_rotary` (_qwen2_kernels.py:66-133) plus the K/V write of the
 * attention step (triton_paged_attention.py:31-104, 498-517); the attention
 * then runs without writing K/V.  head_size % 16 == 0, row_stride a multiple
 * of 8 covering the Q, K and V heads, 16-byte aligned rows, tables, caches. */
LVB_API int lvb_rope_kv_write(uint16_t *qkv, int64_t row_stride, int64_t tokens, int64_t num_query_heads,
                              int64_t num_kv_heads, int64_t head_size, const int32_t *positions,
                              const uint16_t *cos_table, const uint16_t *sin_table, int64_t table_rows,
                              uint16_t *key_cache, uint16_t *value_cache, const int32_t *block_tables,
                              int64_t table_stride, const int32_t *num_computed, const int32_t *query_start_loc,
                              const int32_t *request_indices, int64_t block_size, lvb_stream_t stream);

/* out[t][c] = silu(g) * u for g = gate_up[t][c], u = gate_up[t][I + c]
 * (fp32 arithmetic, one fp16 rounding).  Replaces `silu_and_mul`
 * (modeling/models/_qwen2_kernels.py:45-64, 183-202) on the merged gate/up
 * output (qwen2.py:237-247).  I and both row strides are multiples of 8;
 * tensors 16-byte aligned. */
LVB_API int lvb_silu_mul(const uint16_t *gate_up, int64_t in_stride, int64_t tokens, int64_t intermediate,
                         uint16_t *out, int64_t out_stride, lvb_stream_t stream);

/* Greedy pick of the vocabulary head without writing logits: for each of
 * tokens (1..4) hidden rows, logit[t][v] = fp16(fp32 sum_k hidden[t][k] *
 * weight[v][k]) over this rank's vocab_rows rows of weight ([vocab_rows]
 * [hidden_size] fp16, the nn.Linear layout), and out_index[t] = vocab_offset
 * + the lowest row holding the maximum; out_value[t] (optional) = that
 * maximum, for the cross-rank pick of a vocab-parallel head.  Replaces the
 * lm_head F.linear + greedy argmax (modeling/models/qwen2.py:665-673,
 * runtime/sampling.py:103-112) at decode batch sizes.  workspace:
 * lvb_lm_head_workspace_bytes() bytes, zero-filled once; every call leaves
 * it zero.  Calls sharing a workspace must not overlap on the GPU. */
LVB_API size_t lvb_lm_head_workspace_bytes(void);
LVB_API int lvb_lm_head_argmax(const uint16_t *hidden, int64_t hidden_stride, int64_t tokens,
                               const uint16_t *weight, int64_t vocab_rows, int64_t hidden_size,
                               int64_t vocab_offset, int64_t *out_index, float *out_value, void *workspace,
                               lvb_stream_t stream);

/* out[t] = table[ids[t] - vocab_start] for vocab_start <= ids[t] < vocab_end,
 * else zeros (int64 ids; fp16 rows of hidden_size, a multiple of 8).  The
 * masked lookup of `VocabParallelEmbedding.forward`
 * (modeling/tensor_parallel.py:296-306); the cross-rank sum is the all-reduce
 * that follows. */
LVB_API int lvb_embedding(const int64_t *ids, int64_t tokens, const uint16_t *table, int64_t vocab_start,
                          int64_t vocab_end, int64_t hidden_size, uint16_t *out, int64_t out_stride,
                          lvb_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* LVB200_H_ */
