/*
 * hayate_b200 — C ABI of the B200 paged-KV attention path.
 *
 * Drop-in for hayate's paged attention seam: the Python side keeps the
 * reference's PagedKVCacheManager / PagedKVBatch API and calls these entry
 * points with raw device pointers (no torch types cross this boundary).
 *
 * Conventions shared by every entry point:
 *  - Pools are the reference's layout, [num_layers, 1, num_kv_heads,
 *    capacity_tokens, head_dim], contiguous, one for K and one for V
 *    (hayate/engine/paged_cache.py:104-109).
 *  - page_table is int32 [batch, page_table_stride] on the device; row b lists
 *    request b's physical page ids in logical order. cache_lens is int32 [batch]
 *    on the device: the tokens cached BEFORE this step. Every request appends
 *    query_len tokens, so kv_len[b] = cache_lens[b] + query_len
 *    (paged_cache.py:216-217).
 *  - q/out/k_new/v_new are [batch, heads, query_len, head_dim] with the last
 *    dimension contiguous; the other three strides are passed in ELEMENTS as
 *    {stride_b, stride_h, stride_t}, so the strided views hayate's attention
 *    module produces (hayate/model/attention.py:66-71) need no copy.
 *  - dtype: HYT_DTYPE_BF16 / F16 / F32 for every tensor of the call.
 *  - stream is a cudaStream_t (NULL = legacy default stream). Calls only
 *    enqueue work; none of them synchronises the host.
 *  - error_word (nullable) is a device int32 the kernels OR error bits into
 *    when they meet a page id or length they refuse to use; the offending
 *    access is skipped, never performed. Host-side argument errors are
 *    returned as negative codes with a message in hyt_last_error().
 */
#ifndef HAYATE_B200_H
#define HAYATE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  HYT_OK = 0,
  HYT_ERR_INVALID = -1,     /* bad argument (null pointer, negative size, ...) */
  HYT_ERR_UNSUPPORTED = -2, /* valid but not served by this build (dtype/shape) */
  HYT_ERR_CUDA = -3,        /* a CUDA runtime/driver call failed */
  HYT_ERR_WORKSPACE = -4    /* workspace missing, too small or not 16-byte aligned */
};

enum { HYT_DTYPE_BF16 = 0, HYT_DTYPE_F16 = 1, HYT_DTYPE_F32 = 2 };

/* Device error bits written into error_word. */
enum {
  HYT_DEVERR_PAGE_RANGE = 1,   /* page id outside [0, capacity_tokens / page_size) */
  HYT_DEVERR_TABLE_RANGE = 2,  /* kv_len needs more pages than page_table_stride */
  HYT_DEVERR_SPLIT_RANGE = 4,  /* kv_len > max_kv_len given at launch */
  HYT_DEVERR_WAIT_TIMEOUT = 8, /* a bounded pipeline wait gave up */
  HYT_DEVERR_ISSUE_LANE = 16,  /* tensor-core issue ran on other than exactly one lane (work skipped) */
  HYT_DEVERR_PACKED_RANGE = 32, /* packed batch: q_start/q_len/request id out of range (work skipped) */
  HYT_DEVERR_PLAN_RANGE = 64    /* prefill plan item out of range (work skipped) */
};

/* Message of the last failed call on this thread ("" if none). */
const char* hyt_last_error(void);

/* ABI version of this library (major * 100 + minor). */
int hyt_version(void);

/*
 * Page-table KV scatter.
 * Replaces PagedKVBatch.write_layer (hayate/engine/paged_cache.py:44-60):
 * token t of row b goes to slot page_table[b][(cache_lens[b]+t)/P]*P +
 * (cache_lens[b]+t)%P of pool[layer, 0, h, :, :], for K and V in one launch.
 * new_strides = {k_b, k_h, k_t, v_b, v_h, v_t} in elements.
 */
int hyt_kv_scatter(const void* k_new, const void* v_new, const int64_t* new_strides,
                   void* k_pool, void* v_pool, int32_t num_layers, int32_t layer,
                   int64_t capacity_tokens, const int32_t* page_table,
                   int32_t page_table_stride, const int32_t* cache_lens, int32_t batch,
                   int32_t query_len, int32_t num_kv_heads, int32_t head_dim,
                   int32_t page_size, int32_t dtype, int32_t* error_word, void* stream);

/*
 * Paged causal GQA attention, any supported shape.
 * Replaces PagedKVBatch.attend_layer (hayate/engine/paged_cache.py:62-71) with
 * the reference's mask (paged_cache.py:266-271): query t of row b sees logical
 * keys 0 .. cache_lens[b] + t. Query head h reads KV head h / (H_q / H_kv).
 * Dispatches to the split-KV decode kernel (query_len * group <= 16,
 * bf16/f16, head_dim 128), the tcgen05 chunked-prefill kernel (bf16/f16,
 * head_dim 128, larger chunks) or the CUDA-core kernel (any other shape, f32).
 * q_strides/out_strides = {b, h, t} in elements. max_kv_len bounds
 * cache_lens[b] + query_len over the batch (sizes the split grid).
 * workspace: see hyt_attention_workspace_bytes (16-byte aligned); the counter area at
 * its start (4 bytes per (request, KV head), rounded up to 256) must be zero when a call
 * starts and is left zero. A buffer reused for a call with more (request, KV head) units
 * than an earlier one must have the newly covered counter bytes zeroed first (they held
 * that call's partials), or be zeroed whole (hyt_workspace_init).
 */
int hyt_paged_attention(const void* q, const int64_t* q_strides, const void* k_pool,
                        const void* v_pool, int32_t num_layers, int32_t layer,
                        int64_t capacity_tokens, const int32_t* page_table,
                        int32_t page_table_stride, const int32_t* cache_lens, void* out,
                        const int64_t* out_strides, int32_t batch, int32_t query_len,
                        int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                        int32_t page_size, int32_t dtype, float scale, int32_t max_kv_len,
                        int32_t split_tokens, void* workspace, size_t workspace_bytes,
                        int32_t* error_word, void* stream);

/*
 * Write the step's new K/V rows, then attend: hyt_kv_scatter (k_new, v_new, new_strides
 * as there) followed by hyt_paged_attention on the same stream, with the same results.
 * Replaces PagedKVBatch.write_layer + attend_layer (hayate/engine/paged_cache.py:44-71),
 * the pair hayate's attention layer calls back to back for every decode step. When the
 * decode kernel serves the step and every new row is 16-byte aligned this is ONE launch:
 * the split that attends a new row copies it into its pool slot first. Otherwise the two
 * kernels run in turn. A split with a refused page id writes none of its new rows (the
 * separate scatter would still write the rows whose pages are valid); both flag it.
 */
int hyt_paged_attention_scatter(const void* q, const int64_t* q_strides, const void* k_new,
                                const void* v_new, const int64_t* new_strides, void* k_pool,
                                void* v_pool, int32_t num_layers, int32_t layer,
                                int64_t capacity_tokens, const int32_t* page_table,
                                int32_t page_table_stride, const int32_t* cache_lens, void* out,
                                const int64_t* out_strides, int32_t batch, int32_t query_len,
                                int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                int32_t page_size, int32_t dtype, float scale, int32_t max_kv_len,
                                int32_t split_tokens, void* workspace, size_t workspace_bytes,
                                int32_t* error_word, void* stream);

/* Split-KV decode kernel only (query_len * (H_q / H_kv) <= 16, bf16/f16, D = 128).
 * split_tokens: tokens per split, a multiple of 64; 0 picks one for this GPU. */
int hyt_decode_attention(const void* q, const int64_t* q_strides, const void* k_pool,
                         const void* v_pool, int32_t num_layers, int32_t layer,
                         int64_t capacity_tokens, const int32_t* page_table,
                         int32_t page_table_stride, const int32_t* cache_lens, void* out,
                         const int64_t* out_strides, int32_t batch, int32_t query_len,
                         int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                         int32_t page_size, int32_t dtype, float scale, int32_t max_kv_len,
                         int32_t split_tokens, void* workspace, size_t workspace_bytes,
                         int32_t* error_word, void* stream);

/*
 * Split-KV decode that allocates nothing. No counterpart in the reference.
 *
 * For callers that cannot allocate device memory: a C or FFI host that only
 * borrows tensors from another framework's caching allocator and has no
 * allocator of its own, or a serving loop that must not call cudaMalloc
 * (which can synchronise the whole device) once it is running. Same arguments
 * and results as hyt_decode_attention, minus the workspace: the split partials
 * and arrival counters live in one static device array of
 * HYT_NOALLOC_SCRATCH_BYTES that every GPU loading this library holds until
 * the process exits. Sizes whose workspace (hyt_attention_workspace_bytes)
 * exceeds it are refused with HYT_ERR_WORKSPACE; a larger split_tokens needs
 * less. Every call made outside stream capture looks the array's address up
 * on the current device (so a context re-created after cudaDeviceReset gets
 * the new address); a call made while `stream` is being captured reuses the
 * address its device's last uncaptured call found, so make the first call on
 * each device before any stream capture (a captured first call is refused
 * with HYT_ERR_INVALID). Every call clears the counter area on `stream` and
 * then reuses the array, so calls that overlap on the GPU (other streams,
 * other threads) race on it.
 */
#define HYT_NOALLOC_SCRATCH_BYTES (8u << 20)
int hyt_decode_attention_noalloc(const void* q, const int64_t* q_strides, const void* k_pool,
                                 const void* v_pool, int32_t num_layers, int32_t layer,
                                 int64_t capacity_tokens, const int32_t* page_table,
                                 int32_t page_table_stride, const int32_t* cache_lens, void* out,
                                 const int64_t* out_strides, int32_t batch, int32_t query_len,
                                 int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                 int32_t page_size, int32_t dtype, float scale,
                                 int32_t max_kv_len, int32_t split_tokens, int32_t* error_word,
                                 void* stream);

/* tcgen05/TMEM chunked-prefill kernel only (bf16/f16, head_dim 128). */
int hyt_prefill_attention(const void* q, const int64_t* q_strides, const void* k_pool,
                          const void* v_pool, int32_t num_layers, int32_t layer,
                          int64_t capacity_tokens, const int32_t* page_table,
                          int32_t page_table_stride, const int32_t* cache_lens, void* out,
                          const int64_t* out_strides, int32_t batch, int32_t query_len,
                          int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                          int32_t page_size, int32_t dtype, float scale, int32_t max_kv_len,
                          int32_t* error_word, void* stream);

/*
 * Fused QK-norm + RoPE + KV scatter (head_dim 128).
 * Replaces, in hayate/model/attention.py:62-75, q_norm/k_norm (nn.RMSNorm over
 * head_dim, attention.py:34-35), apply_rope_vectorized at position cache_lens[b] + t
 * with the model's fp32 cos/sin tables (hayate/model/rope.py:31-47) and
 * PagedKVBatch.write_layer (paged_cache.py:44-60), in one launch. Inputs are the
 * projections before the transpose: q [B, T, H_q, 128], k/v [B, T, H_kv, 128] with
 * element strides {b, t, h} (qkv_strides = q's 3, then k's, then v's). q_out is
 * [B, H_q, T, 128] with strides {b, h, t}. cos/sin are [rope_positions, 128] fp32.
 * Every row starts on a 16-byte boundary: q, k, v, q_out, both norm weights, both pools
 * and cos/sin 16-byte aligned, all strides multiples of 16 bytes (HYT_ERR_INVALID
 * otherwise).
 */
int hyt_norm_rope_scatter(const void* q, const void* k, const void* v, const int64_t* qkv_strides,
                          const void* q_norm_weight, const void* k_norm_weight, float eps,
                          const float* cos, const float* sin, int32_t rope_positions,
                          void* q_out, const int64_t* q_out_strides, void* k_pool, void* v_pool,
                          int32_t num_layers, int32_t layer, int64_t capacity_tokens,
                          const int32_t* page_table, int32_t page_table_stride,
                          const int32_t* cache_lens, int32_t batch, int32_t query_len,
                          int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                          int32_t page_size, int32_t dtype, int32_t* error_word, void* stream);

/* CUDA-core kernel only (any dtype, head_dim a multiple of 8 up to 256). */
int hyt_generic_attention(const void* q, const int64_t* q_strides, const void* k_pool,
                          const void* v_pool, int32_t num_layers, int32_t layer,
                          int64_t capacity_tokens, const int32_t* page_table,
                          int32_t page_table_stride, const int32_t* cache_lens, void* out,
                          const int64_t* out_strides, int32_t batch, int32_t query_len,
                          int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                          int32_t page_size, int32_t dtype, float scale,
                          int32_t* error_word, void* stream);

/*
 * Packed (mixed prefill + decode) batches. No single counterpart in the reference:
 * its engine runs one forward pass per distinct prefill chunk length plus one for
 * decoding (hayate/engine/engine.py:226-283, 306-312), each with its own
 * write_layer/attend_layer calls (paged_cache.py:44-71). Here the new tokens of all
 * requests share one token axis: request b owns rows q_start[b] .. q_start[b] +
 * q_len[b] - 1 (total_tokens rows in all), and token_request[i] names the request
 * of row i. Same slot formula and causal rule as the calls above, per request.
 */

/* Packed write_layer. new_strides = {k_t, k_h, v_t, v_h} in elements. */
int hyt_kv_scatter_packed(const void* k_new, const void* v_new, const int64_t* new_strides,
                          void* k_pool, void* v_pool, int32_t num_layers, int32_t layer,
                          int64_t capacity_tokens, const int32_t* page_table,
                          int32_t page_table_stride, const int32_t* cache_lens,
                          const int32_t* q_start, const int32_t* token_request, int32_t batch,
                          int32_t total_tokens, int32_t num_kv_heads, int32_t head_dim,
                          int32_t page_size, int32_t dtype, int32_t* error_word, void* stream);

/* Packed hyt_norm_rope_scatter: qkv_strides = {q_t, q_h, k_t, k_h, v_t, v_h},
 * q_out_strides = {t, h}; token i is at position cache_lens[b] + i - q_start[b]. */
int hyt_norm_rope_scatter_packed(const void* q, const void* k, const void* v,
                                 const int64_t* qkv_strides, const void* q_norm_weight,
                                 const void* k_norm_weight, float eps, const float* cos,
                                 const float* sin, int32_t rope_positions, void* q_out,
                                 const int64_t* q_out_strides, void* k_pool, void* v_pool,
                                 int32_t num_layers, int32_t layer, int64_t capacity_tokens,
                                 const int32_t* page_table, int32_t page_table_stride,
                                 const int32_t* cache_lens, const int32_t* q_start,
                                 const int32_t* token_request, int32_t batch,
                                 int32_t total_tokens, int32_t num_q_heads, int32_t num_kv_heads,
                                 int32_t head_dim, int32_t page_size, int32_t dtype,
                                 int32_t* error_word, void* stream);

/*
 * Packed attend_layer in one call: the requests listed in decode_ids (one query
 * each) go to the split-KV decode kernel, those in prefill_ids (any chunk length up
 * to max_query_len) to the tcgen05 prefill kernel, both on `stream` (the CUDA-core
 * kernel serves shapes those two do not take). q_strides/out_strides = {t, h}.
 * The workspace is the decode kernel's for num_decode requests of one query:
 * hyt_attention_workspace_bytes(num_decode, 1, ...).
 */
int hyt_paged_attention_packed(const void* q, const int64_t* q_strides, const void* k_pool,
                               const void* v_pool, int32_t num_layers, int32_t layer,
                               int64_t capacity_tokens, const int32_t* page_table,
                               int32_t page_table_stride, const int32_t* cache_lens,
                               const int32_t* q_start, const int32_t* q_len, void* out,
                               const int64_t* out_strides, int32_t batch, int32_t total_tokens,
                               int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                               int32_t page_size, int32_t dtype, float scale,
                               const int32_t* decode_ids, int32_t num_decode,
                               const int32_t* prefill_ids, int32_t num_prefill,
                               int32_t max_query_len, int32_t max_kv_len, int32_t split_tokens,
                               void* workspace, size_t workspace_bytes, int32_t* error_word,
                               void* stream);

/*
 * Prefill schedule (host function, no GPU): the order in which the tcgen05 prefill
 * kernel's work items (query tile, head pair, request) start, and which of the heaviest
 * are cut in two along their keys (the halves merged by whichever finishes second), so
 * that the last wave of CTAs ends evenly. Replaces nothing in hayate (its FlexAttention
 * grid is fixed); a planned launch computes the same rows as hyt_prefill_attention.
 * cache_lens / q_lens are HOST arrays (q_lens NULL: every request has query_len queries).
 * The plan is chosen by simulating the block scheduler on num_sms SMs for the default
 * grid and for longest-first orders with 0..max_splits items cut, in a cost model
 * counted in key tiles: an item costs its tiles + item_overhead, a half of a cut item
 * also pays merge_cost (<= 0: the defaults fitted on a B200); items (4 int32 each,
 * room for max_items) receives it. Returns the number of items, 0 when the default grid
 * is at least as good (launch without a plan), negative on bad arguments.
 * *num_splits receives the number of split slots the plan uses.
 */
int32_t hyt_prefill_plan(const int32_t* cache_lens, const int32_t* q_lens, int32_t batch,
                         int32_t query_len, int32_t num_q_heads, int32_t num_sms,
                         int32_t max_splits, float item_overhead, float merge_cost,
                         int32_t* items, int32_t max_items, int32_t* num_splits);

/* Workspace bytes a plan with num_splits split slots needs (its counters, 4 bytes per
 * slot rounded up to 256 at the start, must be zero before first use, hyt_workspace_init;
 * the kernel leaves them zero; a buffer reused for a plan with more slots than an earlier
 * one needs the newly covered counter bytes zeroed first). */
size_t hyt_prefill_workspace_bytes(int32_t num_splits);

/* hyt_prefill_attention launched on a plan from hyt_prefill_plan: items is the plan in
 * DEVICE memory (num_items entries of 4 int32; num_items 0 = the default grid). */
int hyt_prefill_attention_planned(const void* q, const int64_t* q_strides, const void* k_pool,
                                  const void* v_pool, int32_t num_layers, int32_t layer,
                                  int64_t capacity_tokens, const int32_t* page_table,
                                  int32_t page_table_stride, const int32_t* cache_lens, void* out,
                                  const int64_t* out_strides, int32_t batch, int32_t query_len,
                                  int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                  int32_t page_size, int32_t dtype, float scale,
                                  const int32_t* items, int32_t num_items, int32_t num_splits,
                                  void* workspace, size_t workspace_bytes, int32_t* error_word,
                                  void* stream);

/* hyt_paged_attention_packed with its prefill launch on a plan from hyt_prefill_plan (made
 * with the prefill requests' cache lengths and chunk lengths, in prefill_ids order: an
 * item's request index is a position in prefill_ids); items in DEVICE memory, num_items 0
 * = the default grid; plan_workspace as for hyt_prefill_attention_planned. */
int hyt_paged_attention_packed_planned(
    const void* q, const int64_t* q_strides, const void* k_pool, const void* v_pool,
    int32_t num_layers, int32_t layer, int64_t capacity_tokens, const int32_t* page_table,
    int32_t page_table_stride, const int32_t* cache_lens, const int32_t* q_start,
    const int32_t* q_len, void* out, const int64_t* out_strides, int32_t batch,
    int32_t total_tokens, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
    int32_t page_size, int32_t dtype, float scale, const int32_t* decode_ids, int32_t num_decode,
    const int32_t* prefill_ids, int32_t num_prefill, int32_t max_query_len, int32_t max_kv_len,
    int32_t split_tokens, void* workspace, size_t workspace_bytes, const int32_t* items,
    int32_t num_items, int32_t num_splits, void* plan_workspace, size_t plan_workspace_bytes,
    int32_t* error_word, void* stream);

/* Workspace bytes hyt_paged_attention / hyt_decode_attention need for these sizes
 * (0 when the dispatched kernel needs none). split_tokens as in the call. */
size_t hyt_attention_workspace_bytes(int32_t batch, int32_t query_len, int32_t num_q_heads,
                                     int32_t num_kv_heads, int32_t head_dim,
                                     int32_t max_kv_len, int32_t split_tokens, int32_t dtype);

/* Zero a workspace's counter area (enqueued on stream). */
int hyt_workspace_init(void* workspace, size_t workspace_bytes, void* stream);

/* Self-test of the bounded pipeline wait (no hayate counterpart: hayate's PyTorch path
 * has no device-side waits). One tiny kernel waits on an mbarrier that nothing signals;
 * the wait gives up after its 1 s limit and ORs HYT_DEVERR_WAIT_TIMEOUT into
 * *error_word, and a second wait of the same CTA returns at once through the CTA's
 * abort flag. elapsed_ns (device, int64[2]) receives both waits' durations. No copy is
 * in flight when the kernel exits, so the context stays usable. Takes about 1 s. */
int hyt_wait_self_test(int32_t* error_word, int64_t* elapsed_ns, void* stream);

/* Measurement only (no hayate counterpart): a plain streaming read of `bytes` (a positive
 * multiple of 16, src 16-byte aligned) by `ctas` CTAs of 512 threads, 16-byte loads, four
 * in flight per thread; writes one XOR word per CTA to sink (device, uint32[ctas]). Timed
 * around, it gives the HBM read ceiling the memory-bound decode kernel is compared with. */
int hyt_read_probe(const void* src, size_t bytes, uint32_t* sink, int32_t ctas, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HAYATE_B200_H */
