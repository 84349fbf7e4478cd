// Launch parameters and host launchers of the hayate_b200 kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hyt {

// ------------------------------------------------------------ (a) KV scatter
struct ScatterParams {
  const uint8_t* k_new;
  const uint8_t* v_new;
  int64_t k_sb, k_sh, k_st, v_sb, v_sh, v_st;  // element strides
  uint8_t* k_pool;
  uint8_t* v_pool;
  int64_t layer_offset;  // elements: layer * H_kv * capacity * D
  int64_t capacity;
  const int32_t* page_table;
  int32_t page_table_stride;
  const int32_t* cache_lens;
  int32_t batch, query_len, heads, head_dim, page_shift, num_pages;
  int32_t* error_word;
  // Packed batch (token_request != nullptr): the new K/V rows of all requests share one
  // token axis of total_tokens rows (strides k_st/v_st; k_sb/v_sb unused); token i
  // belongs to request token_request[i] at position i - q_start[request] of its chunk.
  const int32_t* q_start;
  const int32_t* token_request;
  int32_t total_tokens;
};
cudaError_t run_kv_scatter(const ScatterParams& p, int elem_bytes, cudaStream_t stream);

// ------------------------------------------------------------ attention (shared fields)
struct AttentionParams {
  const void* q;
  int64_t q_sb, q_sh, q_st;  // element strides
  void* out;
  int64_t o_sb, o_sh, o_st;
  const void* k_pool;
  const void* v_pool;
  int64_t capacity;
  int32_t num_layers, layer;
  const int32_t* page_table;
  int32_t page_table_stride;
  const int32_t* cache_lens;
  int32_t batch, query_len, num_q_heads, num_kv_heads, head_dim, page_shift, num_pages;
  float scale;
  int32_t* error_word;
  // Packed batch (q_start != nullptr): request b's queries are rows q_start[b] ..
  // q_start[b] + q_len[b] - 1 of one token axis of total_tokens rows (strides q_st /
  // o_st; q_sb / o_sb unused) and query_len is the longest q_len. req_ids, if set,
  // lists the requests one launch serves (launch index z -> request req_ids[z], z <
  // the launch's count); the other kernels of the same call serve the rest.
  const int32_t* q_start;
  const int32_t* q_len;
  const int32_t* req_ids;
  int32_t num_listed;  // entries of req_ids
  int32_t total_tokens;
};

// Requests one launch serves (its grid's request dimension).
__host__ __device__ inline int32_t att_launch_count(const AttentionParams& p) {
  return p.req_ids != nullptr ? p.num_listed : p.batch;
}

#ifdef __CUDACC__
// Request served by launch index z.
__device__ __forceinline__ int att_request(const AttentionParams& p, int z) {
  return p.req_ids != nullptr ? p.req_ids[z] : z;
}
// Queries of request b.
__device__ __forceinline__ int att_query_len(const AttentionParams& p, int b) {
  return p.q_start != nullptr ? p.q_len[b] : p.query_len;
}
// Element offset of query t of request b in q (head offset not included), and in out.
__device__ __forceinline__ int64_t att_q_row(const AttentionParams& p, int b, int t) {
  return p.q_start != nullptr ? (int64_t(p.q_start[b]) + t) * p.q_st
                              : int64_t(b) * p.q_sb + int64_t(t) * p.q_st;
}
__device__ __forceinline__ int64_t att_o_row(const AttentionParams& p, int b, int t) {
  return p.q_start != nullptr ? (int64_t(p.q_start[b]) + t) * p.o_st
                              : int64_t(b) * p.o_sb + int64_t(t) * p.o_st;
}
// A packed request whose rows leave the token axis or exceed query_len, or a request id
// outside the batch: refused (flagged, no work) so no q/out access leaves its tensor.
__device__ __forceinline__ bool att_request_ok(const AttentionParams& p, int b) {
  if (b < 0 || b >= p.batch) return false;
  if (p.q_start == nullptr) return true;
  const int s = p.q_start[b], n = p.q_len[b];
  return s >= 0 && n >= 1 && n <= p.query_len && int64_t(s) + n <= p.total_tokens;
}
#endif

// CUDA-core path: any dtype (0 bf16, 1 f16, 2 f32), head_dim % 8 == 0, <= 256.
cudaError_t run_generic_attention(const AttentionParams& p, int dtype, cudaStream_t stream);

// ------------------------------------------------------------ (c) split-KV decode
struct DecodeLaunch {
  int32_t split_tokens;  // multiple of 64
  int32_t max_splits;    // splits per (request, kv head) the grid covers
  float* ws_o;           // [batch, H_kv, max_splits, rows, 128] f32 partial outputs
  float* ws_ml;          // [batch, H_kv, max_splits, rows, 2] f32 running max / sum
  int32_t* ws_counter;   // [batch, H_kv] arrival counters (zero between calls)
  // Fused scatter (k_new != nullptr, uniform batches only): before attending, the step's
  // new K/V rows [B, H_kv, T, 128] (element strides, rows 16-byte aligned) are written to
  // their pool slots at positions cache_lens[b] + t, each by the split that attends it.
  const uint8_t* k_new;
  const uint8_t* v_new;
  int64_t k_sb, k_sh, k_st, v_sb, v_sh, v_st;
  uint8_t* k_pool;
  uint8_t* v_pool;
};
constexpr int kDecodeMaxRows = 16;  // query rows per (request, kv head): group * query_len
cudaError_t run_decode_attention(const AttentionParams& p, const DecodeLaunch& d,
                                 const CUtensorMap& k_map, const CUtensorMap& v_map, int dtype,
                                 cudaStream_t stream);

// ------------------------------------------------------------ (b) tcgen05 chunked prefill
// bf16/f16, head_dim 128, page_size % 128 == 0, q/out rows 16-byte aligned.
// Planned schedule (optional): the grid is plan.num_items CTAs, CTA i computing item
// plan.items[i] = {z (launch request index), query tile | head pair << 16, first key
// tile | end key tile << 16, split}. split = slot * 2 + part for one half of an item cut
// in two along its keys, -1 for a whole item; the two halves write their partial
// (O, max, sum) into slot `slot` of the split workspace and the second to arrive merges
// them (atomic counter per slot, no waiting) and resets the counter.
struct PrefillItem {
  int32_t z, tile_pair, keys, split;
};
struct PrefillPlan {
  const PrefillItem* items;  // device; nullptr: the default grid
  int32_t num_items;
  int32_t num_splits;   // slots the workspace holds
  float* ws_o;          // [slots, 2 parts, 2 heads, 32 column chunks, 128 rows, 4] f32
  float* ws_ml;         // [slots, 2 parts, 2 heads, 128 rows, 2] f32 (max, sum)
  int32_t* ws_counter;  // [slots] arrival counters (zero between calls)
};
constexpr int64_t kPrefillSplitSlotBytes = 2 * (2 * 128 * 128 * 4 + 2 * 128 * 2 * 4);

// q_map (optional): a 4-D tensor map over q, dims (head_dim, T, H_q, B) or, with q_ht,
// (head_dim, H_q, T, B), box 64 x 128 rows, 128-byte swizzle; T is query_len (the token
// axis for packed batches, B = 1). Without it the softmax warps load Q themselves.
cudaError_t run_prefill_attention(const AttentionParams& p, const CUtensorMap& k_map,
                                  const CUtensorMap& v_map, const CUtensorMap* q_map, bool q_ht,
                                  int dtype, cudaStream_t stream,
                                  const PrefillPlan* plan = nullptr);

// ------------------------------------------------------------ fused QK-norm + RoPE + scatter
struct NormRopeParams {
  const void* q;  // [B, T, H_q, 128] element strides {b, t, h}
  int64_t q_sb, q_st, q_sh;
  const void* k;  // [B, T, H_kv, 128]
  int64_t k_sb, k_st, k_sh;
  const void* v;
  int64_t v_sb, v_st, v_sh;
  void* q_out;    // [B, H_q, T, 128] element strides {b, h, t}
  int64_t o_sb, o_sh, o_st;
  const void* q_norm_weight;
  const void* k_norm_weight;
  float eps;
  const float* cos;  // [rope_positions, 128] fp32
  const float* sin;
  int32_t rope_positions;
  void* k_pool;
  void* v_pool;
  int64_t capacity;
  int32_t layer;
  const int32_t* page_table;
  int32_t page_table_stride;
  const int32_t* cache_lens;
  int32_t batch, query_len, num_q_heads, num_kv_heads, page_shift, num_pages;
  int32_t* error_word;
  // Packed batch, as in ScatterParams: q/k/v/q_out rows on one token axis of
  // total_tokens rows (b strides unused), token i of request token_request[i].
  const int32_t* q_start;
  const int32_t* token_request;
  int32_t total_tokens;
};
cudaError_t run_norm_rope_scatter(const NormRopeParams& p, int dtype, cudaStream_t stream);

// Runs the bounded mbarrier wait into its time limit (see self_test.cu).
cudaError_t run_wait_self_test(int32_t* error_word, int64_t* elapsed_ns, cudaStream_t stream);
cudaError_t run_read_probe(const void* src, size_t bytes, uint32_t* sink, int ctas, cudaStream_t stream);

}  // namespace hyt
