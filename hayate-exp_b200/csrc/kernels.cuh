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
};

// CUDA-core path: any dtype (0 bf16, 1 f16, 2 f32), head_dim % 8 == 0, <= 256.
cudaError_t run_generic_attention(const AttentionParams& p, int dtype, cudaStream_t stream);

// ------------------------------------------------------------ (c) split-KV decode
struct DecodeLaunch {
  int32_t split_tokens;  // multiple of 64
  int32_t max_splits;    // splits per (request, kv head) the grid covers
  float* ws_o;           // [batch, H_kv, max_splits, rows, 128] f32 partial outputs
  float* ws_ml;          // [batch, H_kv, max_splits, rows, 2] f32 running max / sum
  int32_t* ws_counter;   // [batch, H_kv] arrival counters (zero between calls)
};
constexpr int kDecodeMaxRows = 16;  // query rows per (request, kv head): group * query_len
cudaError_t run_decode_attention(const AttentionParams& p, const DecodeLaunch& d,
                                 const CUtensorMap& k_map, const CUtensorMap& v_map, int dtype,
                                 cudaStream_t stream);

// ------------------------------------------------------------ (b) tcgen05 chunked prefill
// bf16/f16, head_dim 128, page_size % 128 == 0, q/out rows 16-byte aligned.
cudaError_t run_prefill_attention(const AttentionParams& p, const CUtensorMap& k_map,
                                  const CUtensorMap& v_map, int dtype, cudaStream_t stream);

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
};
cudaError_t run_norm_rope_scatter(const NormRopeParams& p, int dtype, cudaStream_t stream);

}  // namespace hyt
