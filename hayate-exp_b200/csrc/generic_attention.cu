// CUDA-core paged attention for the shapes the tensor-core kernels do not take:
// fp32 pools (the reference's CPU dtype, checked at 1e-4), head_dim other than
// 128 (the reference's own parity test uses 16) and any GQA ratio.
//
// Same mask as hayate/engine/paged_cache.py:266-271: query t of row b sees
// logical keys 0 .. cache_lens[b] + t, gathered through the page table; query
// head h reads KV head h / (H_q / H_kv) (FlexAttention's enable_gqa mapping).
//
// Packed batches (per-request chunk lengths on one token axis) and request lists
// (AttentionParams::req_ids) are served row by row the same way.
//
// One warp per query row; lane l holds dims l, l + 32, ... so every K/V row is
// read by one coalesced warp access. Keys are taken four at a time so the four
// warp reductions overlap. fp32 accumulation, base-2 online softmax.
#include "common.cuh"
#include "kernels.cuh"

namespace hyt {

constexpr int kGenericMaxPerLane = 8;  // head_dim <= 256
constexpr int kGenericWarps = 4;

template <typename T>
__global__ void __launch_bounds__(kGenericWarps * 32) generic_attention_kernel(const AttentionParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * kGenericWarps + warp;
  const int64_t rows = int64_t(att_launch_count(p)) * p.num_q_heads * p.query_len;
  if (row >= rows) return;
  const int t = int(row % p.query_len);
  const int h = int((row / p.query_len) % p.num_q_heads);
  const int z = int(row / (int64_t(p.query_len) * p.num_q_heads));
  const int b = att_request(p, z);
  if (!att_request_ok(p, b)) {
    if (t == 0 && h == 0 && lane == 0) flag_error(p.error_word, HYT_DEVERR_PACKED_RANGE);
    return;
  }
  if (t >= att_query_len(p, b)) return;  // packed batch: past this request's chunk
  const int g = h / (p.num_q_heads / p.num_kv_heads);
  const int D = p.head_dim;
  const int n_keys = p.cache_lens[b] + t + 1;
  const int32_t page_mask = (1 << p.page_shift) - 1;

  const T* q = static_cast<const T*>(p.q) + att_q_row(p, b, t) + h * p.q_sh;
  const int64_t plane = (int64_t(p.layer) * p.num_kv_heads + g) * p.capacity;
  const T* kp = static_cast<const T*>(p.k_pool) + plane * D;
  const T* vp = static_cast<const T*>(p.v_pool) + plane * D;
  const int32_t* table = p.page_table + int64_t(b) * p.page_table_stride;
  const float scale_log2 = p.scale * kLog2e;

  float qr[kGenericMaxPerLane], o[kGenericMaxPerLane];
#pragma unroll
  for (int e = 0; e < kGenericMaxPerLane; ++e) {
    const int d = lane + 32 * e;
    qr[e] = d < D ? Elem<T>::to_float(q[d]) : 0.f;
    o[e] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  bool bad = false;

  for (int j0 = 0; j0 < n_keys; j0 += 4) {
    float s[4];
    int64_t slot[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = j0 + u;
      s[u] = 0.f;
      slot[u] = -1;
      if (j < n_keys) {
        const int lp = j >> p.page_shift;
        const int32_t page = lp < p.page_table_stride ? table[lp] : -1;
        if (page >= 0 && page < p.num_pages) {
          slot[u] = (int64_t(page) << p.page_shift) + (j & page_mask);
          const T* krow = kp + slot[u] * D;
#pragma unroll
          for (int e = 0; e < kGenericMaxPerLane; ++e) {
            const int d = lane + 32 * e;
            if (d < D) s[u] += qr[e] * Elem<T>::to_float(krow[d]);
          }
        } else {
          bad = true;
        }
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
      for (int u = 0; u < 4; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], off);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (slot[u] < 0) continue;  // past the row's keys, or a refused page
      const float x = s[u] * scale_log2;
      const float m_new = fmaxf(m, x);
      const float alpha = ex2(m - m_new);
      const float pw = ex2(x - m_new);
      l = l * alpha + pw;
      const T* vrow = vp + slot[u] * D;
#pragma unroll
      for (int e = 0; e < kGenericMaxPerLane; ++e) {
        const int d = lane + 32 * e;
        if (d < D) o[e] = o[e] * alpha + pw * Elem<T>::to_float(vrow[d]);
      }
      m = m_new;
    }
  }
  if (bad && lane == 0) flag_error(p.error_word, HYT_DEVERR_PAGE_RANGE);
  const float inv = l > 0.f ? 1.f / l : 0.f;
  T* out = static_cast<T*>(p.out) + att_o_row(p, b, t) + h * p.o_sh;
#pragma unroll
  for (int e = 0; e < kGenericMaxPerLane; ++e) {
    const int d = lane + 32 * e;
    if (d < D) out[d] = Elem<T>::from_float(o[e] * inv);
  }
}

cudaError_t run_generic_attention(const AttentionParams& p, int dtype, cudaStream_t stream) {
  const int64_t rows = int64_t(att_launch_count(p)) * p.num_q_heads * p.query_len;
  const int64_t blocks = (rows + kGenericWarps - 1) / kGenericWarps;
  if (blocks <= 0) return cudaSuccess;
  if (blocks > INT32_MAX) return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>(blocks)), block(kGenericWarps * 32);
  switch (dtype) {
    case HYT_DTYPE_BF16: generic_attention_kernel<__nv_bfloat16><<<grid, block, 0, stream>>>(p); break;
    case HYT_DTYPE_F16: generic_attention_kernel<__half><<<grid, block, 0, stream>>>(p); break;
    default: generic_attention_kernel<float><<<grid, block, 0, stream>>>(p); break;
  }
  return cudaGetLastError();
}

}  // namespace hyt
