// Fused QK-norm + RoPE + KV scatter for one layer step.
//
// Replaces, in hayate's GroupedQueryAttention.forward (hayate/model/attention.py:62-75),
// the per-head RMSNorm of q and k (nn.RMSNorm(head_dim, eps), attention.py:34-35,62-63),
// the half-split rotary embedding at each token's position (rope.py:31-47: x * cos +
// cat(-x2, x1) * sin with fp32 cos/sin tables, result cast back to the input dtype) and
// PagedKVBatch.write_layer (paged_cache.py:44-60) with ONE launch:
//   q_out[b, h, t, :] = rope(rmsnorm(q[b, t, h, :]) ,  pos = cache_lens[b] + t)
//   pool_k[layer, 0, g, slot(b, t), :] = rope(rmsnorm(k[b, t, g, :]), pos)
//   pool_v[layer, 0, g, slot(b, t), :] = v[b, t, g, :]
// The arithmetic follows the reference's dtype steps: the norm is computed in fp32 and
// rounded to the storage dtype (the module returns a bf16 tensor), the rotation uses
// fp32 products of that rounded value with the fp32 tables (separate multiply and add,
// as torch evaluates them) and is rounded once more.
//
// Packed batches (token_request set) look each token's request and position up.
//
// One warp per (token, head row); each lane holds 4 consecutive features, so the
// rotation partner (feature i +/- 64) sits in lane ^ 16. HBM-bound: every byte of
// q, k, v is read once and written once.
#include "common.cuh"
#include "kernels.cuh"

namespace hyt {

namespace {

constexpr int kWarps = 8;

template <typename T>
__device__ __forceinline__ void load4(const T* src, float (&x)[4]) {
  if constexpr (sizeof(T) == 2) {
    const uint2 raw = *reinterpret_cast<const uint2*>(src);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = Elem<T>::to_float(e[i]);
  } else {
    const float4 raw = *reinterpret_cast<const float4*>(src);
    x[0] = raw.x; x[1] = raw.y; x[2] = raw.z; x[3] = raw.w;
  }
}

template <typename T>
__device__ __forceinline__ void store4(T* dst, const float (&x)[4]) {
  if constexpr (sizeof(T) == 2) {
    uint2 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) e[i] = Elem<T>::from_float(x[i]);
    *reinterpret_cast<uint2*>(dst) = raw;
  } else {
    *reinterpret_cast<float4*>(dst) = make_float4(x[0], x[1], x[2], x[3]);
  }
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) norm_rope_scatter_kernel(const NormRopeParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = p.num_q_heads + 2 * p.num_kv_heads;
  const bool packed = p.token_request != nullptr;
  const int64_t tokens = packed ? int64_t(p.total_tokens) : int64_t(p.batch) * p.query_len;
  const int64_t row = int64_t(blockIdx.x) * kWarps + warp;
  if (row >= tokens * heads) return;
  const int which = int(row % heads);
  const int64_t token = row / heads;
  int t, b;
  if (packed) {
    b = p.token_request[token];
    t = (b >= 0 && b < p.batch) ? int(token - p.q_start[b]) : -1;
    if (t < 0) {
      flag_error(p.error_word, HYT_DEVERR_PACKED_RANGE);
      return;
    }
  } else {
    t = int(token % p.query_len);
    b = int(token / p.query_len);
  }
  // element offsets of this token in q/k/v ({b, t} part) and in q_out
  const int64_t q_tok = packed ? token * p.q_st : b * p.q_sb + t * p.q_st;
  const int64_t k_tok = packed ? token * p.k_st : b * p.k_sb + t * p.k_st;
  const int64_t v_tok = packed ? token * p.v_st : b * p.v_sb + t * p.v_st;
  const int64_t o_tok = packed ? token * p.o_st : b * p.o_sb + t * p.o_st;
  const int pos = p.cache_lens[b] + t;
  const int d0 = lane * 4;  // this lane's features d0 .. d0 + 3 (head_dim 128)

  const T* src;
  int kind;  // 0 q, 1 k, 2 v
  int h;
  if (which < p.num_q_heads) {
    kind = 0, h = which;
    src = static_cast<const T*>(p.q) + q_tok + int64_t(h) * p.q_sh;
  } else if (which < p.num_q_heads + p.num_kv_heads) {
    kind = 1, h = which - p.num_q_heads;
    src = static_cast<const T*>(p.k) + k_tok + int64_t(h) * p.k_sh;
  } else {
    kind = 2, h = which - p.num_q_heads - p.num_kv_heads;
    src = static_cast<const T*>(p.v) + v_tok + int64_t(h) * p.v_sh;
  }
  float x[4];
  load4<T>(src + d0, x);

  if (kind != 2) {
    // RMSNorm in fp32, rounded to the storage dtype (the module's output tensor)
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float rstd = rsqrtf(ss / 128.f + p.eps);
    const T* w = static_cast<const T*>(kind == 0 ? p.q_norm_weight : p.k_norm_weight);
    float wf[4];
    load4<T>(w + d0, wf);
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = Elem<T>::to_float(Elem<T>::from_float((x[i] * rstd) * wf[i]));
    // half-split rotation at position pos: rotated = cat(-x2, x1)
    if (pos < 0 || pos >= p.rope_positions) {
      flag_error(p.error_word, HYT_DEVERR_TABLE_RANGE);
      return;
    }
    const float* cs = p.cos + int64_t(pos) * 128 + d0;
    const float* sn = p.sin + int64_t(pos) * 128 + d0;
    const float4 c4 = *reinterpret_cast<const float4*>(cs), s4 = *reinterpret_cast<const float4*>(sn);
    const float cv[4] = {c4.x, c4.y, c4.z, c4.w}, sv[4] = {s4.x, s4.y, s4.z, s4.w};
    float y[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float partner = __shfl_xor_sync(0xffffffffu, x[i], 16);
      const float rotated = lane < 16 ? -partner : partner;
      y[i] = __fadd_rn(__fmul_rn(x[i], cv[i]), __fmul_rn(rotated, sv[i]));
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = y[i];
  }

  if (kind == 0) {
    T* dst = static_cast<T*>(p.q_out) + o_tok + int64_t(h) * p.o_sh;
    store4<T>(dst + d0, x);
    return;
  }
  // K / V: page-table slot of logical position pos (write_layer's index math)
  const int64_t logical_page = pos >> p.page_shift;
  if (logical_page >= p.page_table_stride) {
    flag_error(p.error_word, HYT_DEVERR_TABLE_RANGE);
    return;
  }
  const int32_t page = p.page_table[int64_t(b) * p.page_table_stride + logical_page];
  if (page < 0 || page >= p.num_pages) {
    flag_error(p.error_word, HYT_DEVERR_PAGE_RANGE);
    return;
  }
  const int64_t slot = (int64_t(page) << p.page_shift) + (pos & ((1 << p.page_shift) - 1));
  T* pool = static_cast<T*>(kind == 1 ? p.k_pool : p.v_pool);
  T* dst = pool + ((int64_t(p.layer) * p.num_kv_heads + h) * p.capacity + slot) * 128;
  store4<T>(dst + d0, x);
}

}  // namespace

cudaError_t run_norm_rope_scatter(const NormRopeParams& p, int dtype, cudaStream_t stream) {
  const int64_t tokens = p.token_request != nullptr ? int64_t(p.total_tokens) : int64_t(p.batch) * p.query_len;
  const int64_t rows = tokens * (p.num_q_heads + 2 * p.num_kv_heads);
  const int64_t blocks = (rows + kWarps - 1) / kWarps;
  if (blocks <= 0) return cudaSuccess;
  if (blocks > INT32_MAX) return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>(blocks)), block(kWarps * 32);
  switch (dtype) {
    case HYT_DTYPE_BF16: norm_rope_scatter_kernel<__nv_bfloat16><<<grid, block, 0, stream>>>(p); break;
    case HYT_DTYPE_F16: norm_rope_scatter_kernel<__half><<<grid, block, 0, stream>>>(p); break;
    default: norm_rope_scatter_kernel<float><<<grid, block, 0, stream>>>(p); break;
  }
  return cudaGetLastError();
}

}  // namespace hyt
