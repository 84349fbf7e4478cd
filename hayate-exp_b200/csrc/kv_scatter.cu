// Kernel (a): page-table KV scatter.
//
// Restates PagedKVBatch.write_layer (hayate/engine/paged_cache.py:44-60) as one
// launch for K and V: token t of batch row b sits at logical position
// pos = cache_lens[b] + t and is copied, unchanged, to slot
// page_table[b][pos / P] * P + pos % P of pool[layer, 0, h]. The copy is a byte
// move (bit-exact with the reference's index_put).
//
// Packed batches (chunks of different lengths on one token axis, token_request set)
// take the same copy with each token's request and position looked up per token.
//
// Layout: consecutive threads take consecutive VEC-byte chunks of one row, so a
// warp moves whole 256-byte rows of a bf16 head_dim-128 vector with coalesced
// 16-byte loads and stores. HBM-bound; the work per launch is tiny at decode
// (B * T * H_kv * D * 2 elements per tensor), so the grid is sized by the work.
#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"

namespace hyt {

// One VEC-byte chunk per thread. The source chunk is loaded first: its address depends
// only on the thread's (row, chunk), so the load overlaps the dependent cache-length ->
// page-table lookups that give the destination. Index arithmetic runs in Index (32-bit
// whenever the launch's chunk count fits, the common case).
template <int kElemBytes, int kVecBytes, typename Index>
__global__ void __launch_bounds__(256) kv_scatter_kernel(const ScatterParams p) {
  using Vec = typename std::conditional<
      kVecBytes == 16, uint4,
      typename std::conditional<kVecBytes == 8, uint2,
                                typename std::conditional<kVecBytes == 4, uint32_t,
                                                          uint16_t>::type>::type>::type;
  constexpr int kVecElems = kVecBytes / kElemBytes;
  const Index chunks = Index(p.head_dim / kVecElems);
  const bool packed = p.token_request != nullptr;
  const Index rows = Index(packed ? int64_t(p.total_tokens) : int64_t(p.batch) * p.query_len) * Index(p.heads);
  const Index total = 2 * rows * chunks;
  const int32_t page_mask = (1 << p.page_shift) - 1;
  for (Index i = Index(blockIdx.x) * Index(blockDim.x) + Index(threadIdx.x); i < total;
       i += Index(gridDim.x) * Index(blockDim.x)) {
    const Index chunk = i % chunks;
    Index row = i / chunks;
    const bool is_v = row >= rows;
    if (is_v) row -= rows;
    const Index h = row % Index(p.heads);
    const Index tok = row / Index(p.heads);  // packed: token index; else b * query_len + t
    int t, b;
    int64_t token_elem;  // element offset of this token's row (head offset not included)
    if (packed) {
      token_elem = int64_t(tok) * (is_v ? p.v_st : p.k_st);
    } else {
      t = int(tok % Index(p.query_len));
      b = int(tok / Index(p.query_len));
      token_elem = is_v ? (b * p.v_sb + t * p.v_st) : (b * p.k_sb + t * p.k_st);
    }
    const int64_t src_elem = token_elem + int64_t(h) * (is_v ? p.v_sh : p.k_sh);
    const Vec v = *reinterpret_cast<const Vec*>((is_v ? p.v_new : p.k_new) +
                                                (src_elem + int64_t(chunk) * kVecElems) * kElemBytes);
    if (packed) {
      b = p.token_request[tok];
      if (b < 0 || b >= p.batch) {
        flag_error(p.error_word, HYT_DEVERR_PACKED_RANGE);
        continue;
      }
      t = int(int64_t(tok) - p.q_start[b]);
      if (t < 0) {
        flag_error(p.error_word, HYT_DEVERR_PACKED_RANGE);
        continue;
      }
    }
    const int64_t pos = int64_t(p.cache_lens[b]) + t;
    const int64_t logical_page = pos >> p.page_shift;
    if (pos < 0 || logical_page >= p.page_table_stride) {
      flag_error(p.error_word, HYT_DEVERR_TABLE_RANGE);
      continue;
    }
    const int32_t page = p.page_table[int64_t(b) * p.page_table_stride + logical_page];
    if (page < 0 || page >= p.num_pages) {
      flag_error(p.error_word, HYT_DEVERR_PAGE_RANGE);
      continue;
    }
    const int64_t slot = (int64_t(page) << p.page_shift) + (pos & page_mask);
    const int64_t dst_elem = p.layer_offset + (int64_t(h) * p.capacity + slot) * p.head_dim;
    uint8_t* dst = (is_v ? p.v_pool : p.k_pool) + (dst_elem + int64_t(chunk) * kVecElems) * kElemBytes;
    *reinterpret_cast<Vec*>(dst) = v;
  }
}

template <int kElemBytes, int kVecBytes>
static cudaError_t launch_scatter(const ScatterParams& p, cudaStream_t stream) {
  constexpr int kVecElems = kVecBytes / kElemBytes;
  const int64_t tokens = p.token_request != nullptr ? int64_t(p.total_tokens) : int64_t(p.batch) * p.query_len;
  const int64_t total = 2 * tokens * p.heads * (p.head_dim / kVecElems);
  const int threads = 256;
  // one chunk per thread (a single pass: each thread's dependent lookups are paid once);
  // grid-stride only beyond 64 resident-size waves. Four chunks per thread with all
  // source loads first measured slower at decode sizes (fewer threads) and equal at
  // prefill sizes.
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 8 * 64) blocks = 148 * 8 * 64;
  if (blocks < 1) blocks = 1;
  if (total + int64_t(blocks) * threads < (int64_t(1) << 31))
    kv_scatter_kernel<kElemBytes, kVecBytes, int32_t><<<int(blocks), threads, 0, stream>>>(p);
  else
    kv_scatter_kernel<kElemBytes, kVecBytes, int64_t><<<int(blocks), threads, 0, stream>>>(p);
  return cudaGetLastError();
}

// Widest vector every address of the copy is aligned to.
static int scatter_vec_bytes(const ScatterParams& p, int elem_bytes) {
  auto aligned = [&](int v) {
    if ((int64_t(p.head_dim) * elem_bytes) % v) return false;
    const int64_t strides[6] = {p.k_sb, p.k_sh, p.k_st, p.v_sb, p.v_sh, p.v_st};
    for (int64_t s : strides)
      if ((s * elem_bytes) % v) return false;
    const uintptr_t ptrs[4] = {uintptr_t(p.k_new), uintptr_t(p.v_new), uintptr_t(p.k_pool),
                               uintptr_t(p.v_pool)};
    for (uintptr_t a : ptrs)
      if (a % v) return false;
    return true;
  };
  for (int v : {16, 8, 4})
    if (v >= elem_bytes && aligned(v)) return v;
  return elem_bytes;
}

cudaError_t run_kv_scatter(const ScatterParams& p, int elem_bytes, cudaStream_t stream) {
  const int vec = scatter_vec_bytes(p, elem_bytes);
  if (elem_bytes == 2) {
    switch (vec) {
      case 16: return launch_scatter<2, 16>(p, stream);
      case 8: return launch_scatter<2, 8>(p, stream);
      case 4: return launch_scatter<2, 4>(p, stream);
      default: return launch_scatter<2, 2>(p, stream);
    }
  }
  switch (vec) {
    case 16: return launch_scatter<4, 16>(p, stream);
    case 8: return launch_scatter<4, 8>(p, stream);
    default: return launch_scatter<4, 4>(p, stream);
  }
}

}  // namespace hyt
