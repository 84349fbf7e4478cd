// Kernel (c): split-KV paged decode attention (HBM-bound).
//
// Semantics: PagedKVBatch.attend_layer (hayate/engine/paged_cache.py:62-71) for
// short query chunks: query t of request b sees logical keys
// 0 .. cache_lens[b] + t (paged_cache.py:266-271), query head h reads KV head
// h / group (FlexAttention enable_gqa), softmax scale 1/sqrt(128) by default.
//
// Work unit: one CTA per (split of up to split_tokens keys, KV head g, request b); a
// request's keys are cut into equal 64-token-aligned pieces, no short last piece.
// All group * query_len (<= 16) query rows that share KV head g ride in one
// 16-row mma tile, so every K/V byte is read from HBM exactly once per step.
//
//   warp 4 (producer): walks the split's 64-token tiles, looks each one up in the
//     page table and issues TMA loads of the K and V tiles (4 boxes of
//     [64 tokens x 64 dims], 128-byte swizzle) into a 3-stage ring of 32 KB
//     stages, signalling a full-barrier with the byte count.
//   warps 0-3 (consumers): each takes 16 of the tile's 64 keys; S = Q K^T and
//     O += P V with mma.sync m16n8k16 (fp32 accumulate) fed by ldmatrix from the
//     swizzled tiles; base-2 online softmax with quad shuffles; release the stage.
//   epilogue: the 4 warps' (max, sum, O) are merged through shared memory; a
//     single-split request writes the normalised output directly, otherwise the
//     split writes its partial to the workspace and the last split to arrive
//     (atomic counter, no waiting) merges all partials and resets the counter.
//
// Fused scatter (DecodeLaunch::k_new, uniform batches): the consumer warps of the split
// that attends a new row first copy it from the step's K/V into its pool slot (the copy
// kernel (a) makes) and fence the async proxy; the producer loads that tile only after
// they have all arrived on an mbarrier. One launch then does write_layer + attend_layer.
//
// Packed batches: a launch may serve a list of requests (AttentionParams::req_ids)
// whose one-token chunks sit on a shared token axis; workspace slots follow the
// launch index, so the workspace is sized for the list.
//
// Bytes per launch: sum_b kv_len[b] * H_kv * 128 * 2 (K and V) * elem_bytes,
// which is what the roofline counts.
#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"

namespace hyt {

namespace {

constexpr int kTile = 64;                       // tokens per stage
constexpr int kStages = 3;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kD = 128;
constexpr int kBoxBytes = kTile * 128;          // [64 tokens x 64 dims] x 2 B
constexpr int kStageBytes = 4 * kBoxBytes;      // K lo, K hi, V lo, V hi
constexpr int kRingBytes = kStages * kStageBytes;
constexpr int kSmemBytes = kRingBytes + 1024 /*align*/ + 256 /*barriers*/;
static_assert(kConsumerWarps * kDecodeMaxRows * kD * 4 + 2 * kConsumerWarps * kDecodeMaxRows * 4 <= kRingBytes,
              "merge scratch must fit in the ring");

struct DecodeKernelParams {
  AttentionParams a;
  DecodeLaunch d;
  int32_t group, rows;
};

// Byte offset of 16-byte chunk `chunk` (0..15 over 128 dims) of token row `r` in a
// [64 x 128] tile stored as two 128B-swizzled [64 x 64] boxes.
__device__ __forceinline__ uint32_t tile_offset(int r, int chunk) {
  return uint32_t((chunk >> 3) * kBoxBytes + r * 128 + (((chunk & 7) ^ (r & 7)) << 4));
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
    decode_attention_kernel(const __grid_constant__ CUtensorMap k_map,
                            const __grid_constant__ CUtensorMap v_map,
                            const DecodeKernelParams P) {
  constexpr bool kHalf = std::is_same<T, __half>::value;
  const AttentionParams& p = P.a;
  const int split = blockIdx.x, g = blockIdx.y, z = blockIdx.z;
  const int b = att_request(p, z);  // z == b unless the launch serves a request list
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // packed batches send only requests whose chunk has exactly query_len queries here
  if (!att_request_ok(p, b) || att_query_len(p, b) != p.query_len) {
    if (split == 0 && g == 0 && threadIdx.x == 0) flag_error(p.error_word, HYT_DEVERR_PACKED_RANGE);
    return;
  }

  const int cache_len = p.cache_lens[b];
  const int kv_len = cache_len + p.query_len;
  // this request's keys in nsplits pieces of equal size (a multiple of the 64-token tile,
  // at most split_tokens): no short last piece. (nsplits - 1) * piece < kv_len, so every
  // one of the nsplits pieces holds keys and the last-arriver count stays nsplits.
  int nsplits = (kv_len + P.d.split_tokens - 1) / P.d.split_tokens;
  const int piece = nsplits > 0 ? ((kv_len + nsplits - 1) / nsplits + kTile - 1) / kTile * kTile : P.d.split_tokens;
  const int tok_begin = split * piece;
  if (tok_begin >= kv_len) return;  // uniform per CTA, before any barrier
  const int tok_end = min(kv_len, tok_begin + piece);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRingBytes);
  uint64_t* empty = full + kStages;
  uint64_t* scattered = empty + kStages;  // fused scatter: the split's new rows are in the pool
  int* s_last = reinterpret_cast<int*>(scattered + 1);
  volatile int* s_abort = s_last + 1;  // set once a bounded wait gave up

  // ---- refuse page ids / lengths that would address outside the pool
  int bad = 0;
  if (kv_len > P.d.max_splits * P.d.split_tokens) bad |= HYT_DEVERR_SPLIT_RANGE;
  const int32_t* table = p.page_table + int64_t(b) * p.page_table_stride;
  for (int tok = tok_begin + int(threadIdx.x) * kTile; tok < tok_end; tok += kThreads * kTile) {
    const int lp = tok >> p.page_shift;
    if (lp >= p.page_table_stride) {
      bad |= HYT_DEVERR_TABLE_RANGE;
    } else {
      const int32_t page = table[lp];
      if (page < 0 || page >= p.num_pages) bad |= HYT_DEVERR_PAGE_RANGE;
    }
  }
  if (p.error_word != nullptr && (*reinterpret_cast<volatile int32_t*>(p.error_word) & HYT_DEVERR_WAIT_TIMEOUT))
    bad |= HYT_DEVERR_WAIT_TIMEOUT;  // an earlier CTA's wait gave up: start no pipeline
  bad = __syncthreads_or(bad);
  if (bad && threadIdx.x == 0) flag_error(p.error_word, bad);
  if (nsplits > P.d.max_splits) nsplits = P.d.max_splits;
  // fused scatter: this split attends positions [new_lo, tok_end) of the step's new rows
  // (a refused split writes nothing)
  const int new_lo = max(cache_len, tok_begin);
  const bool has_new = P.d.k_new != nullptr && !bad && new_lo < tok_end;

  if (threadIdx.x == 0) {
    *s_abort = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    mbar_init(scattered, kConsumerWarps * 32);
    fence_barrier_init();
  }
  __syncthreads();

  const int n_tiles = bad ? 0 : (tok_end - tok_begin + kTile - 1) / kTile;
  const int plane = p.layer * p.num_kv_heads + g;
  const int page_mask = (1 << p.page_shift) - 1;

  // per-thread softmax state for rows lane/4 and lane/4 + 8 (consumers only)
  float o[16][4];
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&k_map);
      tma_prefetch_desc(&v_map);
      for (int i = 0; i < n_tiles; ++i) {
        const int stage = i % kStages;
        if (i >= kStages) mbar_wait(&empty[stage], ((i / kStages) - 1) & 1, p.error_word, s_abort);
        const int tok = tok_begin + i * kTile;
        // the tile holding the first new row is read only once the consumers wrote it
        if (has_new && i == (new_lo - tok_begin) / kTile) mbar_wait(scattered, 0, p.error_word, s_abort);
        const int32_t page = table[tok >> p.page_shift];
        const int row = (page << p.page_shift) + (tok & page_mask);
        uint8_t* dst = smem + stage * kStageBytes;
        mbar_arrive_expect_tx(&full[stage], kStageBytes);
        tma_load_3d(dst, &k_map, &full[stage], 0, row, plane);
        tma_load_3d(dst + kBoxBytes, &k_map, &full[stage], 64, row, plane);
        tma_load_3d(dst + 2 * kBoxBytes, &v_map, &full[stage], 0, row, plane);
        tma_load_3d(dst + 3 * kBoxBytes, &v_map, &full[stage], 64, row, plane);
      }
      // no TMA write may still be in flight when the ring is reused or the CTA exits
      for (int i = max(0, n_tiles - kStages); i < n_tiles; ++i)
        mbar_drain(&full[i % kStages], (i / kStages) & 1);
    }
  } else {
    // ------------------------------------------------------------ consumers
    // fused scatter (kv_scatter's copy for this split's rows of KV head g), in two halves
    // around the Q load so that its source loads and Q's share one memory round trip:
    // up to kScatterPerThread 16-byte chunks per thread are loaded here and stored after
    // the Q loads were issued, then a proxy fence lets the producer's TMA, ordered after
    // the `scattered` barrier, read the new rows.
    constexpr int kChunks = kD * int(sizeof(T)) / 16;
    constexpr int kScatterPerThread = 2 * (kDecodeMaxRows * kChunks) / (kConsumerWarps * 32);
    const int n_chunks = has_new ? 2 * (tok_end - new_lo) * kChunks : 0;
    uint4 scat_v[kScatterPerThread];
    uint8_t* scat_dst[kScatterPerThread];
#pragma unroll
    for (int c = 0; c < kScatterPerThread; ++c) {
      const int idx = int(threadIdx.x) + c * kConsumerWarps * 32;
      scat_dst[c] = nullptr;
      if (idx < n_chunks) {
        const int nrows = tok_end - new_lo;
        const bool is_v = idx >= nrows * kChunks;
        const int rem = is_v ? idx - nrows * kChunks : idx;
        const int row = rem / kChunks, chunk = rem - row * kChunks;
        const int pos = new_lo + row, t = pos - cache_len;
        const int64_t src_elem = int64_t(b) * (is_v ? P.d.v_sb : P.d.k_sb) +
                                 int64_t(g) * (is_v ? P.d.v_sh : P.d.k_sh) +
                                 int64_t(t) * (is_v ? P.d.v_st : P.d.k_st);
        scat_v[c] = *reinterpret_cast<const uint4*>((is_v ? P.d.v_new : P.d.k_new) +
                                                    src_elem * int64_t(sizeof(T)) + chunk * 16);
        const int32_t page = table[pos >> p.page_shift];  // checked with the split's pages
        const int64_t slot = (int64_t(page) << p.page_shift) + (pos & page_mask);
        const int64_t layer_off = int64_t(p.layer) * p.num_kv_heads * p.capacity * kD;
        scat_dst[c] = (is_v ? P.d.v_pool : P.d.k_pool) +
                      (layer_off + (int64_t(g) * p.capacity + slot) * kD) * int64_t(sizeof(T)) + chunk * 16;
      }
    }
    const int r0 = lane >> 2, c2 = (lane & 3) * 2;
    // Q rows: row r = local_head * query_len + t, zero past group * query_len.
    uint32_t qa[8][4];
    {
      const T* qbase = static_cast<const T*>(p.q);
      const T* qrow[2] = {nullptr, nullptr};
      for (int half = 0; half < 2; ++half) {
        const int r = r0 + half * 8;
        if (r < P.rows) {
          const int hl = r / p.query_len, t = r - hl * p.query_len;
          qrow[half] = qbase + att_q_row(p, b, t) + int64_t(g * P.group + hl) * p.q_sh;
        }
      }
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const T* src = qrow[j & 1];
          const int d = kk * 16 + c2 + (j >> 1) * 8;
          if (src != nullptr) {
            const T lo = src[d], hi = src[d + 1];
            qa[kk][j] = uint32_t(*reinterpret_cast<const uint16_t*>(&lo)) |
                        (uint32_t(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
          } else {
            qa[kk][j] = 0u;
          }
        }
      }
    }
    if (has_new) {  // second half of the fused scatter (see above)
#pragma unroll
      for (int c = 0; c < kScatterPerThread; ++c)
        if (scat_dst[c] != nullptr) *reinterpret_cast<uint4*>(scat_dst[c]) = scat_v[c];
      fence_proxy_async_global();
      mbar_arrive(scattered);
    }
    // last visible key of each of this thread's two rows
    int limit[2];
    for (int half = 0; half < 2; ++half) {
      const int r = r0 + half * 8;
      const int t = r < P.rows ? r % p.query_len : 0;
      limit[half] = cache_len + t;
    }
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    const float scale_log2 = p.scale * kLog2e;
    const uint32_t ring = smem_u32(smem);

    for (int i = 0; i < n_tiles; ++i) {
      const int stage = i % kStages;
      mbar_wait(&full[stage], (i / kStages) & 1, p.error_word, s_abort);
      const uint32_t kbase = ring + stage * kStageBytes;
      const uint32_t vbase = kbase + 2 * kBoxBytes;
      const int key0 = warp * 16;  // this warp's keys inside the tile

      // ---- S = Q K^T for 16 keys (2 n-tiles of 8)
      float s[2][4];
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
        const int r = key0 + n * 8 + (lane & 7);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(kbase + tile_offset(r, 4 * c + (lane >> 3)), b0, b1, b2, b3);
          mma_16816<kHalf>(s[n], qa[2 * c], b0, b1);
          mma_16816<kHalf>(s[n], qa[2 * c + 1], b2, b3);
        }
      }

      // ---- mask, online softmax (base 2)
      const int tok0 = tok_begin + i * kTile + key0;
      float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int n = 0; n < 2; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int half = e >> 1;
          const int key = tok0 + n * 8 + c2 + (e & 1);
          const float x = key <= limit[half] ? s[n][e] * scale_log2 : -INFINITY;
          s[n][e] = x;
          tmax[half] = fmaxf(tmax[half], x);
        }
      }
      float alpha[2], m_use[2];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        tmax[half] = fmaxf(tmax[half], __shfl_xor_sync(0xffffffffu, tmax[half], 1));
        tmax[half] = fmaxf(tmax[half], __shfl_xor_sync(0xffffffffu, tmax[half], 2));
        const float m_new = fmaxf(m_run[half], tmax[half]);
        m_use[half] = m_new == -INFINITY ? 0.f : m_new;
        alpha[half] = ex2(m_run[half] - m_use[half]);
        m_run[half] = m_new;
      }
      float psum[2] = {0.f, 0.f};
#pragma unroll
      for (int n = 0; n < 2; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int half = e >> 1;
          s[n][e] = ex2(s[n][e] - m_use[half]);
          psum[half] += s[n][e];
        }
      }
#pragma unroll
      for (int half = 0; half < 2; ++half) l_run[half] = l_run[half] * alpha[half] + psum[half];
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        o[n][0] *= alpha[0];
        o[n][1] *= alpha[0];
        o[n][2] *= alpha[1];
        o[n][3] *= alpha[1];
      }

      // ---- O += P V  (P: 16 rows x 16 keys as one A fragment)
      uint32_t pa[4];
      pa[0] = Elem<T>::pack2(s[0][0], s[0][1]);
      pa[1] = Elem<T>::pack2(s[0][2], s[0][3]);
      pa[2] = Elem<T>::pack2(s[1][0], s[1][1]);
      pa[3] = Elem<T>::pack2(s[1][2], s[1][3]);
      const int vr = key0 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
      for (int dc = 0; dc < 8; ++dc) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(vbase + tile_offset(vr, 2 * dc + (lane >> 4)), b0, b1, b2, b3);
        mma_16816<kHalf>(o[2 * dc], pa, b0, b1);
        mma_16816<kHalf>(o[2 * dc + 1], pa, b2, b3);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      l_run[half] += __shfl_xor_sync(0xffffffffu, l_run[half], 1);
      l_run[half] += __shfl_xor_sync(0xffffffffu, l_run[half], 2);
    }
  }
  __syncthreads();  // every TMA write has been consumed: the ring is free

  // ---- merge the 4 consumer warps through shared memory
  float* red_o = reinterpret_cast<float*>(smem);                       // [warp][16][128]
  float* red_m = red_o + kConsumerWarps * kDecodeMaxRows * kD;         // [warp][16]
  float* red_l = red_m + kConsumerWarps * kDecodeMaxRows;              // [warp][16]
  if (warp < kConsumerWarps) {
    const int r0 = lane >> 2, c2 = (lane & 3) * 2;
    float* wo = red_o + warp * kDecodeMaxRows * kD;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      wo[r0 * kD + n * 8 + c2] = o[n][0];
      wo[r0 * kD + n * 8 + c2 + 1] = o[n][1];
      wo[(r0 + 8) * kD + n * 8 + c2] = o[n][2];
      wo[(r0 + 8) * kD + n * 8 + c2 + 1] = o[n][3];
    }
    if ((lane & 3) == 0) {
      red_m[warp * kDecodeMaxRows + r0] = m_run[0];
      red_m[warp * kDecodeMaxRows + r0 + 8] = m_run[1];
      red_l[warp * kDecodeMaxRows + r0] = l_run[0];
      red_l[warp * kDecodeMaxRows + r0 + 8] = l_run[1];
    }
  }
  __syncthreads();

  const int64_t unit = int64_t(z) * p.num_kv_heads + g;  // (launch request index, kv head)
  const int rows = P.rows;
  float* ws_o = P.d.ws_o + (unit * P.d.max_splits + split) * rows * kD;
  float* ws_ml = P.d.ws_ml + (unit * P.d.max_splits + split) * rows * 2;
  for (int idx = threadIdx.x; idx < rows * kD; idx += kThreads) {
    const int r = idx / kD, d = idx - r * kD;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) mx = fmaxf(mx, red_m[w * kDecodeMaxRows + r]);
    const float mu = mx == -INFINITY ? 0.f : mx;
    float lsum = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float f = ex2(red_m[w * kDecodeMaxRows + r] - mu);
      lsum += red_l[w * kDecodeMaxRows + r] * f;
      acc += red_o[(w * kDecodeMaxRows + r) * kD + d] * f;
    }
    if (nsplits == 1) {
      const int hl = r / p.query_len, t = r - hl * p.query_len;
      T* out = static_cast<T*>(p.out) + att_o_row(p, b, t) + int64_t(g * P.group + hl) * p.o_sh;
      out[d] = Elem<T>::from_float(lsum > 0.f ? acc / lsum : 0.f);
    } else {
      ws_o[idx] = acc;
      if (d == 0) {
        ws_ml[r * 2] = mx;
        ws_ml[r * 2 + 1] = lsum;
      }
    }
  }
  if (nsplits == 1) return;

  // ---- last split to arrive merges every split's partial (no waiting)
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(&P.d.ws_counter[unit], 1);
    *s_last = prev == nsplits - 1;
  }
  __syncthreads();
  if (!*s_last) return;
  __threadfence();
  const float* all_o = P.d.ws_o + unit * P.d.max_splits * rows * kD;
  const float* all_ml = P.d.ws_ml + unit * P.d.max_splits * rows * 2;
  for (int idx = threadIdx.x; idx < rows * kD; idx += kThreads) {
    const int r = idx / kD, d = idx - r * kD;
    float mx = -INFINITY;
    for (int s = 0; s < nsplits; ++s) mx = fmaxf(mx, __ldcg(&all_ml[(s * rows + r) * 2]));
    const float mu = mx == -INFINITY ? 0.f : mx;
    float lsum = 0.f, acc = 0.f;
    for (int s = 0; s < nsplits; ++s) {
      const float f = ex2(__ldcg(&all_ml[(s * rows + r) * 2]) - mu);
      lsum += __ldcg(&all_ml[(s * rows + r) * 2 + 1]) * f;
      acc += __ldcg(&all_o[(int64_t(s) * rows + r) * kD + d]) * f;
    }
    const int hl = r / p.query_len, t = r - hl * p.query_len;
    T* out = static_cast<T*>(p.out) + att_o_row(p, b, t) + int64_t(g * P.group + hl) * p.o_sh;
    out[d] = Elem<T>::from_float(lsum > 0.f ? acc / lsum : 0.f);
  }
  if (threadIdx.x == 0) P.d.ws_counter[unit] = 0;  // leave the counter zero for the next call
}

}  // namespace

cudaError_t run_decode_attention(const AttentionParams& p, const DecodeLaunch& d,
                                 const CUtensorMap& k_map, const CUtensorMap& v_map, int dtype,
                                 cudaStream_t stream) {
  DecodeKernelParams P;
  P.a = p;
  P.d = d;
  P.group = p.num_q_heads / p.num_kv_heads;
  P.rows = P.group * p.query_len;
  const dim3 grid(unsigned(d.max_splits), unsigned(p.num_kv_heads), unsigned(att_launch_count(p)));
  if (dtype == HYT_DTYPE_F16) {
    auto kernel = decode_attention_kernel<__half>;
    cudaError_t err = allow_smem(kernel, kSmemBytes, stream);
    if (err != cudaSuccess) return err;
    kernel<<<grid, kThreads, kSmemBytes, stream>>>(k_map, v_map, P);
  } else {
    auto kernel = decode_attention_kernel<__nv_bfloat16>;
    cudaError_t err = allow_smem(kernel, kSmemBytes, stream);
    if (err != cudaSuccess) return err;
    kernel<<<grid, kThreads, kSmemBytes, stream>>>(k_map, v_map, P);
  }
  return cudaGetLastError();
}

}  // namespace hyt
