// Kernel (b): chunked-prefill causal GQA attention on tcgen05 tensor cores.
//
// Semantics: PagedKVBatch.attend_layer (hayate/engine/paged_cache.py:62-71) for a
// chunk of T new tokens per request on top of cache_lens[b] cached ones: query t
// of request b sees logical keys 0 .. cache_lens[b] + t (paged_cache.py:266-271),
// query head h reads KV head h / (H_q / H_kv), scale 1/sqrt(128) by default.
//
// Work unit: one CTA per (128 consecutive queries of one query head, request).
// 192 threads, warp-specialised:
//   warps 0-3 (softmax warpgroup): thread r owns query row r. It loads its Q row
//     into 128B-swizzled shared memory, then for every 128-key tile reads its S
//     row from TMEM (tcgen05.ld), applies the causal mask, runs a base-2 online
//     softmax (the running max is only moved when it grows by more than 2^8, so
//     O is rescaled rarely; the final O / l is exact either way), writes its P row
//     as bf16/f16 into swizzled shared memory and, when the max moved, rescales
//     its O row in TMEM. At the end it normalises O and stores the output row.
//   warp 4 (producer): per 128-key tile looks the page up in the page table and
//     TMA-loads the K and V tiles (2 boxes of [128 tokens x 64 dims] each, 128B
//     swizzle) into 2-stage rings.
//   warp 5 (MMA issuer, one thread): S = Q K^T into one of two TMEM S buffers
//     (M=128, N=128, 8 x K=16), then O += P V (V as an MN-major operand), each
//     batch closed by tcgen05.commit onto the mbarriers the other warps wait on.
//     QK of tile j+1 is issued before PV of tile j so the tensor core works on
//     it while the softmax warps handle tile j.
// TMEM: S0 cols [0,128), S1 [128,256), O [256,384) of a 512-column allocation.
// Shared memory: Q 32 KB, K 2x32 KB, V 2x32 KB, P 2x32 KB (about 225 KB).
//
// FLOPs per launch counted by the roofline: 4 * H_q * 128 per causal-valid
// (query, key) pair.
#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"

namespace hyt {

namespace {

constexpr int kRows = 128;  // queries per CTA
constexpr int kKeys = 128;  // keys per tile
constexpr int kD = 128;
constexpr int kThreads = 192;
constexpr int kTileBytes = kRows * kD * 2;  // 32 KB
constexpr int kChunkBytes = kTileBytes / 2; // [128 rows x 64 elements]
constexpr int kQOff = 0;
constexpr int kKOff = kQOff + kTileBytes;
constexpr int kVOff = kKOff + 2 * kTileBytes;
constexpr int kPOff = kVOff + 2 * kTileBytes;
constexpr int kBarOff = kPOff + 2 * kTileBytes;
constexpr int kSmemBytes = kBarOff + 256 + 1024;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kOCol = 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct PrefillKernelParams {
  AttentionParams a;
  int32_t group;
};

// Byte offset of 16-byte chunk `chunk` (0..15) of row `r` in a [128 x 128] tile
// stored as two 128B-swizzled [128 x 64] chunks (the layout TMA SWIZZLE_128B writes).
__device__ __forceinline__ uint32_t sw128_offset(int r, int chunk) {
  return uint32_t((chunk >> 3) * kChunkBytes + r * 128 + (((chunk & 7) ^ (r & 7)) << 4));
}

struct Barriers {
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
  uint64_t s_full[2], s_free[2], p_full[2], p_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int32_t abort;  // set once a bounded wait gave up: later waits return at once
};
static_assert(sizeof(Barriers) <= 256, "barrier block");

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_attention_kernel(const __grid_constant__ CUtensorMap k_map,
                             const __grid_constant__ CUtensorMap v_map,
                             const PrefillKernelParams P) {
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const AttentionParams& p = P.a;
  const int q_tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int g = h / P.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + kBarOff);

  const int cache_len = p.cache_lens[b];
  const int t0 = q_tile * kRows;
  const int t_last = min(t0 + kRows, p.query_len) - 1;
  const int n_tiles = (cache_len + t_last) / kKeys + 1;
  const int32_t* table = p.page_table + int64_t(b) * p.page_table_stride;
  const int page_mask = (1 << p.page_shift) - 1;

  // ---- refuse page ids that would address outside the pool (before any load)
  int bad = cache_len < 0 ? HYT_DEVERR_TABLE_RANGE : 0;
  // a wait of an earlier CTA already gave up: do not start another pipeline
  if (p.error_word != nullptr && (*reinterpret_cast<volatile int32_t*>(p.error_word) & HYT_DEVERR_WAIT_TIMEOUT))
    bad |= HYT_DEVERR_WAIT_TIMEOUT;
  for (int j = threadIdx.x; j < n_tiles && !bad; j += kThreads) {
    const int lp = (j * kKeys) >> p.page_shift;
    if (lp >= p.page_table_stride) {
      bad |= HYT_DEVERR_TABLE_RANGE;
    } else {
      const int32_t page = table[lp];
      if (page < 0 || page >= p.num_pages) bad |= HYT_DEVERR_PAGE_RANGE;
    }
  }
  bad = __syncthreads_or(bad);
  if (bad) {
    if (threadIdx.x == 0) flag_error(p.error_word, bad);
    // write zeros for this CTA's rows so the output is defined
    for (int idx = threadIdx.x; idx < kRows * kD; idx += kThreads) {
      const int r = idx / kD, d = idx - r * kD;
      if (t0 + r < p.query_len) {
        T* out = static_cast<T*>(p.out) + b * p.o_sb + int64_t(h) * p.o_sh + int64_t(t0 + r) * p.o_st;
        out[d] = Elem<T>::from_float(0.f);
      }
    }
    return;
  }

  if (threadIdx.x == 0) {
    bars->abort = 0;
    mbar_init(&bars->drain, 1);
    mbar_init(&bars->q_full, 128);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->s_free[s], 128);
      mbar_init(&bars->p_full[s], 128);
      mbar_init(&bars->p_empty[s], 1);
    }
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const uint32_t smem_base = smem_u32(smem);
  int32_t* err = p.error_word;

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&k_map);
      tma_prefetch_desc(&v_map);
      const int plane = p.layer * p.num_kv_heads + g;
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        const int tok = j * kKeys;
        const int32_t page = table[tok >> p.page_shift];
        const int row = (page << p.page_shift) + (tok & page_mask);
        if (j >= 2) mbar_wait(&bars->k_empty[st], ph ^ 1, err, &bars->abort);
        uint8_t* kdst = smem + kKOff + st * kTileBytes;
        mbar_arrive_expect_tx(&bars->k_full[st], kTileBytes);
        tma_load_3d(kdst, &k_map, &bars->k_full[st], 0, row, plane);
        tma_load_3d(kdst + kChunkBytes, &k_map, &bars->k_full[st], 64, row, plane);
        if (j >= 2) mbar_wait(&bars->v_empty[st], ph ^ 1, err, &bars->abort);
        uint8_t* vdst = smem + kVOff + st * kTileBytes;
        mbar_arrive_expect_tx(&bars->v_full[st], kTileBytes);
        tma_load_3d(vdst, &v_map, &bars->v_full[st], 0, row, plane);
        tma_load_3d(vdst + kChunkBytes, &v_map, &bars->v_full[st], 64, row, plane);
      }
      // no TMA write may still be in flight when the CTA exits
      for (int j = max(0, n_tiles - 2); j < n_tiles; ++j) {
        mbar_drain(&bars->k_full[j & 1], (j >> 1) & 1);
        mbar_drain(&bars->v_full[j & 1], (j >> 1) & 1);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = umma_idesc_f16(kBf16, 128, 128, false, false);
      constexpr uint32_t idesc_pv = umma_idesc_f16(kBf16, 128, 128, false, true);
      auto kmajor = [&](uint32_t base, int kk) {
        // k-step kk (16 elements): chunk kk/4, 32-byte step inside the 128B atom
        return umma_desc_sw128(base + (kk >> 2) * kChunkBytes + (kk & 3) * 32, 16);
      };
      auto issue_pv = [&](int i) {
        const int st = i & 1;
        const uint32_t ph = (i >> 1) & 1;
        mbar_wait(&bars->v_full[st], ph, err, &bars->abort);
        mbar_wait(&bars->p_full[st], ph, err, &bars->abort);
        tc_fence_after();
        const uint32_t pbase = smem_base + kPOff + st * kTileBytes;
        const uint32_t vbase = smem_base + kVOff + st * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          // V is [keys x dims]: K-dim = keys (16 per step = 2048 bytes), N = dims (LBO = chunk)
          const uint64_t vdesc = umma_desc_sw128(vbase + kk * 2048, kChunkBytes);
          umma_f16_ss(tmem + kOCol, kmajor(pbase, kk), vdesc, idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars->p_empty[st]);
        umma_commit(&bars->v_empty[st]);
      };
      mbar_wait(&bars->q_full, 0, err, &bars->abort);
      tc_fence_after();
      const uint32_t qbase = smem_base + kQOff;
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        mbar_wait(&bars->k_full[st], ph, err, &bars->abort);
        if (j >= 2) mbar_wait(&bars->s_free[st], ph ^ 1, err, &bars->abort);
        tc_fence_after();
        const uint32_t kbase = smem_base + kKOff + st * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          umma_f16_ss(tmem + st * 128, kmajor(qbase, kk), kmajor(kbase, kk), idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full[st]);
        umma_commit(&bars->k_empty[st]);
        if (j >= 1) issue_pv(j - 1);
      }
      issue_pv(n_tiles - 1);
      umma_commit(&bars->drain);  // every MMA done before TMEM is released
      mbar_drain(&bars->drain, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroup
    const int r = threadIdx.x;  // 0..127: query row == TMEM lane
    const int t = t0 + r;
    const bool row_valid = t < p.query_len;
    const int limit = cache_len + min(t, p.query_len - 1);  // last visible key
    const uint32_t lane_addr = tmem + (uint32_t(warp * 32) << 16);

    // Q row -> swizzled shared memory (zeros past the chunk)
    {
      const T* qrow = static_cast<const T*>(p.q) + b * p.q_sb + int64_t(h) * p.q_sh + int64_t(t) * p.q_st;
      uint8_t* qdst = smem + kQOff;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (row_valid) v = reinterpret_cast<const uint4*>(qrow)[c];
        *reinterpret_cast<uint4*>(qdst + sw128_offset(r, c)) = v;
      }
      fence_proxy_async_smem();
      mbar_arrive(&bars->q_full);
    }

    const float scale_log2 = p.scale * kLog2e;
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      mbar_wait(&bars->s_full[st], ph, err, &bars->abort);
      tc_fence_after();
      float s[128];
      {
        uint32_t raw[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          tmem_ld32(lane_addr + st * 128 + c * 32, raw);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(raw[i]);
        }
      }
      tc_fence_before();
      mbar_arrive(&bars->s_free[st]);

      // mask + tile max (scores in log2 units)
      const int key0 = j * kKeys;
      float mx = -INFINITY;
      if (key0 + kKeys - 1 <= limit) {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          s[c] *= scale_log2;
          mx = fmaxf(mx, s[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          s[c] = (key0 + c <= limit) ? s[c] * scale_log2 : -INFINITY;
          mx = fmaxf(mx, s[c]);
        }
      }
      const float m_new = fmaxf(m_run, mx);
      const bool warp_moves = __any_sync(0xffffffffu, m_new > m_run + kRescaleThreshold);
      float alpha = 1.f;
      if (warp_moves) {
        alpha = ex2(m_run - m_new);  // 0 on the first tile (m_run = -inf)
        m_run = m_new;
      }
      float rowsum = 0.f;
      uint32_t packed[64];
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float p0 = ex2(s[2 * c] - m_run);
        const float p1 = ex2(s[2 * c + 1] - m_run);
        rowsum += p0 + p1;
        packed[c] = Elem<T>::pack2(p0, p1);
      }
      l_run = l_run * alpha + rowsum;

      // P row -> swizzled shared memory (buffer st is free once PV(j-2) completed)
      if (j >= 2) mbar_wait(&bars->p_empty[st], ph ^ 1, err, &bars->abort);
      uint8_t* pdst = smem + kPOff + st * kTileBytes;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        *reinterpret_cast<uint4*>(pdst + sw128_offset(r, c)) =
            make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
      }

      // rescale O (the running max moved) once PV(j-1) has landed in TMEM
      if (warp_moves && j >= 1) {
        mbar_wait(&bars->p_empty[(j - 1) & 1], ((j - 1) >> 1) & 1, err, &bars->abort);
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(lane_addr + kOCol + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(lane_addr + kOCol + c * 32, o);
        }
        tmem_wait_st();
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->p_full[st]);
    }

    // ---- epilogue: O / l -> out[b, h, t, :]
    mbar_wait(&bars->p_empty[(n_tiles - 1) & 1], ((n_tiles - 1) >> 1) & 1, err, &bars->abort);
    tc_fence_after();
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    T* out = static_cast<T*>(p.out) + b * p.o_sb + int64_t(h) * p.o_sh + int64_t(t) * p.o_st;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t o[32];
      tmem_ld32(lane_addr + kOCol + c * 32, o);
      tmem_wait_ld();
      if (row_valid) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 w;
          w.x = Elem<T>::pack2(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
          w.y = Elem<T>::pack2(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
          w.z = Elem<T>::pack2(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
          w.w = Elem<T>::pack2(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
          reinterpret_cast<uint4*>(out)[c * 4 + v] = w;
        }
      }
    }
  }

  // ---- release TMEM once every warp is done with it
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

cudaError_t run_prefill_attention(const AttentionParams& p, const CUtensorMap& k_map,
                                  const CUtensorMap& v_map, int dtype, cudaStream_t stream) {
  PrefillKernelParams P;
  P.a = p;
  P.group = p.num_q_heads / p.num_kv_heads;
  const dim3 grid(unsigned((p.query_len + kRows - 1) / kRows), unsigned(p.num_q_heads),
                  unsigned(p.batch));
  if (dtype == HYT_DTYPE_F16) {
    auto kernel = prefill_attention_kernel<__half>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    kernel<<<grid, kThreads, kSmemBytes, stream>>>(k_map, v_map, P);
  } else {
    auto kernel = prefill_attention_kernel<__nv_bfloat16>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    kernel<<<grid, kThreads, kSmemBytes, stream>>>(k_map, v_map, P);
  }
  return cudaGetLastError();
}

}  // namespace hyt
