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
// One CTA per token, one half-warp per head row at a time; each lane holds 8 consecutive
// features, so the rotation partner (feature i +/- 64) sits in lane ^ 8. HBM-bound: every
// byte of q, k, v is read once and written once, the token's cos/sin rows once per warp.
#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"

namespace hyt {

namespace {

constexpr int kWarps = 8;
constexpr int kPairsPerWarp = 3;  // row pairs of one token a warp has in flight at once

// Two storage-dtype values packed in a 32-bit word, as fp32 (exact).
template <typename T>
__device__ __forceinline__ void unpack2(uint32_t w, float& lo, float& hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    lo = __uint_as_float(w << 16);
    hi = __uint_as_float(w & 0xFFFF0000u);
  } else {
    lo = __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu)));
    hi = __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
  }
}

// This lane's 8 consecutive features of a row as loaded: packed 16-bit values (4 words),
// or fp32 (8 words) for fp32 pools.
template <typename T>
struct RowBits {
  static constexpr int kWords = sizeof(T) == 2 ? 4 : 8;
  uint32_t w[kWords];
};
template <typename T>
__device__ __forceinline__ void load_row(const T* src, RowBits<T>& r) {
  if constexpr (sizeof(T) == 2) {
    const uint4 raw = *reinterpret_cast<const uint4*>(src);
    r.w[0] = raw.x, r.w[1] = raw.y, r.w[2] = raw.z, r.w[3] = raw.w;
  } else {
    const uint4 a = *reinterpret_cast<const uint4*>(src);
    const uint4 b = *reinterpret_cast<const uint4*>(src + 4);
    r.w[0] = a.x, r.w[1] = a.y, r.w[2] = a.z, r.w[3] = a.w, r.w[4] = b.x, r.w[5] = b.y, r.w[6] = b.z, r.w[7] = b.w;
  }
}
template <typename T>
__device__ __forceinline__ void unpack_row(const RowBits<T>& r, float (&x)[8]) {
  if constexpr (sizeof(T) == 2) {
#pragma unroll
    for (int i = 0; i < 4; ++i) unpack2<T>(r.w[i], x[2 * i], x[2 * i + 1]);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = __uint_as_float(r.w[i]);
  }
}

template <typename T>
__device__ __forceinline__ void store_row(T* dst, const RowBits<T>& r) {
  if constexpr (sizeof(T) == 2) {
    *reinterpret_cast<uint4*>(dst) = make_uint4(r.w[0], r.w[1], r.w[2], r.w[3]);
  } else {
    *reinterpret_cast<uint4*>(dst) = make_uint4(r.w[0], r.w[1], r.w[2], r.w[3]);
    *reinterpret_cast<uint4*>(dst + 4) = make_uint4(r.w[4], r.w[5], r.w[6], r.w[7]);
  }
}

// This lane's 8 consecutive features of a row, as fp32.
template <typename T>
__device__ __forceinline__ void load8(const T* src, float (&x)[8]) {
  if constexpr (sizeof(T) == 2) {
    const uint4 raw = *reinterpret_cast<const uint4*>(src);
    unpack2<T>(raw.x, x[0], x[1]);
    unpack2<T>(raw.y, x[2], x[3]);
    unpack2<T>(raw.z, x[4], x[5]);
    unpack2<T>(raw.w, x[6], x[7]);
  } else {
    const float4 a = *reinterpret_cast<const float4*>(src);
    const float4 b = *reinterpret_cast<const float4*>(src + 4);
    x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
  }
}

// One CTA per token: the token's rows live at offsets known from the grid alone, so their
// loads go out first; then the request, position, rotation tables and pool slot are looked
// up once. A half-warp takes a row (8 features a lane: the rotation partner, feature
// i +/- 64, sits in lane ^ 8), a warp a pair of rows, warp w the pairs w, w + 8, ...: with
// 32 + 8 + 8 rows, two q pairs and one k or v pair each. Arithmetic in fp32 on packed
// pairs (f32x2: the same IEEE results as scalar fp32, half the instructions).
template <typename T>
__global__ void __launch_bounds__(kWarps * 32, 4) norm_rope_scatter_kernel(const NormRopeParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hl = lane & 15, half = lane >> 4;
  const int heads = p.num_q_heads + 2 * p.num_kv_heads;
  const bool packed = p.token_request != nullptr;
  const int token = int(blockIdx.x);
  const int b_grid = packed ? 0 : token / p.query_len;
  const int t_grid = packed ? 0 : token - b_grid * p.query_len;
  const int64_t q_tok = packed ? int64_t(token) * p.q_st : b_grid * p.q_sb + int64_t(t_grid) * p.q_st;
  const int64_t k_tok = packed ? int64_t(token) * p.k_st : b_grid * p.k_sb + int64_t(t_grid) * p.k_st;
  const int64_t v_tok = packed ? int64_t(token) * p.v_st : b_grid * p.v_sb + int64_t(t_grid) * p.v_st;
  const int d0 = hl * 8;  // this lane's features d0 .. d0 + 7 (head_dim 128)
  // row r of the token: q head r, k head r - H_q, v head r - H_q - H_kv
  auto row_src = [&](int r) -> const T* {
    if (r < p.num_q_heads) return static_cast<const T*>(p.q) + q_tok + int64_t(r) * p.q_sh;
    if (r < p.num_q_heads + p.num_kv_heads)
      return static_cast<const T*>(p.k) + k_tok + int64_t(r - p.num_q_heads) * p.k_sh;
    return static_cast<const T*>(p.v) + v_tok + int64_t(r - p.num_q_heads - p.num_kv_heads) * p.v_sh;
  };
  auto issue_loads = [&](int pair0, RowBits<T> (&x)[kPairsPerWarp]) {
#pragma unroll
    for (int k = 0; k < kPairsPerWarp; ++k) {
      const int r = 2 * (pair0 + k * kWarps) + half;
      if (r < heads) load_row<T>(row_src(r) + d0, x[k]);
    }
  };
  RowBits<T> x[kPairsPerWarp];
  issue_loads(warp, x);

  int t = t_grid, b = b_grid;
  if (packed) {
    b = p.token_request[token];
    t = (b >= 0 && b < p.batch) ? token - p.q_start[b] : -1;
    if (t < 0) {
      if (threadIdx.x == 0) flag_error(p.error_word, HYT_DEVERR_PACKED_RANGE);
      return;
    }
  }
  const int64_t o_tok = packed ? int64_t(token) * p.o_st : b * p.o_sb + int64_t(t) * p.o_st;
  const int pos = p.cache_lens[b] + t;

  // rotation at `pos` (q and k rows) and the pool slot of `pos` (k and v rows)
  const bool rope_ok = pos >= 0 && pos < p.rope_positions;
  uint64_t c2[4], s2[4];
  {
    float c[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, sn[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (rope_ok) {
      load8<float>(p.cos + int64_t(pos) * 128 + d0, c);
      load8<float>(p.sin + int64_t(pos) * 128 + d0, sn);
    } else if (threadIdx.x == 0) {
      flag_error(p.error_word, HYT_DEVERR_TABLE_RANGE);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      c2[i] = f2_pack(c[2 * i], c[2 * i + 1]);
      s2[i] = f2_pack(sn[2 * i], sn[2 * i + 1]);
    }
  }
  int64_t slot = -1;  // -1: the token's K/V rows are not written (flagged)
  if (pos >= 0) {
    const int64_t logical_page = pos >> p.page_shift;
    if (logical_page < p.page_table_stride) {
      const int32_t page = p.page_table[int64_t(b) * p.page_table_stride + logical_page];
      if (page >= 0 && page < p.num_pages)
        slot = (int64_t(page) << p.page_shift) + (pos & ((1 << p.page_shift) - 1));
      else if (threadIdx.x == 0)
        flag_error(p.error_word, HYT_DEVERR_PAGE_RANGE);
    } else if (threadIdx.x == 0) {
      flag_error(p.error_word, HYT_DEVERR_TABLE_RANGE);
    }
  } else if (threadIdx.x == 0) {
    flag_error(p.error_word, HYT_DEVERR_TABLE_RANGE);
  }
  for (int pair0 = warp;;) {
#pragma unroll
    for (int k = 0; k < kPairsPerWarp; ++k) {
      const int pair = pair0 + k * kWarps;
      if (2 * pair >= heads) break;  // warp-uniform: the shuffles below see the whole warp
      const int r = 2 * pair + half;
      const int kind = r < p.num_q_heads ? 0 : (r < p.num_q_heads + p.num_kv_heads ? 1 : (r < heads ? 2 : 3));
      float xr[8];
      unpack_row<T>(x[k], xr);
      // RMSNorm in fp32 over the half-warp's 128 features, rounded to the storage dtype
      // (the module's output tensor); every lane computes it, v rows keep their input
      uint64_t ss2 = f2_mul(f2_pack(xr[0], xr[1]), f2_pack(xr[0], xr[1]));
#pragma unroll
      for (int i = 1; i < 4; ++i)
        ss2 = f2_fma(f2_pack(xr[2 * i], xr[2 * i + 1]), f2_pack(xr[2 * i], xr[2 * i + 1]), ss2);
      float ss_lo, ss_hi;
      f2_unpack(ss2, ss_lo, ss_hi);
      float ss = ss_lo + ss_hi;
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      const float rstd = rsqrtf(ss / 128.f + p.eps);
      const uint64_t rstd2 = f2_pack(rstd, rstd);
      RowBits<T> wb;
      load_row<T>(static_cast<const T*>(kind == 0 ? p.q_norm_weight : p.k_norm_weight) + d0, wb);
      float wv[8];
      unpack_row<T>(wb, wv);
      RowBits<T> out;
      if constexpr (sizeof(T) == 2) {
        // normalised values rounded to the storage dtype, as packed pairs: the rotation
        // partner moves in one shuffle per pair, its sign in one XOR of both sign bits
        uint32_t u[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint64_t v2 = f2_mul(f2_mul(f2_pack(xr[2 * i], xr[2 * i + 1]), rstd2), f2_pack(wv[2 * i], wv[2 * i + 1]));
          float lo, hi;
          f2_unpack(v2, lo, hi);
          u[i] = Elem<T>::pack2(lo, hi);
        }
        const uint32_t flip = hl < 8 ? 0x80008000u : 0u;  // rotated = cat(-x2, x1)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t pw = __shfl_xor_sync(0xffffffffu, u[i], 8) ^ flip;
          float n0, n1, p0, p1;
          unpack2<T>(u[i], n0, n1);
          unpack2<T>(pw, p0, p1);
          const uint64_t y2 = f2_add(f2_mul(f2_pack(n0, n1), c2[i]), f2_mul(f2_pack(p0, p1), s2[i]));
          float y0, y1;
          f2_unpack(y2, y0, y1);
          out.w[i] = Elem<T>::pack2(y0, y1);
        }
      } else {
        float xn[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint64_t v2 = f2_mul(f2_mul(f2_pack(xr[2 * i], xr[2 * i + 1]), rstd2), f2_pack(wv[2 * i], wv[2 * i + 1]));
          f2_unpack(v2, xn[2 * i], xn[2 * i + 1]);
        }
        const float sign = hl < 8 ? -1.f : 1.f;
        const uint64_t sign2 = f2_pack(sign, sign);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float plo = __shfl_xor_sync(0xffffffffu, xn[2 * i], 8);
          const float phi = __shfl_xor_sync(0xffffffffu, xn[2 * i + 1], 8);
          const uint64_t y2 = f2_add(f2_mul(f2_pack(xn[2 * i], xn[2 * i + 1]), c2[i]),
                                     f2_mul(f2_mul(f2_pack(plo, phi), sign2), s2[i]));
          float y0, y1;
          f2_unpack(y2, y0, y1);
          out.w[2 * i] = __float_as_uint(y0);
          out.w[2 * i + 1] = __float_as_uint(y1);
        }
      }
      if (kind == 0) {
        if (rope_ok) store_row<T>(static_cast<T*>(p.q_out) + o_tok + int64_t(r) * p.o_sh + d0, out);
      } else if (kind <= 2 && slot >= 0 && (kind == 2 || rope_ok)) {
        const int h = kind == 1 ? r - p.num_q_heads : r - p.num_q_heads - p.num_kv_heads;
        T* pool = static_cast<T*>(kind == 1 ? p.k_pool : p.v_pool);
        store_row<T>(pool + ((int64_t(p.layer) * p.num_kv_heads + h) * p.capacity + slot) * 128 + d0,
                     kind == 1 ? out : x[k]);
      }
    }
    // more head rows than one pass holds (more than 2 * kWarps * kPairsPerWarp heads)
    pair0 += kWarps * kPairsPerWarp;
    if (2 * pair0 >= heads) break;
    issue_loads(pair0, x);
  }
}

}  // namespace

cudaError_t run_norm_rope_scatter(const NormRopeParams& p, int dtype, cudaStream_t stream) {
  const int64_t tokens = p.token_request != nullptr ? int64_t(p.total_tokens) : int64_t(p.batch) * p.query_len;
  if (tokens <= 0) return cudaSuccess;
  if (tokens > INT32_MAX) return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>(tokens)), block(kWarps * 32);
  switch (dtype) {
    case HYT_DTYPE_BF16: norm_rope_scatter_kernel<__nv_bfloat16><<<grid, block, 0, stream>>>(p); break;
    case HYT_DTYPE_F16: norm_rope_scatter_kernel<__half><<<grid, block, 0, stream>>>(p); break;
    default: norm_rope_scatter_kernel<float><<<grid, block, 0, stream>>>(p); break;
  }
  return cudaGetLastError();
}

}  // namespace hyt
