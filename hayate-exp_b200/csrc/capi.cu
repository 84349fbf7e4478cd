// C ABI of hayate_b200 (declared in include/hayate_b200.h).
//
// Host-side argument checks, TMA tensor maps over the KV pools, workspace
// sizing and the choice between the decode, prefill and CUDA-core kernels.
// Every entry point only enqueues work on the caller's stream.
#include <algorithm>
#include <functional>
#include <mutex>
#include <queue>
#include <vector>
#include <string>

#include "common.cuh"
#include "kernels.cuh"

// Split partials + arrival counters of hyt_decode_attention_noalloc, one copy per
// GPU that loads this library. In host code this name is only a stand-in for the
// symbol: its device address is looked up per device (decode_scratch_address).
static __device__ __align__(256) uint8_t g_decode_scratch[HYT_NOALLOC_SCRATCH_BYTES];

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t err, const char* what) {
  return fail(HYT_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
}

bool is_pow2(int64_t v) { return v > 0 && (v & (v - 1)) == 0; }

int log2_int(int64_t v) {
  int s = 0;
  while ((int64_t(1) << s) < v) ++s;
  return s;
}

int elem_bytes(int dtype) { return dtype == HYT_DTYPE_F32 ? 4 : 2; }

// ------------------------------------------------------------------ tensor maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult status;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status) ==
            cudaSuccess &&
        status == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
  });
  return fn;
}

struct MapKey {
  const void* ptr;
  int dtype, head_dim, box_rows;
  int64_t capacity, planes;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && dtype == o.dtype && head_dim == o.head_dim && box_rows == o.box_rows &&
           capacity == o.capacity && planes == o.planes;
  }
};

struct MapCache {
  static constexpr int kEntries = 32;
  MapKey keys[kEntries];
  CUtensorMap maps[kEntries];
  bool used[kEntries] = {};
  int next = 0;
  std::mutex mu;
};

MapCache& map_cache() {
  static MapCache cache;
  return cache;
}

// Tensor map over a whole pool viewed as [planes = layers * H_kv][capacity][head_dim],
// box = [box_rows tokens x 64 dims], 128-byte swizzle (the layout the kernels index).
int pool_tensor_map(const void* pool, int dtype, int head_dim, int64_t capacity, int64_t planes,
                    int box_rows, CUtensorMap* out) {
  MapKey key{pool, dtype, head_dim, box_rows, capacity, planes};
  MapCache& cache = map_cache();
  std::lock_guard<std::mutex> lock(cache.mu);
  for (int i = 0; i < MapCache::kEntries; ++i) {
    if (cache.used[i] && cache.keys[i] == key) {
      *out = cache.maps[i];
      return HYT_OK;
    }
  }
  EncodeTiledFn encode = encode_fn();
  if (encode == nullptr) return fail(HYT_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (reinterpret_cast<uintptr_t>(pool) % 16)
    return fail(HYT_ERR_INVALID, "KV pool base address must be 16-byte aligned for TMA");
  const int eb = elem_bytes(dtype);
  cuuint64_t dims[3] = {cuuint64_t(head_dim), cuuint64_t(capacity), cuuint64_t(planes)};
  cuuint64_t strides[2] = {cuuint64_t(head_dim) * eb, cuuint64_t(capacity) * head_dim * eb};
  cuuint32_t box[3] = {64, cuuint32_t(box_rows), 1};
  cuuint32_t estrides[3] = {1, 1, 1};
  CUtensorMap map;
  CUresult res = encode(&map,
                        dtype == HYT_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                        3, const_cast<void*>(pool), dims, strides, box, estrides,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS)
    return fail(HYT_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string(int(res)));
  const int slot = cache.next;
  cache.next = (cache.next + 1) % MapCache::kEntries;
  cache.keys[slot] = key;
  cache.maps[slot] = map;
  cache.used[slot] = true;
  *out = map;
  return HYT_OK;
}

// Tensor map over q for the prefill kernel's Q load: dims (head_dim, T, H, B), or
// (head_dim, H, T, B) when the head stride is the smaller one (q viewed from a
// [B, T, H, D] tensor), box [128 rows x 64 dims], 128-byte swizzle: the same shared-memory
// layout as the K tiles. qs = {b, h, t} in elements (b unused when requests == 1).
// Returns false, with nothing recorded as an error, when q cannot be described (the kernel
// then loads Q with plain loads). Cached like the pool maps: the engine's q buffers come
// back at the same addresses layer after layer.
struct QMapKey {
  const void* ptr;
  int dtype, heads;
  int64_t tokens, requests, sb, sh, st;
  bool operator==(const QMapKey& o) const {
    return ptr == o.ptr && dtype == o.dtype && heads == o.heads && tokens == o.tokens &&
           requests == o.requests && sb == o.sb && sh == o.sh && st == o.st;
  }
};

struct QMapCache {
  static constexpr int kEntries = 64;
  QMapKey keys[kEntries];
  CUtensorMap maps[kEntries];
  bool ht[kEntries];
  bool used[kEntries] = {};
  int next = 0;
  std::mutex mu;
};

bool q_tensor_map(const void* q, const int64_t* qs, int dtype, int64_t tokens, int heads,
                  int64_t requests, CUtensorMap* out, bool* ht_out) {
  const int64_t eb = elem_bytes(dtype);
  const int64_t sh = qs[1] * eb, st = qs[2] * eb;
  if (reinterpret_cast<uintptr_t>(q) % 16 || sh <= 0 || st <= 0 || sh % 16 || st % 16 ||
      tokens < 1 || heads < 1 || requests < 1)
    return false;
  int64_t sb = qs[0] * eb;
  if (requests == 1) sb = std::max(sh * heads, st * tokens);  // any valid stride: one request
  if (sb <= 0 || sb % 16) return false;
  const int64_t kMaxStride = int64_t(1) << 40;
  if (sh >= kMaxStride || st >= kMaxStride || sb >= kMaxStride || tokens >= (int64_t(1) << 31) ||
      requests >= (int64_t(1) << 31))
    return false;
  static QMapCache cache;
  const QMapKey key{q, dtype, heads, tokens, requests, sb, sh, st};
  std::lock_guard<std::mutex> lock(cache.mu);
  for (int i = 0; i < QMapCache::kEntries; ++i) {
    if (cache.used[i] && cache.keys[i] == key) {
      *out = cache.maps[i];
      *ht_out = cache.ht[i];
      return true;
    }
  }
  EncodeTiledFn encode = encode_fn();
  if (encode == nullptr) return false;
  const bool ht = sh < st;
  cuuint64_t dims[4] = {128, cuuint64_t(ht ? heads : tokens), cuuint64_t(ht ? tokens : heads),
                        cuuint64_t(requests)};
  cuuint64_t strides[3] = {cuuint64_t(ht ? sh : st), cuuint64_t(ht ? st : sh), cuuint64_t(sb)};
  cuuint32_t box[4] = {64, ht ? 1u : 128u, ht ? 128u : 1u, 1};
  cuuint32_t estrides[4] = {1, 1, 1, 1};
  CUtensorMap map;
  CUresult res = encode(&map,
                        dtype == HYT_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                        4, const_cast<void*>(q), dims, strides, box, estrides,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) return false;
  const int slot = cache.next;
  cache.next = (cache.next + 1) % QMapCache::kEntries;
  cache.keys[slot] = key;
  cache.maps[slot] = map;
  cache.ht[slot] = ht;
  cache.used[slot] = true;
  *out = map;
  *ht_out = ht;
  return true;
}

// ------------------------------------------------------------------ argument checks
struct Geometry {
  int32_t num_layers, layer;
  int64_t capacity;
  int32_t page_table_stride;
  int32_t batch, query_len, num_q_heads, num_kv_heads, head_dim, page_size, dtype;
};

int check_geometry(const Geometry& g) {
  if (g.batch < 1) return fail(HYT_ERR_INVALID, "batch must be positive");
  if (g.query_len < 1) return fail(HYT_ERR_INVALID, "query_len must be positive");
  if (g.num_kv_heads < 1 || g.num_q_heads < 1 || g.num_q_heads % g.num_kv_heads)
    return fail(HYT_ERR_INVALID, "num_q_heads must be a positive multiple of num_kv_heads");
  if (g.head_dim < 1) return fail(HYT_ERR_INVALID, "head_dim must be positive");
  if (!is_pow2(g.page_size)) return fail(HYT_ERR_INVALID, "page_size must be a positive power of two");
  if (g.capacity < g.page_size || g.capacity % g.page_size)
    return fail(HYT_ERR_INVALID, "capacity_tokens must be a positive multiple of page_size");
  if (g.capacity / g.page_size > INT32_MAX) return fail(HYT_ERR_INVALID, "too many pages");
  if (g.num_layers < 1 || g.layer < 0 || g.layer >= g.num_layers)
    return fail(HYT_ERR_INVALID, "layer must be within [0, num_layers)");
  if (g.page_table_stride < 1) return fail(HYT_ERR_INVALID, "page_table_stride must be positive");
  if (g.dtype != HYT_DTYPE_BF16 && g.dtype != HYT_DTYPE_F16 && g.dtype != HYT_DTYPE_F32)
    return fail(HYT_ERR_INVALID, "unknown dtype");
  return HYT_OK;
}

hyt::AttentionParams attention_params(const void* q, const int64_t* qs, const void* k_pool,
                                      const void* v_pool, const Geometry& g,
                                      const int32_t* page_table, const int32_t* cache_lens,
                                      void* out, const int64_t* os, float scale,
                                      int32_t* error_word) {
  hyt::AttentionParams p;
  p.q = q;
  p.q_sb = qs[0];
  p.q_sh = qs[1];
  p.q_st = qs[2];
  p.out = out;
  p.o_sb = os[0];
  p.o_sh = os[1];
  p.o_st = os[2];
  p.k_pool = k_pool;
  p.v_pool = v_pool;
  p.capacity = g.capacity;
  p.num_layers = g.num_layers;
  p.layer = g.layer;
  p.page_table = page_table;
  p.page_table_stride = g.page_table_stride;
  p.cache_lens = cache_lens;
  p.batch = g.batch;
  p.query_len = g.query_len;
  p.num_q_heads = g.num_q_heads;
  p.num_kv_heads = g.num_kv_heads;
  p.head_dim = g.head_dim;
  p.page_shift = log2_int(g.page_size);
  p.num_pages = int32_t(g.capacity / g.page_size);
  p.scale = scale;
  p.error_word = error_word;
  p.q_start = nullptr;
  p.q_len = nullptr;
  p.req_ids = nullptr;
  p.num_listed = 0;
  p.total_tokens = 0;
  return p;
}

// Per-request addressing of a packed batch, and the request list one launch serves.
struct PackedArgs {
  const int32_t* q_start;
  const int32_t* q_len;
  const int32_t* req_ids;
  int32_t num_listed;
  int32_t total_tokens;
};

void apply_packed(hyt::AttentionParams& p, const PackedArgs* pk) {
  if (pk == nullptr) return;
  p.q_start = pk->q_start;
  p.q_len = pk->q_len;
  p.req_ids = pk->req_ids;
  p.num_listed = pk->num_listed;
  p.total_tokens = pk->total_tokens;
}

int check_attention_pointers(const void* q, const int64_t* qs, const void* k_pool,
                             const void* v_pool, const int32_t* page_table,
                             const int32_t* cache_lens, const void* out, const int64_t* os) {
  if (!q || !qs || !k_pool || !v_pool || !page_table || !cache_lens || !out || !os)
    return fail(HYT_ERR_INVALID, "null pointer argument");
  return HYT_OK;
}

// ------------------------------------------------------------------ decode sizing
constexpr int64_t kB200Slots = 148 * 2;  // resident decode CTAs on one B200

bool decode_eligible(const Geometry& g) {
  return (g.dtype == HYT_DTYPE_BF16 || g.dtype == HYT_DTYPE_F16) && g.head_dim == 128 &&
         g.page_size % 64 == 0 &&
         (g.num_q_heads / g.num_kv_heads) * g.query_len <= hyt::kDecodeMaxRows;
}

int32_t decode_split_tokens(int32_t batch, int32_t num_kv_heads, int32_t max_kv_len,
                            int32_t requested) {
  const int64_t tiles_per_seq = (int64_t(max_kv_len) + 63) / 64;
  int64_t split_tiles;
  if (requested > 0) {
    split_tiles = (int64_t(requested) + 63) / 64;
  } else {
    const int64_t total = int64_t(batch) * num_kv_heads * tiles_per_seq;
    const int64_t target = 7 * kB200Slots;  // ~7 waves: measured best on the config-2 sweep
    split_tiles = (total + target - 1) / target;
    if (split_tiles < 8) split_tiles = 8;
  }
  if (split_tiles > tiles_per_seq) split_tiles = tiles_per_seq;
  if (split_tiles < 1) split_tiles = 1;
  return int32_t(split_tiles * 64);
}

struct DecodeLayout {
  int32_t split_tokens, max_splits, rows;
  size_t counter_bytes, ml_bytes, o_bytes, total;
};

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

DecodeLayout decode_layout(int32_t batch, int32_t query_len, int32_t num_q_heads,
                           int32_t num_kv_heads, int32_t max_kv_len, int32_t split_tokens) {
  DecodeLayout L;
  L.split_tokens = decode_split_tokens(batch, num_kv_heads, max_kv_len, split_tokens);
  L.max_splits = int32_t((int64_t(max_kv_len) + L.split_tokens - 1) / L.split_tokens);
  L.rows = (num_q_heads / num_kv_heads) * query_len;
  const size_t units = size_t(batch) * num_kv_heads;
  if (L.max_splits <= 1) {
    L.counter_bytes = L.ml_bytes = L.o_bytes = L.total = 0;
    return L;
  }
  L.counter_bytes = align256(units * sizeof(int32_t));
  L.ml_bytes = align256(units * L.max_splits * L.rows * 2 * sizeof(float));
  L.o_bytes = units * L.max_splits * L.rows * 128 * sizeof(float);
  L.total = L.counter_bytes + L.ml_bytes + L.o_bytes;
  return L;
}

// The step's new K/V rows for a decode launch that writes them itself (fused scatter).
struct FusedScatter {
  const void* k_new;
  const void* v_new;
  const int64_t* strides;  // {k_b, k_h, k_t, v_b, v_h, v_t} in elements
};

int launch_decode(const void* q, const int64_t* qs, const void* k_pool, const void* v_pool,
                  const Geometry& g, const int32_t* page_table, const int32_t* cache_lens,
                  void* out, const int64_t* os, float scale, int32_t max_kv_len,
                  int32_t split_tokens, void* workspace, size_t workspace_bytes,
                  int32_t* error_word, cudaStream_t stream, const PackedArgs* pk = nullptr,
                  const FusedScatter* fs = nullptr) {
  if (max_kv_len < g.query_len) return fail(HYT_ERR_INVALID, "max_kv_len must be >= query_len");
  if (split_tokens < 0) return fail(HYT_ERR_INVALID, "split_tokens must be >= 0");
  const int32_t count = pk != nullptr && pk->req_ids != nullptr ? pk->num_listed : g.batch;
  const DecodeLayout L = decode_layout(count, g.query_len, g.num_q_heads, g.num_kv_heads,
                                       max_kv_len, split_tokens);
  if (L.max_splits > 65535) return fail(HYT_ERR_UNSUPPORTED, "too many splits for one launch");
  if (count > 65535 || g.num_kv_heads > 65535) return fail(HYT_ERR_UNSUPPORTED, "batch too large");
  if (L.total > 0 && (workspace == nullptr || workspace_bytes < L.total || reinterpret_cast<uintptr_t>(workspace) % 16))
    return fail(HYT_ERR_WORKSPACE,
                "workspace missing, not 16-byte aligned or smaller than hyt_attention_workspace_bytes()");
  CUtensorMap k_map, v_map;
  const int64_t planes = int64_t(g.num_layers) * g.num_kv_heads;
  int rc = pool_tensor_map(k_pool, g.dtype, g.head_dim, g.capacity, planes, 64, &k_map);
  if (rc != HYT_OK) return rc;
  rc = pool_tensor_map(v_pool, g.dtype, g.head_dim, g.capacity, planes, 64, &v_map);
  if (rc != HYT_OK) return rc;
  hyt::AttentionParams p = attention_params(q, qs, k_pool, v_pool, g, page_table, cache_lens,
                                            out, os, scale, error_word);
  apply_packed(p, pk);
  hyt::DecodeLaunch d;
  d.split_tokens = L.split_tokens;
  d.max_splits = L.max_splits;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  d.ws_counter = L.total ? reinterpret_cast<int32_t*>(ws) : nullptr;
  d.ws_ml = L.total ? reinterpret_cast<float*>(ws + L.counter_bytes) : nullptr;
  d.ws_o = L.total ? reinterpret_cast<float*>(ws + L.counter_bytes + L.ml_bytes) : nullptr;
  d.k_new = fs != nullptr ? static_cast<const uint8_t*>(fs->k_new) : nullptr;
  d.v_new = fs != nullptr ? static_cast<const uint8_t*>(fs->v_new) : nullptr;
  d.k_sb = fs != nullptr ? fs->strides[0] : 0;
  d.k_sh = fs != nullptr ? fs->strides[1] : 0;
  d.k_st = fs != nullptr ? fs->strides[2] : 0;
  d.v_sb = fs != nullptr ? fs->strides[3] : 0;
  d.v_sh = fs != nullptr ? fs->strides[4] : 0;
  d.v_st = fs != nullptr ? fs->strides[5] : 0;
  d.k_pool = static_cast<uint8_t*>(const_cast<void*>(k_pool));
  d.v_pool = static_cast<uint8_t*>(const_cast<void*>(v_pool));
  cudaError_t err = hyt::run_decode_attention(p, d, k_map, v_map, g.dtype, stream);
  if (err != cudaSuccess) return cuda_fail(err, "decode attention launch");
  return HYT_OK;
}

bool rows_16b_aligned(const void* ptr, const int64_t* strides) {
  if (reinterpret_cast<uintptr_t>(ptr) % 16) return false;
  for (int i = 0; i < 3; ++i)
    if (strides[i] % 8) return false;  // 8 elements of 2 bytes
  return true;
}

bool prefill_eligible(const Geometry& g, const void* q, const int64_t* qs, const void* out,
                      const int64_t* os) {
  // the kernel pairs two query heads of one KV group per CTA
  return (g.dtype == HYT_DTYPE_BF16 || g.dtype == HYT_DTYPE_F16) && g.head_dim == 128 &&
         g.page_size % 128 == 0 && (g.num_q_heads / g.num_kv_heads) % 2 == 0 &&
         rows_16b_aligned(q, qs) && rows_16b_aligned(out, os);
}

int launch_prefill(const void* q, const int64_t* qs, const void* k_pool, const void* v_pool,
                   const Geometry& g, const int32_t* page_table, const int32_t* cache_lens,
                   void* out, const int64_t* os, float scale, int32_t* error_word,
                   cudaStream_t stream, const PackedArgs* pk = nullptr,
                   const hyt::PrefillPlan* plan = nullptr) {
  const int32_t count = pk != nullptr && pk->req_ids != nullptr ? pk->num_listed : g.batch;
  if (count > 65535 || g.num_q_heads > 65535) return fail(HYT_ERR_UNSUPPORTED, "batch too large");
  CUtensorMap k_map, v_map;
  const int64_t planes = int64_t(g.num_layers) * g.num_kv_heads;
  int rc = pool_tensor_map(k_pool, g.dtype, g.head_dim, g.capacity, planes, 128, &k_map);
  if (rc != HYT_OK) return rc;
  rc = pool_tensor_map(v_pool, g.dtype, g.head_dim, g.capacity, planes, 128, &v_map);
  if (rc != HYT_OK) return rc;
  hyt::AttentionParams p = attention_params(q, qs, k_pool, v_pool, g, page_table, cache_lens,
                                            out, os, scale, error_word);
  apply_packed(p, pk);
  CUtensorMap q_map;
  bool q_ht = false;
  const bool packed = pk != nullptr;
  const bool q_tma = q_tensor_map(q, qs, g.dtype, packed ? pk->total_tokens : g.query_len,
                                  g.num_q_heads, packed ? 1 : g.batch, &q_map, &q_ht);
  cudaError_t err = hyt::run_prefill_attention(p, k_map, v_map, q_tma ? &q_map : nullptr, q_ht,
                                               g.dtype, stream, plan);
  if (err != cudaSuccess) return cuda_fail(err, "prefill attention launch");
  return HYT_OK;
}

int launch_generic(const void* q, const int64_t* qs, const void* k_pool, const void* v_pool,
                   const Geometry& g, const int32_t* page_table, const int32_t* cache_lens,
                   void* out, const int64_t* os, float scale, int32_t* error_word,
                   cudaStream_t stream, const PackedArgs* pk = nullptr) {
  if (g.head_dim % 8 || g.head_dim > 256)
    return fail(HYT_ERR_UNSUPPORTED, "head_dim must be a multiple of 8 and at most 256");
  hyt::AttentionParams p = attention_params(q, qs, k_pool, v_pool, g, page_table, cache_lens,
                                            out, os, scale, error_word);
  apply_packed(p, pk);
  cudaError_t err = hyt::run_generic_attention(p, g.dtype, stream);
  if (err != cudaSuccess) return cuda_fail(err, "generic attention launch");
  return HYT_OK;
}

// ------------------------------------------------------------------ prefill schedule
// Cost model of one prefill work item, in key tiles (~2 us each on a B200): the tiles it
// streams plus a fixed start-up/epilogue cost; a half of a split item pays the start-up
// again plus the merge (its partial out to the workspace, both read back by the second
// half). The two constants are fitted to B200 timings of the default grid, longest-first
// orders and split plans on four prefix sets (config 3, two random U[0, 4096] sets and
// U[0, 32768]); a plan is used only when the model predicts it at least kMinGain faster.
constexpr double kItemOverhead = 5.0, kMergeCost = 8.0, kMinGain = 0.03;  // defaults
constexpr int kMaxPlannedItemsPerSm = 24;  // beyond this many items per SM: the default grid

struct PlanEntry {
  int32_t z, q_tile, pair, k_lo, k_hi, split;  // split: slot * 2 + part, or -1
  double cost;
};

// Longest time any of `sms` SMs is busy when the items start in `order` on whichever SM
// frees first (the block scheduler's greedy order, one CTA per SM).
double greedy_makespan(const std::vector<double>& costs, int sms) {
  std::priority_queue<double, std::vector<double>, std::greater<double>> free_at;
  for (int i = 0; i < sms; ++i) free_at.push(0.0);
  double end = 0.0;
  for (double c : costs) {
    const double t = free_at.top() + c;
    free_at.pop();
    free_at.push(t);
    end = std::max(end, t);
  }
  return end;
}

// Items of the default grid, in its launch order (request, head pair, query tile from the
// last), with their key-tile counts; false when a count does not fit the item encoding.
bool prefill_items(const int32_t* cache_lens, const int32_t* q_lens, int32_t batch,
                   int32_t query_len, int32_t pairs, double overhead, std::vector<PlanEntry>* items) {
  for (int32_t z = 0; z < batch; ++z) {
    const int64_t ql = q_lens != nullptr ? q_lens[z] : query_len;
    if (ql <= 0 || cache_lens[z] < 0) continue;
    const int32_t tiles = int32_t((ql + 127) / 128);
    for (int32_t pair = 0; pair < pairs; ++pair)
      for (int32_t qt = tiles - 1; qt >= 0; --qt) {
        const int64_t t_last = std::min<int64_t>(int64_t(qt) * 128 + 127, ql - 1);
        const int64_t n = (int64_t(cache_lens[z]) + t_last) / 128 + 1;
        if (n > 0xFFFF || qt > 0xFFFF || pair > 0xFFFF) return false;
        items->push_back({z, qt, pair, 0, int32_t(n), -1, double(n) + overhead});
      }
  }
  return true;
}

// Split workspace of a plan: [counters (int32 per slot, 256-byte padded) | (max, sum) per
// slot, half, head and row | partial O per slot, half, head, 16-byte column chunk and row].
size_t split_counter_bytes(int32_t num_splits) { return (size_t(num_splits) * 4 + 255) / 256 * 256; }

hyt::PrefillPlan make_prefill_plan(const int32_t* items, int32_t num_items, int32_t num_splits,
                                   void* workspace) {
  hyt::PrefillPlan plan{nullptr, 0, 0, nullptr, nullptr, nullptr};
  if (num_items <= 0) return plan;
  plan.items = reinterpret_cast<const hyt::PrefillItem*>(items);
  plan.num_items = num_items;
  plan.num_splits = num_splits;
  if (num_splits > 0) {
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const size_t cb = split_counter_bytes(num_splits), ml_bytes = size_t(num_splits) * 2 * 2 * 128 * 2 * 4;
    plan.ws_counter = reinterpret_cast<int32_t*>(ws);
    plan.ws_ml = reinterpret_cast<float*>(ws + cb);
    plan.ws_o = reinterpret_cast<float*>(ws + cb + ml_bytes);
  }
  return plan;
}

// ------------------------------------------------------------------ static decode scratch
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_decode_scratch on the current device. Looked up afresh on every
// call made outside stream capture (cheap), so a context re-created after
// cudaDeviceReset gets its own address; a call made while `stream` is being captured
// uses the address the last uncaptured call on this device found (and fails if there
// was none).
int decode_scratch_address(cudaStream_t stream, void** out) {
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
  if (device < 0 || device >= kMaxDevices) return fail(HYT_ERR_UNSUPPORTED, "device index too large");
  cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
  err = cudaStreamIsCapturing(stream, &status);
  if (err != cudaSuccess) return cuda_fail(err, "cudaStreamIsCapturing");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (status == cudaStreamCaptureStatusNone) {
    void* addr = nullptr;
    err = cudaGetSymbolAddress(&addr, g_decode_scratch);
    if (err != cudaSuccess) return cuda_fail(err, "cudaGetSymbolAddress(decode scratch)");
    g_scratch_addr[device] = addr;
  } else if (g_scratch_addr[device] == nullptr) {
    return fail(HYT_ERR_INVALID,
                "hyt_decode_attention_noalloc: the first call on a device must come before any "
                "stream capture (it looks the static scratch's address up)");
  }
  *out = g_scratch_addr[device];
  return HYT_OK;
}

// The fused norm/RoPE/scatter kernels move 16 bytes per lane (8 features of a 16-bit row, 4
// of an fp32 one) between global memory and registers or shared memory: every row they
// read or write must start on a 16-byte boundary.
int check_norm_rope_alignment(int dtype, const void* q, const void* k, const void* v, const void* q_out,
                              const int64_t* qkv_strides, int n_qkv, const int64_t* q_out_strides,
                              int n_out, const void* q_norm_weight, const void* k_norm_weight,
                              const void* k_pool, const void* v_pool, const float* cos, const float* sin) {
  const int per16 = 16 / elem_bytes(dtype);  // elements in 16 bytes
  const void* ptrs[8] = {q, k, v, q_out, q_norm_weight, k_norm_weight, k_pool, v_pool};
  for (const void* ptr : ptrs)
    if (reinterpret_cast<uintptr_t>(ptr) % 16)
      return fail(HYT_ERR_INVALID, "q/k/v/q_out, the norm weights and the pools must be 16-byte aligned");
  for (int i = 0; i < n_qkv; ++i)
    if (qkv_strides[i] % per16) return fail(HYT_ERR_INVALID, "q/k/v strides must be multiples of 16 bytes");
  for (int i = 0; i < n_out; ++i)
    if (q_out_strides[i] % per16) return fail(HYT_ERR_INVALID, "q_out strides must be multiples of 16 bytes");
  if (reinterpret_cast<uintptr_t>(cos) % 16 || reinterpret_cast<uintptr_t>(sin) % 16)
    return fail(HYT_ERR_INVALID, "cos/sin tables must be 16-byte aligned");
  return HYT_OK;
}

}  // namespace

extern "C" {

const char* hyt_last_error(void) { return g_last_error.c_str(); }

int hyt_version(void) { return 100; }

int hyt_kv_scatter(const void* k_new, const void* v_new, const int64_t* new_strides,
                   void* k_pool, void* v_pool, int32_t num_layers, int32_t layer,
                   int64_t capacity_tokens, const int32_t* page_table,
                   int32_t page_table_stride, const int32_t* cache_lens, int32_t batch,
                   int32_t query_len, int32_t num_kv_heads, int32_t head_dim,
                   int32_t page_size, int32_t dtype, int32_t* error_word, void* stream) {
  g_last_error.clear();
  if (!k_new || !v_new || !new_strides || !k_pool || !v_pool || !page_table || !cache_lens)
    return fail(HYT_ERR_INVALID, "null pointer argument");
  Geometry g{num_layers, layer, capacity_tokens, page_table_stride, batch, query_len,
             num_kv_heads, num_kv_heads, head_dim, page_size, dtype};
  int rc = check_geometry(g);
  if (rc != HYT_OK) return rc;
  hyt::ScatterParams p;
  p.k_new = static_cast<const uint8_t*>(k_new);
  p.v_new = static_cast<const uint8_t*>(v_new);
  p.k_sb = new_strides[0];
  p.k_sh = new_strides[1];
  p.k_st = new_strides[2];
  p.v_sb = new_strides[3];
  p.v_sh = new_strides[4];
  p.v_st = new_strides[5];
  p.k_pool = static_cast<uint8_t*>(k_pool);
  p.v_pool = static_cast<uint8_t*>(v_pool);
  p.layer_offset = int64_t(layer) * num_kv_heads * capacity_tokens * head_dim;
  p.capacity = capacity_tokens;
  p.page_table = page_table;
  p.page_table_stride = page_table_stride;
  p.cache_lens = cache_lens;
  p.batch = batch;
  p.query_len = query_len;
  p.heads = num_kv_heads;
  p.head_dim = head_dim;
  p.page_shift = log2_int(page_size);
  p.num_pages = int32_t(capacity_tokens / page_size);
  p.error_word = error_word;
  p.q_start = nullptr;
  p.token_request = nullptr;
  p.total_tokens = 0;
  cudaError_t err = hyt::run_kv_scatter(p, elem_bytes(dtype), static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "kv scatter launch");
  return HYT_OK;
}

int hyt_norm_rope_scatter(const void* q, const void* k, const void* v, const int64_t* qkv_strides,
                          const void* q_norm_weight, const void* k_norm_weight, float eps,
                          const float* cos, const float* sin, int32_t rope_positions,
                          void* q_out, const int64_t* q_out_strides, void* k_pool, void* v_pool,
                          int32_t num_layers, int32_t layer, int64_t capacity_tokens,
                          const int32_t* page_table, int32_t page_table_stride,
                          const int32_t* cache_lens, int32_t batch, int32_t query_len,
                          int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                          int32_t page_size, int32_t dtype, int32_t* error_word, void* stream) {
  g_last_error.clear();
  if (!q || !k || !v || !qkv_strides || !q_norm_weight || !k_norm_weight || !cos || !sin ||
      !q_out || !q_out_strides || !k_pool || !v_pool || !page_table || !cache_lens)
    return fail(HYT_ERR_INVALID, "null pointer argument");
  Geometry g{num_layers, layer, capacity_tokens, page_table_stride, batch, query_len,
             num_q_heads, num_kv_heads, head_dim, page_size, dtype};
  int rc = check_geometry(g);
  if (rc != HYT_OK) return rc;
  if (head_dim != 128) return fail(HYT_ERR_UNSUPPORTED, "fused norm/RoPE/scatter needs head_dim 128");
  if (rope_positions < 1) return fail(HYT_ERR_INVALID, "rope_positions must be positive");
  rc = check_norm_rope_alignment(dtype, q, k, v, q_out, qkv_strides, 9, q_out_strides, 3,
                                 q_norm_weight, k_norm_weight, k_pool, v_pool, cos, sin);
  if (rc != HYT_OK) return rc;
  hyt::NormRopeParams p;
  p.q = q;
  p.q_sb = qkv_strides[0]; p.q_st = qkv_strides[1]; p.q_sh = qkv_strides[2];
  p.k = k;
  p.k_sb = qkv_strides[3]; p.k_st = qkv_strides[4]; p.k_sh = qkv_strides[5];
  p.v = v;
  p.v_sb = qkv_strides[6]; p.v_st = qkv_strides[7]; p.v_sh = qkv_strides[8];
  p.q_out = q_out;
  p.o_sb = q_out_strides[0]; p.o_sh = q_out_strides[1]; p.o_st = q_out_strides[2];
  p.q_norm_weight = q_norm_weight;
  p.k_norm_weight = k_norm_weight;
  p.eps = eps;
  p.cos = cos;
  p.sin = sin;
  p.rope_positions = rope_positions;
  p.k_pool = k_pool;
  p.v_pool = v_pool;
  p.capacity = capacity_tokens;
  p.layer = layer;
  p.page_table = page_table;
  p.page_table_stride = page_table_stride;
  p.cache_lens = cache_lens;
  p.batch = batch;
  p.query_len = query_len;
  p.num_q_heads = num_q_heads;
  p.num_kv_heads = num_kv_heads;
  p.page_shift = log2_int(page_size);
  p.num_pages = int32_t(capacity_tokens / page_size);
  p.error_word = error_word;
  p.q_start = nullptr;
  p.token_request = nullptr;
  p.total_tokens = 0;
  cudaError_t err = hyt::run_norm_rope_scatter(p, dtype, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "norm/RoPE/scatter launch");
  return HYT_OK;
}

int hyt_generic_attention(const void* q, const int64_t* q_strides, const void* k_pool,
                          const void* v_pool, int32_t num_layers, int32_t layer,
                          int64_t capacity_tokens, const int32_t* page_table,
                          int32_t page_table_stride, const int32_t* cache_lens, void* out,
                          const int64_t* out_strides, int32_t batch, int32_t query_len,
                          int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                          int32_t page_size, int32_t dtype, float scale,
                          int32_t* error_word, void* stream) {
  g_last_error.clear();
  int rc = check_attention_pointers(q, q_strides, k_pool, v_pool, page_table, cache_lens, out,
                                    out_strides);
  if (rc != HYT_OK) return rc;
  Geometry g{num_layers, layer, capacity_tokens, page_table_stride, batch, query_len,
             num_q_heads, num_kv_heads, head_dim, page_size, dtype};
  rc = check_geometry(g);
  if (rc != HYT_OK) return rc;
  return launch_generic(q, q_strides, k_pool, v_pool, g, page_table, cache_lens, out,
                        out_strides, scale, error_word, static_cast<cudaStream_t>(stream));
}

int hyt_decode_attention(const void* q, const int64_t* q_strides, const void* k_pool,
                         const void* v_pool, int32_t num_layers, int32_t layer,
                         int64_t capacity_tokens, const int32_t* page_table,
                         int32_t page_table_stride, const int32_t* cache_lens, void* out,
                         const int64_t* out_strides, int32_t batch, int32_t query_len,
                         int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                         int32_t page_size, int32_t dtype, float scale, int32_t max_kv_len,
                         int32_t split_tokens, void* workspace, size_t workspace_bytes,
                         int32_t* error_word, void* stream) {
  g_last_error.clear();
  int rc = check_attention_pointers(q, q_strides, k_pool, v_pool, page_table, cache_lens, out,
                                    out_strides);
  if (rc != HYT_OK) return rc;
  Geometry g{num_layers, layer, capacity_tokens, page_table_stride, batch, query_len,
             num_q_heads, num_kv_heads, head_dim, page_size, dtype};
  rc = check_geometry(g);
  if (rc != HYT_OK) return rc;
  if (!decode_eligible(g))
    return fail(HYT_ERR_UNSUPPORTED,
                "decode kernel needs bf16/f16, head_dim 128, page_size % 64 == 0 and "
                "group * query_len <= 16");
  return launch_decode(q, q_strides, k_pool, v_pool, g, page_table, cache_lens, out,
                       out_strides, scale, max_kv_len, split_tokens, workspace, workspace_bytes,
                       error_word, static_cast<cudaStream_t>(stream));
}

int hyt_decode_attention_noalloc(const void* q, const int64_t* q_strides, const void* k_pool,
                                 const void* v_pool, int32_t num_layers, int32_t layer,
                                 int64_t capacity_tokens, const int32_t* page_table,
                                 int32_t page_table_stride, const int32_t* cache_lens, void* out,
                                 const int64_t* out_strides, int32_t batch, int32_t query_len,
                                 int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                 int32_t page_size, int32_t dtype, float scale,
                                 int32_t max_kv_len, int32_t split_tokens, int32_t* error_word,
                                 void* stream) {
  g_last_error.clear();
  int rc = check_attention_pointers(q, q_strides, k_pool, v_pool, page_table, cache_lens, out,
                                    out_strides);
  if (rc != HYT_OK) return rc;
  Geometry g{num_layers, layer, capacity_tokens, page_table_stride, batch, query_len,
             num_q_heads, num_kv_heads, head_dim, page_size, dtype};
  rc = check_geometry(g);
  if (rc != HYT_OK) return rc;
  if (!decode_eligible(g))
    return fail(HYT_ERR_UNSUPPORTED,
                "decode kernel needs bf16/f16, head_dim 128, page_size % 64 == 0 and "
                "group * query_len <= 16");
  if (max_kv_len < query_len) return fail(HYT_ERR_INVALID, "max_kv_len must be >= query_len");
  if (split_tokens < 0) return fail(HYT_ERR_INVALID, "split_tokens must be >= 0");
  const DecodeLayout L = decode_layout(batch, query_len, num_q_heads, num_kv_heads, max_kv_len,
                                       split_tokens);
  if (L.total > size_t(HYT_NOALLOC_SCRATCH_BYTES))
    return fail(HYT_ERR_WORKSPACE,
                "decode scratch of " + std::to_string(L.total) + " bytes exceeds the static " +
                    std::to_string(HYT_NOALLOC_SCRATCH_BYTES) +
                    "-byte buffer; pass a larger split_tokens or use hyt_decode_attention");
  void* scratch = nullptr;
  rc = decode_scratch_address(static_cast<cudaStream_t>(stream), &scratch);
  if (rc != HYT_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (L.total > 0) {
    // the array keeps the previous call's bytes: the counters must start at zero
    cudaError_t err = cudaMemsetAsync(scratch, 0, L.counter_bytes, s);
    if (err != cudaSuccess) return cuda_fail(err, "clearing the decode scratch counters");
  }
  return launch_decode(q, q_strides, k_pool, v_pool, g, page_table, cache_lens, out, out_strides,
                       scale, max_kv_len, split_tokens, scratch, HYT_NOALLOC_SCRATCH_BYTES,
                       error_word, s);
}

int hyt_prefill_attention(const void* q, const int64_t* q_strides, const void* k_pool,
                          const void* v_pool, int32_t num_layers, int32_t layer,
                          int64_t capacity_tokens, const int32_t* page_table,
                          int32_t page_table_stride, const int32_t* cache_lens, void* out,
                          const int64_t* out_strides, int32_t batch, int32_t query_len,
                          int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                          int32_t page_size, int32_t dtype, float scale, int32_t max_kv_len,
                          int32_t* error_word, void* stream) {
  g_last_error.clear();
  (void)max_kv_len;  // the prefill grid is sized by query_len, not by the longest request
  int rc = check_attention_pointers(q, q_strides, k_pool, v_pool, page_table, cache_lens, out,
                                    out_strides);
  if (rc != HYT_OK) return rc;
  Geometry g{num_layers, layer, capacity_tokens, page_table_stride, batch, query_len,
             num_q_heads, num_kv_heads, head_dim, page_size, dtype};
  rc = check_geometry(g);
  if (rc != HYT_OK) return rc;
  if (!prefill_eligible(g, q, q_strides, out, out_strides))
    return fail(HYT_ERR_UNSUPPORTED,
                "prefill kernel needs bf16/f16, head_dim 128, page_size % 128 == 0, an even "
                "query-head group and 16-byte aligned q/out rows");
  return launch_prefill(q, q_strides, k_pool, v_pool, g, page_table, cache_lens, out,
                        out_strides, scale, error_word, static_cast<cudaStream_t>(stream));
}

int hyt_paged_attention(const void* q, const int64_t* q_strides, const void* k_pool,
                        const void* v_pool, int32_t num_layers, int32_t layer,
                        int64_t capacity_tokens, const int32_t* page_table,
                        int32_t page_table_stride, const int32_t* cache_lens, void* out,
                        const int64_t* out_strides, int32_t batch, int32_t query_len,
                        int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                        int32_t page_size, int32_t dtype, float scale, int32_t max_kv_len,
                        int32_t split_tokens, void* workspace, size_t workspace_bytes,
                        int32_t* error_word, void* stream) {
  g_last_error.clear();
  int rc = check_attention_pointers(q, q_strides, k_pool, v_pool, page_table, cache_lens, out,
                                    out_strides);
  if (rc != HYT_OK) return rc;
  Geometry g{num_layers, layer, capacity_tokens, page_table_stride, batch, query_len,
             num_q_heads, num_kv_heads, head_dim, page_size, dtype};
  rc = check_geometry(g);
  if (rc != HYT_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (decode_eligible(g))
    return launch_decode(q, q_strides, k_pool, v_pool, g, page_table, cache_lens, out,
                         out_strides, scale, max_kv_len, split_tokens, workspace,
                         workspace_bytes, error_word, s);
  if (prefill_eligible(g, q, q_strides, out, out_strides))
    return launch_prefill(q, q_strides, k_pool, v_pool, g, page_table, cache_lens, out,
                          out_strides, scale, error_word, s);
  return launch_generic(q, q_strides, k_pool, v_pool, g, page_table, cache_lens, out,
                        out_strides, scale, error_word, s);
}

int hyt_paged_attention_scatter(const void* q, const int64_t* q_strides, const void* k_new,
                                const void* v_new, const int64_t* new_strides, void* k_pool,
                                void* v_pool, int32_t num_layers, int32_t layer,
                                int64_t capacity_tokens, const int32_t* page_table,
                                int32_t page_table_stride, const int32_t* cache_lens, void* out,
                                const int64_t* out_strides, int32_t batch, int32_t query_len,
                                int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                int32_t page_size, int32_t dtype, float scale, int32_t max_kv_len,
                                int32_t split_tokens, void* workspace, size_t workspace_bytes,
                                int32_t* error_word, void* stream) {
  g_last_error.clear();
  int rc = check_attention_pointers(q, q_strides, k_pool, v_pool, page_table, cache_lens, out,
                                    out_strides);
  if (rc != HYT_OK) return rc;
  if (!k_new || !v_new || !new_strides) return fail(HYT_ERR_INVALID, "null pointer argument");
  Geometry g{num_layers, layer, capacity_tokens, page_table_stride, batch, query_len,
             num_q_heads, num_kv_heads, head_dim, page_size, dtype};
  rc = check_geometry(g);
  if (rc != HYT_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // one launch when the decode kernel serves the step and every new row is 16-byte aligned
  bool rows16 = reinterpret_cast<uintptr_t>(k_new) % 16 == 0 && reinterpret_cast<uintptr_t>(v_new) % 16 == 0;
  for (int i = 0; i < 6; ++i) rows16 = rows16 && (new_strides[i] * elem_bytes(dtype)) % 16 == 0;
  if (decode_eligible(g) && rows16) {
    const FusedScatter fs{k_new, v_new, new_strides};
    return launch_decode(q, q_strides, k_pool, v_pool, g, page_table, cache_lens, out,
                         out_strides, scale, max_kv_len, split_tokens, workspace,
                         workspace_bytes, error_word, s, nullptr, &fs);
  }
  rc = hyt_kv_scatter(k_new, v_new, new_strides, k_pool, v_pool, num_layers, layer,
                      capacity_tokens, page_table, page_table_stride, cache_lens, batch, query_len,
                      num_kv_heads, head_dim, page_size, dtype, error_word, stream);
  if (rc != HYT_OK) return rc;
  return hyt_paged_attention(q, q_strides, k_pool, v_pool, num_layers, layer, capacity_tokens,
                             page_table, page_table_stride, cache_lens, out, out_strides, batch,
                             query_len, num_q_heads, num_kv_heads, head_dim, page_size, dtype,
                             scale, max_kv_len, split_tokens, workspace, workspace_bytes,
                             error_word, stream);
}

int hyt_kv_scatter_packed(const void* k_new, const void* v_new, const int64_t* new_strides,
                          void* k_pool, void* v_pool, int32_t num_layers, int32_t layer,
                          int64_t capacity_tokens, const int32_t* page_table,
                          int32_t page_table_stride, const int32_t* cache_lens,
                          const int32_t* q_start, const int32_t* token_request, int32_t batch,
                          int32_t total_tokens, int32_t num_kv_heads, int32_t head_dim,
                          int32_t page_size, int32_t dtype, int32_t* error_word, void* stream) {
  g_last_error.clear();
  if (!k_new || !v_new || !new_strides || !k_pool || !v_pool || !page_table || !cache_lens ||
      !q_start || !token_request)
    return fail(HYT_ERR_INVALID, "null pointer argument");
  if (total_tokens < 1) return fail(HYT_ERR_INVALID, "total_tokens must be positive");
  Geometry g{num_layers, layer, capacity_tokens, page_table_stride, batch, 1,
             num_kv_heads, num_kv_heads, head_dim, page_size, dtype};
  int rc = check_geometry(g);
  if (rc != HYT_OK) return rc;
  hyt::ScatterParams p;
  p.k_new = static_cast<const uint8_t*>(k_new);
  p.v_new = static_cast<const uint8_t*>(v_new);
  p.k_sb = 0;
  p.k_st = new_strides[0];
  p.k_sh = new_strides[1];
  p.v_sb = 0;
  p.v_st = new_strides[2];
  p.v_sh = new_strides[3];
  p.k_pool = static_cast<uint8_t*>(k_pool);
  p.v_pool = static_cast<uint8_t*>(v_pool);
  p.layer_offset = int64_t(layer) * num_kv_heads * capacity_tokens * head_dim;
  p.capacity = capacity_tokens;
  p.page_table = page_table;
  p.page_table_stride = page_table_stride;
  p.cache_lens = cache_lens;
  p.batch = batch;
  p.query_len = 1;
  p.heads = num_kv_heads;
  p.head_dim = head_dim;
  p.page_shift = log2_int(page_size);
  p.num_pages = int32_t(capacity_tokens / page_size);
  p.error_word = error_word;
  p.q_start = q_start;
  p.token_request = token_request;
  p.total_tokens = total_tokens;
  cudaError_t err = hyt::run_kv_scatter(p, elem_bytes(dtype), static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "packed kv scatter launch");
  return HYT_OK;
}

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
                                 int32_t* error_word, void* stream) {
  g_last_error.clear();
  if (!q || !k || !v || !qkv_strides || !q_norm_weight || !k_norm_weight || !cos || !sin ||
      !q_out || !q_out_strides || !k_pool || !v_pool || !page_table || !cache_lens || !q_start ||
      !token_request)
    return fail(HYT_ERR_INVALID, "null pointer argument");
  if (total_tokens < 1) return fail(HYT_ERR_INVALID, "total_tokens must be positive");
  Geometry g{num_layers, layer, capacity_tokens, page_table_stride, batch, 1,
             num_q_heads, num_kv_heads, head_dim, page_size, dtype};
  int rc = check_geometry(g);
  if (rc != HYT_OK) return rc;
  if (head_dim != 128) return fail(HYT_ERR_UNSUPPORTED, "fused norm/RoPE/scatter needs head_dim 128");
  if (rope_positions < 1) return fail(HYT_ERR_INVALID, "rope_positions must be positive");
  rc = check_norm_rope_alignment(dtype, q, k, v, q_out, qkv_strides, 6, q_out_strides, 2,
                                 q_norm_weight, k_norm_weight, k_pool, v_pool, cos, sin);
  if (rc != HYT_OK) return rc;
  hyt::NormRopeParams p;
  p.q = q;
  p.q_sb = 0; p.q_st = qkv_strides[0]; p.q_sh = qkv_strides[1];
  p.k = k;
  p.k_sb = 0; p.k_st = qkv_strides[2]; p.k_sh = qkv_strides[3];
  p.v = v;
  p.v_sb = 0; p.v_st = qkv_strides[4]; p.v_sh = qkv_strides[5];
  p.q_out = q_out;
  p.o_sb = 0; p.o_st = q_out_strides[0]; p.o_sh = q_out_strides[1];
  p.q_norm_weight = q_norm_weight;
  p.k_norm_weight = k_norm_weight;
  p.eps = eps;
  p.cos = cos;
  p.sin = sin;
  p.rope_positions = rope_positions;
  p.k_pool = k_pool;
  p.v_pool = v_pool;
  p.capacity = capacity_tokens;
  p.layer = layer;
  p.page_table = page_table;
  p.page_table_stride = page_table_stride;
  p.cache_lens = cache_lens;
  p.batch = batch;
  p.query_len = 1;
  p.num_q_heads = num_q_heads;
  p.num_kv_heads = num_kv_heads;
  p.page_shift = log2_int(page_size);
  p.num_pages = int32_t(capacity_tokens / page_size);
  p.error_word = error_word;
  p.q_start = q_start;
  p.token_request = token_request;
  p.total_tokens = total_tokens;
  cudaError_t err = hyt::run_norm_rope_scatter(p, dtype, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "packed norm/RoPE/scatter launch");
  return HYT_OK;
}

static int packed_attention(const void* q, const int64_t* q_strides, const void* k_pool,
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
                            void* stream, const hyt::PrefillPlan* plan) {
  if (!q || !q_strides || !k_pool || !v_pool || !page_table || !cache_lens || !q_start ||
      !q_len || !out || !out_strides)
    return fail(HYT_ERR_INVALID, "null pointer argument");
  if (num_decode < 0 || num_prefill < 0 || num_decode + num_prefill < 1)
    return fail(HYT_ERR_INVALID, "the decode and prefill lists must hold at least one request");
  if ((num_decode > 0 && !decode_ids) || (num_prefill > 0 && !prefill_ids))
    return fail(HYT_ERR_INVALID, "null request list");
  if (total_tokens < 1) return fail(HYT_ERR_INVALID, "total_tokens must be positive");
  if (max_query_len < 1 || max_query_len > total_tokens)
    return fail(HYT_ERR_INVALID, "max_query_len must be within [1, total_tokens]");
  // b strides are unused for a packed batch: the kernels index rows by q_start
  const int64_t qs[3] = {0, q_strides[1], q_strides[0]};
  const int64_t os[3] = {0, out_strides[1], out_strides[0]};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = HYT_OK;
  if (num_decode > 0) {
    Geometry g{num_layers, layer, capacity_tokens, page_table_stride, batch, 1,
               num_q_heads, num_kv_heads, head_dim, page_size, dtype};
    rc = check_geometry(g);
    if (rc != HYT_OK) return rc;
    const PackedArgs pk{q_start, q_len, decode_ids, num_decode, total_tokens};
    if (decode_eligible(g))
      rc = launch_decode(q, qs, k_pool, v_pool, g, page_table, cache_lens, out, os, scale,
                         max_kv_len, split_tokens, workspace, workspace_bytes, error_word, st, &pk);
    else
      rc = launch_generic(q, qs, k_pool, v_pool, g, page_table, cache_lens, out, os, scale,
                          error_word, st, &pk);
    if (rc != HYT_OK) return rc;
  }
  if (num_prefill > 0) {
    Geometry g{num_layers, layer, capacity_tokens, page_table_stride, batch, max_query_len,
               num_q_heads, num_kv_heads, head_dim, page_size, dtype};
    rc = check_geometry(g);
    if (rc != HYT_OK) return rc;
    const PackedArgs pk{q_start, q_len, prefill_ids, num_prefill, total_tokens};
    if (prefill_eligible(g, q, qs, out, os))
      rc = launch_prefill(q, qs, k_pool, v_pool, g, page_table, cache_lens, out, os, scale,
                          error_word, st, &pk, plan);
    else if (plan != nullptr)
      rc = fail(HYT_ERR_UNSUPPORTED, "a prefill plan needs the tcgen05 prefill kernel's shapes");
    else
      rc = launch_generic(q, qs, k_pool, v_pool, g, page_table, cache_lens, out, os, scale,
                          error_word, st, &pk);
  }
  return rc;
}

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
                               void* stream) {
  g_last_error.clear();
  return packed_attention(q, q_strides, k_pool, v_pool, num_layers, layer, capacity_tokens,
                          page_table, page_table_stride, cache_lens, q_start, q_len, out,
                          out_strides, batch, total_tokens, num_q_heads, num_kv_heads, head_dim,
                          page_size, dtype, scale, decode_ids, num_decode, prefill_ids,
                          num_prefill, max_query_len, max_kv_len, split_tokens, workspace,
                          workspace_bytes, error_word, stream, nullptr);
}

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
    int32_t* error_word, void* stream) {
  g_last_error.clear();
  if (num_items < 0 || num_splits < 0 || (num_items > 0 && items == nullptr))
    return fail(HYT_ERR_INVALID, "bad plan");
  if (num_items > 0 && num_splits > 0 &&
      (plan_workspace == nullptr || plan_workspace_bytes < hyt_prefill_workspace_bytes(num_splits) ||
       reinterpret_cast<uintptr_t>(plan_workspace) % 16))
    return fail(HYT_ERR_WORKSPACE,
                "plan workspace missing, not 16-byte aligned or smaller than hyt_prefill_workspace_bytes()");
  const hyt::PrefillPlan plan = make_prefill_plan(items, num_items, num_splits, plan_workspace);
  return packed_attention(q, q_strides, k_pool, v_pool, num_layers, layer, capacity_tokens,
                          page_table, page_table_stride, cache_lens, q_start, q_len, out,
                          out_strides, batch, total_tokens, num_q_heads, num_kv_heads, head_dim,
                          page_size, dtype, scale, decode_ids, num_decode, prefill_ids,
                          num_prefill, max_query_len, max_kv_len, split_tokens, workspace,
                          workspace_bytes, error_word, stream, num_items > 0 ? &plan : nullptr);
}

int32_t hyt_prefill_plan(const int32_t* cache_lens, const int32_t* q_lens, int32_t batch,
                         int32_t query_len, int32_t num_q_heads, int32_t num_sms,
                         int32_t max_splits, float item_overhead, float merge_cost,
                         int32_t* items, int32_t max_items, int32_t* num_splits) {
  g_last_error.clear();
  if (cache_lens == nullptr || items == nullptr || num_splits == nullptr)
    return fail(HYT_ERR_INVALID, "null pointer argument");
  if (batch < 1 || num_q_heads < 2 || num_sms < 1 || max_splits < 0 || max_items < 0 ||
      (q_lens == nullptr && query_len < 1))
    return fail(HYT_ERR_INVALID, "bad plan sizes");
  *num_splits = 0;
  const double ov = item_overhead > 0.f ? item_overhead : kItemOverhead;
  const double mc = merge_cost > 0.f ? merge_cost : kMergeCost;
  std::vector<PlanEntry> base;
  if (!prefill_items(cache_lens, q_lens, batch, query_len, num_q_heads / 2, ov, &base)) return 0;
  // with many waves the last one is a small share of the launch: not worth the host time
  // (about 1 ms per 500 items)
  if (base.empty() || base.size() > size_t(kMaxPlannedItemsPerSm) * size_t(num_sms)) return 0;
  std::vector<double> costs;
  for (const PlanEntry& e : base) costs.push_back(e.cost);
  const double grid = greedy_makespan(costs, num_sms);  // the default grid
  double best = grid;
  int best_k = -1;
  // longest first, the k heaviest items cut in two along their keys
  std::vector<PlanEntry> lpt = base;
  std::stable_sort(lpt.begin(), lpt.end(),
                   [](const PlanEntry& a, const PlanEntry& b) { return a.cost > b.cost; });
  int splittable = 0;
  for (const PlanEntry& e : lpt) splittable += e.k_hi >= 2;
  auto build = [&](int k, std::vector<PlanEntry>* out) {
    out->clear();
    int slot = 0;
    for (const PlanEntry& e : lpt) {
      if (slot < k && e.k_hi >= 2) {
        const int32_t mid = e.k_hi / 2;
        const double c0 = mid + ov + mc, c1 = (e.k_hi - mid) + ov + mc;
        out->push_back({e.z, e.q_tile, e.pair, 0, mid, slot * 2, c0});
        out->push_back({e.z, e.q_tile, e.pair, mid, e.k_hi, slot * 2 + 1, c1});
        ++slot;
      } else {
        out->push_back(e);
      }
    }
    std::stable_sort(out->begin(), out->end(),
                     [](const PlanEntry& a, const PlanEntry& b) { return a.cost > b.cost; });
  };
  std::vector<PlanEntry> cand;
  const int limit = std::min(max_splits, splittable);
  for (int k : {0, 8, 16, 24, 32, 48, 64, 96, 128, 192, 256, 384, 512}) {
    if (k > limit) break;
    if (int64_t(base.size()) + k > max_items) break;
    build(k, &cand);
    costs.clear();
    for (const PlanEntry& e : cand) costs.push_back(e.cost);
    const double m = greedy_makespan(costs, num_sms);
    if (m < best - 1e-9) {
      best = m;
      best_k = k;
    }
  }
  if (best_k < 0 || best > (1.0 - kMinGain) * grid) return 0;  // the default grid: no plan
  build(best_k, &cand);
  for (size_t i = 0; i < cand.size(); ++i) {
    const PlanEntry& e = cand[i];
    items[4 * i + 0] = e.z;
    items[4 * i + 1] = e.q_tile | (e.pair << 16);
    items[4 * i + 2] = e.k_lo | (e.k_hi << 16);
    items[4 * i + 3] = e.split;
  }
  *num_splits = best_k;
  return int32_t(cand.size());
}

size_t hyt_prefill_workspace_bytes(int32_t num_splits) {
  if (num_splits <= 0) return 0;
  return split_counter_bytes(num_splits) + size_t(num_splits) * size_t(hyt::kPrefillSplitSlotBytes);
}

int hyt_prefill_attention_planned(const void* q, const int64_t* q_strides, const void* k_pool,
                                  const void* v_pool, int32_t num_layers, int32_t layer,
                                  int64_t capacity_tokens, const int32_t* page_table,
                                  int32_t page_table_stride, const int32_t* cache_lens, void* out,
                                  const int64_t* out_strides, int32_t batch, int32_t query_len,
                                  int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                  int32_t page_size, int32_t dtype, float scale,
                                  const int32_t* items, int32_t num_items, int32_t num_splits,
                                  void* workspace, size_t workspace_bytes, int32_t* error_word,
                                  void* stream) {
  g_last_error.clear();
  int rc = check_attention_pointers(q, q_strides, k_pool, v_pool, page_table, cache_lens, out,
                                    out_strides);
  if (rc != HYT_OK) return rc;
  Geometry g{num_layers, layer, capacity_tokens, page_table_stride, batch, query_len,
             num_q_heads, num_kv_heads, head_dim, page_size, dtype};
  rc = check_geometry(g);
  if (rc != HYT_OK) return rc;
  if (!prefill_eligible(g, q, q_strides, out, out_strides))
    return fail(HYT_ERR_UNSUPPORTED,
                "prefill kernel needs bf16/f16, head_dim 128, page_size % 128 == 0, an even "
                "query-head group and 16-byte aligned q/out rows");
  if (num_items < 0 || num_splits < 0 || (num_items > 0 && items == nullptr))
    return fail(HYT_ERR_INVALID, "bad plan");
  if (num_splits > 0 && (workspace == nullptr || workspace_bytes < hyt_prefill_workspace_bytes(num_splits) ||
                         reinterpret_cast<uintptr_t>(workspace) % 16))
    return fail(HYT_ERR_WORKSPACE,
                "workspace missing, not 16-byte aligned or smaller than hyt_prefill_workspace_bytes()");
  if (num_items == 0)  // no plan: the default grid
    return launch_prefill(q, q_strides, k_pool, v_pool, g, page_table, cache_lens, out,
                          out_strides, scale, error_word, static_cast<cudaStream_t>(stream));
  const hyt::PrefillPlan plan = make_prefill_plan(items, num_items, num_splits, workspace);
  return launch_prefill(q, q_strides, k_pool, v_pool, g, page_table, cache_lens, out,
                        out_strides, scale, error_word, static_cast<cudaStream_t>(stream), nullptr,
                        &plan);
}

size_t hyt_attention_workspace_bytes(int32_t batch, int32_t query_len, int32_t num_q_heads,
                                     int32_t num_kv_heads, int32_t head_dim,
                                     int32_t max_kv_len, int32_t split_tokens, int32_t dtype) {
  if (batch < 1 || query_len < 1 || num_kv_heads < 1 || num_q_heads < 1 ||
      num_q_heads % num_kv_heads || max_kv_len < 1 || split_tokens < 0)
    return 0;
  Geometry g{1, 0, 128, 1, batch, query_len, num_q_heads, num_kv_heads, head_dim, 128, dtype};
  if (!decode_eligible(g)) return 0;
  return decode_layout(batch, query_len, num_q_heads, num_kv_heads, max_kv_len, split_tokens).total;
}

int hyt_workspace_init(void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (workspace_bytes == 0) return HYT_OK;
  if (workspace == nullptr) return fail(HYT_ERR_INVALID, "null workspace");
  cudaError_t err = cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "workspace memset");
  return HYT_OK;
}

int hyt_wait_self_test(int32_t* error_word, int64_t* elapsed_ns, void* stream) {
  g_last_error.clear();
  if (error_word == nullptr || elapsed_ns == nullptr)
    return fail(HYT_ERR_INVALID, "null error_word or elapsed_ns");
  cudaError_t err = hyt::run_wait_self_test(error_word, elapsed_ns, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "wait self-test launch");
  return HYT_OK;
}

int hyt_read_probe(const void* src, size_t bytes, uint32_t* sink, int32_t ctas, void* stream) {
  g_last_error.clear();
  if (src == nullptr || sink == nullptr) return fail(HYT_ERR_INVALID, "null src or sink");
  if (bytes == 0 || bytes % 16 || reinterpret_cast<uintptr_t>(src) % 16)
    return fail(HYT_ERR_INVALID, "src must be 16-byte aligned and bytes a positive multiple of 16");
  if (ctas < 1 || ctas > 65535) return fail(HYT_ERR_INVALID, "ctas must be in [1, 65535]");
  cudaError_t err = hyt::run_read_probe(src, bytes, sink, ctas, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "read probe launch");
  return HYT_OK;
}

}  // extern "C"
