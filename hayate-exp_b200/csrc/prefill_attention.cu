// Kernel (b): chunked-prefill causal GQA attention on tcgen05 tensor cores.
//
// Semantics: PagedKVBatch.attend_layer (hayate/engine/paged_cache.py:62-71) for a
// chunk of T new tokens per request on top of cache_lens[b] cached ones: query t
// of request b sees logical keys 0 .. cache_lens[b] + t (paged_cache.py:266-271),
// query head h reads KV head h / (H_q / H_kv), scale 1/sqrt(128) by default.
//
// Work unit: one CTA per (128 consecutive query positions, pair of query heads of
// one KV group, request). The two heads are two 128-row tiles, A and B, that see the
// same keys under the same causal mask, so every K/V tile loaded serves both.
// 576 threads, warp-specialised:
//   warps 0-15 (softmax): warps 0-7 handle tile A and 8-15 tile B, both at once.
//     In a tile, warps w and w + 4 own rows 32 * (w % 4) .. + 31 (TMEM lanes) and
//     split the 128 key columns, exchanging row maxima through shared memory. Per
//     tile a thread reads its 64 scores (tcgen05.ld), masks `key <= cache_len + t`,
//     keeps a stale running max unless the true one grows by more than 2^8 (then
//     rescales its O half-row in TMEM; O / l stays exact), turns the scores into P
//     (scale-and-shift and row sums on packed f32x2 pairs, 7 of 8 exponentials on
//     MUFU and 1 of 8 on the FMA pipe via ex2_poly; masked keys give exact 0 on
//     both) and writes P as packed bf16/f16 back over its S columns (tcgen05.st).
//     At the end the pair adds its row sums and each warp normalises its half of the
//     O rows, stages them in shared memory (the idle K/V stages) and stores them with
//     coalesced 128-byte row segments.
//   warp 16 (producer): first TMA-loads Q_A and Q_B (through a tensor map over q; when
//     q has none, the softmax warps load Q with one warp load per two whole rows), then
//     per 128-key tile looks the page up, checks it, and TMA-loads K and V (2 boxes of
//     [128 tokens x 64 dims] each, 128B swizzle) into 2-stage rings, prefetching the
//     tile kPrefetchTiles ahead into L2.
//   warp 17 (MMA issuer): S_x = Q_x K^T (M=128, N=128, 8 x K=16) and O_x += P_x V with
//     P read straight from TMEM (tcgen05.mma, A in TMEM) and V as an MN-major
//     shared-memory operand. The whole warp walks the loop and waits on the barriers;
//     each group of MMAs and its commits is issued by the lane elect.sync picks at that
//     site (lane 0, checked): on this B200 a warp-uniform elected issue costs ~39 cycles
//     per MMA next to busy softmax warps, a lone-lane branch 67-95. Issue order per key
//     tile j:
//       PV_A(j), QK_A(j+1), PV_B(j), QK_B(j+1)
//     so the softmax of tile A overlaps the tensor core working on B and vice
//     versa. tcgen05.mma ops of one thread execute in issue order, which
//     is what lets QK_x(j+1) overwrite the columns PV_x(j) reads P from, and makes
//     O_x stable whenever S_x(j) is (its commit covers PV_x(j-1)).
// TMEM (512 columns): S_A/P_A [0,128), S_B/P_B [128,256), O_A [256,384), O_B [384,512).
// Shared memory: Q_A, Q_B 32 KB each, K and V 2 x 32 KB each (192 KB), 6 KB exchange.
//
// Packed batches (AttentionParams::q_start) give each request its own chunk length on a
// shared token axis; query tiles past a request's chunk exit at once, and a request
// list (req_ids) picks the requests the launch serves.
//
// Planned launches (PrefillPlan, made on the host by hyt_prefill_plan): a 1-D grid whose
// CTA i takes item i of the plan (request, query tile, head pair, key-tile range), so
// that the longest items start first. An item cut in two runs as two CTAs over the two
// halves of its key tiles: the first to finish writes its partial (unnormalised O,
// running max, sum) to its slot of the split workspace and publishes it; the second
// merges it with its own O from TMEM (the same online-softmax merge as across tiles),
// writes the rows and resets the slot's counter.
//
// FLOPs per launch counted by the roofline: 4 * H_q * 128 per causal-valid
// (query, key) pair.
#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"

namespace hyt {

namespace {

constexpr int kRows = 128;  // query positions per CTA (per tile)
constexpr int kKeys = 128;  // keys per KV tile
constexpr int kD = 128;
constexpr int kSoftmaxThreads = 512;  // 8 warps per tile
constexpr int kProducerWarp = 16, kMmaWarp = 17;
constexpr int kSoftmaxBar = 9;  // named barrier of all 16 softmax warps (1..8: row-quarter pairs)
constexpr int kThreads = 576;
constexpr int kTileBytes = kRows * kD * 2;   // 32 KB
constexpr int kChunkBytes = kTileBytes / 2;  // [128 rows x 64 elements]
constexpr int kQOff = 0;                     // Q_A, Q_B
constexpr int kKOff = kQOff + 2 * kTileBytes;
constexpr int kVOff = kKOff + 2 * kTileBytes;
constexpr int kBarOff = kVOff + 2 * kTileBytes;
constexpr int kRedOff = kBarOff + 256;       // row-max and row-sum exchange, 6 KB
constexpr int kSmemBytes = kRedOff + 6 * 2 * 128 * 4 + 1024;
// output staging row (256 B of bf16 plus 16 B so consecutive rows start 4 banks apart)
constexpr int kStageRowBytes = 272;
static_assert(2 * kRows * kStageRowBytes <= 4 * kTileBytes, "O staging must fit in the K/V stages");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kOCol = 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr int kPrefetchTiles = 3;          // L2 prefetch distance of the K/V stream (tiles)

struct PrefillKernelParams {
  AttentionParams a;
  PrefillPlan plan;  // items == nullptr: the default grid (query tile, head pair, request)
  int32_t group;
  int32_t q_tma;  // Q arrives by TMA through q_map (else the softmax warps load it)
  int32_t q_ht;   // q_map's dims are (d, head, token, request), else (d, token, head, request)
};

// Byte offset of 16-byte chunk `chunk` (0..15) of row `r` in a [128 x 128] tile
// stored as two 128B-swizzled [128 x 64] chunks (the layout TMA SWIZZLE_128B writes).
__device__ __forceinline__ uint32_t sw128_offset(int r, int chunk) {
  return uint32_t((chunk >> 3) * kChunkBytes + r * 128 + (((chunk & 7) ^ (r & 7)) << 4));
}

// P = 2^(s * scale_log2 - m) for one thread's 64 scores, written to TMEM as 32
// packed 16-bit pairs at `p_addr`; returns the row-sum contribution. Scale-and-shift
// and the sum run on packed f32x2 pairs; 7 of 8 exponentials on MUFU (ex2), 1 of 8
// on the FMA pipe (ex2_poly). Masked scores (-inf) give exact zeros on both paths.
template <typename T>
__device__ __forceinline__ float exp_tile(const float (&s)[64], uint64_t scale2, float m,
                                          uint32_t p_addr) {
  const uint64_t neg_m2 = f2_pack(-m, -m);
  uint64_t sum2a = f2_pack(0.f, 0.f), sum2b = sum2a;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint32_t packed[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int k = c * 32 + 2 * i;
      const uint64_t x2 = f2_fma(f2_pack(s[k], s[k + 1]), scale2, neg_m2);
      float a, b;
      f2_unpack(x2, a, b);
      const float pa = ex2(a);
      const float pb = (i & 3) == 3 ? ex2_poly(b) : ex2(b);
      if (i & 1) sum2b = f2_add(sum2b, f2_pack(pa, pb));
      else sum2a = f2_add(sum2a, f2_pack(pa, pb));
      packed[i] = Elem<T>::pack2(pa, pb);
    }
    tmem_st16(p_addr + c * 16, packed);
  }
  float sa0, sa1, sb0, sb1;
  f2_unpack(sum2a, sa0, sa1);
  f2_unpack(sum2b, sb0, sb1);
  return (sa0 + sb0) + (sa1 + sb1);
}

struct Barriers {
  uint64_t q_full[2];  // Q_A, Q_B
  uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
  uint64_t s_full[2], p_full[2];  // per tile (A, B)
  uint64_t o_done, drain;
  uint64_t prod_done;  // the producer has issued its last load (and set `bad`)
  uint32_t tmem_base;
  int32_t abort;  // set once a bounded wait gave up: later waits return at once
  int32_t bad;    // device error bits of a refused page table: the CTA writes zeros
  int32_t last;   // split item: this half arrived second and merges the two
};
static_assert(sizeof(Barriers) <= 256, "barrier block");

// Split items: both halves' partials are in the workspace; write out = (O0 a0 + O1 a1) /
// (l0 a0 + l1 a1), a_i = 2^(m_i - max(m0, m1)), for rows t0 .. of heads h0, h0 + 1. A half
// with l = 0 (nothing visible, or refused) contributes nothing. Threads tid, tid + nthreads
// ... take (head, 16-byte column chunk, row) entries, consecutive threads consecutive rows.
template <typename T, typename RowFn>
__device__ __forceinline__ void merge_split(const PrefillPlan& plan, int slot, const AttentionParams& p,
                                            int h0, int t0, int query_len, RowFn o_row, int tid,
                                            int nthreads) {
  const float4* wo = reinterpret_cast<const float4*>(plan.ws_o);
  const float2* ml = reinterpret_cast<const float2*>(plan.ws_ml);
  for (int idx = tid; idx < 2 * 32 * kRows; idx += nthreads) {
    const int r = idx & (kRows - 1), c4 = (idx >> 7) & 31, x = idx >> 12;
    if (t0 + r >= query_len) continue;
    const int64_t u0 = (int64_t(slot) * 2 + 0) * 2 + x, u1 = (int64_t(slot) * 2 + 1) * 2 + x;
    const float2 a = __ldcg(&ml[u0 * kRows + r]), c = __ldcg(&ml[u1 * kRows + r]);
    const bool use0 = a.y > 0.f, use1 = c.y > 0.f;
    const float m = use0 && use1 ? fmaxf(a.x, c.x) : (use0 ? a.x : (use1 ? c.x : 0.f));
    const float f0 = use0 ? ex2(a.x - m) : 0.f, f1 = use1 ? ex2(c.x - m) : 0.f;
    const float l = __fadd_rn(__fmul_rn(a.y, f0), __fmul_rn(c.y, f1));  // as the in-kernel merge
    const float inv = l > 0.f ? 1.f / l : 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    if (use0) {  // part 0's term rounded, part 1's fused into it (the in-kernel merge's order)
      const float4 v = __ldcg(&wo[(u0 * 32 + c4) * kRows + r]);
      o = make_float4(__fmul_rn(v.x, f0), __fmul_rn(v.y, f0), __fmul_rn(v.z, f0), __fmul_rn(v.w, f0));
    }
    if (use1) {
      const float4 v = __ldcg(&wo[(u1 * 32 + c4) * kRows + r]);
      o = make_float4(__fmaf_rn(v.x, f1, o.x), __fmaf_rn(v.y, f1, o.y), __fmaf_rn(v.z, f1, o.z),
                      __fmaf_rn(v.w, f1, o.w));
    }
    uint2 w;
    w.x = Elem<T>::pack2(o.x * inv, o.y * inv);
    w.y = Elem<T>::pack2(o.z * inv, o.w * inv);
    T* out = static_cast<T*>(p.out) + o_row(t0 + r) + int64_t(h0 + x) * p.o_sh + c4 * 4;
    *reinterpret_cast<uint2*>(out) = w;
  }
}

// Split slot counter: each half adds 1 when it arrives (bits 0-1 count arrivals) and the
// first to arrive adds kPublished once its partial is in the workspace. The second half
// (its add returned an arrival count of 1) waits, bounded by the pipeline-wait limit, for
// that bit, then merges and zeroes the counter.
constexpr int kPublished = 4;
__device__ __forceinline__ void wait_published(int* counter, int prev, int32_t* error_word) {
  if (prev & kPublished) return;
  const uint64_t start = global_ns();
  while (!(*reinterpret_cast<volatile int*>(counter) & kPublished)) {
    if (global_ns() - start > kWaitLimitNs) {
      flag_error(error_word, HYT_DEVERR_WAIT_TIMEOUT);
      return;
    }
  }
}

// 96 registers: 18 warps over 4 sub-partitions put 5 warps on one 16K-register file.
template <typename T, bool kPacked>
__global__ void __maxnreg__(96)
    prefill_attention_kernel(const __grid_constant__ CUtensorMap k_map,
                             const __grid_constant__ CUtensorMap v_map,
                             const __grid_constant__ CUtensorMap q_map,
                             const PrefillKernelParams P) {
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  const AttentionParams& p = P.a;
  // work item: from the default grid, or planned (item check uniform per CTA)
  int q_tile, pair, z, k_first = 0, k_end = 1 << 30, split = -1;
  bool item_ok = true;
  if (P.plan.items != nullptr) {
    const PrefillItem it = P.plan.items[blockIdx.x];
    z = it.z;
    q_tile = it.tile_pair & 0xFFFF;
    pair = int(uint32_t(it.tile_pair) >> 16);
    k_first = it.keys & 0xFFFF;
    k_end = int(uint32_t(it.keys) >> 16);
    split = it.split;
    if (split >= 0 && (split >> 1) >= P.plan.num_splits) {  // no slot to report through
      if (threadIdx.x == 0) flag_error(p.error_word, HYT_DEVERR_PLAN_RANGE);
      return;
    }
    item_ok = z >= 0 && z < att_launch_count(p) && pair < p.num_q_heads / 2 && k_first < k_end;
  } else {
    q_tile = int(gridDim.x) - 1 - int(blockIdx.x);  // heavier (later) query tiles first
    pair = blockIdx.y;
    z = blockIdx.z;
  }
  const int b = !item_ok ? 0 : (kPacked ? att_request(p, z) : z);
  const int h0 = pair * 2;  // tiles A and B: heads h0 and h0 + 1 of KV group g
  const int g = h0 / P.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + kBarOff);

  // element offsets of query row t of this request in q and in out (head offset apart)
  auto q_row = [&](int t) -> int64_t {
    return kPacked ? (int64_t(p.q_start[b]) + t) * p.q_st : int64_t(b) * p.q_sb + int64_t(t) * p.q_st;
  };
  auto o_row = [&](int t) -> int64_t {
    return kPacked ? (int64_t(p.q_start[b]) + t) * p.o_st : int64_t(b) * p.o_sb + int64_t(t) * p.o_st;
  };
  const int t0 = q_tile * kRows;
  // A half of a split item with nothing to contribute still takes its turn in the slot's
  // protocol: an empty partial (sum 0), then, if it arrived second, the merge.
  auto empty_split = [&](bool rows_known, int query_len) {
    if (split < 0) return;
    const int slot = split >> 1, part = split & 1;
    int* counter = P.plan.ws_counter + slot;
    float2* ml = reinterpret_cast<float2*>(P.plan.ws_ml) + (int64_t(slot) * 2 + part) * 2 * kRows;
    for (int i = threadIdx.x; i < 2 * kRows; i += kThreads) ml[i] = make_float2(-INFINITY, 0.f);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) bars->last = atomicAdd(counter, 1);
    __syncthreads();
    const int prev = *reinterpret_cast<volatile int32_t*>(&bars->last);
    if ((prev & 3) == 0) {  // first: the empty partial is published
      if (threadIdx.x == 0) atomicAdd(counter, kPublished);
    } else {  // second: merge the partner's partial with the empty one
      if (threadIdx.x == 0) wait_published(counter, prev, p.error_word);
      __syncthreads();
      __threadfence();
      if (rows_known) merge_split<T>(P.plan, slot, p, h0, t0, query_len, o_row, threadIdx.x, kThreads);
      if (threadIdx.x == 0) *counter = 0;
    }
  };
  if (!item_ok) {
    if (threadIdx.x == 0) flag_error(p.error_word, HYT_DEVERR_PLAN_RANGE);
    empty_split(false, 0);
    return;
  }

  // packed batches: this request's chunk length; tiles past it have no work (uniform
  // per CTA, decided before any barrier or TMEM allocation)
  if (kPacked && !att_request_ok(p, b)) {
    if ((q_tile == 0 && pair == 0) || P.plan.items != nullptr)
      if (threadIdx.x == 0) flag_error(p.error_word, HYT_DEVERR_PACKED_RANGE);
    empty_split(false, 0);
    return;
  }
  const int query_len = kPacked ? p.q_len[b] : p.query_len;
  if (t0 >= query_len) {
    if (P.plan.items != nullptr && threadIdx.x == 0) flag_error(p.error_word, HYT_DEVERR_PLAN_RANGE);
    empty_split(false, 0);
    return;
  }
  const int cache_len = p.cache_lens[b];
  const int t_last = min(t0 + kRows, query_len) - 1;
  const int n_tiles = (cache_len + t_last) / kKeys + 1;
  const int32_t* table = p.page_table + int64_t(b) * p.page_table_stride;
  const int page_mask = (1 << p.page_shift) - 1;

  // ---- a negative cache length, or one that needs more pages than the table row holds,
  // refuses the CTA before any load (arithmetic only). Page ids are checked by the
  // producer as it reaches each tile (off the start-up path); a refused tile is not
  // loaded and the CTA writes zeros.
  if (cache_len < 0 || ((int64_t(n_tiles - 1) * kKeys) >> p.page_shift) >= p.page_table_stride) {
    if (threadIdx.x == 0) flag_error(p.error_word, HYT_DEVERR_TABLE_RANGE);
    for (int idx = threadIdx.x; idx < 2 * kRows * kD; idx += kThreads) {
      const int x = idx / (kRows * kD), r = (idx / kD) % kRows, d = idx % kD;
      if (t0 + r < query_len) {
        T* out = static_cast<T*>(p.out) + o_row(t0 + r) + int64_t(h0 + x) * p.o_sh;
        out[d] = Elem<T>::from_float(0.f);
      }
    }
    __syncthreads();  // the zeros before a merge that may overwrite them
    empty_split(true, query_len);
    return;
  }
  // key tiles [k_lo, k_lo + n_loop) of the item's n_tiles (all of them unless split)
  const int k_lo = k_first;
  const int n_loop = min(k_end, n_tiles) - k_first;
  if (n_loop <= 0) {
    if (threadIdx.x == 0) flag_error(p.error_word, HYT_DEVERR_PLAN_RANGE);
    empty_split(true, query_len);
    return;
  }

  int32_t* err = p.error_word;
  volatile int* abort = &bars->abort;
  const int plane = p.layer * p.num_kv_heads + g;
  // producer state, shared by its start-up loads (issued before the CTA-wide barrier) and
  // its loop; an earlier CTA's wait gave up: load nothing (the CTA writes zeros)
  int bad = 0;
  // pool row of key tile j, or -1 (and the error bit in `why`) for a page id outside the
  // pool; the table row is long enough for every tile (checked above)
  auto tile_row = [&](int j, int& why) {
    const int tok = j * kKeys;
    const int32_t page = table[tok >> p.page_shift];
    if (page < 0 || page >= p.num_pages) {
      why |= HYT_DEVERR_PAGE_RANGE;
      return -1;
    }
    return (page << p.page_shift) + (tok & page_mask);
  };
  // K and V of ring position j (key tile k_lo + j) into stage j & 1: a TMA load, or, once a
  // page id was refused, a plain arrival so every role still walks the same tiles
  auto load_tile = [&](int j) {
    const int st = j & 1;
    const uint32_t ph = (j >> 1) & 1;
    const int row = bad ? -1 : tile_row(k_lo + j, bad);
    if (j >= 2) mbar_wait(&bars->k_empty[st], ph ^ 1, err, abort);
    uint8_t* kdst = smem + kKOff + st * kTileBytes;
    if (!bad) {
      mbar_arrive_expect_tx(&bars->k_full[st], kTileBytes);
      tma_load_3d(kdst, &k_map, &bars->k_full[st], 0, row, plane);
      tma_load_3d(kdst + kChunkBytes, &k_map, &bars->k_full[st], 64, row, plane);
    } else {
      mbar_arrive(&bars->k_full[st]);
    }
    if (j >= 2) mbar_wait(&bars->v_empty[st], ph ^ 1, err, abort);
    uint8_t* vdst = smem + kVOff + st * kTileBytes;
    if (!bad) {
      mbar_arrive_expect_tx(&bars->v_full[st], kTileBytes);
      tma_load_3d(vdst, &v_map, &bars->v_full[st], 0, row, plane);
      tma_load_3d(vdst + kChunkBytes, &v_map, &bars->v_full[st], 64, row, plane);
    } else {
      mbar_arrive(&bars->v_full[st]);
    }
  };
  const int n_early = min(n_loop, 2);  // ring positions the producer loads before the barrier

  if (warp == kProducerWarp && lane == 0) {
    // Start-up: the producer initialises the barriers and issues Q_A, Q_B and the first
    // two K/V tiles at once, while warp 0 allocates tensor memory; the CTA-wide barrier
    // below then publishes the barriers to every other thread.
    bars->abort = 0;
    bars->bad = 0;
    for (int x = 0; x < 2; ++x) mbar_init(&bars->q_full[x], P.q_tma ? 1 : kSoftmaxThreads);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->p_full[s], kSoftmaxThreads / 2);
    }
    mbar_init(&bars->o_done, 1);
    mbar_init(&bars->drain, 1);
    mbar_init(&bars->prod_done, 1);
    fence_barrier_init();
    fence_proxy_async_smem();  // the initialised barriers, before this thread's TMA uses them
    bad = (err != nullptr && (*reinterpret_cast<volatile int32_t*>(err) & HYT_DEVERR_WAIT_TIMEOUT))
              ? HYT_DEVERR_WAIT_TIMEOUT : 0;
    if (P.q_tma) {  // Q first: QK_x waits for Q_x and K tile 0
      const int q_row0 = kPacked ? p.q_start[b] + t0 : t0;
      const int q_req = kPacked ? 0 : b;
#pragma unroll
      for (int qx = 0; qx < 2; ++qx) {
        mbar_arrive_expect_tx(&bars->q_full[qx], kTileBytes);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint8_t* dst = smem + kQOff + qx * kTileBytes + c * kChunkBytes;
          if (P.q_ht)
            tma_load_4d(dst, &q_map, &bars->q_full[qx], c * 64, h0 + qx, q_row0, q_req);
          else
            tma_load_4d(dst, &q_map, &bars->q_full[qx], c * 64, q_row0, h0 + qx, q_req);
        }
      }
    }
    tma_prefetch_desc(&k_map);
    tma_prefetch_desc(&v_map);
    for (int j = 0; j < n_early; ++j) load_tile(j);
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

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      auto prefetch = [&](int j) {  // K and V of tile j into L2
        int why = 0;
        const int row = tile_row(j, why);
        if (why) return;  // refused when its turn to load comes
        tma_prefetch_l2_3d(&k_map, 0, row, plane);
        tma_prefetch_l2_3d(&k_map, 64, row, plane);
        tma_prefetch_l2_3d(&v_map, 0, row, plane);
        tma_prefetch_l2_3d(&v_map, 64, row, plane);
      };
      // Positions 0 and 1 were loaded at start-up (both ring stages are free); from
      // iteration 1 on, each iteration prefetches into L2 the tile kPrefetchTiles beyond the
      // one it loads. No prefetch burst at start-up: the whole first wave loads Q and its
      // first tiles then, sharing HBM.
      if (!bad && n_early > 1 && 1 + kPrefetchTiles < n_loop) prefetch(k_lo + 1 + kPrefetchTiles);
      for (int j = n_early; j < n_loop; ++j) {  // ring position j holds key tile k_lo + j
        if (!bad && j + kPrefetchTiles < n_loop) prefetch(k_lo + j + kPrefetchTiles);
        load_tile(j);
      }
      if (bad) {
        flag_error(err, bad);
        bars->bad = bad;
      }
      mbar_arrive(&bars->prod_done);  // release: `bad` is visible to whoever waits on it
      for (int j = max(0, n_loop - 2); j < n_loop; ++j) {  // nothing in flight at exit
        mbar_drain(&bars->k_full[j & 1], (j >> 1) & 1);
        mbar_drain(&bars->v_full[j & 1], (j >> 1) & 1);
      }
      if (P.q_tma) {
        mbar_drain(&bars->q_full[0], 0);
        mbar_drain(&bars->q_full[1], 0);
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp walks the loop and waits on the barriers (descriptors stay
    // warp-uniform); each group of tcgen05 ops and its commit is issued by one lane
    // chosen by elect.sync at that site.
    constexpr uint32_t idesc_qk = umma_idesc_f16(kBf16, 128, 128, false, false);
    constexpr uint32_t idesc_pv = umma_idesc_f16(kBf16, 128, 128, false, true);
    // all descriptors share their high halves (layout, SBO); the low halves hold the start
    // address, which never carries into the high half (shared memory < 256 KB)
    const uint64_t q_desc0 = umma_desc_sw128(smem_base + kQOff, 16);
    const uint32_t hi = uint32_t(q_desc0 >> 32);
    const uint32_t q_lo0 = uint32_t(q_desc0);
    const uint32_t q_lo1 = uint32_t(umma_desc_sw128(smem_base + kQOff + kTileBytes, 16));
    const uint32_t k_lo0 = uint32_t(umma_desc_sw128(smem_base + kKOff, 16));
    const uint32_t k_lo1 = uint32_t(umma_desc_sw128(smem_base + kKOff + kTileBytes, 16));
    const uint32_t v_lo0 = uint32_t(umma_desc_sw128(smem_base + kVOff, kChunkBytes));
    const uint32_t v_lo1 = uint32_t(umma_desc_sw128(smem_base + kVOff + kTileBytes, kChunkBytes));
    // self-check: an issuing block must run on exactly one lane, always the same one
    // (lane 0), so that every commit covers every tcgen05 op issued before it
    auto single_lane = [&]() {
      if (__activemask() != (1u << lane) || lane != 0) {
        flag_error(err, HYT_DEVERR_ISSUE_LANE);
        return false;
      }
      return true;
    };
    // PV_x(j) (optional) then, if qk, S_x = Q_x K_{j+1}^T with its commit, one lane
    auto issue = [&](int x, int j, bool pv, bool qk, uint64_t* extra_commit, uint64_t* extra_commit2) {
      if (elect_one()) {
        if (single_lane()) {
          tc_fence_after();
          if (pv) {
            const uint32_t b0 = (j & 1) ? v_lo1 : v_lo0;
            const uint32_t d = tmem + kOCol + x * 128, a = tmem + x * 128;
            const uint32_t first = j > 0 ? 1u : 0u;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              umma_f16_ts_lh(d, a + kk * 8, b0 + uint32_t((kk * 2048) >> 4), hi, idesc_pv, kk > 0 ? 1u : first);
          }
          if (qk) {
            const int jq = pv ? j + 1 : j;
            const uint32_t a0 = x ? q_lo1 : q_lo0, b0 = (jq & 1) ? k_lo1 : k_lo0;
            const uint32_t d = tmem + x * 128;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint32_t off = uint32_t(((kk >> 2) * kChunkBytes + (kk & 3) * 32) >> 4);
              umma_f16_ss_lh(d, a0 + off, hi, b0 + off, hi, idesc_qk, kk > 0 ? 1u : 0u);
            }
            umma_commit(&bars->s_full[x]);
          }
          if (extra_commit != nullptr) umma_commit(extra_commit);
          if (extra_commit2 != nullptr) umma_commit(extra_commit2);
        }
      }
      __syncwarp();
    };
    mbar_wait(&bars->q_full[0], 0, err, abort);
    mbar_wait(&bars->k_full[0], 0, err, abort);
    issue(0, 0, false, true, nullptr, nullptr);
    mbar_wait(&bars->q_full[1], 0, err, abort);
    issue(1, 0, false, true, &bars->k_empty[0], nullptr);
    for (int j = 0; j < n_loop; ++j) {
      const bool more = j + 1 < n_loop;
      mbar_wait(&bars->v_full[j & 1], (j >> 1) & 1, err, abort);
      mbar_wait(&bars->p_full[0], j & 1, err, abort);  // tile A
      if (more) mbar_wait(&bars->k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, err, abort);
      issue(0, j, true, more, nullptr, nullptr);
      mbar_wait(&bars->p_full[1], j & 1, err, abort);  // tile B
      issue(1, j, true, more, &bars->v_empty[j & 1], more ? &bars->k_empty[(j + 1) & 1] : nullptr);
    }
    if (elect_one()) {
      if (single_lane()) {
        umma_commit(&bars->o_done);
        umma_commit(&bars->drain);  // every MMA done before TMEM is released
      }
    }
    __syncwarp();
    mbar_drain(&bars->drain, 0);
  } else {
    // ------------------------------------------------------------ softmax warps
    // Warps 0-7 handle tile A and warps 8-15 tile B, both at once. Within a tile,
    // warps w and w + 4 own rows 32 * (w % 4) .. + 31 (TMEM lanes) and split the 128
    // key columns, exchanging row maxima through shared memory; row sums are added
    // once, in the epilogue. Each sub-partition thus runs four softmax warps.
    const int x = warp >> 3, half = (warp >> 2) & 1, quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row == TMEM lane
    const int t = t0 + r;
    const int limit = cache_len + min(t, query_len - 1);  // last visible key
    const uint32_t lane_addr = tmem + (uint32_t(quarter * 32) << 16);
    const int pair_bar = 1 + x * 4 + quarter;  // named barrier of the two warps of this row quarter
    float* red_max = reinterpret_cast<float*>(smem + kRedOff) + x * (2 * 2 * kRows);  // [parity][half][row]
    float* red_sum = reinterpret_cast<float*>(smem + kRedOff) + 2 * (2 * 2 * kRows) + x * (2 * kRows);

    if (!P.q_tma) {  // Q rows -> swizzled shared memory (when q has no tensor map); one
       // warp load covers 2 whole rows (512 B). All eight loads are issued before the first
       // shared store (one memory round trip, not eight: the stores would otherwise be
       // ordered behind each load).
      uint4 v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int idx = i * kSoftmaxThreads + int(threadIdx.x);  // (tile, row, 16-byte chunk)
        const int c = idx & 15, qr = (idx >> 4) & (kRows - 1), qx = idx >> 11;
        const int qt = t0 + qr;
        v[i] = make_uint4(0u, 0u, 0u, 0u);
        if (qt < query_len)
          v[i] = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(p.q) + q_row(qt) +
                                                       int64_t(h0 + qx) * p.q_sh) + c);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int idx = i * kSoftmaxThreads + int(threadIdx.x);
        const int c = idx & 15, qr = (idx >> 4) & (kRows - 1), qx = idx >> 11;
        *reinterpret_cast<uint4*>(smem + kQOff + qx * kTileBytes + sw128_offset(qr, c)) = v[i];
      }
      fence_proxy_async_smem();
      mbar_arrive(&bars->q_full[0]);
      mbar_arrive(&bars->q_full[1]);
    }

    const float scale_log2 = p.scale * kLog2e;
    const uint64_t scale2 = f2_pack(scale_log2, scale_log2);
    const uint32_t s_col = x * 128 + half * 64;
    const uint32_t p_col = x * 128 + half * 32;
    const uint32_t o_col = kOCol + x * 128 + half * 64;
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = 0; j < n_loop; ++j) {
      mbar_wait(&bars->s_full[x], j & 1, err, abort);
      tc_fence_after();
      float s[64];
      {
        uint32_t raw[2][32];
        tmem_ld32(lane_addr + s_col, raw[0]);
        tmem_ld32(lane_addr + s_col + 32, raw[1]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(raw[c][i]);
      }
      // mask + this half's row max on the raw scores (scale > 0 keeps the order)
      const int key0 = (k_lo + j) * kKeys + half * 64;
      if (key0 + 63 > limit) {  // only the diagonal tiles
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (key0 + c > limit) s[c] = -INFINITY;
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int c = 0; c < 64; c += 4) {
        mx0 = fmax3(mx0, s[c], s[c + 1]);
        mx1 = fmax3(mx1, s[c + 2], s[c + 3]);
      }
      float* slot = red_max + (j & 1) * 2 * kRows;
      slot[half * kRows + r] = fmaxf(mx0, mx1);
      named_bar_sync(pair_bar, 64);
      const float m_tile = fmaxf(slot[r], slot[kRows + r]) * scale_log2;
      const float m_new = fmaxf(m_run, m_tile);
      const bool moves = __any_sync(0xffffffffu, m_new > m_run + kRescaleThreshold);
      float alpha = 1.f;
      if (moves) {
        alpha = ex2(m_run - m_new);  // 0 on the first tile (m_run = -inf)
        m_run = m_new;
      }
      const float tile_sum = exp_tile<T>(s, scale2, m_run, lane_addr + p_col);
      l_run = l_run * alpha + tile_sum;
      if (moves && j > 0) {  // O_x is stable: PV_x(j-1) completed before S_x(j) did
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          tmem_ld32(lane_addr + o_col + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(lane_addr + o_col + c * 32, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->p_full[x]);
    }

    // ---- epilogue: O / l -> out[b, h0 + x, t, half * 64 ..]. Rows go through shared memory
    // (the K/V stages are idle once o_done fired) so that each warp store writes four whole
    // 128-byte row segments instead of 16 bytes of 32 different rows.
    red_sum[half * kRows + r] = l_run;
    mbar_wait(&bars->o_done, 0, err, abort);
    mbar_wait(&bars->prod_done, 0, err, abort);
    tc_fence_after();
    named_bar_sync(pair_bar, 64);
    const float l = red_sum[r] + red_sum[kRows + r];
    // a refused page table: zeros (`bad` is published by the producer's prod_done arrival)
    const bool refused = *reinterpret_cast<volatile int32_t*>(&bars->bad) != 0;
    // split item: the half that arrives first writes its partial (unnormalised O, running
    // max, sum; consecutive lanes -> consecutive rows of a 16-byte column chunk) and
    // publishes it; the second merges it with its own O (still in TMEM) and writes the
    // rows. A refused half contributes nothing (sum 0).
    float own_scale = 1.f, partner_scale = 0.f, inv = l > 0.f ? 1.f / l : 0.f;
    bool use_own = !refused;
    const float4* partner = nullptr;
    bool write_rows = true;
    if (split >= 0) {
      const int slot = split >> 1, part = split & 1;
      int* counter = P.plan.ws_counter + slot;
      if (threadIdx.x == 0) bars->last = atomicAdd(counter, 1);
      named_bar_sync(kSoftmaxBar, kSoftmaxThreads);
      const int prev = *reinterpret_cast<volatile int32_t*>(&bars->last);
      if ((prev & 3) == 0) {  // first
        const int64_t unit = (int64_t(slot) * 2 + part) * 2 + x;
        float4* wo = reinterpret_cast<float4*>(P.plan.ws_o) + unit * 32 * kRows;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          tmem_ld32(lane_addr + o_col + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int v = 0; v < 8; ++v)
            wo[(half * 16 + c * 8 + v) * kRows + r] =
                make_float4(__uint_as_float(o[4 * v]), __uint_as_float(o[4 * v + 1]),
                            __uint_as_float(o[4 * v + 2]), __uint_as_float(o[4 * v + 3]));
        }
        if (half == 0)
          reinterpret_cast<float2*>(P.plan.ws_ml)[unit * kRows + r] = make_float2(m_run, refused ? 0.f : l);
        __threadfence();
        named_bar_sync(kSoftmaxBar, kSoftmaxThreads);
        if (threadIdx.x == 0) atomicAdd(counter, kPublished);
        write_rows = false;
      } else {  // second
        if (threadIdx.x == 0) wait_published(counter, prev, err);
        named_bar_sync(kSoftmaxBar, kSoftmaxThreads);
        __threadfence();
        const int64_t unit = (int64_t(slot) * 2 + (part ^ 1)) * 2 + x;
        const float2 other = __ldcg(reinterpret_cast<const float2*>(P.plan.ws_ml) + unit * kRows + r);
        const float own_l = refused ? 0.f : l;
        const bool use_other = other.y > 0.f;
        use_own = own_l > 0.f;
        const float m = use_own && use_other ? fmaxf(m_run, other.x) : (use_own ? m_run : (use_other ? other.x : 0.f));
        own_scale = use_own ? ex2(m_run - m) : 0.f;
        partner_scale = use_other ? ex2(other.x - m) : 0.f;
        // products rounded on their own and added (no fused multiply-add): the same sum
        // whichever half arrived second
        const float lsum = __fadd_rn(__fmul_rn(own_l, own_scale), __fmul_rn(other.y, partner_scale));
        inv = lsum > 0.f ? 1.f / lsum : 0.f;
        if (use_other) partner = reinterpret_cast<const float4*>(P.plan.ws_o) + unit * 32 * kRows;
        if (threadIdx.x == 0) *counter = 0;  // both halves are done with the slot
      }
    }
    if (write_rows) {
    uint8_t* stage = smem + kKOff + x * kRows * kStageRowBytes + half * 128;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      uint32_t o[32];
      tmem_ld32(lane_addr + o_col + c * 32, o);
      tmem_wait_ld();
      float f[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) f[i] = use_own ? __uint_as_float(o[i]) * own_scale : 0.f;
      if (partner != nullptr) {
        // the two halves combine in one fixed order, part 0's term rounded, part 1's fused
        // into it, so the rows do not depend on which half arrived second
        const bool own_first = (split & 1) == 0;
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const float4 q4 = __ldcg(&partner[(half * 16 + c * 8 + v) * kRows + r]);
          const float pv[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float mine = use_own ? __uint_as_float(o[4 * v + e]) : 0.f;
            f[4 * v + e] = own_first ? __fmaf_rn(pv[e], partner_scale, __fmul_rn(mine, own_scale))
                                     : __fmaf_rn(mine, own_scale, __fmul_rn(pv[e], partner_scale));
          }
        }
      }
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        uint4 w;
        w.x = Elem<T>::pack2(f[8 * v + 0] * inv, f[8 * v + 1] * inv);
        w.y = Elem<T>::pack2(f[8 * v + 2] * inv, f[8 * v + 3] * inv);
        w.z = Elem<T>::pack2(f[8 * v + 4] * inv, f[8 * v + 5] * inv);
        w.w = Elem<T>::pack2(f[8 * v + 6] * inv, f[8 * v + 7] * inv);
        *reinterpret_cast<uint4*>(stage + r * kStageRowBytes + (c * 4 + v) * 16) = w;
      }
    }
    __syncwarp();
    T* out_head = static_cast<T*>(p.out) + int64_t(h0 + x) * p.o_sh + half * 64;
#pragma unroll
    for (int i = 0; i < 8; ++i) {  // this warp's 32 rows, 4 per store, lane -> 16-byte chunk
      const int rr = quarter * 32 + i * 4 + (lane >> 3), ch = lane & 7;
      const uint4 w = *reinterpret_cast<const uint4*>(stage + rr * kStageRowBytes + ch * 16);
      if (t0 + rr < query_len) reinterpret_cast<uint4*>(out_head + o_row(t0 + rr))[ch] = w;
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
                                  const CUtensorMap& v_map, const CUtensorMap* q_map, bool q_ht,
                                  int dtype, cudaStream_t stream, const PrefillPlan* plan) {
  PrefillKernelParams P;
  P.a = p;
  P.plan = plan != nullptr ? *plan : PrefillPlan{nullptr, 0, 0, nullptr, nullptr, nullptr};
  P.group = p.num_q_heads / p.num_kv_heads;
  P.q_tma = q_map != nullptr ? 1 : 0;
  P.q_ht = q_ht ? 1 : 0;
  const dim3 grid = P.plan.items != nullptr
                        ? dim3(unsigned(P.plan.num_items), 1u, 1u)
                        : dim3(unsigned((p.query_len + kRows - 1) / kRows), unsigned(p.num_q_heads / 2),
                               unsigned(att_launch_count(p)));
  auto launch = [&](auto kernel) {
    cudaError_t e = allow_smem(kernel, kSmemBytes, stream);
    if (e != cudaSuccess) return e;
    kernel<<<grid, kThreads, kSmemBytes, stream>>>(k_map, v_map, q_map != nullptr ? *q_map : k_map, P);
    return cudaSuccess;
  };
  const bool packed = p.q_start != nullptr;
  cudaError_t e;
  if (dtype == HYT_DTYPE_F16)
    e = packed ? launch(prefill_attention_kernel<__half, true>) : launch(prefill_attention_kernel<__half, false>);
  else
    e = packed ? launch(prefill_attention_kernel<__nv_bfloat16, true>)
               : launch(prefill_attention_kernel<__nv_bfloat16, false>);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace hyt
