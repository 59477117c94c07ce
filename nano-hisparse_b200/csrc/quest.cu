// (1) Quest page selection: page scoring over the K min/max metadata, shared
// top-k with forced sink/tail pages and page->token expansion, in one launch.
//
// Reference: nano_hisparse/selection.py:69-91 (quest_selection),
// selection.py:45-62 (Selection.from_pages), row_index.py:20-24
// (LogicalTopK.from_selection, shared case).
//
// Grid (ctas_per_request, batch). A CTA scores one tile of pages of one
// request; a warp serves one (KV head, group of 4 query heads) and scores
// 32 / L pages at a time, L = the lanes sharing one page's row (L = 16 at
// head_dim 128): each lane holds its 8 head-dim elements of q for the 4 heads,
// widens 8 min and 8 max elements into packed pairs and runs 32 packed FMAs;
// a 4-value lane reduction (two halving levels, then whole values) leaves one
// (page, head) sum per lane group. Head sums meet in shared memory and are
// combined per page. The last CTA of a request to finish (a completion counter
// in the workspace) runs the top-k: an MSB-first radix select over
// order-preserving score keys, then the chosen pages are scanned in page order
// so tokens come out sorted.
//
// Fixed fp32 order (reproducible bit for bit; the oracle restates it):
//   L           = smallest power of two >= ceil(D / 8)
//   a[h, j]     = terms d = 8j, 8j+2, 8j+4, 8j+6 (d < D) of max(q*min, q*max),
//                 left to right; b[h, j] the same at 8j+1, 8j+3, ...
//   part[h, j]  = a + b
//   s[h]        = xor tree over lanes j < L: pairs (j, j^(L/2)), ..., (j, j^1)
//   u[j]        = sum over heads h = j, j+32, ... of s[h], left to right
//   score       = (xor tree over 32 lanes of u[j]) / q_heads
// For 16-bit q and metadata, max(q*min, q*max) is evaluated as
// fma(q+, max, .) then fma(q-, min, .) with q+ = max(q, 0), q- = min(q, 0):
// the products of two 16-bit floats are exact in fp32 and min <= max, so the
// sums are bit-identical and an (even, odd) pair of terms costs two packed FMAs.
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace hs {
namespace {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kHeadsPerItem = 4;
constexpr int kPagesPerItem = 32 / kHeadsPerItem;  // 8

template <typename TQ, typename TKV> struct QuestParams {
  int batch;
  Batched<TQ> query;
  Batched<TKV> minimum;
  Batched<TKV> maximum;
  Lengths lengths;
  int q_heads, kv_heads, head_dim, page_size, top_pages, keep_sink;
  int64_t max_pages;
  int tile_pages;  // pages per CTA (multiple of kPagesPerItem)
  float *scores;   // workspace [batch, max_pages] (partial mode: the caller's output)
  unsigned *done;  // workspace [batch] completion counters (zero between calls)
  int partial;     // 1: write head sums without the division and skip the selection
  int32_t *out_tokens;
  int64_t capacity;
  int32_t *out_counts;
  int32_t *status;
};

template <typename T> constexpr bool is16() { return sizeof(T) == 2; }

// C consecutive elements of one metadata row, kept in their storage type until
// use (halves the registers held by in-flight loads for 16-bit metadata).
template <typename T, int C> struct Raw {
  T e[C];
  __device__ __forceinline__ void load(const T *src, bool in, int d0, int D) {
    constexpr int bytes = C * (int)sizeof(T);
    if (in && d0 + C <= D) {
      if constexpr (bytes == 16 || bytes == 8 || bytes == 4) {
        if ((reinterpret_cast<uintptr_t>(src) & (bytes - 1)) == 0) {
          if constexpr (bytes == 16) *reinterpret_cast<uint4 *>(e) = __ldg(reinterpret_cast<const uint4 *>(src));
          if constexpr (bytes == 8) *reinterpret_cast<uint2 *>(e) = __ldg(reinterpret_cast<const uint2 *>(src));
          if constexpr (bytes == 4) *reinterpret_cast<uint32_t *>(e) = __ldg(reinterpret_cast<const uint32_t *>(src));
          return;
        }
      }
    }
#pragma unroll
    for (int c = 0; c < C; ++c) e[c] = (in && d0 + c < D) ? src[c] : T(0.f);
  }
  // Same from a shared-memory address (plain loads: __ldg is global-only).
  __device__ __forceinline__ void load_shared(const T *src, bool in, int d0, int D) {
    constexpr int bytes = C * (int)sizeof(T);
    if (in && d0 + C <= D) {
      if constexpr (bytes == 16 || bytes == 8 || bytes == 4) {
        if ((reinterpret_cast<uintptr_t>(src) & (bytes - 1)) == 0) {
          if constexpr (bytes == 16) *reinterpret_cast<uint4 *>(e) = *reinterpret_cast<const uint4 *>(src);
          if constexpr (bytes == 8) *reinterpret_cast<uint2 *>(e) = *reinterpret_cast<const uint2 *>(src);
          if constexpr (bytes == 4) *reinterpret_cast<uint32_t *>(e) = *reinterpret_cast<const uint32_t *>(src);
          return;
        }
      }
    }
#pragma unroll
    for (int c = 0; c < C; ++c) e[c] = (in && d0 + c < D) ? src[c] : T(0.f);
  }
  // Whole, aligned row slice from shared memory (the staged path's layout).
  __device__ __forceinline__ void load_shared_full(const T *src, bool in) {
    constexpr int bytes = C * (int)sizeof(T);
    if constexpr (bytes == 16) {
      *reinterpret_cast<uint4 *>(e) = in ? *reinterpret_cast<const uint4 *>(src) : make_uint4(0, 0, 0, 0);
    } else if constexpr (bytes == 8) {
      *reinterpret_cast<uint2 *>(e) = in ? *reinterpret_cast<const uint2 *>(src) : make_uint2(0, 0);
    } else if constexpr (bytes == 4) {
      *reinterpret_cast<uint32_t *>(e) = in ? *reinterpret_cast<const uint32_t *>(src) : 0u;
    } else {
#pragma unroll
      for (int c = 0; c < C; ++c) e[c] = in ? src[c] : T(0.f);
    }
  }
  __device__ __forceinline__ void unpack(float (&out)[C]) const {
#pragma unroll
    for (int c = 0; c < C; ++c) out[c] = to_f32(e[c]);
  }
};

// Order-preserving map of a float score to an unsigned key. -0 is folded onto
// +0; NaN ranks above +inf (as in torch.topk); forced pages take the maximum.
__device__ __forceinline__ uint32_t score_key(float s) {
  if (isnan(s)) return 0xfffffffeu;
  const uint32_t bits = __float_as_uint(s + 0.0f);
  return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
}

__device__ __forceinline__ uint32_t page_key(const float *sc, int64_t page, int64_t n, bool sink) {
  if (page == n - 1 || (sink && page == 0)) return 0xffffffffu;
  return score_key(__ldcg(sc + page));
}

constexpr int kSmemKeys = 16384;  // pages whose keys the select phase caches in shared memory
constexpr int kMaxChosenPages = 2048;  // chosen-page list of the cooperative token expansion

// Keys of one request: from shared memory when cached, else recomputed from
// the scores in global memory.
struct KeySource {
  const uint32_t *cached;
  const float *scores;
  int64_t n;
  bool sink;
  __device__ __forceinline__ uint32_t operator()(int64_t page) const {
    return cached ? cached[page] : page_key(scores, page, n, sink);
  }
};

// One radix step, run by one warp: the digit of the k-th largest key among the
// keys counted in `h` (256 bins; bins above the digit's width are empty).
// Lane l owns digits [8*(31-l), 8*(31-l)+7], so the lanes in order walk the
// digits from the top. Narrows prefix/mask by the digit and leaves in *k the
// rank of the wanted key among the keys with that digit.
__device__ __forceinline__ void pick_digit(const uint32_t *h, uint32_t prefix, uint32_t mask,
                                           int shift, uint32_t digit_mask, uint32_t *s_prefix,
                                           uint32_t *s_mask, uint32_t *s_k) {
  const int lane = threadIdx.x & 31;
  uint32_t local = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) local += h[8 * (31 - lane) + i];
  const uint32_t inc = warp_inclusive_scan(local);
  const uint32_t k = *s_k;
  const unsigned ballot = __ballot_sync(kFullMask, inc >= k);
  const int owner = __ffs(ballot) - 1;
  if (lane == owner) {
    uint32_t above = inc - local;
    int digit = 8 * (31 - lane) + 7;
    for (; digit > 8 * (31 - lane); --digit) {
      if (above + h[digit] >= k) break;
      above += h[digit];
    }
    *s_k = k - above;
    *s_prefix = prefix | ((uint32_t)digit << shift);
    *s_mask = mask | (digit_mask << shift);
  }
}

// ---- top-k + expansion for one request (run by the last CTA) ------------------
template <typename TQ, typename TKV>
__device__ void select_request(const QuestParams<TQ, TKV> &p, int b, int64_t length, int64_t n,
                               uint32_t *key_cache) {
  __shared__ uint32_t hist[256];
  __shared__ int64_t scan_scratch[33];
  __shared__ uint32_t s_prefix, s_mask, s_k, s_lo, s_hi;
  const int tid = threadIdx.x;
  int32_t *out = p.out_tokens + (int64_t)b * p.capacity;
  if (length <= 0 || n > p.max_pages) {
    if (n > p.max_pages && tid == 0) flag(p.status, HS_DEV_PAGES_EXCEED_TABLE);
    for (int64_t i = tid; i < p.capacity; i += blockDim.x) out[i] = -1;
    if (tid == 0) p.out_counts[b] = 0;
    return;
  }
  if (p.top_pages >= n) {  // every page (selection.py:80-81)
    for (int64_t i = tid; i < p.capacity; i += blockDim.x) out[i] = i < length ? (int32_t)i : -1;
    if (tid == 0) p.out_counts[b] = (int32_t)length;
    return;
  }
  const float *sc = p.scores + (int64_t)b * p.max_pages;
  const bool sink = p.keep_sink && p.top_pages > 1 && n > 1;
  KeySource key_of{nullptr, sc, n, sink};
  if (key_cache != nullptr && n <= kSmemKeys) {
    // eight independent score loads in flight per thread (the scores sit in L2:
    // one load at a time would cost a full L2 round trip per page)
    for (int64_t pg0 = tid; pg0 < n; pg0 += 8 * (int64_t)blockDim.x) {
      uint32_t key[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t pg = pg0 + (int64_t)u * blockDim.x;
        key[u] = pg < n ? page_key(sc, pg, n, sink) : 0u;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t pg = pg0 + (int64_t)u * blockDim.x;
        if (pg < n) key_cache[pg] = key[u];
      }
    }
    key_of.cached = key_cache;
  }
  // The forced pages (key kForcedKey: the tail, and the sink when kept) are
  // always chosen, so the radix select ranks only the other pages, for the
  // rest of the budget, and starts at the highest bit in which their keys
  // differ: the scores of one request share their sign and most exponent
  // bits, and a digit over those bits sends every page to one histogram bin
  // (every atomic on one shared-memory word).
  constexpr uint32_t kForcedKey = 0xffffffffu;  // no score maps here (NaN: 0xfffffffe)
  const int forced = sink ? 2 : 1;
  const int lane = tid & 31, warp = tid >> 5, warps = (int)(blockDim.x >> 5);
  if (tid == 0) {
    s_lo = 0xffffffffu;
    s_hi = 0u;
  }
  __syncthreads();
  {
    uint32_t lo = 0xffffffffu, hi = 0u;
    for (int64_t pg = tid; pg < n; pg += blockDim.x) {
      const uint32_t key = key_of(pg);
      if (key != kForcedKey) {
        lo = min(lo, key);
        hi = max(hi, key);
      }
    }
    lo = __reduce_min_sync(kFullMask, lo);
    hi = __reduce_max_sync(kFullMask, hi);
    if (lane == 0) {
      atomicMin(&s_lo, lo);
      atomicMax(&s_hi, hi);
    }
  }
  __syncthreads();
  // budget left after the forced pages; fewer than the unforced pages (n > top_pages)
  const uint32_t rest = (uint32_t)(p.top_pages - forced);
  const uint32_t differ = s_lo ^ s_hi;
  const int top_bit = differ ? 31 - __clz((int)differ) : -1;
  if (tid == 0) {
    // the bits above top_bit are the same in every unforced key
    const uint32_t common =
        top_bit < 0 ? 0xffffffffu : top_bit < 31 ? ~((2u << top_bit) - 1u) : 0u;
    s_prefix = s_hi & common;
    s_mask = common;
    s_k = rest;
  }
  __syncthreads();
  for (int high = rest > 0 ? top_bit : -1; high >= 0; high -= 8) {
    const int shift = high >= 7 ? high - 7 : 0;
    const uint32_t digit_mask = (2u << (high - shift)) - 1u;  // up to 8 bits
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    for (int64_t pg = tid; pg < n; pg += blockDim.x) {
      const uint32_t key = key_of(pg);
      if (key != kForcedKey && (key & mask) == prefix)
        atomicAdd(&hist[(key >> shift) & digit_mask], 1u);
    }
    __syncthreads();
    if (tid < 32) pick_digit(hist, prefix, mask, shift, digit_mask, &s_prefix, &s_mask, &s_k);
    __syncthreads();
  }
  // rest == 0: the forced pages alone (threshold = their key, all of them
  // kept); else every key above the threshold, forced pages included, and the
  // first take_equal keys equal to it
  const uint32_t threshold = rest > 0 ? s_prefix : kForcedKey;
  const int64_t take_equal = rest > 0 ? (int64_t)s_k : forced;  // lowest pages first
  // Keep every key above the threshold and the first take_equal keys equal to
  // it, in page order. Warp-major: warp w owns the pages [w*span, (w+1)*span)
  // (span a multiple of 32) and walks them 32 at a time with lane = page, so
  // the shared-memory key reads are consecutive; ballots give each lane the
  // number of equal and of chosen pages before it.
  const unsigned before_me = (1u << lane) - 1u;
  const int64_t span = ceil_div(ceil_div(n, (int64_t)warps), 32) * 32;
  const int64_t w_lo = min(n, warp * span), w_hi = min(n, w_lo + span);
  int64_t eq_local = 0;
  for (int64_t base = w_lo; base < w_hi; base += 32) {
    const int64_t pg = base + lane;
    eq_local += __popc(__ballot_sync(kFullMask, pg < w_hi && key_of(pg) == threshold));
  }
  int64_t eq_total;
  // lane 0 carries its warp's count; the other lanes take lane 0's prefix
  const int64_t eq_before = __shfl_sync(
      kFullMask, block_exclusive_scan<int64_t>(lane == 0 ? eq_local : 0, scan_scratch, &eq_total),
      0);
  // one step of the walk: is this lane's page chosen? (eq_run: equal keys before the step)
#define HS_TAKE(pg, eq_run, eq_mask)                                                     \
  ([&]() -> bool {                                                                       \
    const uint32_t key_ = (pg) < w_hi ? key_of(pg) : 0u;                                 \
    const bool eq_ = (pg) < w_hi && key_ == threshold;                                   \
    eq_mask = __ballot_sync(kFullMask, eq_);                                             \
    return ((pg) < w_hi && key_ > threshold) ||                                          \
           (eq_ && (eq_run) + __popc(eq_mask & before_me) < take_equal);                 \
  }())
  int64_t chosen_local = 0;
  {
    int64_t eq_run = eq_before;
    for (int64_t base = w_lo; base < w_hi; base += 32) {
      unsigned eq_mask;
      const bool t = HS_TAKE(base + lane, eq_run, eq_mask);
      chosen_local += __popc(__ballot_sync(kFullMask, t));
      eq_run += __popc(eq_mask);
    }
  }
  int64_t chosen_total;
  const int64_t chosen_before = __shfl_sync(
      kFullMask,
      block_exclusive_scan<int64_t>(lane == 0 ? chosen_local : 0, scan_scratch, &chosen_total),
      0);
  if (chosen_total <= kMaxChosenPages) {
    // the chosen pages by rank, then every thread writes tokens: coalesced
    // stores spread over the block instead of a page's tokens from one thread
    __shared__ int32_t chosen_pages[kMaxChosenPages];
    int64_t eq_run = eq_before, rank = chosen_before;
    for (int64_t base = w_lo; base < w_hi; base += 32) {
      unsigned eq_mask;
      const int64_t pg = base + lane;
      const bool t = HS_TAKE(pg, eq_run, eq_mask);
      const unsigned t_mask = __ballot_sync(kFullMask, t);
      if (t) chosen_pages[rank + __popc(t_mask & before_me)] = (int32_t)pg;
      rank += __popc(t_mask);
      eq_run += __popc(eq_mask);
    }
    __syncthreads();
    // 32-bit index arithmetic: max_pages * page_size <= INT32_MAX (host check)
    const uint32_t P = (uint32_t)p.page_size, tokens = (uint32_t)chosen_total * P;
    for (uint32_t t = tid; t < tokens; t += blockDim.x) {
      const uint32_t r = t / P;
      const int64_t tok = (int64_t)chosen_pages[r] * P + (t - r * P);
      out[t] = tok < length ? (int32_t)tok : -1;  // only the tail page is partial
    }
  } else {
    int64_t eq_run = eq_before, rank = chosen_before;
    for (int64_t base = w_lo; base < w_hi; base += 32) {
      unsigned eq_mask;
      const int64_t pg = base + lane;
      const bool t = HS_TAKE(pg, eq_run, eq_mask);
      const unsigned t_mask = __ballot_sync(kFullMask, t);
      if (t) {
        const int64_t r = rank + __popc(t_mask & before_me);
        const int64_t first = pg * p.page_size;
        const int64_t cnt = min((int64_t)p.page_size, length - first);
        for (int64_t i = 0; i < cnt; ++i) out[r * p.page_size + i] = (int32_t)(first + i);
      }
      rank += __popc(t_mask);
      eq_run += __popc(eq_mask);
    }
  }
#undef HS_TAKE
  // only the tail page (always chosen, always last) can be partial
  const int64_t count = (chosen_total - 1) * p.page_size + (length - (n - 1) * p.page_size);
  for (int64_t i = count + tid; i < p.capacity; i += blockDim.x) out[i] = -1;
  if (tid == 0) p.out_counts[b] = (int32_t)count;
}

// ---- the per-lane arithmetic of the fixed order ------------------------------
// Lane j of the L lanes that share a (page, KV head) row owns elements
// d = 8j .. 8j+7. For each of up to 4 query heads it adds the terms
// max(q*min, q*max) at even offsets left to right and those at odd offsets
// left to right, then even + odd; lane_reduce4 combines the L lanes by the xor
// tree. L = the smallest power of two >= ceil(head_dim / 8).
constexpr int kMaxQuestLanes = 32;

__host__ __device__ inline int quest_lanes(int head_dim) {
  int L = 1;
  while (L * 8 < head_dim) L *= 2;
  return L;
}

// Two packed 16-bit elements (element 2k in the low half) widened to fp32.
template <typename T> __device__ __forceinline__ float2 pair_f32(uint32_t w);
template <> __device__ __forceinline__ float2 pair_f32<__nv_bfloat16>(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <> __device__ __forceinline__ float2 pair_f32<__half>(uint32_t w) {
  __half2 h;
  *reinterpret_cast<uint32_t *>(&h) = w;
  return __half22float2(h);
}

// 16-bit q and metadata: q+ = max(q, 0) and q- = min(q, 0) as packed pairs
// (qa, qb: [head][pair]); one packed FMA serves the even and the odd term of a
// pair. max(q*min, q*max) = q+*max + q-*min exactly (products of 16-bit floats
// are exact in fp32, min <= max, one of q+ / q- is zero), so each term is one
// rounding of acc + term.
template <typename TKV>
__device__ __forceinline__ void score16(const uint4 &mn, const uint4 &mx, const float2 (&qa)[4][4],
                                        const float2 (&qb)[4][4], float (&v)[4]) {
  float2 acc[4];
#pragma unroll
  for (int h = 0; h < 4; ++h) acc[h] = make_float2(0.f, 0.f);
  const uint32_t lw[4] = {mn.x, mn.y, mn.z, mn.w}, hw[4] = {mx.x, mx.y, mx.z, mx.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 hi = pair_f32<TKV>(hw[k]), lo = pair_f32<TKV>(lw[k]);
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      acc[h] = __ffma2_rn(qa[h][k], hi, acc[h]);
      acc[h] = __ffma2_rn(qb[h][k], lo, acc[h]);
    }
  }
#pragma unroll
  for (int h = 0; h < 4; ++h) v[h] = __fadd_rn(acc[h].x, acc[h].y);
}

// Any other types: the terms computed and added one by one; `ne` of the 8
// elements exist (head_dim - 8j, clamped to [0, 8]).
__device__ __forceinline__ void score_f32(const float (&lo)[8], const float (&hi)[8], int ne,
                                          const float (&q)[4][8], float (&v)[4]) {
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (e < ne) {
        const float t = fmaxf(__fmul_rn(q[h][e], lo[e]), __fmul_rn(q[h][e], hi[e]));
        if (e & 1) b = e == 1 ? t : __fadd_rn(b, t);
        else a = e == 0 ? t : __fadd_rn(a, t);
      }
    }
    v[h] = ne > 1 ? __fadd_rn(a, b) : (ne == 1 ? a : 0.f);
  }
}

// Xor tree over the L lanes of a group for 4 values at once: the first two
// levels halve the values each lane keeps (recursive halving), the rest add
// whole values. Afterwards the lane holds kValues head sums, heads
// hbase .. hbase + kValues - 1; `writer` marks one lane per group and head.
template <int L> struct LaneReduce {
  static constexpr int kValues = L >= 4 ? 1 : (L == 2 ? 2 : 4);
  float out[kValues];
  int hbase;
  bool writer;
  __device__ __forceinline__ LaneReduce(const float (&v)[4], int lane) {
    float w[4] = {v[0], v[1], v[2], v[3]};
    hbase = 0;
    if constexpr (L >= 2) {
      constexpr int o = L / 2;
      const bool up = (lane & o) != 0;
      const float s0 = up ? w[0] : w[2], s1 = up ? w[1] : w[3];
      const float k0 = up ? w[2] : w[0], k1 = up ? w[3] : w[1];
      w[0] = __fadd_rn(k0, __shfl_xor_sync(kFullMask, s0, o));
      w[1] = __fadd_rn(k1, __shfl_xor_sync(kFullMask, s1, o));
      hbase = up ? 2 : 0;
    }
    if constexpr (L >= 4) {
      constexpr int o = L / 4;
      const bool up = (lane & o) != 0;
      const float sd = up ? w[0] : w[1], kp = up ? w[1] : w[0];
      w[0] = __fadd_rn(kp, __shfl_xor_sync(kFullMask, sd, o));
      hbase += up ? 1 : 0;
#pragma unroll
      for (int o2 = L / 8; o2 > 0; o2 >>= 1) w[0] = __fadd_rn(w[0], __shfl_xor_sync(kFullMask, w[0], o2));
      writer = (lane & (L / 4 - 1)) == 0;
    } else {
      writer = true;
    }
#pragma unroll
    for (int i = 0; i < kValues; ++i) out[i] = w[i];
  }
};

// ---- scoring ------------------------------------------------------------------------
template <typename TQ, typename TKV, int L>
__global__ void __launch_bounds__(kThreads, 2) quest_kernel(QuestParams<TQ, TKV> p) {
  extern __shared__ float head_sums[];  // [tile_pages][q_heads]
  __shared__ int s_last;
  constexpr bool kFma = is16<TQ>() && is16<TKV>();
  constexpr int kPass = 32 / L;   // pages a warp scores at once
  constexpr int kUnroll = 4;      // passes whose loads are in flight together
  const int b = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t length = p.lengths.at(b);
  const int64_t n = length > 0 ? ceil_div(length, p.page_size) : 0;
  const bool score = length > 0 && n <= p.max_pages && p.top_pages < n;
  const int64_t tile0 = (int64_t)blockIdx.x * p.tile_pages;
  const int D = p.head_dim, Hq = p.q_heads;
  if (score && tile0 < n) {
    const int64_t tile_n = min((int64_t)p.tile_pages, n - tile0);
    const int groups = Hq / p.kv_heads;
    const int chunks = (groups + kHeadsPerItem - 1) / kHeadsPerItem;
    const int passes = (int)ceil_div(tile_n, (int64_t)kPass);
    const TQ *q = p.query.at(b);
    const TKV *mn_base = p.minimum.at(b);
    const TKV *mx_base = p.maximum.at(b);
    const int pl = lane / L, j = lane % L, d0 = 8 * j;
    const int ne = D - d0 < 0 ? 0 : (D - d0 > 8 ? 8 : D - d0);
    const bool vec = ne == 8 && sizeof(TKV) == 2 && (D % 8) == 0 &&
                     ((reinterpret_cast<uintptr_t>(mn_base) | reinterpret_cast<uintptr_t>(mx_base)) & 15) == 0;
    // Each warp keeps one (KV head, head chunk) and its q slice in registers
    // while it walks the tile's pages, kPass pages per pass.
    for (int khc = warp; khc < p.kv_heads * chunks; khc += kWarps) {
      const int hc = khc % chunks, kh = khc / chunks;
      const int h_begin = kh * groups + hc * kHeadsPerItem;
      const int h_count = min(kHeadsPerItem, kh * groups + groups - h_begin);
      float qf[4][8];
#pragma unroll
      for (int h = 0; h < 4; ++h)
#pragma unroll
        for (int e = 0; e < 8; ++e)
          qf[h][e] = (h < h_count && e < ne) ? to_f32(q[(int64_t)(h_begin + h) * D + d0 + e]) : 0.f;
      float2 qa[4][4], qb[4][4];
#pragma unroll
      for (int h = 0; h < 4; ++h)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          qa[h][k] = make_float2(fmaxf(qf[h][2 * k], 0.f), fmaxf(qf[h][2 * k + 1], 0.f));
          qb[h][k] = make_float2(fminf(qf[h][2 * k], 0.f), fminf(qf[h][2 * k + 1], 0.f));
        }
      for (int ps0 = 0; ps0 < passes; ps0 += kUnroll) {
        // kUnroll passes' min/max slices, every load issued before any use
        uint4 lo_w[kUnroll], hi_w[kUnroll];
        float lo_f[kUnroll][8], hi_f[kUnroll][8];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int64_t lp = (int64_t)(ps0 + u) * kPass + pl;
          const bool in = ps0 + u < passes && lp < tile_n;
          const int64_t off = ((tile0 + lp) * p.kv_heads + kh) * D + d0;
          if constexpr (kFma) {
            if (vec) {
              lo_w[u] = in ? __ldg(reinterpret_cast<const uint4 *>(mn_base + off)) : make_uint4(0, 0, 0, 0);
              hi_w[u] = in ? __ldg(reinterpret_cast<const uint4 *>(mx_base + off)) : make_uint4(0, 0, 0, 0);
            } else {
              uint16_t lw[8], hw[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                lw[e] = (in && e < ne) ? reinterpret_cast<const uint16_t *>(mn_base)[off + e] : 0;
                hw[e] = (in && e < ne) ? reinterpret_cast<const uint16_t *>(mx_base)[off + e] : 0;
              }
              lo_w[u] = make_uint4(lw[0] | (uint32_t)lw[1] << 16, lw[2] | (uint32_t)lw[3] << 16,
                                   lw[4] | (uint32_t)lw[5] << 16, lw[6] | (uint32_t)lw[7] << 16);
              hi_w[u] = make_uint4(hw[0] | (uint32_t)hw[1] << 16, hw[2] | (uint32_t)hw[3] << 16,
                                   hw[4] | (uint32_t)hw[5] << 16, hw[6] | (uint32_t)hw[7] << 16);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              lo_f[u][e] = (in && e < ne) ? to_f32(mn_base[off + e]) : 0.f;
              hi_f[u][e] = (in && e < ne) ? to_f32(mx_base[off + e]) : 0.f;
            }
          }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          if (ps0 + u >= passes) break;  // warp-uniform
          float v[4];
          if constexpr (kFma) score16<TKV>(lo_w[u], hi_w[u], qa, qb, v);
          else score_f32(lo_f[u], hi_f[u], ne, qf, v);
          const LaneReduce<L> r(v, lane);
          const int64_t lp = (int64_t)(ps0 + u) * kPass + pl;
#pragma unroll
          for (int i = 0; i < LaneReduce<L>::kValues; ++i) {
            const int h = r.hbase + i;
            if (r.writer && h < h_count && lp < tile_n) head_sums[lp * Hq + h_begin + h] = r.out[i];
          }
        }
      }
    }
    __syncthreads();
    // per page: lane j adds heads j, j+32, ... then the xor tree; divide by q_heads
    for (int64_t lp = warp; lp < tile_n; lp += kWarps) {
      float u = 0.f;
      for (int h = lane; h < Hq; h += 32) u = __fadd_rn(u, head_sums[lp * Hq + h]);
      const float total = warp_xor_tree_sum(u);
      if (lane == 0)
        p.scores[(int64_t)b * p.max_pages + tile0 + lp] =
            p.partial ? total : __fdiv_rn(total, (float)Hq);
    }
  }
  if (p.partial) return;  // shard of a head-sharded selection: no top-k here
  // completion: the last CTA of this request selects
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&p.done[b], 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  select_request(p, b, length, n, reinterpret_cast<uint32_t *>(head_sums));
  if (threadIdx.x == 0) p.done[b] = 0;  // ready for the next call
}

// ---- TMA-staged path (16-bit data, page rows a multiple of 16 bytes) ----------
//
// One CTA of 16 warps per SM streams a tile of one request's pages through a
// 3-stage ring of shared-memory buffers. Thread 0 issues, per stage, two 1-D
// bulk copies (cp.async.bulk, min and max of 16 consecutive pages: one
// contiguous range each) that complete on the stage's mbarrier; every warp
// waits on that barrier, computes its (KV head, 4 heads, 8 pages) item from
// shared memory, and the CTA barrier at the end of a stage hands the buffer
// back to the producer. The arithmetic and its order are those of
// quest_kernel; head sums are double buffered so a stage's per-page combine
// overlaps the next stage's compute.
constexpr int kTmaThreads = 512;
constexpr int kTmaWarps = kTmaThreads / 32;
constexpr int kTmaStagePages = 16;
constexpr int kTmaStages = 3;
template <typename TQ, typename TKV, int D>
__global__ void __launch_bounds__(kTmaThreads, 1) quest_tma_kernel(QuestParams<TQ, TKV> p) {
  extern __shared__ __align__(128) char smem[];
  __shared__ __align__(8) uint64_t full[kTmaStages];
  __shared__ int s_last, s_ok;
  const int b = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t length = p.lengths.at(b);
  const int64_t n = length > 0 ? ceil_div(length, p.page_size) : 0;
  const bool score = length > 0 && n <= p.max_pages && p.top_pages < n;
  const int64_t tile0 = (int64_t)blockIdx.x * p.tile_pages;
  const int Hq = p.q_heads, Hkv = p.kv_heads;
  const int64_t page_elems = (int64_t)Hkv * D;
  const unsigned page_bytes = (unsigned)(page_elems * sizeof(TKV));
  const size_t stage_bytes = (size_t)2 * kTmaStagePages * page_bytes;
  float *sums = reinterpret_cast<float *>(smem + kTmaStages * stage_bytes);  // [2][16][Hq]
  if (tid == 0) s_ok = 1;
  if (score && tile0 < n) {
    const int64_t tile_n = min((int64_t)p.tile_pages, n - tile0);
    const int nstages = (int)ceil_div(tile_n, kTmaStagePages);
    const TKV *mn_base = p.minimum.at(b) + tile0 * page_elems;
    const TKV *mx_base = p.maximum.at(b) + tile0 * page_elems;
    if (((reinterpret_cast<uintptr_t>(mn_base) | reinterpret_cast<uintptr_t>(mx_base)) & 15) != 0) {
      // bulk copies need 16-byte aligned sources; the callers guarantee it
      if (tid == 0) flag(p.status, HS_DEV_MISALIGNED);
      goto done;
    }
    auto issue = [&](int g) {
      char *buf = smem + (g % kTmaStages) * stage_bytes;
      const int64_t pages = min((int64_t)kTmaStagePages, tile_n - (int64_t)g * kTmaStagePages);
      const unsigned bytes = (unsigned)(pages * page_bytes);
      mbar_expect_tx(&full[g % kTmaStages], 2 * bytes);
      bulk_copy(buf, mn_base + (int64_t)g * kTmaStagePages * page_elems, bytes,
                &full[g % kTmaStages]);
      bulk_copy(buf + kTmaStagePages * page_bytes,
                mx_base + (int64_t)g * kTmaStagePages * page_elems, bytes, &full[g % kTmaStages]);
    };
    if (tid == 0) {
      for (int s = 0; s < kTmaStages; ++s) mbar_init(&full[s], 1);
      asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();
    if (tid == 0)
      for (int g = 0; g < kTmaStages && g < nstages; ++g) issue(g);

    const int groups = Hq / Hkv;
    const int chunks = (groups + kHeadsPerItem - 1) / kHeadsPerItem;
    constexpr int L = D / 8;                            // lanes per page row (4, 8 or 16)
    constexpr int kPass = 32 / L;                       // pages per warp pass
    constexpr int kPassesPerStage = kTmaStagePages / kPass;
    const int roles = Hkv * chunks;
    const int items = roles * kPassesPerStage;
    const TQ *q = p.query.at(b);
    const int pl = lane / L, d0 = 8 * (lane % L);
    const int role0 = warp % roles, pass0 = warp / roles;
    const int role_step = kTmaWarps % roles, pass_step = kTmaWarps / roles;
    int cur = -1, hc = 0, kh = 0, h_begin = 0, h_count = 0;
    // q+ and q- of the item's 4 heads as packed (even, odd) pairs, loaded when
    // the warp's (KV head, head chunk) changes
    float2 qa[4][4], qb[4][4];
    for (int g = 0; g < nstages; ++g) {
      const int64_t pages = min((int64_t)kTmaStagePages, tile_n - (int64_t)g * kTmaStagePages);
      const char *buf = smem + (g % kTmaStages) * stage_bytes;
      const TKV *lo_s = reinterpret_cast<const TKV *>(buf);
      const TKV *hi_s = reinterpret_cast<const TKV *>(buf + kTmaStagePages * page_bytes);
      float *stage_sums = sums + (g & 1) * kTmaStagePages * Hq;
      const bool ready = mbar_wait(&full[g % kTmaStages], (g / kTmaStages) & 1, p.status);
      if (!ready) s_ok = 0;
      // item = pass * roles + role: with roles dividing the warp count a warp
      // keeps one role (and its q registers) for the whole tile. role and pass
      // advance incrementally (no division per item).
      int role = role0, pass = pass0;
      for (int item = warp; ready && item < items; item += kTmaWarps) {
        if (role != cur) {
          cur = role;
          hc = role % chunks;
          kh = role / chunks;
          h_begin = kh * groups + hc * kHeadsPerItem;
          h_count = min(kHeadsPerItem, kh * groups + groups - h_begin);
#pragma unroll
          for (int h = 0; h < 4; ++h)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              float x0 = 0.f, x1 = 0.f;
              if (h < h_count) {
                x0 = to_f32(q[(int64_t)(h_begin + h) * D + d0 + 2 * k]);
                x1 = to_f32(q[(int64_t)(h_begin + h) * D + d0 + 2 * k + 1]);
              }
              qa[h][k] = make_float2(fmaxf(x0, 0.f), fmaxf(x1, 0.f));
              qb[h][k] = make_float2(fminf(x0, 0.f), fminf(x1, 0.f));
            }
        }
        // Pages past the tile's last page hold stale data; their sums are
        // never stored (lp < pages below), so the loads need no predicate.
        const int lp = pass * kPass + pl;
        const int off = lp * (int)page_elems + kh * D + d0;
        const uint4 lo = *reinterpret_cast<const uint4 *>(lo_s + off);
        const uint4 hi = *reinterpret_cast<const uint4 *>(hi_s + off);
        float v[4];
        score16<TKV>(lo, hi, qa, qb, v);
        const LaneReduce<L> r(v, lane);
        if (r.writer && r.hbase < h_count && lp < pages)
          stage_sums[lp * Hq + h_begin + r.hbase] = r.out[0];
        role += role_step;
        pass += pass_step;
        if (role >= roles) {
          role -= roles;
          ++pass;
        }
      }
      __syncthreads();  // buffer g % kTmaStages consumed; stage sums complete
      if (tid == 0 && s_ok && g + kTmaStages < nstages) issue(g + kTmaStages);
      // per page: lane j adds heads j, j+32, ... then the xor tree; divide by q_heads
      for (int lp = warp; lp < pages; lp += kTmaWarps) {
        float u = 0.f;
        for (int h = lane; h < Hq; h += 32) u = __fadd_rn(u, stage_sums[lp * Hq + h]);
        const float total = warp_xor_tree_sum(u);
        if (lane == 0)
          p.scores[(int64_t)b * p.max_pages + tile0 + (int64_t)g * kTmaStagePages + lp] =
              p.partial ? total : __fdiv_rn(total, (float)Hq);
      }
      if (!s_ok) {
        // a copy never completed: wait (bounded) for the stages still in
        // flight, so no copy lands in shared memory after this CTA exits
        for (int gg = g + 1; gg < nstages && gg < g + kTmaStages; ++gg)
          mbar_wait(&full[gg % kTmaStages], (gg / kTmaStages) & 1, p.status);
        break;
      }
    }
  }
done:
  if (p.partial) return;  // shard of a head-sharded selection: no top-k here
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&p.done[b], 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int64_t cap_keys = (int64_t)(kTmaStages * stage_bytes / sizeof(uint32_t));
  select_request(p, b, length, n, n <= cap_keys ? reinterpret_cast<uint32_t *>(smem) : nullptr);
  if (tid == 0) p.done[b] = 0;
}

// Head-sharded selection, second half: the shards' per-page head sums are
// added in shard order (left to right, fp32), divided by the total query
// heads, and the usual top-k + expansion runs on the result — the same tokens
// on every rank. With one shard this equals the unsharded selection bit for
// bit (0 + s = s, and the same division).
constexpr int kSelectThreads = 512;

__global__ void __launch_bounds__(kSelectThreads, 1)
    select_partials_kernel(QuestParams<float, float> p, const float *partials, int shards) {
  extern __shared__ uint32_t key_cache[];
  const int b = blockIdx.x;
  const int64_t length = p.lengths.at(b);
  const int64_t n = length > 0 ? ceil_div(length, (int64_t)p.page_size) : 0;
  float *sc = p.scores + (int64_t)b * p.max_pages;
  if (n <= p.max_pages) {
    // four pages per thread at a time, their shard loads all in flight
    for (int64_t pg0 = threadIdx.x; pg0 < n; pg0 += 4 * (int64_t)blockDim.x) {
      float total[4] = {0.f, 0.f, 0.f, 0.f};
      for (int r = 0; r < shards; ++r) {
        const float *row = partials + ((int64_t)r * p.batch + b) * p.max_pages;
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t pg = pg0 + (int64_t)u * blockDim.x;
          v[u] = pg < n ? __ldcg(row + pg) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) total[u] = __fadd_rn(total[u], v[u]);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t pg = pg0 + (int64_t)u * blockDim.x;
        if (pg < n) sc[pg] = __fdiv_rn(total[u], (float)p.q_heads);
      }
    }
  }
  __syncthreads();
  select_request(p, b, length, n, n <= kSmemKeys ? key_cache : nullptr);
}

// ---- cluster select: one request's top-k spread over a thread-block cluster -----
//
// For long requests the single-CTA selection above is latency-bound (one SM
// walks every page several times). Here a cluster of kSelectCluster CTAs
// shares one request: CTA r owns a contiguous chunk of its pages (a multiple
// of 32), turns the shard partials into keys in its shared memory (the same
// shard-ordered fp32 sum and division as select_partials_kernel), and each
// radix pass counts the chunk into a local histogram that every CTA then sums
// over the cluster through distributed shared memory, so all CTAs take the
// same digit. The final walk needs only per-CTA totals of keys above and equal
// to the threshold: the chosen pages before any position are those above it
// plus min(equal ones before it, take_equal). Same selection and token order
// as select_request, bit for bit.
//
// Every CTA of a cluster takes the same branch (one request) and so reaches
// the same cluster barriers: one before the first remote read, one per radix
// pass (histograms double-buffered, so a pass never clears a buffer a peer may
// still read), one before the CTA totals are read, one before exit.
constexpr int kSelectCluster = 8;                 // CTAs per request (portable cluster size)
constexpr int kClusterSelectThreads = 512;
constexpr int64_t kClusterSelectMinPages = 4096;  // shorter tables: one CTA is as fast
constexpr int64_t kClusterChunkMax = 8192;        // pages per CTA: 32 KiB keys + 32 KiB chosen

__global__ void __launch_bounds__(kClusterSelectThreads, 1)
    select_cluster_kernel(QuestParams<float, float> p, const float *partials, int shards,
                          int64_t chunk_cap) {
  extern __shared__ __align__(16) uint32_t cs_keys[];  // [chunk_cap] keys, [chunk_cap] chosen
  __shared__ uint32_t hist[2][256];
  __shared__ uint32_t ghist[256];
  __shared__ int64_t scan_scratch[33];
  __shared__ uint32_t s_lo, s_hi, g_lo, g_hi, s_prefix, s_mask, s_k;
  __shared__ long long s_eq_total, s_gt_total;  // this CTA's counts, read by the peers
  __shared__ long long s_eq_before, s_gt_before;
  constexpr uint32_t kForcedKey = 0xffffffffu;
  const unsigned S = kSelectCluster, rank = cluster_rank();
  const int b = (int)(blockIdx.x / S);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, warps = (int)(blockDim.x >> 5);
  const int64_t ctid = (int64_t)rank * blockDim.x + tid, cthreads = (int64_t)S * blockDim.x;
  const int64_t length = p.lengths.at(b);
  const int64_t n = length > 0 ? ceil_div(length, (int64_t)p.page_size) : 0;
  const int64_t P = p.page_size;
  int32_t *out = p.out_tokens + (int64_t)b * p.capacity;
  if (length <= 0 || n > p.max_pages || p.top_pages >= n) {
    // no ranking (same results as select_request); no shared memory is shared
    const bool all = length > 0 && n <= p.max_pages;
    if (n > p.max_pages && ctid == 0) flag(p.status, HS_DEV_PAGES_EXCEED_TABLE);
    for (int64_t i = ctid; i < p.capacity; i += cthreads)
      out[i] = all && i < length ? (int32_t)i : -1;
    if (ctid == 0) p.out_counts[b] = all ? (int32_t)length : 0;
    return;
  }
  const bool sink = p.keep_sink && p.top_pages > 1 && n > 1;
  const int forced = sink ? 2 : 1;
  const int64_t chunk = ceil_div(ceil_div(n, (int64_t)S), (int64_t)32) * 32;  // <= chunk_cap
  const int64_t c_lo = min(n, (int64_t)rank * chunk), c_len = min(n, c_lo + chunk) - c_lo;
  uint32_t *keys = cs_keys;
  int32_t *chosen = reinterpret_cast<int32_t *>(cs_keys + chunk_cap);
  if (tid == 0) {
    s_lo = 0xffffffffu;
    s_hi = 0u;
  }
  __syncthreads();
  {
    uint32_t lo = 0xffffffffu, hi = 0u;
    for (int64_t i0 = tid; i0 < c_len; i0 += 4 * (int64_t)blockDim.x) {
      float total[4] = {0.f, 0.f, 0.f, 0.f};
      for (int r = 0; r < shards; ++r) {
        const float *row = partials + ((int64_t)r * p.batch + b) * p.max_pages + c_lo;
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t i = i0 + (int64_t)u * blockDim.x;
          v[u] = i < c_len ? __ldcg(row + i) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) total[u] = __fadd_rn(total[u], v[u]);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t i = i0 + (int64_t)u * blockDim.x, pg = c_lo + i;
        if (i < c_len) {
          const bool is_forced = pg == n - 1 || (sink && pg == 0);
          const uint32_t key =
              is_forced ? kForcedKey : score_key(__fdiv_rn(total[u], (float)p.q_heads));
          keys[i] = key;
          if (!is_forced) {
            lo = min(lo, key);
            hi = max(hi, key);
          }
        }
      }
    }
    lo = __reduce_min_sync(kFullMask, lo);
    hi = __reduce_max_sync(kFullMask, hi);
    if (lane == 0) {
      atomicMin(&s_lo, lo);
      atomicMax(&s_hi, hi);
    }
  }
  cluster_barrier();  // keys and every CTA's key range are complete
  if (tid == 0) {
    uint32_t lo = 0xffffffffu, hi = 0u;
    for (unsigned r = 0; r < S; ++r) {
      lo = min(lo, *map_rank(&s_lo, r));
      hi = max(hi, *map_rank(&s_hi, r));
    }
    g_lo = lo;
    g_hi = hi;
  }
  __syncthreads();
  const uint32_t rest = (uint32_t)(p.top_pages - forced);  // < the unforced pages
  const uint32_t differ = g_lo ^ g_hi;
  const int top_bit = differ ? 31 - __clz((int)differ) : -1;
  if (tid == 0) {
    const uint32_t common =
        top_bit < 0 ? 0xffffffffu : top_bit < 31 ? ~((2u << top_bit) - 1u) : 0u;
    s_prefix = g_hi & common;
    s_mask = common;
    s_k = rest;
  }
  __syncthreads();
  int pass = 0;
  for (int high = rest > 0 ? top_bit : -1; high >= 0; high -= 8, ++pass) {
    const int shift = high >= 7 ? high - 7 : 0;
    const uint32_t digit_mask = (2u << (high - shift)) - 1u;
    uint32_t *h = hist[pass & 1];
    for (int i = tid; i < 256; i += blockDim.x) h[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    for (int64_t i = tid; i < c_len; i += blockDim.x) {
      const uint32_t key = keys[i];
      if (key != kForcedKey && (key & mask) == prefix)
        atomicAdd(&h[(key >> shift) & digit_mask], 1u);
    }
    cluster_barrier();  // every CTA's histogram of this pass is complete
    for (int d = tid; d < 256; d += blockDim.x) {
      uint32_t sum = 0;
      for (unsigned r = 0; r < S; ++r) sum += *map_rank(&h[d], r);
      ghist[d] = sum;
    }
    __syncthreads();
    if (tid < 32) pick_digit(ghist, prefix, mask, shift, digit_mask, &s_prefix, &s_mask, &s_k);
    __syncthreads();
  }
  const uint32_t threshold = rest > 0 ? s_prefix : kForcedKey;
  const int64_t take_equal = rest > 0 ? (int64_t)s_k : forced;
  // per warp: keys equal to and above the threshold in its span of the chunk
  const unsigned before_me = (1u << lane) - 1u;
  const int64_t span = ceil_div(ceil_div(c_len, (int64_t)warps), (int64_t)32) * 32;
  const int64_t w_lo = min(c_len, warp * span), w_hi = min(c_len, w_lo + span);
  int64_t eq_local = 0, gt_local = 0;
  for (int64_t base = w_lo; base < w_hi; base += 32) {
    const int64_t i = base + lane;
    const uint32_t key = i < w_hi ? keys[i] : 0u;
    eq_local += __popc(__ballot_sync(kFullMask, i < w_hi && key == threshold));
    gt_local += __popc(__ballot_sync(kFullMask, i < w_hi && key > threshold));
  }
  int64_t eq_cta, gt_cta;
  const int64_t eq_in = __shfl_sync(
      kFullMask, block_exclusive_scan<int64_t>(lane == 0 ? eq_local : 0, scan_scratch, &eq_cta),
      0);
  const int64_t gt_in = __shfl_sync(
      kFullMask, block_exclusive_scan<int64_t>(lane == 0 ? gt_local : 0, scan_scratch, &gt_cta),
      0);
  if (tid == 0) {
    s_eq_total = eq_cta;
    s_gt_total = gt_cta;
  }
  cluster_barrier();  // every CTA's totals are published
  if (tid == 0) {
    long long eq = 0, gt = 0;
    for (unsigned r = 0; r < rank; ++r) {
      eq += *map_rank(&s_eq_total, r);
      gt += *map_rank(&s_gt_total, r);
    }
    s_eq_before = eq;
    s_gt_before = gt;
  }
  __syncthreads();
  const int64_t eq_cta_before = s_eq_before, gt_cta_before = s_gt_before;
  const int64_t chosen_cta_before = gt_cta_before + min(eq_cta_before, take_equal);
  const int64_t chosen_cta =
      gt_cta_before + gt_cta + min(eq_cta_before + eq_cta, take_equal) - chosen_cta_before;
  {
    int64_t eq_run = eq_cta_before + eq_in;
    int64_t at = gt_cta_before + gt_in + min(eq_run, take_equal) - chosen_cta_before;
    for (int64_t base = w_lo; base < w_hi; base += 32) {
      const int64_t i = base + lane;
      const uint32_t key = i < w_hi ? keys[i] : 0u;
      const bool eq = i < w_hi && key == threshold;
      const unsigned eq_mask = __ballot_sync(kFullMask, eq);
      const bool take = (i < w_hi && key > threshold) ||
                        (eq && eq_run + __popc(eq_mask & before_me) < take_equal);
      const unsigned t_mask = __ballot_sync(kFullMask, take);
      if (take) chosen[at + __popc(t_mask & before_me)] = (int32_t)(c_lo + i);
      at += __popc(t_mask);
      eq_run += __popc(eq_mask);
    }
  }
  __syncthreads();
  // this CTA's chosen pages hold ranks [chosen_cta_before, +chosen_cta) of the selection
  {
    const uint32_t Pu = (uint32_t)P, tokens = (uint32_t)chosen_cta * Pu;
    int32_t *dst = out + chosen_cta_before * P;
    for (uint32_t t = tid; t < tokens; t += blockDim.x) {
      const uint32_t r = t / Pu;
      const int64_t tok = (int64_t)chosen[r] * P + (t - r * Pu);
      dst[t] = tok < length ? (int32_t)tok : -1;  // only the tail page is partial
    }
  }
  const int64_t count = (int64_t)(p.top_pages - 1) * P + (length - (n - 1) * P);
  for (int64_t i = count + ctid; i < p.capacity; i += cthreads) out[i] = -1;
  if (ctid == 0) p.out_counts[b] = (int32_t)count;
  cluster_barrier();  // no CTA exits while a peer may still read its shared memory
}

// Whether clusters of kSelectCluster select CTAs with `smem` bytes of dynamic
// shared memory fit the device; asked once per device (the answer is kept for
// the largest size that fits).
bool select_cluster_fits(size_t smem) {
  static std::mutex lock;
  static size_t fits[64];  // largest dynamic shared memory known to fit, per device
  static bool asked[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  std::lock_guard<std::mutex> guard(lock);
  if (asked[dev]) return smem <= fits[dev];
  asked[dev] = true;
  const size_t most = 2 * (size_t)kClusterChunkMax * sizeof(uint32_t);
  if (reserve_smem((const void *)select_cluster_kernel, most, "quest select") != HS_OK) {
    cudaGetLastError();
    return false;
  }
  cudaLaunchConfig_t config{};
  config.gridDim = dim3((unsigned)kSelectCluster);
  config.blockDim = dim3(kClusterSelectThreads);
  config.dynamicSmemBytes = most;
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = (unsigned)kSelectCluster;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  config.attrs = &attr;
  config.numAttrs = 1;
  int clusters = 0;
  const bool ok = cudaOccupancyMaxActiveClusters(&clusters, (const void *)select_cluster_kernel,
                                                 &config) == cudaSuccess &&
                  clusters > 0;
  cudaGetLastError();
  fits[dev] = ok ? most : 0;
  return ok && smem <= most;
}

// Pages per CTA of the cluster select for a table of `max_pages`, or 0 when the
// single-CTA select is used (short tables, or tables beyond the chunk limit).
int64_t select_cluster_chunk(int64_t max_pages) {
  if (max_pages < kClusterSelectMinPages) return 0;
  const int64_t chunk = ceil_div(ceil_div(max_pages, (int64_t)kSelectCluster), (int64_t)32) * 32;
  if (chunk > kClusterChunkMax) return 0;
  return select_cluster_fits(2 * (size_t)chunk * sizeof(uint32_t)) ? chunk : 0;
}

int launch_select_cluster(const QuestParams<float, float> &p, const float *partials, int shards,
                          int64_t chunk, cudaStream_t stream) {
  cudaLaunchConfig_t config{};
  config.gridDim = dim3((unsigned)(p.batch * kSelectCluster));
  config.blockDim = dim3(kClusterSelectThreads);
  config.dynamicSmemBytes = 2 * (size_t)chunk * sizeof(uint32_t);
  config.stream = stream;
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = (unsigned)kSelectCluster;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  config.attrs = &attr;
  config.numAttrs = 1;
  const cudaError_t err =
      cudaLaunchKernelEx(&config, select_cluster_kernel, p, partials, shards, chunk);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return set_error(HS_ERR_CUDA, "select_cluster_kernel: launch failed: %s",
                     cudaGetErrorString(err));
  }
  return HS_OK;
}

int launch_select_partials(int shards, const float *partials, int batch, const int32_t *lengths,
                           int q_heads, int64_t max_pages, int page_size, int top_pages,
                           int keep_sink, int32_t *out_tokens, int64_t capacity,
                           int32_t *out_counts, float *scores, int32_t *status,
                           cudaStream_t stream) {
  QuestParams<float, float> p{};
  p.batch = batch;
  p.lengths = Lengths{lengths, 0};
  p.q_heads = q_heads;
  p.page_size = page_size;
  p.top_pages = top_pages;
  p.keep_sink = keep_sink;
  p.max_pages = max_pages;
  p.scores = scores;
  p.out_tokens = out_tokens;
  p.capacity = capacity;
  p.out_counts = out_counts;
  p.status = status;
  const int64_t chunk = select_cluster_chunk(max_pages);
  if (chunk > 0) return launch_select_cluster(p, partials, shards, chunk, stream);
  const size_t smem = (size_t)(max_pages < kSmemKeys ? max_pages : kSmemKeys) * sizeof(uint32_t);
  const int rc = reserve_smem((const void *)select_partials_kernel, smem, "quest select");
  if (rc != HS_OK) return rc;
  select_partials_kernel<<<batch, kSelectThreads, smem, stream>>>(p, partials, shards);
  return check_launch("select_partials_kernel");
}

int tile_pages_for(int batch, int64_t max_pages) {
  const int64_t target_ctas = (int64_t)sm_count() * 3 * 2;  // two waves at 3 CTAs per SM
  int64_t per_req = ceil_div(target_ctas, batch);
  if (per_req < 1) per_req = 1;
  int64_t tile = ceil_div(max_pages, per_req);
  tile = ceil_div(tile, kPagesPerItem) * kPagesPerItem;
  if (tile < kPagesPerItem) tile = kPagesPerItem;
  if (tile > 256) tile = 256;
  return (int)tile;
}

template <typename TQ, typename TKV>
int launch_tma(QuestParams<TQ, TKV> &p, cudaStream_t stream) {
  const size_t page_bytes = (size_t)p.kv_heads * p.head_dim * sizeof(TKV);
  const size_t smem = kTmaStages * 2 * kTmaStagePages * page_bytes +
                      2 * kTmaStagePages * (size_t)p.q_heads * sizeof(float);
  int64_t per_req = sm_count() / p.batch;
  if (per_req < 1) per_req = 1;
  int64_t tile = ceil_div(p.max_pages, per_req);
  tile = ceil_div(tile, kTmaStagePages) * kTmaStagePages;
  p.tile_pages = (int)tile;
  dim3 grid((unsigned)ceil_div(p.max_pages, tile), (unsigned)p.batch);
#define HS_QUEST_TMA(DD)                                                                  \
  case DD: {                                                                              \
    auto k = quest_tma_kernel<TQ, TKV, DD>;                                               \
    const int rc = reserve_smem((const void *)k, smem, "quest");                          \
    if (rc != HS_OK) return rc;                                                           \
    k<<<grid, kTmaThreads, smem, stream>>>(p);                                            \
    break;                                                                                \
  }
  switch (p.head_dim) {
    HS_QUEST_TMA(32)
    HS_QUEST_TMA(64)
    HS_QUEST_TMA(128)
    default:
      return set_error(HS_ERR_UNSUPPORTED, "quest: no staged path for head_dim %d", p.head_dim);
  }
#undef HS_QUEST_TMA
  return check_launch("quest_tma_kernel");
}

// The staged path needs 16-bit data, head_dim 32, 64 or 128 (whole 16-byte
// lane slices), 16-byte aligned metadata and a ring that fits shared memory;
// other shapes use quest_kernel.
template <typename TQ, typename TKV>
bool tma_eligible(const QuestParams<TQ, TKV> &p, bool aligned) {
  const size_t page_bytes = (size_t)p.kv_heads * p.head_dim * sizeof(TKV);
  const size_t smem = kTmaStages * 2 * kTmaStagePages * page_bytes +
                      2 * kTmaStagePages * (size_t)p.q_heads * sizeof(float);
  return is16<TQ>() && is16<TKV>() && aligned && page_bytes % 16 == 0 &&
         smem <= 200 * 1024 && (p.head_dim == 32 || p.head_dim == 64 || p.head_dim == 128);
}

template <typename TQ, typename TKV>
int launch(QuestParams<TQ, TKV> &p, cudaStream_t stream, bool aligned) {
  if constexpr (is16<TQ>() && is16<TKV>()) {
    if (tma_eligible(p, aligned)) return launch_tma(p, stream);
  }
  p.tile_pages = tile_pages_for(p.batch, p.max_pages);
  const size_t sums_bytes = (size_t)p.tile_pages * p.q_heads * sizeof(float);
  const size_t keys_bytes =
      (size_t)(p.max_pages < kSmemKeys ? p.max_pages : kSmemKeys) * sizeof(uint32_t);
  const size_t smem = sums_bytes > keys_bytes ? sums_bytes : keys_bytes;
  dim3 grid((unsigned)ceil_div(p.max_pages, p.tile_pages), (unsigned)p.batch);
#define HS_QUEST_CASE(LL)                                                                 \
  case LL: {                                                                              \
    auto k = quest_kernel<TQ, TKV, LL>;                                                   \
    const int rc = reserve_smem((const void *)k, smem, "quest");                          \
    if (rc != HS_OK) return rc;                                                           \
    k<<<grid, kThreads, smem, stream>>>(p);                                               \
    break;                                                                                \
  }
  if (p.head_dim > 8 * kMaxQuestLanes)
    return set_error(HS_ERR_UNSUPPORTED, "quest: head_dim %d > 256 is not supported",
                     p.head_dim);
  switch (quest_lanes(p.head_dim)) {
    HS_QUEST_CASE(1)
    HS_QUEST_CASE(2)
    HS_QUEST_CASE(4)
    HS_QUEST_CASE(8)
    HS_QUEST_CASE(16)
    HS_QUEST_CASE(32)
    default:
      return set_error(HS_ERR_UNSUPPORTED, "quest: head_dim %d is not supported", p.head_dim);
  }
#undef HS_QUEST_CASE
  return check_launch("quest_kernel");
}

struct Common {
  int batch;
  const void *query;
  int64_t qstride;
  int query_dtype;
  const void *mn, *mx;
  const uint64_t *mn_ptrs, *mx_ptrs;
  int kv_dtype;
  Lengths lengths;
  int q_heads, kv_heads, head_dim, page_size, top_pages, keep_sink;
  int64_t max_pages;
  int32_t *out_tokens;
  int64_t capacity;
  int32_t *out_counts;
  void *workspace;
  size_t workspace_bytes;
  int32_t *status;
  float *partial_out;  // head-sharded selection: per-page head sums of this shard
};

template <typename TQ, typename TKV> int run(const Common &c, cudaStream_t stream) {
  QuestParams<TQ, TKV> p;
  p.batch = c.batch;
  p.query = Batched<TQ>{static_cast<const TQ *>(c.query), c.qstride, nullptr};
  p.minimum = Batched<TKV>{static_cast<const TKV *>(c.mn), 0, c.mn_ptrs};
  p.maximum = Batched<TKV>{static_cast<const TKV *>(c.mx), 0, c.mx_ptrs};
  p.lengths = c.lengths;
  p.q_heads = c.q_heads;
  p.kv_heads = c.kv_heads;
  p.head_dim = c.head_dim;
  p.page_size = c.page_size;
  p.top_pages = c.top_pages;
  p.keep_sink = c.keep_sink;
  p.max_pages = c.max_pages;
  if (c.partial_out != nullptr) {
    p.scores = c.partial_out;
    p.done = nullptr;
    p.partial = 1;
  } else {
    p.scores = static_cast<float *>(c.workspace);
    p.done = reinterpret_cast<unsigned *>(static_cast<char *>(c.workspace) +
                                          (size_t)c.batch * c.max_pages * sizeof(float));
    p.partial = 0;
  }
  p.out_tokens = c.out_tokens;
  p.capacity = c.capacity;
  p.out_counts = c.out_counts;
  p.status = c.status;
  // pointer arrays (batched calls) are required to be 16-byte aligned
  const bool aligned = c.mn_ptrs != nullptr ||
                       ((reinterpret_cast<uintptr_t>(c.mn) | reinterpret_cast<uintptr_t>(c.mx)) &
                        15) == 0;
  // Long tables with few requests: score in partial mode (undivided head sums
  // into the workspace) and rank over a cluster per request, one wave of CTAs.
  // One shard's sum is the head sum itself (0 + s = s), so the keys, and the
  // selection, are those of the fused path bit for bit.
  const int64_t chunk = p.partial || (int64_t)c.batch * kSelectCluster > sm_count()
                            ? 0
                            : select_cluster_chunk(c.max_pages);
  if (chunk == 0) return launch<TQ, TKV>(p, stream, aligned);
  p.partial = 1;
  p.done = nullptr;
  const int rc = launch<TQ, TKV>(p, stream, aligned);
  if (rc != HS_OK) return rc;
  QuestParams<float, float> s{};
  s.batch = c.batch;
  s.lengths = c.lengths;
  s.q_heads = c.q_heads;
  s.page_size = c.page_size;
  s.top_pages = c.top_pages;
  s.keep_sink = c.keep_sink;
  s.max_pages = c.max_pages;
  s.out_tokens = c.out_tokens;
  s.capacity = c.capacity;
  s.out_counts = c.out_counts;
  s.status = c.status;
  return launch_select_cluster(s, p.scores, 1, chunk, stream);
}

template <typename TQ> int dispatch_kv(const Common &c, cudaStream_t s) {
  switch (c.kv_dtype) {
    case HS_FLOAT32: return run<TQ, float>(c, s);
    case HS_FLOAT16: return run<TQ, __half>(c, s);
    case HS_BFLOAT16: return run<TQ, __nv_bfloat16>(c, s);
  }
  return set_error(HS_ERR_INVALID_ARGUMENT, "quest: invalid KV dtype %d", c.kv_dtype);
}

int quest_common(const Common &c, cudaStream_t stream) {
  if (c.batch < 1 || c.q_heads < 1 || c.kv_heads < 1 || c.head_dim < 1 || c.page_size < 1 ||
      c.max_pages < 1)
    return set_error(HS_ERR_INVALID_ARGUMENT, "quest: dimensions must be positive");
  const bool partial = c.partial_out != nullptr;
  if ((!partial && c.top_pages < 1) || c.q_heads % c.kv_heads)
    return set_error(HS_ERR_INVALID_ARGUMENT, "invalid page budget or GQA shape");
  if (c.head_dim > 256)
    return set_error(HS_ERR_UNSUPPORTED, "quest: head_dim %d > 256 is not supported",
                     c.head_dim);
  if (!c.query || (!partial && (!c.out_tokens || !c.out_counts)) || (!c.mn && !c.mn_ptrs) ||
      (!c.mx && !c.mx_ptrs))
    return set_error(HS_ERR_INVALID_ARGUMENT, "quest: null tensor pointer");
  if (partial) {
    if (c.max_pages * (int64_t)c.page_size > INT32_MAX)
      return set_error(HS_ERR_INVALID_ARGUMENT, "quest: token positions must fit int32");
  } else if (c.capacity < (int64_t)c.top_pages * c.page_size)
    return set_error(HS_ERR_INVALID_ARGUMENT,
                     "quest: out_capacity %lld < top_pages * page_size = %lld",
                     (long long)c.capacity, (long long)c.top_pages * c.page_size);
  if (c.capacity > INT32_MAX || c.max_pages * (int64_t)c.page_size > INT32_MAX)
    return set_error(HS_ERR_INVALID_ARGUMENT, "quest: token positions must fit int32");
  if ((size_t)tile_pages_for(c.batch, c.max_pages) * c.q_heads * sizeof(float) > 200 * 1024)
    return set_error(HS_ERR_UNSUPPORTED, "quest: %d query heads do not fit shared memory",
                     c.q_heads);
  const size_t need = hs_quest_workspace_bytes(c.batch, c.max_pages);
  if (!partial && (!c.workspace || c.workspace_bytes < need))
    return set_error(HS_ERR_WORKSPACE, "quest: workspace of %zu bytes < required %zu",
                     c.workspace_bytes, need);
  switch (c.query_dtype) {
    case HS_FLOAT32: return dispatch_kv<float>(c, stream);
    case HS_FLOAT16: return dispatch_kv<__half>(c, stream);
    case HS_BFLOAT16: return dispatch_kv<__nv_bfloat16>(c, stream);
  }
  return set_error(HS_ERR_INVALID_ARGUMENT, "quest: invalid query dtype %d", c.query_dtype);
}

}  // namespace
}  // namespace hs

extern "C" size_t hs_quest_workspace_bytes(int batch, int64_t max_pages) {
  if (batch < 1 || max_pages < 1) return 0;
  // scores [batch, max_pages] fp32, then one completion counter per request
  return (size_t)batch * (size_t)max_pages * sizeof(float) + (size_t)batch * sizeof(unsigned);
}

extern "C" int hs_quest_select(const void *query, int query_dtype, const void *minimum,
                               const void *maximum, int kv_dtype, int q_heads, int kv_heads,
                               int head_dim, int64_t max_pages, int64_t length,
                               int page_size, int top_pages, int keep_sink,
                               int32_t *out_tokens, int64_t out_capacity, int32_t *out_count,
                               void *workspace, size_t workspace_bytes,
                               int32_t *device_status, hs_stream stream) {
  if (length < 1)
    return hs::set_error(HS_ERR_INVALID_ARGUMENT, "selection dimensions must be positive");
  if (hs::ceil_div(length, page_size < 1 ? 1 : page_size) > max_pages)
    return hs::set_error(HS_ERR_INVALID_ARGUMENT,
                         "quest: ceil(length / page_size) exceeds the metadata pages");
  if (!minimum || !maximum)
    return hs::set_error(HS_ERR_INVALID_ARGUMENT, "quest: null metadata pointer");
  hs::Common c{1, query, 0, query_dtype, minimum, maximum, nullptr, nullptr, kv_dtype,
               hs::Lengths{nullptr, length}, q_heads, kv_heads, head_dim, page_size,
               top_pages, keep_sink, max_pages, out_tokens, out_capacity, out_count,
               workspace, workspace_bytes, device_status, nullptr};
  return hs::quest_common(c, static_cast<cudaStream_t>(stream));
}

extern "C" int hs_quest_select_batched(int batch, const void *query,
                                       int64_t query_batch_stride, int query_dtype,
                                       const uint64_t *minimum_ptrs,
                                       const uint64_t *maximum_ptrs, int kv_dtype,
                                       const int32_t *lengths, int q_heads, int kv_heads,
                                       int head_dim, int64_t max_pages, int page_size,
                                       int top_pages, int keep_sink, int32_t *out_tokens,
                                       int64_t out_capacity, int32_t *out_counts,
                                       void *workspace, size_t workspace_bytes,
                                       int32_t *device_status, hs_stream stream) {
  if (!minimum_ptrs || !maximum_ptrs || !lengths)
    return hs::set_error(HS_ERR_INVALID_ARGUMENT, "quest: null pointer array or lengths");
  hs::Common c{batch, query, query_batch_stride, query_dtype, nullptr, nullptr, minimum_ptrs,
               maximum_ptrs, kv_dtype, hs::Lengths{lengths, 0}, q_heads, kv_heads, head_dim,
               page_size, top_pages, keep_sink, max_pages, out_tokens, out_capacity,
               out_counts, workspace, workspace_bytes, device_status, nullptr};
  return hs::quest_common(c, static_cast<cudaStream_t>(stream));
}

// ---- head-sharded selection (a request's KV heads split over ranks) -------------
extern "C" int hs_quest_partial_scores_batched(
    int batch, const void *query, int64_t query_batch_stride, int query_dtype,
    const uint64_t *minimum_ptrs, const uint64_t *maximum_ptrs, int kv_dtype,
    const int32_t *lengths, int q_heads, int kv_heads, int head_dim, int64_t max_pages,
    int page_size, float *out_partial, int32_t *device_status, hs_stream stream) {
  if (!minimum_ptrs || !maximum_ptrs || !lengths || !out_partial)
    return hs::set_error(HS_ERR_INVALID_ARGUMENT, "quest: null pointer array or output");
  hs::Common c{batch, query, query_batch_stride, query_dtype, nullptr, nullptr, minimum_ptrs,
               maximum_ptrs, kv_dtype, hs::Lengths{lengths, 0}, q_heads, kv_heads, head_dim,
               page_size, 1, 0, max_pages, nullptr, 0, nullptr, nullptr, 0, device_status,
               out_partial};
  return hs::quest_common(c, static_cast<cudaStream_t>(stream));
}

extern "C" int hs_quest_select_partials(int shards, const float *partials, int batch,
                                        const int32_t *lengths, int q_heads, int64_t max_pages,
                                        int page_size, int top_pages, int keep_sink,
                                        int32_t *out_tokens, int64_t out_capacity,
                                        int32_t *out_counts, void *workspace,
                                        size_t workspace_bytes, int32_t *device_status,
                                        hs_stream stream) {
  using namespace hs;
  if (shards < 1 || batch < 1 || q_heads < 1 || max_pages < 1 || page_size < 1 ||
      top_pages < 1)
    return set_error(HS_ERR_INVALID_ARGUMENT, "quest: dimensions must be positive");
  if (batch > 65535) return set_error(HS_ERR_UNSUPPORTED, "quest: batch %d > 65535", batch);
  if (!partials || !lengths || !out_tokens || !out_counts)
    return set_error(HS_ERR_INVALID_ARGUMENT, "quest: null tensor pointer");
  if (out_capacity < (int64_t)top_pages * page_size)
    return set_error(HS_ERR_INVALID_ARGUMENT,
                     "quest: out_capacity %lld < top_pages * page_size = %lld",
                     (long long)out_capacity, (long long)top_pages * page_size);
  if (out_capacity > INT32_MAX || max_pages * (int64_t)page_size > INT32_MAX)
    return set_error(HS_ERR_INVALID_ARGUMENT, "quest: token positions must fit int32");
  const size_t need = hs_quest_workspace_bytes(batch, max_pages);
  if (!workspace || workspace_bytes < need)
    return set_error(HS_ERR_WORKSPACE, "quest: workspace of %zu bytes < required %zu",
                     workspace_bytes, need);
  return launch_select_partials(shards, partials, batch, lengths, q_heads, max_pages,
                                page_size, top_pages, keep_sink, out_tokens, out_capacity,
                                out_counts, static_cast<float *>(workspace), device_status,
                                static_cast<cudaStream_t>(stream));
}
