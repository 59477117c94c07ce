// (1) Quest page selection: page scoring over the K min/max metadata, shared
// top-k with forced sink/tail pages and page->token expansion.
//
// Reference: nano_hisparse/selection.py:69-91 (quest_selection),
// selection.py:45-62 (Selection.from_pages), row_index.py:20-24
// (LogicalTopK.from_selection, shared case).
//
// Two launches per call:
//   quest_score_kernel  : HBM-bound streaming pass over min/max [n, Hkv, D];
//                         one warp per page, lanes own C = ceil(D/32)
//                         consecutive head-dim elements; fixed fp32 order.
//   quest_select_kernel : one CTA per request; MSB-first radix select of the
//                         top_pages largest scores, lower page index first on
//                         ties; the chosen-page bitmap is scanned in page order
//                         so the token list comes out sorted.
#include <cstdio>

#include "common.cuh"

namespace hs {
namespace {

constexpr int kScoreThreads = 256;
constexpr int kScoreWarps = kScoreThreads / 32;
constexpr int kPagesPerCta = 64;
constexpr int kSelectThreads = 1024;

template <typename TQ, typename TKV> struct QuestScoreParams {
  int batch;
  Batched<TQ> query;
  Batched<TKV> minimum;
  Batched<TKV> maximum;
  Lengths lengths;
  int q_heads, kv_heads, head_dim, page_size;
  int64_t max_pages;
  float *scores;  // [batch, max_pages]
  int32_t *status;
};

// Each lane j owns head-dim elements d = j*C .. j*C+C-1. For a page, lane j
// computes, for every query head h, part[h] = sum_c max(q*min, q*max) left to
// right; part[] over the 32 lanes is then reduced with a reduce-scatter whose
// pairing is (j, j^16), (j, j^8), ..., (j, j^1), which leaves s[h] on lane
// h % 32. Heads are processed in chunks of 32; lane j accumulates its heads
// j, j+32, ... left to right and the lanes are finally combined with the
// same xor tree. The result divided by q_heads is the page score.
template <typename TQ, typename TKV, int C>
__global__ void __launch_bounds__(kScoreThreads)
    quest_score_kernel(QuestScoreParams<TQ, TKV> p) {
  extern __shared__ float q_smem[];  // [q_heads][32*C], zero padded past head_dim
  const int b = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t length = p.lengths.at(b);
  if (length <= 0) return;
  const int64_t n = ceil_div(length, p.page_size);
  if (n > p.max_pages) return;  // reported by the select kernel
  const int64_t page_begin = (int64_t)blockIdx.x * kPagesPerCta;
  if (page_begin >= n) return;
  const int64_t page_end = min(n, page_begin + kPagesPerCta);

  const int D = p.head_dim, W = 32 * C;
  const TQ *q = p.query.at(b);
  for (int i = threadIdx.x; i < p.q_heads * W; i += blockDim.x) {
    const int h = i / W, d = i % W;
    q_smem[i] = d < D ? to_f32(q[(int64_t)h * D + d]) : 0.f;
  }
  __syncthreads();

  const TKV *mn_base = p.minimum.at(b);
  const TKV *mx_base = p.maximum.at(b);
  const int groups = p.q_heads / p.kv_heads;
  const int d0 = lane * C;
  const float inv_heads_div = (float)p.q_heads;

  for (int64_t page = page_begin + warp; page < page_end; page += kScoreWarps) {
    const int64_t page_off = page * p.kv_heads * D;
    float u = 0.f;
    for (int hc = 0; hc < p.q_heads; hc += 32) {
      float v[32];
      float mn[C], mx[C];
      int cur_kh = -1;
#pragma unroll
      for (int hl = 0; hl < 32; ++hl) {
        v[hl] = 0.f;
        const int h = hc + hl;
        if (h < p.q_heads) {
          const int kh = h / groups;
          if (kh != cur_kh) {
            cur_kh = kh;
            const TKV *a = mn_base + page_off + (int64_t)kh * D + d0;
            const TKV *c = mx_base + page_off + (int64_t)kh * D + d0;
            if (d0 + C <= D) {
              const bool al = ((reinterpret_cast<uintptr_t>(a) |
                                reinterpret_cast<uintptr_t>(c)) &
                               (C * sizeof(TKV) - 1)) == 0;
              load_f32<TKV, C>(a, mn, al);
              load_f32<TKV, C>(c, mx, al);
            } else {
#pragma unroll
              for (int i = 0; i < C; ++i) {
                mn[i] = d0 + i < D ? to_f32(a[i]) : 0.f;
                mx[i] = d0 + i < D ? to_f32(c[i]) : 0.f;
              }
            }
          }
          const float *qh = q_smem + h * W + d0;
          float part = 0.f;
#pragma unroll
          for (int i = 0; i < C; ++i) {
            if (d0 + i < D) {
              const float qq = qh[i];
              const float t = fmaxf(__fmul_rn(qq, mn[i]), __fmul_rn(qq, mx[i]));
              part = i == 0 ? t : __fadd_rn(part, t);
            }
          }
          v[hl] = part;
        }
      }
      // Reduce-scatter: after the step with offset o, v[0..o) hold the heads
      // whose bit pattern in [o, 32) equals the lane's.
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < o; ++i) {
          const float send = upper ? v[i] : v[i + o];
          const float keep = upper ? v[i + o] : v[i];
          v[i] = __fadd_rn(keep, __shfl_xor_sync(kFullMask, send, o));
        }
      }
      u = __fadd_rn(u, v[0]);
    }
    const float total = warp_xor_tree_sum(u);
    if (lane == 0) p.scores[(int64_t)b * p.max_pages + page] = __fdiv_rn(total, inv_heads_div);
  }
}

struct QuestSelectParams {
  int batch;
  Lengths lengths;
  int page_size, top_pages, keep_sink;
  int64_t max_pages;
  const float *scores;
  int32_t *out_tokens;  // [batch, capacity]
  int64_t capacity;
  int32_t *out_counts;
  int32_t *status;
};

// Order-preserving map of a float score to an unsigned key (larger float ->
// larger key). -0 is folded onto +0; NaN ranks above +inf (as in torch.topk);
// forced pages take the maximum key.
__device__ __forceinline__ uint32_t score_key(float s) {
  if (isnan(s)) return 0xfffffffeu;
  const uint32_t bits = __float_as_uint(s + 0.0f);
  return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
}

__device__ __forceinline__ uint32_t page_key(const QuestSelectParams &p, const float *sc,
                                             int64_t page, int64_t n, bool sink) {
  if (page == n - 1 || (sink && page == 0)) return 0xffffffffu;
  return score_key(sc[page]);
}

__global__ void __launch_bounds__(kSelectThreads) quest_select_kernel(QuestSelectParams p) {
  __shared__ uint32_t hist[256];
  __shared__ int64_t scan_scratch[33];
  __shared__ uint32_t s_prefix, s_mask, s_k;
  const int b = blockIdx.x;
  const int tid = threadIdx.x;
  const int64_t length = p.lengths.at(b);
  int32_t *out = p.out_tokens + (int64_t)b * p.capacity;
  const int64_t n = length > 0 ? ceil_div(length, p.page_size) : 0;
  if (length <= 0 || n > p.max_pages) {
    if (n > p.max_pages && tid == 0) flag(p.status, HS_DEV_PAGES_EXCEED_TABLE);
    for (int64_t i = tid; i < p.capacity; i += blockDim.x) out[i] = -1;
    if (tid == 0) p.out_counts[b] = 0;
    return;
  }
  if (p.top_pages >= n) {
    // Every page: tokens 0 .. length-1 (selection.py:80-81).
    for (int64_t i = tid; i < p.capacity; i += blockDim.x) out[i] = i < length ? (int32_t)i : -1;
    if (tid == 0) p.out_counts[b] = (int32_t)length;
    return;
  }
  const float *sc = p.scores + (int64_t)b * p.max_pages;
  const bool sink = p.keep_sink && p.top_pages > 1 && n > 1;

  if (tid == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_k = (uint32_t)p.top_pages;
  }
  __syncthreads();
  // MSB-first radix select of the k-th largest key.
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    for (int64_t pg = tid; pg < n; pg += blockDim.x) {
      const uint32_t key = page_key(p, sc, pg, n, sink);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xffu], 1u);
    }
    __syncthreads();
    if (tid < 32) {
      // Lane l owns digits [8*(31-l), 8*(31-l)+7]; scanning lanes in order walks
      // the digits from the top.
      uint32_t local = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) local += hist[8 * (31 - tid) + i];
      const uint32_t inc = warp_inclusive_scan(local);
      const uint32_t k = s_k;
      const unsigned ballot = __ballot_sync(kFullMask, inc >= k);
      const int owner = __ffs(ballot) - 1;  // first lane whose cumulative count reaches k
      if (tid == owner) {
        uint32_t above = inc - local;
        int digit = 8 * (31 - tid) + 7;
        for (; digit > 8 * (31 - tid); --digit) {
          if (above + hist[digit] >= k) break;
          above += hist[digit];
        }
        s_k = k - above;
        s_prefix = prefix | ((uint32_t)digit << shift);
        s_mask = mask | (0xffu << shift);
      }
    }
    __syncthreads();
  }
  const uint32_t threshold = s_prefix;
  const uint32_t take_equal = s_k;  // how many keys == threshold to keep (lowest pages)

  // Pages are split into contiguous runs per thread so scans follow page order.
  const int64_t per = ceil_div(n, (int64_t)blockDim.x);
  const int64_t lo = min(n, tid * per), hi = min(n, lo + per);
  int64_t eq_local = 0;
  for (int64_t pg = lo; pg < hi; ++pg) eq_local += page_key(p, sc, pg, n, sink) == threshold;
  int64_t eq_total;
  int64_t eq_before = block_exclusive_scan<int64_t>(eq_local, scan_scratch, &eq_total);
  // Chosen-page ranks in page order.
  int64_t chosen_local = 0;
  {
    int64_t eq = eq_before;
    for (int64_t pg = lo; pg < hi; ++pg) {
      const uint32_t key = page_key(p, sc, pg, n, sink);
      const bool take = key > threshold || (key == threshold && eq++ < (int64_t)take_equal);
      chosen_local += take;
    }
  }
  int64_t chosen_total;
  int64_t rank = block_exclusive_scan<int64_t>(chosen_local, scan_scratch, &chosen_total);
  {
    int64_t eq = eq_before;
    for (int64_t pg = lo; pg < hi; ++pg) {
      const uint32_t key = page_key(p, sc, pg, n, sink);
      const bool take = key > threshold || (key == threshold && eq++ < (int64_t)take_equal);
      if (take) {
        const int64_t first = pg * p.page_size;
        const int64_t cnt = min((int64_t)p.page_size, length - first);
        for (int64_t i = 0; i < cnt; ++i) out[rank * p.page_size + i] = (int32_t)(first + i);
        ++rank;
      }
    }
  }
  // Only the tail page (always chosen, always last) can be partial.
  const int64_t count = (chosen_total - 1) * p.page_size + (length - (n - 1) * p.page_size);
  for (int64_t i = count + tid; i < p.capacity; i += blockDim.x) out[i] = -1;
  if (tid == 0) p.out_counts[b] = (int32_t)count;
}

template <typename TQ, typename TKV>
int launch_score(const QuestScoreParams<TQ, TKV> &p, int head_dim, cudaStream_t stream) {
  const int C = (head_dim + 31) / 32;
  const size_t smem = (size_t)p.q_heads * 32 * C * sizeof(float);
  dim3 grid((unsigned)ceil_div(p.max_pages, kPagesPerCta), (unsigned)p.batch);
#define HS_QUEST_CASE(CC)                                                                 \
  case CC: {                                                                              \
    auto k = quest_score_kernel<TQ, TKV, CC>;                                             \
    if (smem > 48 * 1024 &&                                                               \
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != \
            cudaSuccess)                                                                  \
      return set_error(HS_ERR_CUDA, "quest: cannot reserve %zu bytes of shared memory", smem); \
    k<<<grid, kScoreThreads, smem, stream>>>(p);                                          \
    break;                                                                                \
  }
  switch (C) {
    HS_QUEST_CASE(1)
    HS_QUEST_CASE(2)
    HS_QUEST_CASE(3)
    HS_QUEST_CASE(4)
    HS_QUEST_CASE(5)
    HS_QUEST_CASE(6)
    HS_QUEST_CASE(7)
    HS_QUEST_CASE(8)
    default:
      return set_error(HS_ERR_UNSUPPORTED, "quest: head_dim %d > 256 is not supported", head_dim);
  }
#undef HS_QUEST_CASE
  return check_launch("quest_score_kernel");
}

template <typename TQ>
int dispatch_kv(int kv_dtype, const void *query, int64_t qstride, const void *mn,
                const void *mx, const uint64_t *mn_ptrs, const uint64_t *mx_ptrs,
                QuestScoreParams<float, float> proto, int head_dim, cudaStream_t stream) {
  auto fill = [&](auto tag) {
    using TKV = decltype(tag);
    QuestScoreParams<TQ, TKV> p;
    p.batch = proto.batch;
    p.query = Batched<TQ>{static_cast<const TQ *>(query), qstride, nullptr};
    p.minimum = Batched<TKV>{static_cast<const TKV *>(mn), 0, mn_ptrs};
    p.maximum = Batched<TKV>{static_cast<const TKV *>(mx), 0, mx_ptrs};
    p.lengths = proto.lengths;
    p.q_heads = proto.q_heads;
    p.kv_heads = proto.kv_heads;
    p.head_dim = proto.head_dim;
    p.page_size = proto.page_size;
    p.max_pages = proto.max_pages;
    p.scores = proto.scores;
    p.status = proto.status;
    return launch_score<TQ, TKV>(p, head_dim, stream);
  };
  switch (kv_dtype) {
    case HS_FLOAT32: return fill(float{});
    case HS_FLOAT16: return fill(__half{});
    case HS_BFLOAT16: return fill(__nv_bfloat16{});
  }
  return set_error(HS_ERR_INVALID_ARGUMENT, "quest: invalid KV dtype %d", kv_dtype);
}

int quest_common(int batch, const void *query, int64_t qstride, int query_dtype,
                 const void *mn, const void *mx, const uint64_t *mn_ptrs,
                 const uint64_t *mx_ptrs, int kv_dtype, Lengths lengths, int q_heads,
                 int kv_heads, int head_dim, int64_t max_pages, int page_size,
                 int top_pages, int keep_sink, int32_t *out_tokens, int64_t capacity,
                 int32_t *out_counts, void *workspace, size_t workspace_bytes,
                 int32_t *status, cudaStream_t stream) {
  if (batch < 1 || q_heads < 1 || kv_heads < 1 || head_dim < 1 || page_size < 1 ||
      max_pages < 1)
    return set_error(HS_ERR_INVALID_ARGUMENT, "quest: dimensions must be positive");
  if (top_pages < 1 || q_heads % kv_heads)
    return set_error(HS_ERR_INVALID_ARGUMENT, "invalid page budget or GQA shape");
  if (head_dim > 256)
    return set_error(HS_ERR_UNSUPPORTED, "quest: head_dim %d > 256 is not supported", head_dim);
  if ((size_t)q_heads * 32 * ((head_dim + 31) / 32) * sizeof(float) > 200 * 1024)
    return set_error(HS_ERR_UNSUPPORTED, "quest: query of %d heads does not fit shared memory",
                     q_heads);
  if (!query || !out_tokens || !out_counts || (!mn && !mn_ptrs) || (!mx && !mx_ptrs))
    return set_error(HS_ERR_INVALID_ARGUMENT, "quest: null tensor pointer");
  if (capacity < (int64_t)top_pages * page_size)
    return set_error(HS_ERR_INVALID_ARGUMENT,
                     "quest: out_capacity %lld < top_pages * page_size = %lld",
                     (long long)capacity, (long long)top_pages * page_size);
  if (capacity > INT32_MAX || max_pages * (int64_t)page_size > INT32_MAX)
    return set_error(HS_ERR_INVALID_ARGUMENT, "quest: token positions must fit int32");
  const size_t need = hs_quest_workspace_bytes(batch, max_pages);
  if (!workspace || workspace_bytes < need)
    return set_error(HS_ERR_WORKSPACE, "quest: workspace of %zu bytes < required %zu",
                     workspace_bytes, need);
  float *scores = static_cast<float *>(workspace);
  QuestScoreParams<float, float> proto;
  proto.batch = batch;
  proto.lengths = lengths;
  proto.q_heads = q_heads;
  proto.kv_heads = kv_heads;
  proto.head_dim = head_dim;
  proto.page_size = page_size;
  proto.max_pages = max_pages;
  proto.scores = scores;
  proto.status = status;
  int rc;
  switch (query_dtype) {
    case HS_FLOAT32:
      rc = dispatch_kv<float>(kv_dtype, query, qstride, mn, mx, mn_ptrs, mx_ptrs, proto,
                              head_dim, stream);
      break;
    case HS_FLOAT16:
      rc = dispatch_kv<__half>(kv_dtype, query, qstride, mn, mx, mn_ptrs, mx_ptrs, proto,
                               head_dim, stream);
      break;
    case HS_BFLOAT16:
      rc = dispatch_kv<__nv_bfloat16>(kv_dtype, query, qstride, mn, mx, mn_ptrs, mx_ptrs,
                                      proto, head_dim, stream);
      break;
    default:
      return set_error(HS_ERR_INVALID_ARGUMENT, "quest: invalid query dtype %d", query_dtype);
  }
  if (rc != HS_OK) return rc;
  QuestSelectParams s;
  s.batch = batch;
  s.lengths = lengths;
  s.page_size = page_size;
  s.top_pages = top_pages;
  s.keep_sink = keep_sink;
  s.max_pages = max_pages;
  s.scores = scores;
  s.out_tokens = out_tokens;
  s.capacity = capacity;
  s.out_counts = out_counts;
  s.status = status;
  quest_select_kernel<<<batch, kSelectThreads, 0, stream>>>(s);
  return check_launch("quest_select_kernel");
}

}  // namespace
}  // namespace hs

extern "C" size_t hs_quest_workspace_bytes(int batch, int64_t max_pages) {
  if (batch < 1 || max_pages < 1) return 0;
  return (size_t)batch * (size_t)max_pages * sizeof(float);
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
  return hs::quest_common(1, query, 0, query_dtype, minimum, maximum, nullptr, nullptr,
                          kv_dtype, hs::Lengths{nullptr, length}, q_heads, kv_heads,
                          head_dim, max_pages, page_size, top_pages, keep_sink, out_tokens,
                          out_capacity, out_count, workspace, workspace_bytes,
                          device_status, static_cast<cudaStream_t>(stream));
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
  return hs::quest_common(batch, query, query_batch_stride, query_dtype, nullptr, nullptr,
                          minimum_ptrs, maximum_ptrs, kv_dtype, hs::Lengths{lengths, 0},
                          q_heads, kv_heads, head_dim, max_pages, page_size, top_pages,
                          keep_sink, out_tokens, out_capacity, out_counts, workspace,
                          workspace_bytes, device_status,
                          static_cast<cudaStream_t>(stream));
}
