// (4) Physical-row GQA decode attention over the resolved rows.
//
// Reference: nano_hisparse/row_kernels.py:73-135 (_attend, attend_rows) and the
// torch path of attention.py:26-35. The reference runs one program per query
// head, so each KV row is read once per head of its GQA group, and K is a
// compile-time constant. Here one CTA serves a whole GQA group (every K/V row
// slice is read once for all of its query heads) over one split of the rows;
// a second launch merges the splits' (max, sum, accumulator) partials.
// Softmax and accumulation are fp32.
#include <math.h>

#include "common.cuh"

namespace hs {
namespace {

constexpr int kAttendThreads = 128;
constexpr int kAttendWarps = kAttendThreads / 32;
constexpr int kMaxGroup = 8;   // query heads per CTA
constexpr int kRowsInFlight = 4;
constexpr int kMaxSplits = 64;

struct AttendParams {
  int batch;
  const void *query;
  int64_t query_batch_stride;
  const char *pool;
  int64_t pool_blocks;
  const int64_t *rows;
  int64_t rows_batch_stride, rows_head_stride, count;
  void *out;
  int64_t out_batch_stride;
  int q_heads, kv_heads, head_dim, page_size;
  int splits, head_chunks;  // grid.y = kv_heads * head_chunks (shared) or q_heads (per head)
  float scale;
  float *partials;  // [batch, q_heads, splits, head_dim + 2]
  int32_t *status;
};

__host__ __device__ inline int attend_splits(int batch, int kv_heads, int64_t count, int sms) {
  const int64_t target = (int64_t)sms * 8;
  int64_t s = ceil_div(target, (int64_t)batch * kv_heads);
  const int64_t by_rows = ceil_div(count, 32);
  if (s > by_rows) s = by_rows;
  if (s > kMaxSplits) s = kMaxSplits;
  if (s < 1) s = 1;
  return (int)s;
}

template <typename TQ, typename TKV, int C>
__global__ void __launch_bounds__(kAttendThreads) attend_split_kernel(AttendParams p) {
  __shared__ float red_m[kAttendWarps][kMaxGroup];
  __shared__ float red_l[kAttendWarps][kMaxGroup];
  __shared__ float red_acc[kAttendWarps][kMaxGroup][32 * C];
  const int split = blockIdx.x, b = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int D = p.head_dim;
  const int groups = p.q_heads / p.kv_heads;
  const bool shared_rows = p.rows_head_stride == 0;
  int kh, h0, hn;
  if (shared_rows) {
    kh = blockIdx.y / p.head_chunks;
    h0 = kh * groups + (blockIdx.y % p.head_chunks) * kMaxGroup;
    hn = min(kMaxGroup, kh * groups + groups - h0);
  } else {
    h0 = blockIdx.y;
    kh = h0 / groups;
    hn = 1;
  }
  const int d0 = lane * C;
  const bool lane_full = d0 + C <= D;

  // Query slice of every head served here.
  float q[kMaxGroup][C];
  const TQ *qb = static_cast<const TQ *>(p.query) + (int64_t)b * p.query_batch_stride;
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g)
#pragma unroll
    for (int c = 0; c < C; ++c)
      q[g][c] = (g < hn && d0 + c < D) ? to_f32(qb[(int64_t)(h0 + g) * D + d0 + c]) : 0.f;

  float m[kMaxGroup], l[kMaxGroup], acc[kMaxGroup][C];
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int c = 0; c < C; ++c) acc[g][c] = 0.f;
  }

  const int64_t chunk = ceil_div(p.count, p.splits);
  const int64_t begin = split * chunk, end = min(p.count, begin + chunk);
  const int64_t *rows = p.rows + (int64_t)b * p.rows_batch_stride +
                        (shared_rows ? 0 : (int64_t)h0 * p.rows_head_stride);
  const int64_t row_elems = (int64_t)p.kv_heads * D;
  const int64_t plane_elems = (int64_t)p.page_size * row_elems;
  const TKV *pool = reinterpret_cast<const TKV *>(p.pool);

  for (int64_t i0 = begin + warp * kRowsInFlight; i0 < end;
       i0 += (int64_t)kAttendWarps * kRowsInFlight) {
    float kv_k[kRowsInFlight][C], kv_v[kRowsInFlight][C];
    bool ok[kRowsInFlight];
#pragma unroll
    for (int r = 0; r < kRowsInFlight; ++r) {
      const int64_t i = i0 + r;
      int64_t row = i < end ? rows[i] : -1;
      if (row >= 0 && row / p.page_size >= p.pool_blocks) {
        if (lane == 0) flag(p.status, HS_DEV_ROW_OUT_OF_RANGE);
        row = -1;
      }
      ok[r] = row >= 0;
      if (ok[r] && d0 < D) {
        const int64_t blk = row / p.page_size, off = row % p.page_size;
        const TKV *kp = pool + (blk * 2 * p.page_size + off) * row_elems + (int64_t)kh * D + d0;
        const TKV *vp = kp + plane_elems;
        if (lane_full) {
          const bool al = ((reinterpret_cast<uintptr_t>(kp) | reinterpret_cast<uintptr_t>(vp)) &
                           (C * sizeof(TKV) - 1)) == 0;
          load_f32<TKV, C>(kp, kv_k[r], al);
          load_f32<TKV, C>(vp, kv_v[r], al);
        } else {
#pragma unroll
          for (int c = 0; c < C; ++c) {
            kv_k[r][c] = d0 + c < D ? to_f32(kp[c]) : 0.f;
            kv_v[r][c] = d0 + c < D ? to_f32(vp[c]) : 0.f;
          }
        }
      } else {
#pragma unroll
        for (int c = 0; c < C; ++c) kv_k[r][c] = kv_v[r][c] = 0.f;
      }
    }
#pragma unroll
    for (int r = 0; r < kRowsInFlight; ++r) {
      if (!ok[r]) continue;  // warp-uniform
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) {
        if (g >= hn) break;
        float dot = 0.f;
#pragma unroll
        for (int c = 0; c < C; ++c) dot = fmaf(q[g][c], kv_k[r][c], dot);
        const float s = warp_xor_tree_sum(dot) * p.scale;
        const float m_new = fmaxf(m[g], s);
        const float alpha = m[g] == -INFINITY ? 0.f : expf(m[g] - m_new);
        const float w = expf(s - m_new);
        l[g] = l[g] * alpha + w;
#pragma unroll
        for (int c = 0; c < C; ++c) acc[g][c] = fmaf(w, kv_v[r][c], acc[g][c] * alpha);
        m[g] = m_new;
      }
    }
  }
  // Combine the warps of this CTA.
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    if (g >= hn) break;
    if (lane == 0) {
      red_m[warp][g] = m[g];
      red_l[warp][g] = l[g];
    }
#pragma unroll
    for (int c = 0; c < C; ++c) red_acc[warp][g][d0 + c] = acc[g][c];
  }
  __syncthreads();
  const int stride = D + 2;
  for (int idx = threadIdx.x; idx < hn * (D + 2); idx += blockDim.x) {
    const int g = idx / (D + 2), e = idx % (D + 2);
    float mm = -INFINITY;
    for (int w = 0; w < kAttendWarps; ++w) mm = fmaxf(mm, red_m[w][g]);
    float v = 0.f;
    if (e == D) {
      v = mm;
    } else {
      for (int w = 0; w < kAttendWarps; ++w) {
        const float f = red_m[w][g] == -INFINITY ? 0.f : expf(red_m[w][g] - mm);
        v += f * (e == D + 1 ? red_l[w][g] : red_acc[w][g][e]);
      }
    }
    p.partials[(((int64_t)b * p.q_heads + h0 + g) * p.splits + split) * stride + e] = v;
  }
}

template <typename TQ>
__global__ void attend_merge_kernel(AttendParams p) {
  const int h = blockIdx.x, b = blockIdx.y;
  const int D = p.head_dim, stride = D + 2;
  const float *part = p.partials + ((int64_t)b * p.q_heads + h) * p.splits * stride;
  float mm = -INFINITY;
  for (int s = 0; s < p.splits; ++s) mm = fmaxf(mm, part[s * stride + D]);
  float denom = 0.f;
  for (int s = 0; s < p.splits; ++s) {
    const float ms = part[s * stride + D];
    if (ms != -INFINITY) denom += expf(ms - mm) * part[s * stride + D + 1];
  }
  TQ *out = static_cast<TQ *>(p.out) + (int64_t)b * p.out_batch_stride + (int64_t)h * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float num = 0.f;
    for (int s = 0; s < p.splits; ++s) {
      const float ms = part[s * stride + D];
      if (ms != -INFINITY) num += expf(ms - mm) * part[s * stride + d];
    }
    out[d] = from_f32<TQ>(denom > 0.f ? num / denom : 0.f);
  }
}

template <typename TQ, typename TKV>
int launch(AttendParams &p, cudaStream_t stream) {
  const int C = (p.head_dim + 31) / 32;
  const int Cp = C <= 1 ? 1 : C <= 2 ? 2 : C <= 4 ? 4 : 8;
  const int groups = p.q_heads / p.kv_heads;
  p.head_chunks = (groups + kMaxGroup - 1) / kMaxGroup;
  const bool shared_rows = p.rows_head_stride == 0;
  dim3 grid(p.splits, shared_rows ? p.kv_heads * p.head_chunks : p.q_heads, p.batch);
  switch (Cp) {
    case 1: attend_split_kernel<TQ, TKV, 1><<<grid, kAttendThreads, 0, stream>>>(p); break;
    case 2: attend_split_kernel<TQ, TKV, 2><<<grid, kAttendThreads, 0, stream>>>(p); break;
    case 4: attend_split_kernel<TQ, TKV, 4><<<grid, kAttendThreads, 0, stream>>>(p); break;
    default: attend_split_kernel<TQ, TKV, 8><<<grid, kAttendThreads, 0, stream>>>(p); break;
  }
  int rc = check_launch("attend_split_kernel");
  if (rc != HS_OK) return rc;
  attend_merge_kernel<TQ><<<dim3(p.q_heads, p.batch), 128, 0, stream>>>(p);
  return check_launch("attend_merge_kernel");
}

template <typename TQ> int dispatch_kv(int kv_dtype, AttendParams &p, cudaStream_t s) {
  switch (kv_dtype) {
    case HS_FLOAT32: return launch<TQ, float>(p, s);
    case HS_FLOAT16: return launch<TQ, __half>(p, s);
    case HS_BFLOAT16: return launch<TQ, __nv_bfloat16>(p, s);
  }
  return set_error(HS_ERR_INVALID_ARGUMENT, "attend: invalid KV dtype %d", kv_dtype);
}

}  // namespace
}  // namespace hs

extern "C" size_t hs_attend_workspace_bytes(int batch, int q_heads, int kv_heads,
                                            int head_dim, int64_t count) {
  if (batch < 1 || q_heads < 1 || kv_heads < 1 || head_dim < 1 || count < 1) return 0;
  const int splits = hs::attend_splits(batch, kv_heads, count, hs::sm_count());
  return (size_t)batch * q_heads * splits * (head_dim + 2) * sizeof(float);
}

extern "C" int hs_attend_rows(int batch, const void *query, int64_t query_batch_stride,
                              int query_dtype, const void *pool, int64_t pool_blocks,
                              int kv_dtype, const int64_t *rows, int64_t rows_batch_stride,
                              int64_t rows_head_stride, int64_t count, void *out,
                              int64_t out_batch_stride, int q_heads, int kv_heads,
                              int head_dim, int page_size, void *workspace,
                              size_t workspace_bytes, int32_t *device_status,
                              hs_stream stream) {
  using namespace hs;
  if (batch < 1 || q_heads < 1 || kv_heads < 1 || head_dim < 1 || page_size < 1 ||
      count < 1 || pool_blocks < 0)
    return set_error(HS_ERR_INVALID_ARGUMENT, "attend: dimensions must be positive");
  if (q_heads % kv_heads)
    return set_error(HS_ERR_INVALID_ARGUMENT, "query GQA/device mismatch");
  if (head_dim > 256)
    return set_error(HS_ERR_UNSUPPORTED, "attend: head_dim %d > 256 is not supported", head_dim);
  if (!query || !pool || !rows || !out)
    return set_error(HS_ERR_INVALID_ARGUMENT, "attend: null tensor pointer");
  const size_t need = hs_attend_workspace_bytes(batch, q_heads, kv_heads, head_dim, count);
  if (!workspace || workspace_bytes < need)
    return set_error(HS_ERR_WORKSPACE, "attend: workspace of %zu bytes < required %zu",
                     workspace_bytes, need);
  AttendParams p{};
  p.batch = batch;
  p.query = query;
  p.query_batch_stride = query_batch_stride;
  p.pool = static_cast<const char *>(pool);
  p.pool_blocks = pool_blocks;
  p.rows = rows;
  p.rows_batch_stride = rows_batch_stride;
  p.rows_head_stride = rows_head_stride;
  p.count = count;
  p.out = out;
  p.out_batch_stride = out_batch_stride;
  p.q_heads = q_heads;
  p.kv_heads = kv_heads;
  p.head_dim = head_dim;
  p.page_size = page_size;
  p.splits = attend_splits(batch, kv_heads, count, sm_count());
  p.scale = (float)(1.0 / sqrt((double)head_dim));
  p.partials = static_cast<float *>(workspace);
  p.status = device_status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (query_dtype) {
    case HS_FLOAT32: return dispatch_kv<float>(kv_dtype, p, s);
    case HS_FLOAT16: return dispatch_kv<__half>(kv_dtype, p, s);
    case HS_BFLOAT16: return dispatch_kv<__nv_bfloat16>(kv_dtype, p, s);
  }
  return set_error(HS_ERR_INVALID_ARGUMENT, "attend: invalid query dtype %d", query_dtype);
}
