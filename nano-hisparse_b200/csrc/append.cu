// (5) KV append: the tensor work of HostStore.append for one page chunk per
// batch item — new K/V rows into the pool block, the same rows into the pinned
// host mirror (stores through the host alias, so no separate device-to-host
// copy is queued), and the page's Quest metadata: running K min/max in the KV
// dtype and the fp32 mean-K summary.
//
// Reference: nano_hisparse/storage.py:296-321 (pool row copies, the mean of
// :309, torch.minimum/maximum of :311-316, the host mirror copies of
// :320-327). The reference issues about eight small torch operations per page
// chunk plus a copy on the transfer stream; here one launch covers a chunk of
// every request in the batch. One thread owns one (KV head, element) column
// of a chunk: it moves the column's new K/V values, folds them into the
// column's min/max and sums the column's K values over the page's valid rows
// in row order (the order of the reference's CPU mean, reproduced bit for bit).
#include "common.cuh"

namespace hs {
namespace {

constexpr int kAppendThreads = 256;

struct AppendParams {
  int batch;
  const void *k, *v;
  int64_t kv_batch_stride;
  const int32_t *within, *count;
  const int64_t *pool_block, *host_block;
  char *pool;
  char *host;
  int64_t pool_blocks, host_blocks;
  const uint64_t *minimum_ptrs, *maximum_ptrs, *summary_ptrs;
  int64_t elems;  // kv_heads * head_dim
  int page_size;
  int32_t *status;
};

template <typename T>
__global__ void __launch_bounds__(kAppendThreads) append_kernel(AppendParams p) {
  const int b = blockIdx.y;
  const int64_t e = (int64_t)blockIdx.x * kAppendThreads + threadIdx.x;
  if (e >= p.elems) return;
  const int cnt = p.count[b], w = p.within[b];
  if (cnt <= 0) return;
  const int64_t blk = p.pool_block[b], hb = p.host_block[b];
  // pool_block < 0: a host-only chunk (a page with no pool block), which needs a host block
  const bool host_ok = hb >= 0 && p.host != nullptr && hb < p.host_blocks;
  if (w < 0 || w + cnt > p.page_size || blk >= p.pool_blocks || (hb >= 0 && !host_ok) ||
      (blk < 0 && !host_ok)) {
    if (e == 0) flag(p.status, HS_DEV_ROW_OUT_OF_RANGE);
    return;
  }
  const int64_t E = p.elems, plane = (int64_t)p.page_size * E;
  T *pk = blk >= 0 ? reinterpret_cast<T *>(p.pool) + blk * 2 * plane : nullptr;
  T *hk = hb >= 0 ? reinterpret_cast<T *>(p.host) + hb * 2 * plane : nullptr;
  const T *page_k = pk != nullptr ? pk : hk;  // where the page's earlier rows live
  const T *k = static_cast<const T *>(p.k) + (int64_t)b * p.kv_batch_stride;
  const T *v = static_cast<const T *>(p.v) + (int64_t)b * p.kv_batch_stride;

  // rows 0 .. w-1 already in the page come first in the mean
  float sum = 0.f;
  for (int r = 0; r < w; ++r) sum += to_f32(page_k[(int64_t)r * E + e]);
  T lo = k[e], hi = k[e];
  bool nan_seen = false;
  T nan_value = lo;
  for (int i = 0; i < cnt; ++i) {
    const T kx = k[(int64_t)i * E + e], vx = v[(int64_t)i * E + e];
    const int64_t row = (int64_t)(w + i) * E + e;
    if (pk != nullptr) {
      pk[row] = kx;
      pk[plane + row] = vx;
    }
    if (hk != nullptr) {
      hk[row] = kx;
      hk[plane + row] = vx;
    }
    const float x = to_f32(kx);
    sum += x;
    if (x != x && !nan_seen) {
      nan_seen = true;
      nan_value = kx;
    }
    if (x < to_f32(lo)) lo = kx;
    if (to_f32(hi) < x) hi = kx;
  }
  // torch.minimum(old, new) / torch.maximum(old, new): NaN propagates, and an
  // equal new value replaces the old one
  T *mn = reinterpret_cast<T *>(p.minimum_ptrs[b]) + e;
  T *mx = reinterpret_cast<T *>(p.maximum_ptrs[b]) + e;
  const float old_lo = to_f32(*mn), old_hi = to_f32(*mx);
  if (old_lo == old_lo) {
    if (nan_seen) *mn = nan_value;
    else if (!(old_lo < to_f32(lo))) *mn = lo;
  }
  if (old_hi == old_hi) {
    if (nan_seen) *mx = nan_value;
    else if (!(to_f32(hi) < old_hi)) *mx = hi;
  }
  reinterpret_cast<float *>(p.summary_ptrs[b])[e] = sum / (float)(w + cnt);
}

template <typename T> int launch(const AppendParams &p, cudaStream_t s) {
  const dim3 grid((unsigned)ceil_div(p.elems, kAppendThreads), (unsigned)p.batch);
  append_kernel<T><<<grid, kAppendThreads, 0, s>>>(p);
  return check_launch("append_kernel");
}

}  // namespace
}  // namespace hs

extern "C" int hs_append_rows(int batch, const void *k, const void *v, int64_t kv_batch_stride,
                              int kv_dtype, const int32_t *within, const int32_t *count,
                              const int64_t *pool_block, void *pool, int64_t pool_blocks,
                              const int64_t *host_block, void *host_alias, int64_t host_blocks,
                              const uint64_t *minimum_ptrs, const uint64_t *maximum_ptrs,
                              const uint64_t *summary_ptrs, int kv_heads, int head_dim,
                              int page_size, int32_t *device_status, hs_stream stream) {
  using namespace hs;
  if (batch < 0 || kv_heads < 1 || head_dim < 1 || page_size < 1 || pool_blocks < 0 ||
      host_blocks < 0 || kv_batch_stride < 0)
    return set_error(HS_ERR_INVALID_ARGUMENT, "append: invalid sizes");
  if (batch == 0) return HS_OK;
  if (!k || !v || !within || !count || !pool_block || !pool || !host_block || !minimum_ptrs ||
      !maximum_ptrs || !summary_ptrs)
    return set_error(HS_ERR_INVALID_ARGUMENT, "append: null pointer");
  if (batch > 65535) return set_error(HS_ERR_UNSUPPORTED, "append: batch %d > 65535", batch);
  AppendParams p{batch, k, v, kv_batch_stride, within, count, pool_block, host_block,
                 static_cast<char *>(pool), static_cast<char *>(host_alias), pool_blocks,
                 host_blocks, minimum_ptrs, maximum_ptrs, summary_ptrs,
                 (int64_t)kv_heads * head_dim, page_size, device_status};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (kv_dtype) {
    case HS_FLOAT32: return launch<float>(p, s);
    case HS_FLOAT16: return launch<__half>(p, s);
    case HS_BFLOAT16: return launch<__nv_bfloat16>(p, s);
  }
  return set_error(HS_ERR_INVALID_ARGUMENT, "append: invalid KV dtype %d", kv_dtype);
}
