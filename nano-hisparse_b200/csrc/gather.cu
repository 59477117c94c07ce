// (3) Miss gather: copies the K-plane and V-plane rows of every planned miss
// from the pinned host store (read zero-copy through its device alias, over
// the host link) into the shared GPU pool.
//
// Reference: nano_hisparse/row_kernels.py:35-70 (_gather, gather_rows) and the
// CPU loop of hybrid.py:452-459. The reference runs min(n, 64) programs and
// recompiles per plan width; here the plan width is a runtime argument and
// the grid has one 4-warp CTA per SM. One warp moves one row: all 2*row_bytes
// of it are loaded (16-byte vectors when the layout allows) before any store,
// so each warp keeps up to 4 KiB of host-link reads in flight.
#include "common.cuh"

namespace hs {
namespace {

constexpr int kGatherThreads = 128;
constexpr int kGatherWarps = kGatherThreads / 32;
constexpr int kUnroll = 8;  // vectors per lane in flight

struct GatherParams {
  const char *host;
  int64_t host_blocks;
  char *pool;
  int64_t pool_blocks;
  const int64_t *miss_host, *miss_device;
  int64_t count, segment;
  int page_size;
  int64_t row_bytes;
  int32_t *status;
};

template <typename V>
__global__ void __launch_bounds__(kGatherThreads) gather_kernel(GatherParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * kGatherWarps + (threadIdx.x >> 5);
  const int64_t warps = (int64_t)gridDim.x * kGatherWarps;
  const int64_t vecs = p.row_bytes / (int64_t)sizeof(V);  // per plane
  const int64_t plane_stride = (int64_t)p.page_size * p.row_bytes;
  for (int64_t e = warp; e < p.count; e += warps) {
    const int64_t h = p.miss_host[e], d = p.miss_device[e];
    if (h < 0 || d < 0) continue;  // padding after the compact prefix
    const int64_t hb = h / p.page_size, db = d / p.page_size;
    if (hb >= p.host_blocks || db >= p.pool_blocks) {
      if (lane == 0) flag(p.status, HS_DEV_ROW_OUT_OF_RANGE);
      continue;
    }
    const char *src = p.host + (hb * 2 * p.page_size + h % p.page_size) * p.row_bytes;
    char *dst = p.pool + (db * 2 * p.page_size + d % p.page_size) * p.row_bytes;
    const int64_t total = 2 * vecs;  // K plane then V plane
    for (int64_t c0 = 0; c0 < total; c0 += 32 * kUnroll) {
      V buf[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t c = c0 + u * 32 + lane;
        if (c < total) {
          const int64_t plane = c >= vecs;
          buf[u] = *reinterpret_cast<const V *>(src + plane * plane_stride +
                                                (c - plane * vecs) * (int64_t)sizeof(V));
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t c = c0 + u * 32 + lane;
        if (c < total) {
          const int64_t plane = c >= vecs;
          *reinterpret_cast<V *>(dst + plane * plane_stride +
                                 (c - plane * vecs) * (int64_t)sizeof(V)) = buf[u];
        }
      }
    }
  }
}

}  // namespace
}  // namespace hs

extern "C" int hs_gather_rows(const void *host_alias, int64_t host_blocks, void *pool,
                              int64_t pool_blocks, const int64_t *miss_host,
                              const int64_t *miss_device, int64_t count, int64_t segment,
                              int page_size, int64_t row_bytes, int32_t *device_status,
                              hs_stream stream) {
  using namespace hs;
  if (!host_alias || !pool || !miss_host || !miss_device)
    return set_error(HS_ERR_INVALID_ARGUMENT, "gather: null pointer");
  if (count < 0 || page_size < 1 || row_bytes < 1 || host_blocks < 0 || pool_blocks < 0)
    return set_error(HS_ERR_INVALID_ARGUMENT, "gather: invalid sizes");
  if (segment < 1) segment = count > 0 ? count : 1;
  if (count == 0) return HS_OK;
  GatherParams p{static_cast<const char *>(host_alias), host_blocks, static_cast<char *>(pool),
                 pool_blocks, miss_host, miss_device, count, segment, page_size, row_bytes,
                 device_status};
  const uintptr_t align = reinterpret_cast<uintptr_t>(host_alias) |
                          reinterpret_cast<uintptr_t>(pool) | (uintptr_t)row_bytes;
  const int64_t warps_needed = count;
  int64_t blocks = ceil_div(warps_needed, kGatherWarps);
  // One small CTA per SM at most: enough host-link reads in flight (4 KiB per
  // warp) while leaving each SM room for the attention that overlaps the gather.
  const int64_t cap = (int64_t)sm_count();
  if (blocks > cap) blocks = cap;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((align & 15) == 0) gather_kernel<uint4><<<(unsigned)blocks, kGatherThreads, 0, s>>>(p);
  else if ((align & 7) == 0) gather_kernel<uint2><<<(unsigned)blocks, kGatherThreads, 0, s>>>(p);
  else if ((align & 3) == 0) gather_kernel<uint32_t><<<(unsigned)blocks, kGatherThreads, 0, s>>>(p);
  else if ((align & 1) == 0) gather_kernel<uint16_t><<<(unsigned)blocks, kGatherThreads, 0, s>>>(p);
  else gather_kernel<uint8_t><<<(unsigned)blocks, kGatherThreads, 0, s>>>(p);
  return check_launch("gather_kernel");
}
