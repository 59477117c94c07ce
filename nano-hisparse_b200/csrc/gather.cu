// (3) Miss gather: copies the K-plane and V-plane rows of every planned miss
// from the pinned host store (read zero-copy through its device alias, over
// the host link) into the shared GPU pool.
//
// Reference: nano_hisparse/row_kernels.py:35-70 (_gather, gather_rows) and the
// CPU loop of hybrid.py:452-459. The reference runs min(n, 64) programs and
// recompiles per plan width; here the plan width is a runtime argument and
// the grid has one 2-warp CTA per SM. One warp moves one row, K and V planes
// side by side: up to 4 KiB of host-link reads in flight per warp (16-byte
// vectors when the layout allows), about 1 MiB over the grid — several times
// the link's bandwidth-latency product.
#include "common.cuh"

namespace hs {
namespace {

constexpr int kGatherThreads = 64;
constexpr int kGatherWarps = kGatherThreads / 32;
constexpr int kUnroll = 4;  // vectors per lane and plane in flight

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

// Two warps of at most 64 registers (4 K registers a CTA): the gather CTAs of
// two micro-batches fit on an SM beside a Quest or attention CTA, so the
// kernels that overlap the gather are not held back waiting for its registers.
// Entries are dealt to the warps round robin (entry e to warp e % warps, as a
// request's misses form a prefix of its plan segment this spreads them over
// every warp), and a warp reads 32 of its entries per load (lane l: entry
// w + l * warps): reading one entry at a time cost an L2 round trip per entry
// (~0.3 ms for a 64 x 4096-entry plan with nothing to move).
constexpr int kChunks = 2;

template <typename V>
__global__ void __launch_bounds__(kGatherThreads, 16) gather_kernel(GatherParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * kGatherWarps + (threadIdx.x >> 5);
  const int64_t warps = (int64_t)gridDim.x * kGatherWarps;
  const int vecs = (int)(p.row_bytes / (int64_t)sizeof(V));  // per plane
  const int64_t plane_stride = (int64_t)p.page_size * p.row_bytes;
  const int64_t stride = 32 * kChunks * warps;  // entries one pass of this warp covers
  for (int64_t base = warp; base < p.count; base += stride) {
    int64_t hs_[kChunks], ds_[kChunks];
#pragma unroll
    for (int k = 0; k < kChunks; ++k) {
      const int64_t e = base + (int64_t)(k * 32 + lane) * warps;
      const bool in = e < p.count;
      hs_[k] = in ? __ldcg(p.miss_host + e) : -1;
      ds_[k] = in ? __ldcg(p.miss_device + e) : -1;
    }
#pragma unroll
    for (int k = 0; k < kChunks; ++k) {
      unsigned todo = __ballot_sync(kFullMask, hs_[k] >= 0 && ds_[k] >= 0);
      while (todo) {
        const int j = __ffs(todo) - 1;
        todo &= todo - 1;
        const int64_t h = __shfl_sync(kFullMask, hs_[k], j);
        const int64_t d = __shfl_sync(kFullMask, ds_[k], j);
        const int64_t hb = h / p.page_size, db = d / p.page_size;
        if (hb >= p.host_blocks || db >= p.pool_blocks) {
          if (lane == 0) flag(p.status, HS_DEV_ROW_OUT_OF_RANGE);
          continue;
        }
        const char *src = p.host + (hb * 2 * p.page_size + h % p.page_size) * p.row_bytes;
        char *dst = p.pool + (db * 2 * p.page_size + d % p.page_size) * p.row_bytes;
        const V *k_src = reinterpret_cast<const V *>(src);
        const V *v_src = reinterpret_cast<const V *>(src + plane_stride);
        V *k_dst = reinterpret_cast<V *>(dst);
        V *v_dst = reinterpret_cast<V *>(dst + plane_stride);
        for (int c_ = lane; c_ < vecs; c_ += 32 * kUnroll) {
          V kv[kUnroll], vv[kUnroll];
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) {
            const int c = c_ + 32 * u;
            if (c < vecs) {
              kv[u] = __ldcs(k_src + c);  // host rows are read once: stream past the caches
              vv[u] = __ldcs(v_src + c);
            }
          }
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) {
            const int c = c_ + 32 * u;
            if (c < vecs) {
              k_dst[c] = kv[u];
              v_dst[c] = vv[u];
            }
          }
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
  // One small CTA per SM at most: enough host-link reads in flight while leaving
  // each SM room for the kernels that overlap the gather.
#ifdef HS_GATHER_MAX_CTAS
  const int64_t cap = HS_GATHER_MAX_CTAS;
#else
  const int64_t cap = (int64_t)sm_count();
#endif
  if (blocks > cap) blocks = cap;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((align & 15) == 0) gather_kernel<uint4><<<(unsigned)blocks, kGatherThreads, 0, s>>>(p);
  else if ((align & 7) == 0) gather_kernel<uint2><<<(unsigned)blocks, kGatherThreads, 0, s>>>(p);
  else if ((align & 3) == 0) gather_kernel<uint32_t><<<(unsigned)blocks, kGatherThreads, 0, s>>>(p);
  else if ((align & 1) == 0) gather_kernel<uint16_t><<<(unsigned)blocks, kGatherThreads, 0, s>>>(p);
  else gather_kernel<uint8_t><<<(unsigned)blocks, kGatherThreads, 0, s>>>(p);
  return check_launch("gather_kernel");
}
