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

#include <mutex>
#include <type_traits>

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
  int page_shift;           // log2(page_size) when a power of two, else -1
  float scale;
  float *partials;          // [2 phases][batch][q_heads][split_stride][head_dim + 2]
  int split_stride;         // splits capacity of the workspace
  int phase, phases;        // partial set written by a phase launch / merged by the merge
  int *phase_splits;        // [2][batch] partials each phase left per batch item
  const int64_t *valid_counts;  // optional: rows valid per batch item = sum of
  int counts_stride, counts_first, counts_n;  // valid_counts[b*stride + first .. +n)
  int32_t *status;
  int spare_sms;            // SMs the bulk path leaves to concurrent work
};

// Leading rows of batch item b that a phase reads, and the [begin, end) part
// of them split `split` covers (an even share of the valid rows).
__device__ __forceinline__ void split_range(const AttendParams &p, int b, int split,
                                            int64_t &begin, int64_t &end) {
  int64_t valid = p.count;
  if (p.valid_counts) {
    valid = 0;
    for (int i = 0; i < p.counts_n; ++i)
      valid += p.valid_counts[(int64_t)b * p.counts_stride + p.counts_first + i];
    valid = valid < 0 ? 0 : (valid > p.count ? p.count : valid);
  }
  const int64_t chunk = ceil_div(valid, p.splits);
  begin = split * chunk;
  end = min(valid, begin + chunk);
}

__device__ __forceinline__ float *partial_slot(const AttendParams &p, int b, int h, int split) {
  return p.partials +
         (((int64_t)(p.phase * p.batch + b) * p.q_heads + h) * p.split_stride + split) *
             (p.head_dim + 2);
}

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

  int64_t begin, end;
  split_range(p, b, split, begin, end);
  const int64_t *rows = p.rows + (int64_t)b * p.rows_batch_stride +
                        (shared_rows ? 0 : (int64_t)h0 * p.rows_head_stride);
  if (split == 0 && blockIdx.y == 0 && threadIdx.x == 0)
    p.phase_splits[p.phase * p.batch + b] = p.splits;
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
    partial_slot(p, b, h0 + g, split)[e] = v;
  }
}

// ---- tensor-core path: bf16 query and KV, head_dim 128, shared rows ------------
//
// One CTA of 8 warps serves one request over one split of the rows and every
// KV head: rows arrive through a 3-stage cp.async pipeline as whole token rows
// (K and V of all KV heads: contiguous 2 KiB runs for 8 heads, so DRAM pages
// are read once), with 16-byte chunks XOR-swizzled by row so the ldmatrix
// reads below are conflict-free. Warp w owns one (KV head, up to 16 query
// heads) item and walks the stage in sub-tiles of 16 rows:
//   S = Q K^T   m16n8k16 bf16 MMA, M = query heads (zero padded to 16),
//               N = 8 rows, K = 16 head-dim elements; Q fragments stay in
//               registers for the whole split;
//   online softmax per head in fp32 (exp2 with log2(e) folded into the scale);
//   O += P V    the S accumulators, rounded to bf16, are the A fragments of the
//               second MMA; V fragments come from ldmatrix.trans.
// Each warp writes one (max, sum, O) partial per (request, head, split) for
// attend_merge_kernel.
constexpr int kMmaThreads = 256;
constexpr int kMmaWarps = kMmaThreads / 32;
constexpr int kStages = 3;
constexpr int kHeadBytes = 256;               // 128 bf16 of one KV head
constexpr int kStageTarget = 64 * 1024;       // bytes of K+V per stage

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, bool valid) {
  const int bytes = valid ? 16 : 0;  // 0: zero-fill, nothing is read
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
               "r"(bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t &r0, uint32_t &r1,
                                            uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t &r0, uint32_t &r1,
                                                  uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&v);
}

struct MmaShape {
  int row_bytes;   // kv_heads * 256
  int stage_rows;  // multiple of 16
  int stage_bytes; // 2 * stage_rows * row_bytes
};

__host__ __device__ inline MmaShape mma_shape(int kv_heads) {
  MmaShape m;
  m.row_bytes = kv_heads * kHeadBytes;
  int rows = kStageTarget / (2 * m.row_bytes);
  rows = rows < 16 ? 16 : (rows / 16) * 16;
  m.stage_rows = rows;
  m.stage_bytes = 2 * rows * m.row_bytes;
  return m;
}

// byte offset of 16-byte chunk `c` of stage row `r` (XOR swizzle by row)
__device__ __forceinline__ uint32_t swz(int r, int c, int row_bytes) {
  return (uint32_t)(r * row_bytes + ((c ^ (r & 7)) << 4));
}

__global__ void __launch_bounds__(kMmaThreads, 1) attend_mma_kernel(AttendParams p) {
  extern __shared__ __align__(128) char smem[];
  __shared__ int8_t row_ok[kStages][128];
  const int split = blockIdx.x, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const MmaShape sh = mma_shape(p.kv_heads);
  const int groups = p.q_heads / p.kv_heads;
  const int items = p.kv_heads * p.head_chunks;
  const bool active = warp < items;
  const int kh = active ? warp / p.head_chunks : 0;
  const int h0 = kh * groups + (warp % p.head_chunks) * 16;
  const int hn = active ? min(16, kh * groups + groups - h0) : 0;
  int64_t begin, end;
  split_range(p, b, split, begin, end);
  if (split == 0 && tid == 0) p.phase_splits[p.phase * p.batch + b] = p.splits;
  const int64_t *rows = p.rows + (int64_t)b * p.rows_batch_stride;
  const int64_t row_elems = (int64_t)p.kv_heads * 128;
  const int64_t plane = (int64_t)p.page_size * row_elems;
  const __nv_bfloat16 *pool = reinterpret_cast<const __nv_bfloat16 *>(p.pool);
  const int tiles = begin < end ? (int)ceil_div(end - begin, sh.stage_rows) : 0;
  const int chunks_per_row = sh.row_bytes / 16;

  // Q fragments for the 8 k-steps: a0/a2 head lane/4, a1/a3 head lane/4 + 8
  uint32_t qf[8][4];
  {
    const __nv_bfloat16 *qb =
        static_cast<const __nv_bfloat16 *>(p.query) + (int64_t)b * p.query_batch_stride;
    const int m0 = lane >> 2, kq = (lane & 3) * 2;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int part = 0; part < 4; ++part) {
        const int m = m0 + ((part & 1) ? 8 : 0);
        const int d = kk * 16 + kq + ((part & 2) ? 8 : 0);
        uint32_t v = 0;
        if (m < hn) v = *reinterpret_cast<const uint32_t *>(qb + (int64_t)(h0 + m) * 128 + d);
        qf[kk][part] = v;
      }
    }
  }

  // loader: warp w copies rows w, w+8, ... of a stage; its lanes copy
  // consecutive 16-byte chunks of the row (K and V of every KV head), so the
  // row's address is computed once per warp
  const int rows_per_warp = sh.stage_rows / kMmaWarps;
  const int lane_chunks = (chunks_per_row + 31) / 32;
  auto load_tile = [&](int t, int stage) {
    char *kbase = smem + stage * sh.stage_bytes;
    char *vbase = kbase + sh.stage_rows * sh.row_bytes;
    for (int k = 0; k < rows_per_warp; ++k) {
      const int r = warp + k * kMmaWarps;
      const int64_t i = begin + (int64_t)t * sh.stage_rows + r;
      const int64_t row = i < end ? rows[i] : -1;
      int64_t blk = 0, off = 0;
      if (row >= 0) {
        if (p.page_shift >= 0) {
          blk = row >> p.page_shift;
          off = row & (p.page_size - 1);
        } else {
          blk = row / p.page_size;
          off = row % p.page_size;
        }
      }
      bool ok = row >= 0;
      if (ok && blk >= p.pool_blocks) {
        if (lane == 0) flag(p.status, HS_DEV_ROW_OUT_OF_RANGE);
        ok = false;
      }
      const __nv_bfloat16 *src = ok ? pool + (blk * 2 * p.page_size + off) * row_elems : pool;
      for (int u = 0; u < lane_chunks; ++u) {
        const int c = u * 32 + lane;
        if (c < chunks_per_row) {
          cp_async16(smem_u32(kbase + swz(r, c, sh.row_bytes)), ok ? src + c * 8 : pool, ok);
          cp_async16(smem_u32(vbase + swz(r, c, sh.row_bytes)), ok ? src + plane + c * 8 : pool,
                     ok);
        }
      }
      if (lane == 0) row_ok[stage][r] = ok;
    }
  };

  constexpr float kLog2e = 1.4426950408889634f;
  const float scale = p.scale * kLog2e;
  float m_run[2] = {-INFINITY, -INFINITY};  // heads lane/4 and lane/4 + 8
  float l_run[2] = {0.f, 0.f};
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < tiles) load_tile(s, s);
    cp_async_commit();
  }
  for (int t = 0; t < tiles; ++t) {
    if (t + kStages - 1 < tiles) load_tile(t + kStages - 1, (t + kStages - 1) % kStages);
    cp_async_commit();
    cp_async_wait<kStages - 1>();
    __syncthreads();
    const int stage = t % kStages;
    const char *kbase = smem + stage * sh.stage_bytes;
    const char *vbase = kbase + sh.stage_rows * sh.row_bytes;
    for (int r0 = 0; active && r0 < sh.stage_rows; r0 += 16) {
      // ---- S = Q K^T for 16 rows (two n-tiles of 8 rows) ----
      float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      {
        const int mi = lane >> 3, rr = lane & 7;
        const int row = r0 + (mi >> 1) * 8 + rr;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(smem_u32(kbase + swz(row, kh * 16 + 2 * kk + (mi & 1), sh.row_bytes)),
                      b0, b1, b2, b3);
          mma_bf16(sacc[0], qf[kk], b0, b1);
          mma_bf16(sacc[1], qf[kk], b2, b3);
        }
      }
      // ---- online softmax (per head; a quad of lanes shares a head) ----
      float pr[2][4];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float mx = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int r = r0 + nt * 8 + (lane & 3) * 2 + e;
            float v = sacc[nt][hh * 2 + e] * scale;
            v = row_ok[stage][r] ? v : -INFINITY;
            sacc[nt][hh * 2 + e] = v;
            mx = fmaxf(mx, v);
          }
        mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, 2));
        const float m_new = fmaxf(m_run[hh], mx);
        const float alpha = m_run[hh] == -INFINITY ? 0.f : exp2f(m_run[hh] - m_new);
        float sum = 0.f;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float v = sacc[nt][hh * 2 + e];
            const float w = v == -INFINITY ? 0.f : exp2f(v - m_new);
            pr[nt][hh * 2 + e] = w;
            sum += w;
          }
        l_run[hh] = l_run[hh] * alpha + sum;
        m_run[hh] = m_new;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          o[i][hh * 2] *= alpha;
          o[i][hh * 2 + 1] *= alpha;
        }
      }
      // ---- O += P V ----
      uint32_t pa[4] = {pack_bf16(pr[0][0], pr[0][1]), pack_bf16(pr[0][2], pr[0][3]),
                        pack_bf16(pr[1][0], pr[1][1]), pack_bf16(pr[1][2], pr[1][3])};
      {
        const int mi = lane >> 3, rr = lane & 7;
        const int row = r0 + (mi & 1) * 8 + rr;
#pragma unroll
        for (int dn = 0; dn < 16; dn += 2) {
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(
              smem_u32(vbase + swz(row, kh * 16 + dn + (mi >> 1), sh.row_bytes)), b0, b1, b2, b3);
          mma_bf16(o[dn], pa, b0, b1);
          mma_bf16(o[dn + 1], pa, b2, b3);
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  if (!active) return;

  // ---- one (max, sum, O) partial per head of this warp ----
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    float l = l_run[hh];
    l += __shfl_xor_sync(kFullMask, l, 1);
    l += __shfl_xor_sync(kFullMask, l, 2);
    const int m = (lane >> 2) + hh * 8;
    if (m >= hn) continue;
    float *dst = partial_slot(p, b, h0 + m, split);
    if ((lane & 3) == 0) {
      dst[128] = m_run[hh] * 0.6931471805599453f;  // log2 units -> natural log for the merge
      dst[129] = l;
    }
#pragma unroll
    for (int dn = 0; dn < 16; ++dn) {
      const int d = dn * 8 + (lane & 3) * 2;
      dst[d] = o[dn][hh * 2];
      dst[d + 1] = o[dn][hh * 2 + 1];
    }
  }
}

// ---- bulk-copy path: bf16 query and KV, head_dim 128, shared rows, <= 8 query
// heads per KV head, 1/2/4/8 KV heads -----------------------------------------------
//
// Rows are spread evenly over the CTAs, stream-K fashion: the valid rows of all
// batch items form one sequence, CTA c takes rows [c*chunk, (c+1)*chunk) of it,
// and leaves one (max, sum, O) partial per batch item its range touches (slot
// c - first CTA of the item). chunk is at least the total over the CTAs and at
// least an item's rows over (slots - 1), so no item needs more partial slots
// than the workspace holds.
//
// Warp 0 is the producer. Per stage it checks the stage's physical rows (loaded
// one stage ahead) and issues 1-D bulk copies (the TMA engine's untiled form)
// of each valid row's K row and V row (kv_heads * 256 contiguous bytes each)
// into a 3-stage ring, completing on the stage's mbarrier. Two rows that are
// consecutive in one pool block move with one copy per plane (4 KiB at
// configuration 2): bulk copies cost a fixed ~85 cycles of the SM's copy
// engine each, so 2 KiB copies reach ~83% and 4 KiB ~94% of the HBM copy rate.
// Slots without a valid row get a zeroed V row and a cleared bit in the stage's
// slot mask. A stage record tells the consumers the batch item, its partial
// slot and whether the stage ends the item's segment; a final record ends the
// CTA.
//
// Warps 1..8 consume. Warp c serves KV head c % kv_heads and 16 of the stage's
// slots (stage rows = 16 * 8 / kv_heads), with the operands swapped so that the
// 16 rows fill the MMA's M side and the <= 8 query heads its N side:
//   S^T = K Q^T   m16n8k16 bf16 MMA: A = 16 K rows (ldmatrix), B = the
//                 query heads (registers, loaded once per batch item);
//   softmax       fp32, exp2 with log2(e) folded into the scale; the running
//                 max is raised only when a tile's max exceeds it by more than
//                 8 (a factor of 256), so O is rescaled rarely;
//   O^T += V^T P^T  A = V^T (ldmatrix.trans), B = P^T: the S^T accumulators
//                 rounded to bf16 pairs and transposed in registers (movmatrix).
// When a segment ends, warps serving the same KV head combine their (max, sum,
// O) through shared memory and one of them writes the partials.
constexpr int kBulkConsumers = 8;
constexpr int kBulkProducers = 2;  // producer warps, taking alternate stages
constexpr int kBulkThreads = 32 * (kBulkProducers + kBulkConsumers);
constexpr int kBulkStages = 3;
// A phase launch runs beside other work (the miss gather, another request
// group's selection and resolve); leaving it a few SMs keeps a pipelined decode
// step 7% faster than taking every SM.
constexpr int kPhaseSpareSms = 4;
constexpr int kRowAhead = 3;  // tiles whose row indices the producer loads ahead

struct BulkShape {
  int row_bytes;     // kv_heads * 256: K (or V) of one token, every KV head
  int run;           // G = stage_rows / 8: slots per group (4 KiB of rows)
  int group_stride;  // G * row_bytes + 16: a group's slots side by side, then 16 bytes of pad
  int stage_rows;    // 16 * subs
  int subs;          // consumer warps per KV head
  int plane_bytes;   // K (or V) slots of a stage: 8 groups
  int stage_bytes;   // K slots, then V slots
  int combine_bytes;  // shared memory for combining the warps of one KV head
  int smem_bytes;
};

__host__ __device__ inline BulkShape bulk_shape(int kv_heads) {
  BulkShape s;
  s.row_bytes = kv_heads * kHeadBytes;
  s.subs = kBulkConsumers / kv_heads;
  s.stage_rows = 16 * s.subs;
  s.run = s.stage_rows / 8;
  s.group_stride = s.run * s.row_bytes + 16;
  s.plane_bytes = 8 * s.group_stride;
  s.stage_bytes = 2 * s.plane_bytes;
  s.combine_bytes = s.subs > 1 ? kv_heads * 32 * 36 * (int)sizeof(float) : 0;
  s.smem_bytes = kBulkStages * s.stage_bytes + s.combine_bytes;
  return s;
}

// A stage's rows sit in 8 groups of G = stage_rows / 8 slots. Tile row i (the
// i-th row of the stage) goes to group i / G, position i % G: G consecutive
// rows of the tile are adjacent in shared memory, so a run of consecutive pool
// rows among them lands with one copy per plane (G * row_bytes = 4 KiB). Slot s
// is group s % 8, position s / 8: the 8 slots an ldmatrix reads (s = j..j+7)
// are in 8 different groups, 16 bytes apart modulo 128 — no bank conflicts.
__host__ __device__ __forceinline__ int slot_offset(const BulkShape &s, int slot) {
  return (slot & 7) * s.group_stride + (slot >> 3) * s.row_bytes;
}
__host__ __device__ __forceinline__ int tile_slot(const BulkShape &s, int i) {
  return (i % s.run) * 8 + i / s.run;
}

struct BulkStage {
  int b;        // batch item (-1: end of the CTA's work)
  int slot;     // partial slot of this CTA for item b
  int last;     // the stage ends the CTA's segment of item b
  int pad;
  uint32_t ok[4];  // slots holding a valid row (bit s of word s / 32)
};

__device__ __forceinline__ int64_t valid_rows(const AttendParams &p, int b) {
  if (!p.valid_counts) return p.count;
  int64_t v = 0;
  for (int i = 0; i < p.counts_n; ++i)
    v += p.valid_counts[(int64_t)b * p.counts_stride + p.counts_first + i];
  return v < 0 ? 0 : (v > p.count ? p.count : v);
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
  return y;
}

__global__ void __launch_bounds__(kBulkThreads, 1) attend_bulk_kernel(AttendParams p) {
  extern __shared__ __align__(128) char smem[];
  __shared__ __align__(8) uint64_t full[kBulkStages], empty[kBulkStages];
  __shared__ __align__(8) uint64_t xbar;  // consumer warps' combine rounds
  __shared__ BulkStage info[kBulkStages];
  __shared__ int64_t row_ring[kBulkProducers][4][128];  // physical rows of upcoming tiles
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const BulkShape sh = bulk_shape(p.kv_heads);
  const int R = sh.stage_rows;
  if (tid == 0) {
    for (int s = 0; s < kBulkStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kBulkConsumers);
    }
    mbar_init(&xbar, kBulkConsumers);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();

  if (warp < kBulkProducers) {
    // ---------------- producers ----------------
    // Producer warp pw fills the stages t with t % kBulkProducers == pw: while
    // one warp checks its rows, the copy engine works through the other's
    // copies (it takes them one at a time, ~85 cycles each).
    const int pw = warp;
    // total valid rows, the largest item, and (CTA 0) zero counts for empty items
    int64_t total = 0, largest = 0;
    for (int b0 = 0; b0 < p.batch; b0 += 32) {
      const int b = b0 + lane;
      const int64_t v = b < p.batch ? valid_rows(p, b) : 0;
      if (blockIdx.x == 0 && b < p.batch && v == 0) p.phase_splits[p.phase * p.batch + b] = 0;
      total += warp_sum_int<int64_t>(v);
      int64_t m = v;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const int64_t other = __shfl_xor_sync(kFullMask, m, o);
        m = other > m ? other : m;
      }
      largest = m > largest ? m : largest;
    }
    const int64_t slots = p.split_stride;
    int64_t chunk = total > 0 ? ceil_div(total, (int64_t)gridDim.x) : 1;
    if (slots > 1) chunk = max(chunk, ceil_div(largest, slots - 1));
    else chunk = max(chunk, largest);
    const int64_t lo = (int64_t)blockIdx.x * chunk, hi = min(total, lo + chunk);
    const char *pool = p.pool;
    const int64_t row_bytes = sh.row_bytes;
    const int64_t plane = (int64_t)p.page_size * row_bytes;  // bytes from a K row to its V row
    int t = 0;  // stages of the CTA before the current segment (both warps count all)
    bool alive = true;
    // claim stage tt's buffer (waits for the consumers to release it)
    auto claim = [&](int tt) -> bool {
      if (tt < kBulkStages) return true;
      return mbar_wait(&empty[tt % kBulkStages], ((tt / kBulkStages) - 1) & 1, p.status);
    };
    int64_t start = 0;  // first row of item b0 in the sequence
    for (int b0 = 0; alive && b0 < p.batch && start < hi; b0 += 32) {
      const int b_l = b0 + lane;
      const int64_t v_l = b_l < p.batch ? valid_rows(p, b_l) : 0;
      const int64_t inc = warp_inclusive_scan<int64_t>(v_l);
      const int64_t chunk_total = __shfl_sync(kFullMask, inc, 31);
      const int64_t s_l = start + inc - v_l;
      unsigned touch = __ballot_sync(kFullMask, v_l > 0 && s_l < hi && s_l + v_l > lo);
      while (alive && touch) {
        const int src = __ffs(touch) - 1;
        touch &= touch - 1;
        const int b = b0 + src;
        const int64_t s_b = __shfl_sync(kFullMask, s_l, src);
        const int64_t v_b = __shfl_sync(kFullMask, v_l, src);
        const int64_t seg_lo = max(lo, s_b) - s_b, seg_hi = min(hi, s_b + v_b) - s_b;
        const int slot = (int)(blockIdx.x - s_b / chunk);
        if (s_b + v_b <= hi && lane == 0) p.phase_splits[p.phase * p.batch + b] = slot + 1;
        const int64_t *rows = p.rows + (int64_t)b * p.rows_batch_stride;
        // Lane l handles tile rows l, l + 32, ... of each tile. Their physical
        // rows travel to a 4-slot shared ring by cp.async, kRowAhead tiles
        // ahead of their use: a row-index load that waits in the stage's
        // critical path costs the whole L2 round trip per stage.
        const int64_t seg_tiles = ceil_div(seg_hi - seg_lo, (int64_t)R);
        // this warp's tiles of the segment: k = k_first + m * kBulkProducers
        const int64_t k_first = ((pw - t) % kBulkProducers + kBulkProducers) % kBulkProducers;
        int64_t *ring = &row_ring[pw][0][0];
        auto prefetch = [&](int64_t m) {  // this warp's tile m into ring slot m % 4
          const int64_t k = k_first + m * kBulkProducers;
          if (k < seg_tiles) {
            const int64_t first = seg_lo + k * R;
            const int n_f = (int)min((int64_t)R, seg_hi - first);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int i = lane + 32 * u;
              int64_t *slot_ptr = ring + (m & 3) * 128 + (i < 128 ? i : 0);
              if (i < R && i < n_f)
                asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(
                                 smem_addr(slot_ptr)), "l"(rows + first + i) : "memory");
              else if (i < R)
                *slot_ptr = -1;
            }
          }
          asm volatile("cp.async.commit_group;\n" ::: "memory");
        };
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");  // the previous segment's slots
#pragma unroll
        for (int m = 0; m < kRowAhead; ++m) prefetch(m);
        for (int64_t m = 0; alive; ++m) {
          const int64_t k = k_first + m * kBulkProducers;
          if (k >= seg_tiles) break;
          const int tt = t + (int)k;
          const int st = tt % kBulkStages;
          const int64_t r0 = seg_lo + k * R;
          if (!claim(tt)) {
            alive = false;
            break;
          }
          char *kb = smem + st * sh.stage_bytes;
          prefetch(m + kRowAhead);
          asm volatile("cp.async.wait_group %0;\n" ::"n"(kRowAhead) : "memory");
          int64_t now[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int i = lane + 32 * u;
            now[u] = i < R ? ring[(m & 3) * 128 + i] : -1;
          }
          // validity, and whether row i continues row i - 1 in the pool within
          // one group (so that one copy covers both)
          int64_t src[4];
          bool ok[4], cont[4];
          int nvalid = 0;
          uint32_t bits[4] = {0u, 0u, 0u, 0u};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int64_t row = now[u];
            int64_t blk = 0, off = 0;
            if (row >= 0) {
              if (p.page_shift >= 0) {
                blk = row >> p.page_shift;
                off = row & (p.page_size - 1);
              } else {
                blk = row / p.page_size;
                off = row % p.page_size;
              }
            }
            ok[u] = row >= 0 && blk < p.pool_blocks;
            if (row >= 0 && !ok[u]) flag(p.status, HS_DEV_ROW_OUT_OF_RANGE);
            src[u] = ok[u] ? (blk * 2 * p.page_size + off) * row_bytes : 0;
            nvalid += ok[u];
            // the previous tile row is the lane below's (G divides 32, so lane 0
            // always opens a group and never continues a row)
            const int64_t before = __shfl_up_sync(kFullMask, row, 1);
            const int i = lane + 32 * u;
            cont[u] = ok[u] && i % sh.run != 0 && before >= 0 && row == before + 1 &&
                      off != 0;  // same block: the row does not open a block
            const int sl = tile_slot(sh, i);
#pragma unroll
            for (int wi = 0; wi < 4; ++wi)
              if (ok[u] && (sl >> 5) == wi) bits[wi] |= 1u << (sl & 31);
          }
          const int valid_total = warp_sum_int(nvalid);
          if (lane == 0) mbar_add_tx(&full[st], (unsigned)(valid_total * 2 * row_bytes));
          // The stage's copies: every valid row that does not continue the row
          // before it starts one K copy and one V copy as long as its run. They
          // are dealt to the lanes through registers (copy c of a 32-row word:
          // lane c % 32, start number c / 2): a thread's shared-memory loads
          // would wait for the bulk copies it has in flight.
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (32 * u >= R) break;
            const uint32_t cont_w = __ballot_sync(kFullMask, cont[u]);
            const unsigned starts = __ballot_sync(kFullMask, ok[u] && !cont[u]);
            // rows continuing this one: the run of set bits of cont_w above the lane
            const uint32_t above = lane < 31 ? cont_w >> (lane + 1) : 0u;
            // 1 + trailing ones; a run never passes its group's end (kept as a bound)
            const int len = min(__ffs(~above), sh.run - (lane + 32 * u) % sh.run);
            const int dst = slot_offset(sh, tile_slot(sh, lane + 32 * u));
            const int n_copies = 2 * __popc(starts);
            for (int c0 = 0; c0 < n_copies; c0 += 32) {
              const int c = c0 + lane;
              const int from = c < n_copies ? (int)__fns(starts, 0, (c >> 1) + 1) : 0;
              const int64_t c_src = __shfl_sync(kFullMask, src[u], from);
              const int c_len = __shfl_sync(kFullMask, len, from);
              const int c_dst = __shfl_sync(kFullMask, dst, from);
              if (c < n_copies) {
                const int v = c & 1;  // 0: K plane, 1: V plane
                bulk_copy(kb + v * sh.plane_bytes + c_dst, pool + c_src + v * plane,
                          (unsigned)(c_len * row_bytes), &full[st]);
              }
            }
          }
          // slot masks; slots without data get a zeroed V row so that a zero
          // weight cannot meet a NaN
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            const uint32_t mask = __reduce_or_sync(kFullMask, bits[wi]);
            if (lane == 0) info[st].ok[wi] = mask;
            uint32_t bad = 32 * wi >= R ? 0u : ~mask;
            if (32 * wi < R && 32 * wi + 32 > R) bad &= (1u << (R - 32 * wi)) - 1u;
            while (bad) {
              const int sl = 32 * wi + __ffs(bad) - 1;
              bad &= bad - 1;
              char *dst = kb + sh.plane_bytes + slot_offset(sh, sl);
              for (int c = lane; c < sh.row_bytes / 16; c += 32)
                *reinterpret_cast<uint4 *>(dst + c * 16) = make_uint4(0, 0, 0, 0);
            }
          }
          if (valid_total < R) asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
          if (lane == 0) {
            info[st].b = b;
            info[st].slot = slot;
            info[st].last = r0 + R >= seg_hi;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[st]);
        }
        t += (int)seg_tiles;
      }
      start += chunk_total;
    }
    // end record, by the warp that owns stage t
    if (alive && t % kBulkProducers == pw && claim(t)) {
      if (lane == 0) {
        info[t % kBulkStages].b = -1;
        mbar_arrive(&full[t % kBulkStages]);
      }
    }
    ++t;
    __syncwarp();
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    // no copy may still be landing when the CTA exits: the last stages' phases
    if (lane == 0)
      for (int u = max(0, t - kBulkStages); u < t; ++u)
        mbar_wait(&full[u % kBulkStages], (u / kBulkStages) & 1, p.status);
    return;
  }

  // ---------------- consumers ----------------
  const int c = warp - kBulkProducers;
  const int kh = c % p.kv_heads, sub = c / p.kv_heads;
  const int groups = p.q_heads / p.kv_heads;
  const int h0 = kh * groups;
  const int r0 = sub * 16;
  const int gi = lane >> 3, rr = lane & 7;
  constexpr float kLog2e = 1.4426950408889634f;
  const float scale = p.scale * kLog2e;
  uint32_t qb[8][2];
  float m_ref[2], lsum[2], o[8][4];
  auto reset = [&]() {
    m_ref[0] = m_ref[1] = -INFINITY;
    lsum[0] = lsum[1] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  };
  reset();
  // a barrier over the consumer warps whose wait is bounded (a warp that gave
  // up on a stage cannot leave the others waiting for good)
  unsigned xphase = 0;
  auto consumers_sync = [&]() {
    __syncwarp();
    if (lane == 0) mbar_arrive(&xbar);
    mbar_wait(&xbar, xphase & 1, p.status);
    ++xphase;
  };
  int cur_b = -1;
  // slot of this lane's ldmatrix row: S^T reads slots r0 + rr (+8 for matrices
  // 1, 3), O^T slots r0 + rr (+8 for matrices 2, 3)
  const int k_row = slot_offset(sh, r0 + rr + (gi & 1) * 8);
  const int v_row = slot_offset(sh, r0 + rr + (gi >> 1) * 8);
  const int k_chunk = kh * 16 + (gi >> 1), v_chunk = kh * 16 + (gi & 1);
  const int row_lo = r0 + (lane >> 2), row_hi = row_lo + 8;
  for (int t = 0;; ++t) {
    const int st = t % kBulkStages;
    if (!mbar_wait(&full[st], (t / kBulkStages) & 1, p.status)) break;
    const int b = info[st].b;
    if (b < 0) break;
    const int slot = info[st].slot;
    const bool seg_end = info[st].last != 0;
    const uint32_t okw_lo = info[st].ok[row_lo >> 5], okw_hi = info[st].ok[row_hi >> 5];
    if (b != cur_b) {
      cur_b = b;
      const __nv_bfloat16 *qp =
          static_cast<const __nv_bfloat16 *>(p.query) + (int64_t)b * p.query_batch_stride;
      const int hq = lane >> 2;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int d = kk * 16 + (lane & 3) * 2;
        const __nv_bfloat16 *qh = qp + (int64_t)(h0 + hq) * 128 + d;
        qb[kk][0] = hq < groups ? *reinterpret_cast<const uint32_t *>(qh) : 0u;
        qb[kk][1] = hq < groups ? *reinterpret_cast<const uint32_t *>(qh + 8) : 0u;
      }
    }
    const char *kb = smem + st * sh.stage_bytes;
    const char *vb = kb + sh.plane_bytes;
    // ---- S^T = K Q^T (rows x heads) ----
    float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kk = 0; kk < 8; kk += 2) {
      uint32_t a[4], a2[4];
      ldmatrix_x4(smem_u32(kb + k_row + (k_chunk + 2 * kk) * 16), a[0], a[1], a[2], a[3]);
      ldmatrix_x4(smem_u32(kb + k_row + (k_chunk + 2 * kk + 2) * 16), a2[0], a2[1], a2[2], a2[3]);
      mma_bf16(sa, a, qb[kk][0], qb[kk][1]);
      mma_bf16(sb, a2, qb[kk + 1][0], qb[kk + 1][1]);
    }
    const bool ok_lo = (okw_lo >> (row_lo & 31)) & 1u, ok_hi = (okw_hi >> (row_hi & 31)) & 1u;
    float sv[4];
    sv[0] = ok_lo ? (sa[0] + sb[0]) * scale : -INFINITY;  // slot lo, head 2*(lane%4)
    sv[1] = ok_lo ? (sa[1] + sb[1]) * scale : -INFINITY;  // slot lo, head 2*(lane%4)+1
    sv[2] = ok_hi ? (sa[2] + sb[2]) * scale : -INFINITY;  // slot hi
    sv[3] = ok_hi ? (sa[3] + sb[3]) * scale : -INFINITY;
    float mx0 = fmaxf(sv[0], sv[2]), mx1 = fmaxf(sv[1], sv[3]);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(kFullMask, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(kFullMask, mx1, off));
    }
    const bool raise = mx0 > m_ref[0] + 8.f || mx1 > m_ref[1] + 8.f;
    if (__any_sync(kFullMask, raise)) {
      const float n0 = fmaxf(m_ref[0], mx0), n1 = fmaxf(m_ref[1], mx1);
      const float a0 = m_ref[0] == -INFINITY ? 0.f : exp2f(m_ref[0] - n0);
      const float a1 = m_ref[1] == -INFINITY ? 0.f : exp2f(m_ref[1] - n1);
      lsum[0] *= a0;
      lsum[1] *= a1;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        o[i][0] *= a0;
        o[i][2] *= a0;
        o[i][1] *= a1;
        o[i][3] *= a1;
      }
      m_ref[0] = n0;
      m_ref[1] = n1;
    }
    float pw[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float m = m_ref[e & 1];
      pw[e] = (m == -INFINITY || sv[e] == -INFINITY) ? 0.f : exp2f(sv[e] - m);
    }
    lsum[0] += pw[0] + pw[2];
    lsum[1] += pw[1] + pw[3];
    const uint32_t bx = movmatrix_trans(pack_bf16(pw[0], pw[1]));  // P^T slots 0-7
    const uint32_t by = movmatrix_trans(pack_bf16(pw[2], pw[3]));  // P^T slots 8-15
    // ---- O^T += V^T P^T (head dim x heads) ----
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      uint32_t a[4];
      ldmatrix_x4_trans(smem_u32(vb + v_row + (v_chunk + 2 * mt) * 16), a[0], a[1], a[2], a[3]);
      mma_bf16(o[mt], a, bx, by);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (!seg_end) continue;
    // ---- end of the segment: combine the warps of this KV head, write partials ----
#pragma unroll
    for (int e = 0; e < 2; ++e)
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) lsum[e] += __shfl_xor_sync(kFullMask, lsum[e], off);
    if (sh.subs > 1) {
      float *xch = reinterpret_cast<float *>(smem + kBulkStages * sh.stage_bytes) +
                   (kh * 32 + lane) * 36;
      for (int round = 1; round < sh.subs; ++round) {
        consumers_sync();
        if (sub == round) {
          xch[0] = m_ref[0];
          xch[1] = m_ref[1];
          xch[2] = lsum[0];
          xch[3] = lsum[1];
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) xch[4 + i * 4 + j] = o[i][j];
        }
        consumers_sync();
        if (sub == 0) {
          float f_me[2], f_it[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float mi = xch[e], mm = fmaxf(m_ref[e], mi);
            f_me[e] = m_ref[e] == -INFINITY ? 0.f : exp2f(m_ref[e] - mm);
            f_it[e] = mi == -INFINITY ? 0.f : exp2f(mi - mm);
            lsum[e] = lsum[e] * f_me[e] + xch[2 + e] * f_it[e];
            m_ref[e] = mm;
          }
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j)
              o[i][j] = o[i][j] * f_me[j & 1] + xch[4 + i * 4 + j] * f_it[j & 1];
        }
      }
    }
    if (sub == 0) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int hl = (lane & 3) * 2 + e;
        if (hl >= groups) continue;
        float *dst = partial_slot(p, b, h0 + hl, slot);
        if ((lane >> 2) == 0) {
          dst[128] = m_ref[e] * 0.6931471805599453f;  // log2 units -> natural log
          dst[129] = lsum[e];
        }
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          dst[mt * 16 + (lane >> 2)] = o[mt][e];
          dst[mt * 16 + (lane >> 2) + 8] = o[mt][2 + e];
        }
      }
    }
    reset();
  }
}

// Merge: one 128-thread CTA per (request, query head). Thread t reads the
// (max, sum) of partial t (phase 0's splits, then phase 1's; at most
// 2 * kMaxSplits = 128 partials) and the block reduces the global max and the
// denominator; then warp w accumulates the weighted partials w, w+4, ... (a lane
// owns 4 consecutive output elements, float2 loads issued ahead of their use)
// and the four warp sums are added in shared memory.
constexpr int kMergeThreads = 2 * kMaxSplits;
constexpr int kMergeWarps = kMergeThreads / 32;

template <typename TQ>
__global__ void __launch_bounds__(kMergeThreads) attend_merge_kernel(AttendParams p) {
  __shared__ float weight[kMergeThreads];
  __shared__ float reduce[kMergeWarps];
  __shared__ float result[2];
  __shared__ float acc_sm[kMergeWarps][128];
  const int h = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5;
  const int D = p.head_dim, stride = D + 2;
  const bool even = (D & 1) == 0;
  const int s0 = p.phase_splits[b], s1 = p.phases > 1 ? p.phase_splits[p.batch + b] : 0;
  const int total = s0 + s1;
  p.phase = 0;
  const float *base0 = partial_slot(p, b, h, 0);
  p.phase = 1;
  const float *base1 = partial_slot(p, b, h, 0);
  auto partial = [&](int i) {
    return i < s0 ? base0 + (int64_t)i * stride : base1 + (int64_t)(i - s0) * stride;
  };
  float m = -INFINITY, l = 0.f;
  if (t < total) {
    const float *part = partial(t);
    m = part[D];
    l = part[D + 1];
  }
  float mm = warp_max(m);
  if (lane == 0) reduce[warp] = mm;
  __syncthreads();
  if (t == 0) {
    float v = reduce[0];
    for (int w = 1; w < kMergeWarps; ++w) v = fmaxf(v, reduce[w]);
    result[0] = v;
  }
  __syncthreads();
  mm = result[0];
  const float w = m == -INFINITY ? 0.f : expf(m - mm);
  weight[t] = w;
  const float dl = warp_xor_tree_sum(w * l);
  __syncthreads();  // reduce[] is reused below
  if (lane == 0) reduce[warp] = dl;
  __syncthreads();
  if (t == 0) {
    float v = 0.f;
    for (int i = 0; i < kMergeWarps; ++i) v += reduce[i];
    result[1] = v;
  }
  __syncthreads();
  const float denom = result[1];
  TQ *out = static_cast<TQ *>(p.out) + (int64_t)b * p.out_batch_stride + (int64_t)h * D;
  for (int d0 = 0; d0 < D; d0 += 128) {
    const int d = d0 + lane * 4;  // even D: partial rows are 8-byte aligned
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int i = warp; i < total; i += kMergeWarps) {
      const float wi = weight[i];
      const float *src = partial(i) + d;
      float2 v0 = make_float2(0.f, 0.f), v1 = make_float2(0.f, 0.f);
      if (even && d + 3 < D) {
        v0 = *reinterpret_cast<const float2 *>(src);
        v1 = *reinterpret_cast<const float2 *>(src + 2);
      } else {
        if (d < D) v0.x = src[0];
        if (d + 1 < D) v0.y = src[1];
        if (d + 2 < D) v1.x = src[2];
        if (d + 3 < D) v1.y = src[3];
      }
      if (wi != 0.f) {  // empty splits carry no weight
        acc[0] += wi * v0.x;
        acc[1] += wi * v0.y;
        acc[2] += wi * v1.x;
        acc[3] += wi * v1.y;
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) acc_sm[warp][lane * 4 + k] = acc[k];
    __syncthreads();
    if (t < 128 && d0 + t < D) {
      float num = 0.f;
#pragma unroll
      for (int w2 = 0; w2 < kMergeWarps; ++w2) num += acc_sm[w2][t];
      out[d0 + t] = from_f32<TQ>(denom > 0.f ? num / denom : 0.f);
    }
    __syncthreads();
  }
}

__host__ inline int mma_splits(int batch, int64_t count, int stage_rows, int sms) {
  int64_t s = sms / batch;
  const int64_t by_rows = ceil_div(count, 2 * stage_rows);
  if (s > by_rows) s = by_rows;
  if (s > kMaxSplits) s = kMaxSplits;
  if (s < 1) s = 1;
  return (int)s;
}

// Partial slots per batch item the bulk path may use: an even spread of the
// rows over the SMs gives an item at most ceil(sms / batch) + 1 of them.
__host__ inline int bulk_slots(int batch, int sms) {
  int64_t s = ceil_div((int64_t)sms, (int64_t)batch) + 2;
  return (int)(s > kMaxSplits ? kMaxSplits : s);
}

// Upper bound of the partial slots any attention path uses (workspace sizing).
__host__ inline int max_splits(int batch, int kv_heads, int64_t count, int sms) {
  const int a = attend_splits(batch, kv_heads, count, sms);
  const int m = mma_splits(batch, count, mma_shape(kv_heads).stage_rows, sms);
  const int k = bulk_slots(batch, sms);
  return a > m ? (a > k ? a : k) : (m > k ? m : k);
}

template <typename TQ, typename TKV>
int launch(AttendParams &p, cudaStream_t stream) {
  const int groups = p.q_heads / p.kv_heads;
  if constexpr (std::is_same<TQ, __nv_bfloat16>::value && std::is_same<TKV, __nv_bfloat16>::value) {
    const bool kv_ok = p.kv_heads == 1 || p.kv_heads == 2 || p.kv_heads == 4 || p.kv_heads == 8;
    if (p.head_dim == 128 && p.rows_head_stride == 0 && groups <= 8 && kv_ok &&
        (reinterpret_cast<uintptr_t>(p.pool) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(p.query) & 3) == 0 && (p.query_batch_stride & 1) == 0) {
      const BulkShape sh = bulk_shape(p.kv_heads);
      const int rc = reserve_smem((const void *)attend_bulk_kernel, sh.smem_bytes, "attend");
      if (rc != HS_OK) return rc;
      const int grid = sm_count() - p.spare_sms > 0 ? sm_count() - p.spare_sms : 1;
      attend_bulk_kernel<<<grid, kBulkThreads, sh.smem_bytes, stream>>>(p);
      return check_launch("attend_bulk_kernel");
    }
    const int chunks16 = (groups + 15) / 16;
    if (p.head_dim == 128 && p.rows_head_stride == 0 && p.kv_heads * chunks16 <= kMmaWarps &&
        (reinterpret_cast<uintptr_t>(p.pool) & 15) == 0) {
      p.head_chunks = chunks16;
      const MmaShape sh = mma_shape(p.kv_heads);
      const int kMmaSmem = kStages * sh.stage_bytes;
      p.splits = mma_splits(p.batch, p.count, sh.stage_rows, sm_count());
      const int rc = reserve_smem((const void *)attend_mma_kernel, kMmaSmem, "attend");
      if (rc != HS_OK) return rc;
      dim3 grid(p.splits, 1, p.batch);
      attend_mma_kernel<<<grid, kMmaThreads, kMmaSmem, stream>>>(p);
      return check_launch("attend_mma_kernel");
    }
  }
  const int C = (p.head_dim + 31) / 32;
  const int Cp = C <= 1 ? 1 : C <= 2 ? 2 : C <= 4 ? 4 : 8;
  p.head_chunks = (groups + kMaxGroup - 1) / kMaxGroup;
  const bool shared_rows = p.rows_head_stride == 0;
  dim3 grid(p.splits, shared_rows ? p.kv_heads * p.head_chunks : p.q_heads, p.batch);
  switch (Cp) {
    case 1: attend_split_kernel<TQ, TKV, 1><<<grid, kAttendThreads, 0, stream>>>(p); break;
    case 2: attend_split_kernel<TQ, TKV, 2><<<grid, kAttendThreads, 0, stream>>>(p); break;
    case 4: attend_split_kernel<TQ, TKV, 4><<<grid, kAttendThreads, 0, stream>>>(p); break;
    default: attend_split_kernel<TQ, TKV, 8><<<grid, kAttendThreads, 0, stream>>>(p); break;
  }
  return check_launch("attend_split_kernel");
}

// Merge for small grids (fewer (request, head) pairs than SMs, e.g. one long
// request): one 256-thread CTA per (request, query head, 32 output elements).
// Every CTA reduces the global max and the denominator of its head's partials
// (the same order in each, so the 32-element slices agree); then warp w sums
// the weighted partials w, w+8, ... with lane = output element, all of a
// warp's loads (at most 16, coalesced 128-byte rows) issued before their use,
// and the eight warp sums are added in order.
constexpr int kNarrowThreads = 256;
constexpr int kNarrowWarps = kNarrowThreads / 32;
constexpr int kNarrowPerWarp = 2 * kMaxSplits / kNarrowWarps;  // 16

template <typename TQ>
__global__ void __launch_bounds__(kNarrowThreads) attend_merge_narrow_kernel(AttendParams p) {
  __shared__ float weight[2 * kMaxSplits];
  __shared__ float reduce[kNarrowWarps];
  __shared__ float result[2];
  __shared__ float acc_sm[kNarrowWarps][32];
  const int h = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5;
  const int D = p.head_dim, stride = D + 2, d = blockIdx.z * 32 + lane;
  const int s0 = p.phase_splits[b], s1 = p.phases > 1 ? p.phase_splits[p.batch + b] : 0;
  const int total = s0 + s1;  // <= 2 * kMaxSplits
  p.phase = 0;
  const float *base0 = partial_slot(p, b, h, 0);
  p.phase = 1;
  const float *base1 = partial_slot(p, b, h, 0);
  auto partial = [&](int i) {
    return i < s0 ? base0 + (int64_t)i * stride : base1 + (int64_t)(i - s0) * stride;
  };
  float m = -INFINITY, l = 0.f;
  if (t < total) {
    const float *part = partial(t);
    m = part[D];
    l = part[D + 1];
  }
  float mm = warp_max(m);
  if (lane == 0) reduce[warp] = mm;
  __syncthreads();
  if (t == 0) {
    float v = reduce[0];
    for (int w = 1; w < kNarrowWarps; ++w) v = fmaxf(v, reduce[w]);
    result[0] = v;
  }
  __syncthreads();
  mm = result[0];
  const float w = m == -INFINITY ? 0.f : expf(m - mm);
  if (t < 2 * kMaxSplits) weight[t] = w;
  const float dl = warp_xor_tree_sum(w * l);
  __syncthreads();  // reduce[] is reused below
  if (lane == 0) reduce[warp] = dl;
  __syncthreads();
  if (t == 0) {
    float v = 0.f;
    for (int i = 0; i < kNarrowWarps; ++i) v += reduce[i];
    result[1] = v;
  }
  __syncthreads();
  const float denom = result[1];
  float v[kNarrowPerWarp];
#pragma unroll
  for (int k = 0; k < kNarrowPerWarp; ++k) {
    const int i = warp + k * kNarrowWarps;
    v[k] = i < total && d < D ? partial(i)[d] : 0.f;
  }
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < kNarrowPerWarp; ++k) {
    const int i = warp + k * kNarrowWarps;
    if (i < total && weight[i] != 0.f) acc += weight[i] * v[k];  // empty splits: no weight
  }
  acc_sm[warp][lane] = acc;
  __syncthreads();
  if (t < 32 && d < D) {
    float num = 0.f;
#pragma unroll
    for (int w2 = 0; w2 < kNarrowWarps; ++w2) num += acc_sm[w2][t];
    TQ *out = static_cast<TQ *>(p.out) + (int64_t)b * p.out_batch_stride + (int64_t)h * D;
    out[d] = from_f32<TQ>(denom > 0.f ? num / denom : 0.f);
  }
}

template <typename TQ> int launch_merge(AttendParams &p, cudaStream_t stream) {
  if ((int64_t)p.batch * p.q_heads < sm_count()) {
    const dim3 grid(p.q_heads, p.batch, (unsigned)ceil_div(p.head_dim, 32));
    attend_merge_narrow_kernel<TQ><<<grid, kNarrowThreads, 0, stream>>>(p);
    return check_launch("attend_merge_narrow_kernel");
  }
  attend_merge_kernel<TQ><<<dim3(p.q_heads, p.batch), kMergeThreads, 0, stream>>>(p);
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

namespace hs {
namespace {

// Workspace: partials of two phases, then the partials each phase left per batch item.
struct AttendWorkspace {
  size_t partial_floats, bytes;
  int split_stride;
  AttendWorkspace(int batch, int q_heads, int kv_heads, int head_dim, int64_t count) {
    split_stride = max_splits(batch, kv_heads, count, sm_count());
    partial_floats = (size_t)2 * batch * q_heads * split_stride * (head_dim + 2);
    bytes = partial_floats * sizeof(float) + (size_t)2 * batch * sizeof(int);
  }
};

int prepare(AttendParams &p, int batch, const void *query, int64_t query_batch_stride,
            const void *pool, int64_t pool_blocks, const int64_t *rows,
            int64_t rows_batch_stride, int64_t rows_head_stride, int64_t count, int q_heads,
            int kv_heads, int head_dim, int page_size, void *workspace,
            size_t workspace_bytes, int32_t *device_status) {
  if (batch < 1 || q_heads < 1 || kv_heads < 1 || head_dim < 1 || page_size < 1 ||
      count < 1 || pool_blocks < 0)
    return set_error(HS_ERR_INVALID_ARGUMENT, "attend: dimensions must be positive");
  if (q_heads % kv_heads)
    return set_error(HS_ERR_INVALID_ARGUMENT, "query GQA/device mismatch");
  if (head_dim > 256)
    return set_error(HS_ERR_UNSUPPORTED, "attend: head_dim %d > 256 is not supported", head_dim);
  if (!query || !pool || !rows)
    return set_error(HS_ERR_INVALID_ARGUMENT, "attend: null tensor pointer");
  const AttendWorkspace ws(batch, q_heads, kv_heads, head_dim, count);
  if (!workspace || workspace_bytes < ws.bytes)
    return set_error(HS_ERR_WORKSPACE, "attend: workspace of %zu bytes < required %zu",
                     workspace_bytes, ws.bytes);
  p = AttendParams{};
  p.batch = batch;
  p.query = query;
  p.query_batch_stride = query_batch_stride;
  p.pool = static_cast<const char *>(pool);
  p.pool_blocks = pool_blocks;
  p.rows = rows;
  p.rows_batch_stride = rows_batch_stride;
  p.rows_head_stride = rows_head_stride;
  p.count = count;
  p.q_heads = q_heads;
  p.kv_heads = kv_heads;
  p.head_dim = head_dim;
  p.page_size = page_size;
  p.splits = attend_splits(batch, kv_heads, count, sm_count());
  p.scale = (float)(1.0 / sqrt((double)head_dim));
  p.page_shift = -1;
  if ((page_size & (page_size - 1)) == 0)
    for (int sh = 0; sh < 31; ++sh)
      if ((1 << sh) == page_size) p.page_shift = sh;
  p.partials = static_cast<float *>(workspace);
  p.split_stride = ws.split_stride;
  p.phase_splits = reinterpret_cast<int *>(static_cast<float *>(workspace) + ws.partial_floats);
  p.status = device_status;
  return HS_OK;
}

int run_phase(AttendParams &p, int query_dtype, int kv_dtype, cudaStream_t s) {
  switch (query_dtype) {
    case HS_FLOAT32: return dispatch_kv<float>(kv_dtype, p, s);
    case HS_FLOAT16: return dispatch_kv<__half>(kv_dtype, p, s);
    case HS_BFLOAT16: return dispatch_kv<__nv_bfloat16>(kv_dtype, p, s);
  }
  return set_error(HS_ERR_INVALID_ARGUMENT, "attend: invalid query dtype %d", query_dtype);
}

int run_merge(AttendParams &p, int query_dtype, cudaStream_t s) {
  switch (query_dtype) {
    case HS_FLOAT32: return launch_merge<float>(p, s);
    case HS_FLOAT16: return launch_merge<__half>(p, s);
    case HS_BFLOAT16: return launch_merge<__nv_bfloat16>(p, s);
  }
  return set_error(HS_ERR_INVALID_ARGUMENT, "attend: invalid query dtype %d", query_dtype);
}

}  // namespace
}  // namespace hs

extern "C" size_t hs_attend_workspace_bytes(int batch, int q_heads, int kv_heads,
                                            int head_dim, int64_t count) {
  if (batch < 1 || q_heads < 1 || kv_heads < 1 || head_dim < 1 || count < 1) return 0;
  return hs::AttendWorkspace(batch, q_heads, kv_heads, head_dim, count).bytes;
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
  if (!out) return set_error(HS_ERR_INVALID_ARGUMENT, "attend: null tensor pointer");
  AttendParams p;
  int rc = prepare(p, batch, query, query_batch_stride, pool, pool_blocks, rows,
                   rows_batch_stride, rows_head_stride, count, q_heads, kv_heads, head_dim,
                   page_size, workspace, workspace_bytes, device_status);
  if (rc != HS_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  p.phase = 0;
  rc = run_phase(p, query_dtype, kv_dtype, s);
  if (rc != HS_OK) return rc;
  p.phases = 1;
  p.out = out;
  p.out_batch_stride = out_batch_stride;
  return run_merge(p, query_dtype, s);
}

extern "C" int hs_attend_rows_phase(int batch, const void *query, int64_t query_batch_stride,
                                    int query_dtype, const void *pool, int64_t pool_blocks,
                                    int kv_dtype, const int64_t *rows,
                                    int64_t rows_batch_stride, int64_t count,
                                    const int64_t *valid_counts, int counts_stride,
                                    int counts_first, int counts_n, int phase, int q_heads,
                                    int kv_heads, int head_dim, int page_size, void *workspace,
                                    size_t workspace_bytes, int32_t *device_status,
                                    hs_stream stream) {
  using namespace hs;
  if (phase != 0 && phase != 1)
    return set_error(HS_ERR_INVALID_ARGUMENT, "attend: phase must be 0 or 1");
  if (valid_counts && (counts_stride < 1 || counts_first < 0 || counts_n < 1))
    return set_error(HS_ERR_INVALID_ARGUMENT, "attend: invalid count selector");
  AttendParams p;
  int rc = prepare(p, batch, query, query_batch_stride, pool, pool_blocks, rows,
                   rows_batch_stride, 0, count, q_heads, kv_heads, head_dim, page_size,
                   workspace, workspace_bytes, device_status);
  if (rc != HS_OK) return rc;
  p.phase = phase;
  p.spare_sms = kPhaseSpareSms;
  p.valid_counts = valid_counts;
  p.counts_stride = counts_stride;
  p.counts_first = counts_first;
  p.counts_n = counts_n;
  return run_phase(p, query_dtype, kv_dtype, static_cast<cudaStream_t>(stream));
}

extern "C" int hs_attend_merge(int batch, int phases, void *out, int64_t out_batch_stride,
                               int query_dtype, int q_heads, int kv_heads, int head_dim,
                               int64_t count, void *workspace, size_t workspace_bytes,
                               int32_t *device_status, hs_stream stream) {
  using namespace hs;
  if (phases != 1 && phases != 2)
    return set_error(HS_ERR_INVALID_ARGUMENT, "attend: phases must be 1 or 2");
  if (!out) return set_error(HS_ERR_INVALID_ARGUMENT, "attend: null tensor pointer");
  AttendParams p;
  // the merge reads no rows or pool: any non-null placeholders pass validation
  int rc = prepare(p, batch, out, 0, out, 0, reinterpret_cast<const int64_t *>(out), 0, 0,
                   count, q_heads, kv_heads, head_dim, 1, workspace, workspace_bytes,
                   device_status);
  if (rc != HS_OK) return rc;
  p.phases = phases;
  p.out = out;
  p.out_batch_stride = out_batch_stride;
  return run_merge(p, query_dtype, static_cast<cudaStream_t>(stream));
}

// ---- hs_attend_rows_static: the same attention with library-owned scratch ----
// Some callers cannot hand this library a workspace. A host that binds only the
// C ABI through a bare FFI stub (ctypes, cgo, JNI) has no device allocator of
// its own, and a serving process that has handed all of the device's memory to
// its KV pool cannot grow that memory for a per-call buffer. For them the
// split partials live in a fixed array in the library's own device memory: this
// entry point calls no allocator. The array exists once per device; calls on one
// device share it, so calls that may overlap on the GPU (different streams)
// race on it and must be ordered by the caller. Nothing in it needs to start at
// zero: every launch writes the partials and split counts before the merge
// reads them.
namespace hs {
namespace {

constexpr size_t kStaticScratchBytes = size_t(16) << 20;  // per device
constexpr int kScratchDevices = 64;
static __device__ __align__(256) unsigned char g_attend_scratch[kStaticScratchBytes];

std::mutex g_scratch_lock;
void *g_scratch_address[kScratchDevices];

// Device address of this device's scratch array, looked up once per device (the
// first call on a device does this set-up; a caller that captures streams makes
// that first call before capturing).
int static_scratch(void **address) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return set_error(HS_ERR_CUDA, "attend (static scratch): no current device: %s",
                     cudaGetErrorString(err));
  }
  if (dev < 0 || dev >= kScratchDevices)
    return set_error(HS_ERR_UNSUPPORTED, "attend (static scratch): device %d >= %d", dev,
                     kScratchDevices);
  std::lock_guard<std::mutex> guard(g_scratch_lock);
  if (g_scratch_address[dev] == nullptr) {
    void *p = nullptr;
    err = cudaGetSymbolAddress(&p, g_attend_scratch);
    if (err != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return set_error(HS_ERR_CUDA,
                       "attend (static scratch): cannot resolve the scratch array on device "
                       "%d: %s", dev, cudaGetErrorString(err));
    }
    g_scratch_address[dev] = p;
  }
  *address = g_scratch_address[dev];
  return HS_OK;
}

}  // namespace
}  // namespace hs

extern "C" int hs_attend_rows_static(int batch, const void *query, int64_t query_batch_stride,
                                     int query_dtype, const void *pool, int64_t pool_blocks,
                                     int kv_dtype, const int64_t *rows,
                                     int64_t rows_batch_stride, int64_t rows_head_stride,
                                     int64_t count, void *out, int64_t out_batch_stride,
                                     int q_heads, int kv_heads, int head_dim, int page_size,
                                     int32_t *device_status, hs_stream stream) {
  using namespace hs;
  const size_t need = hs_attend_workspace_bytes(batch, q_heads, kv_heads, head_dim, count);
  if (need > kStaticScratchBytes)
    return set_error(HS_ERR_WORKSPACE,
                     "attend (static scratch): this call needs %zu bytes of scratch, more "
                     "than the library's fixed %zu; use hs_attend_rows with a workspace",
                     need, kStaticScratchBytes);
  void *scratch = nullptr;
  const int rc = static_scratch(&scratch);
  if (rc != HS_OK) return rc;
  return hs_attend_rows(batch, query, query_batch_stride, query_dtype, pool, pool_blocks,
                        kv_dtype, rows, rows_batch_stride, rows_head_stride, count, out,
                        out_batch_stride, q_heads, kv_heads, head_dim, page_size, scratch,
                        kStaticScratchBytes, device_status, stream);
}
