// Shared helpers for the libhisparse kernels: element conversion, vector
// loads, warp reductions, device status flags and host-side error reporting.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "hisparse.h"

namespace hs {

constexpr unsigned kFullMask = 0xffffffffu;

// ---- host-side error reporting (hs_last_error) ----------------------------
int set_error(int status, const char *fmt, ...);
int check_launch(const char *what);
int sm_count();
// Raises `func`'s dynamic shared-memory limit to at least `bytes` on the
// current device, calling the runtime only the first time a larger limit is
// needed (so launches inside a CUDA-graph capture make no such call).
int reserve_smem(const void *func, size_t bytes, const char *what);

// ---- element types ---------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_float(float x) { return x; }
  static __device__ __forceinline__ float from_float(float x) { return x; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_float(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_float(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_float(__nv_bfloat16 x) {
    return __bfloat162float(x);
  }
  static __device__ __forceinline__ __nv_bfloat16 from_float(float x) {
    return __float2bfloat16_rn(x);
  }
};

template <typename T> __device__ __forceinline__ float to_f32(T x) {
  return Elem<T>::to_float(x);
}
template <typename T> __device__ __forceinline__ T from_f32(float x) {
  return Elem<T>::from_float(x);
}

// Loads N consecutive elements starting at p (aligned to N * sizeof(T) when
// `aligned` is true) and converts them to fp32.
template <typename T, int N>
__device__ __forceinline__ void load_f32(const T *p, float (&out)[N], bool aligned) {
  constexpr int bytes = N * (int)sizeof(T);
  if (aligned && (bytes == 16 || bytes == 8 || bytes == 4)) {
    if constexpr (bytes == 16) {
      uint4 raw = __ldg(reinterpret_cast<const uint4 *>(p));
      const T *e = reinterpret_cast<const T *>(&raw);
#pragma unroll
      for (int i = 0; i < N; ++i) out[i] = to_f32(e[i]);
      return;
    } else if constexpr (bytes == 8) {
      uint2 raw = __ldg(reinterpret_cast<const uint2 *>(p));
      const T *e = reinterpret_cast<const T *>(&raw);
#pragma unroll
      for (int i = 0; i < N; ++i) out[i] = to_f32(e[i]);
      return;
    } else if constexpr (bytes == 4) {
      uint32_t raw = __ldg(reinterpret_cast<const uint32_t *>(p));
      const T *e = reinterpret_cast<const T *>(&raw);
#pragma unroll
      for (int i = 0; i < N; ++i) out[i] = to_f32(e[i]);
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = to_f32(p[i]);
}

// ---- device status ------------------------------------------------------------
__device__ __forceinline__ void flag(int32_t *status, int bits) {
  if (status != nullptr) atomicOr(status, bits);
}

// ---- warp helpers -------------------------------------------------------------
// Sum over the 32 lanes, pairing (j, j^16), (j, j^8), ..., (j, j^1). Every lane
// receives the same value (fp32 addition is commutative).
__device__ __forceinline__ float warp_xor_tree_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFullMask, v, o));
  return v;
}

template <typename T> __device__ __forceinline__ T warp_sum_int(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
  return v;
}

// Inclusive prefix sum over the 32 lanes.
template <typename T> __device__ __forceinline__ T warp_inclusive_scan(T v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T n = __shfl_up_sync(kFullMask, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

// ---- thread-block clusters -----------------------------------------------------
// Barrier over every thread of every CTA of the cluster; orders the shared-
// memory writes before it (release) with the reads after it (acquire).
__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n"
               "barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ unsigned cluster_rank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
// Generic address of `p` (this CTA's shared memory) in the shared memory of CTA
// `rank` of the cluster.
template <typename T> __device__ __forceinline__ T *map_rank(T *p, unsigned rank) {
  uint64_t out;
  asm volatile("mapa.u64 %0, %1, %2;\n" : "=l"(out) : "l"(reinterpret_cast<uint64_t>(p)),
               "r"(rank));
  return reinterpret_cast<T *>(out);
}

// Block-wide exclusive scan of one value per thread; returns the exclusive
// prefix and writes the block total to *total. `scratch` holds >= 33 T.
// Must be called by every thread of the block.
template <typename T>
__device__ __forceinline__ T block_exclusive_scan(T v, T *scratch, T *total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps = (blockDim.x + 31) >> 5;
  T inc = warp_inclusive_scan(v);
  if (lane == 31) scratch[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    T w = lane < warps ? scratch[lane] : T(0);
    T winc = warp_inclusive_scan(w);
    scratch[lane] = winc - w;  // exclusive prefix of warp totals
    if (lane == 31) scratch[32] = winc;
  }
  __syncthreads();
  T result = scratch[warp] + inc - v;
  *total = scratch[32];
  __syncthreads();
  return result;
}

// Number of elements a thread owns when n elements are split into contiguous
// runs over the block: thread t owns [t*per, min((t+1)*per, n)).
__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) {
  return (a + b - 1) / b;
}

// Operand of a batched launch: either a device array of per-request pointers
// or one base pointer advanced by `stride` elements per request.
template <typename T> struct Batched {
  const T *base;
  int64_t stride;
  const uint64_t *pointers;
  __device__ __forceinline__ const T *at(int b) const {
    return pointers ? reinterpret_cast<const T *>(pointers[b]) : base + (int64_t)b * stride;
  }
};
template <typename T> struct BatchedMut {
  T *base;
  int64_t stride;
  const uint64_t *pointers;
  __device__ __forceinline__ T *at(int b) const {
    return pointers ? reinterpret_cast<T *>(pointers[b]) : base + (int64_t)b * stride;
  }
};

// Lengths: a device array, or one value for a single request.
struct Lengths {
  const int32_t *array;
  int64_t single;
  __device__ __forceinline__ int64_t at(int b) const {
    return array ? (int64_t)array[b] : single;
  }
};

// ---- mbarriers and 1-D bulk copies (the TMA engine's untiled form) ----------------
// Every wait is bounded: kWaitLimit tries, each of which may suspend the warp for
// up to ~1 ms until the phase completes (about 4 s in all), after which the
// caller sets HS_DEV_WAIT_TIMEOUT and winds down. No copy here uses cluster
// multicast.
constexpr long long kWaitLimit = 4000;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count));
}
// Arrive (one of the phase's expected arrivals) and add `bytes` to the
// transaction count that the phase's bulk copies will complete.
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
// Add `bytes` to the phase's transaction count without arriving.
__device__ __forceinline__ void mbar_add_tx(uint64_t *bar, unsigned bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
// Plain arrive (release: the caller's earlier shared-memory writes are visible
// to the threads that wait for the phase).
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_addr(bar)) : "memory");
}
// try_wait with a suspend-time hint: the warp sleeps until the phase
// completes (or about 1 ms passes) instead of spinning through instructions.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, unsigned parity) {
  unsigned done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return done != 0;
}
// Global -> this CTA's shared memory, completing `bytes` on `bar`. Both
// addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_copy(void *dst, const void *src, unsigned bytes,
                                          uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
      ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
// Waits for `parity` of `bar`; false (and a device flag) when the bounded
// wait runs out.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, unsigned parity, int32_t *status) {
  for (long long i = 0; i < kWaitLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  flag(status, HS_DEV_WAIT_TIMEOUT);
  return false;
}

}  // namespace hs
