// (2) Row resolver: resident lookup, hot-tag lookup, LRU replacement and the
// compact miss plan, with the in-place tag/LRU update.
//
// Reference: nano_hisparse/row_index.py:62-140 (resolve_rows). The reference
// expresses the algorithm as ~35 tensor ops (sorts, searchsorted, argsorts,
// scatters). Here one CTA of 1024 threads resolves one request:
//   1. bitonic sort of the normalised logical positions;
//   2. per sorted entry: dedupe, page -> (host row, resident block) lookup;
//   3. open-addressing hash of the hot tags (tag -> slot) shared by the hot-hit
//      lookup and the "protect every hit" pass;
//   4. block scans give each miss its rank (sorted logical order) and each
//      unprotected slot its victim rank (LRU order), so miss r takes victim r;
//   5. a stable 4-way partition of the old LRU order by category
//      (untouched, inserted, protected, inserted+protected) is the new LRU;
//   6. inputs map back to their first occurrence in input order.
// Per-request scratch lives in one CTA's shared memory when it fits; when it
// does not (e.g. 8192 positions against 16384 hot rows, ~660 KiB), a cluster
// of up to 8 CTAs holds it in distributed shared memory; beyond that it lives
// in the caller's workspace (L2-resident). The same code runs in all three
// through the scratch policy (LocalScratch / ClusterScratch). No host round
// trip: the launch is graph-capturable.
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace hs {
namespace {

constexpr int kResolveThreads = 1024;
constexpr size_t kResolveSmemLimit = 200 * 1024;
constexpr unsigned long long kEmpty = ~0ull;
constexpr unsigned long long kWantedBit = 1ull << 31;

enum : uint8_t {
  kValid = 1,        // unique, in range, and source page >= 0
  kResidentHit = 2,  // valid and resident block >= 0
  kNeedsHot = 4,     // valid and not resident
  kHotHit = 8,       // needs hot and its host row is tagged
  kMiss = 16         // needs hot and not tagged
};
enum : uint8_t { kProtected = 1, kInserted = 2 };

__host__ __device__ inline int64_t next_pow2(int64_t x) {
  int64_t p = 1;
  while (p < x) p <<= 1;
  return p;
}

__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

struct Layout {
  int64_t kp, ch;  // padded sort length, hash capacity
  size_t keys, first, flags, slot, rank, host, phys, hash, sflags, lru_old, victims, total;
  __host__ __device__ Layout(int64_t k, int64_t h) {
    kp = next_pow2(k);
    ch = next_pow2(2 * h);
    if (ch < 64) ch = 64;
    size_t o = 0;
    keys = o;    o = align16(o + kp * 4);
    first = o;   o = align16(o + k * 4);
    flags = o;   o = align16(o + k);
    slot = o;    o = align16(o + k * 4);
    rank = o;    o = align16(o + k * 4);
    host = o;    o = align16(o + k * 8);
    phys = o;    o = align16(o + k * 8);
    hash = o;    o = align16(o + ch * 8);
    sflags = o;  o = align16(o + h);
    lru_old = o; o = align16(o + h * 4);
    victims = o; o = align16(o + h * 4);
    total = o;
  }
};

struct ResolveParams {
  int batch;
  const void *positions;  // [batch, count] int32 or int64
  int positions_i64;
  int64_t count;
  Batched<int32_t> source, resident, hot;
  BatchedMut<int32_t> tags;
  BatchedMut<int64_t> lru;
  int64_t table_pages, hot_blocks, hot_rows;
  Lengths lengths;
  int page_size;
  int64_t *out_physical, *out_miss_host, *out_miss_device, *out_counts;
  int64_t *out_ready;  // optional [batch, count]: resident + hot rows, compact
  const int64_t *head_columns;
  int64_t head_count, head_width;
  int64_t *out_head_physical;
  char *workspace;  // nullptr -> shared memory
  int32_t *status;
};

__device__ __forceinline__ uint32_t hash_slot(uint32_t key, int64_t ch) {
  return (uint32_t)((key * 0x9E3779B1u) & (uint32_t)(ch - 1));
}

template <typename Table>
__device__ __forceinline__ void hash_insert(const Table &table, int64_t ch, uint32_t key,
                                            uint32_t slot) {
  const unsigned long long entry = ((unsigned long long)key << 32) | slot;
  uint32_t h = hash_slot(key, ch);
  while (true) {
    unsigned long long cur = table[h];
    if (cur == kEmpty) {
      cur = atomicCAS(&table[h], kEmpty, entry);
      if (cur == kEmpty) return;
    }
    if ((uint32_t)(cur >> 32) == key) {
      atomicMin(&table[h], entry);  // duplicate tags: keep the lowest slot
      return;
    }
    h = (h + 1) & (uint32_t)(ch - 1);
  }
}

template <typename Table>
__device__ __forceinline__ int hash_find(const Table &table, int64_t ch, uint32_t key) {
  uint32_t h = hash_slot(key, ch);
  while (true) {
    const unsigned long long cur = table[h];
    if (cur == kEmpty) return -1;
    if ((uint32_t)(cur >> 32) == key) return (int)h;
    h = (h + 1) & (uint32_t)(ch - 1);
  }
}

__device__ __forceinline__ int64_t load_position(const ResolveParams &p, int b, int64_t i) {
  const int64_t idx = (int64_t)b * p.count + i;
  return p.positions_i64 ? static_cast<const int64_t *>(p.positions)[idx]
                         : (int64_t) static_cast<const int32_t *>(p.positions)[idx];
}

// Smallest j in [0, n) with keys[j] >= v (n if none).
template <typename Keys>
__device__ __forceinline__ int lower_bound(const Keys &keys, int n, int64_t v) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if ((int64_t)keys[mid] < v) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// ---- scratch access --------------------------------------------------------------
// The per-request scratch (Layout) is one logical byte buffer. LocalScratch is
// one CTA's view of it (its shared memory, or the workspace in global memory);
// ClusterScratch spreads it over the shared memory of the CTAs of a thread-
// block cluster (distributed shared memory), 4 KiB granules dealt round-robin
// to the CTAs, so scratch too large for one SM still stays on chip and every
// array's traffic is shared by all the cluster's SMs. Both give the thread index and count, the barrier, a block- or
// cluster-wide OR and exclusive scan, and element addresses.
struct LocalScratch {
  char *base;
  __device__ __forceinline__ int tid() const { return (int)threadIdx.x; }
  __device__ __forceinline__ int nthreads() const { return (int)blockDim.x; }
  __device__ __forceinline__ void sync() const { __syncthreads(); }
  __device__ __forceinline__ bool any(int v) const { return __syncthreads_or(v) != 0; }
  template <typename T> __device__ __forceinline__ T *at(size_t off) const {
    return reinterpret_cast<T *>(base + off);
  }
  template <typename T> __device__ __forceinline__ T scan(T v, T *scratch, T *total) const {
    return block_exclusive_scan<T>(v, scratch, total);
  }
};

constexpr int kClusterShift = 17;   // 128 KiB of scratch per CTA of a cluster
constexpr int kPortableCluster = 8;  // largest portable cluster size
constexpr int kMaxCluster = 16;      // with the non-portable opt-in (powers of two are used)
constexpr int kGranuleShift = 12;   // 4 KiB granules dealt round-robin to the CTAs

struct ClusterScratch {
  char *base;                   // this CTA's part
  unsigned rank, size;          // this CTA's cluster rank, CTAs in the cluster (power of 2)
  unsigned size_log2;
  unsigned long long *totals;   // [kMaxCluster] scan totals, in this CTA's shared memory
  __device__ __forceinline__ int tid() const { return (int)(rank * blockDim.x + threadIdx.x); }
  __device__ __forceinline__ int nthreads() const { return (int)(size * blockDim.x); }
  __device__ __forceinline__ void sync() const { cluster_barrier(); }
  template <typename T> __device__ __forceinline__ T *at(size_t off) const {
    const size_t granule = off >> kGranuleShift;
    const size_t local = ((granule >> size_log2) << kGranuleShift) |
                         (off & ((size_t(1) << kGranuleShift) - 1));
    return map_rank(reinterpret_cast<T *>(base + local), (unsigned)(granule & (size - 1)));
  }
  // Exclusive scan in cluster thread order (rank-major): the block scan, then
  // each CTA's total is written into every CTA's `totals` and summed in rank order.
  template <typename T> __device__ __forceinline__ T scan(T v, T *scratch, T *total) const {
    T block_total;
    const T prefix = block_exclusive_scan<T>(v, scratch, &block_total);
    if (threadIdx.x == 0)
      for (unsigned r = 0; r < size; ++r)
        *map_rank(totals + rank, r) = (unsigned long long)block_total;
    cluster_barrier();
    T before = 0, all = 0;
    for (unsigned r = 0; r < size; ++r) {
      const T t = (T)totals[r];
      all += t;
      if (r < rank) before += t;
    }
    *total = all;
    cluster_barrier();  // `totals` is rewritten by the next scan
    return before + prefix;
  }
  __device__ __forceinline__ bool any(int v) const {
    __shared__ unsigned long long any_scratch[33];
    unsigned long long total;
    scan<unsigned long long>(v ? 1ull : 0ull, any_scratch, &total);
    return total != 0;
  }
};

template <typename T, typename S> struct Arr {
  S s;
  size_t off;
  __device__ __forceinline__ T &operator[](int64_t i) const {
    return *s.template at<T>(off + (size_t)i * sizeof(T));
  }
};

// Packed counters for one scan: misses in bits 0-20, hot hits 21-41, resident
// hits 42-62 (count < 2^21, checked on the host).
constexpr int kCountBits = 21;
constexpr unsigned long long kCountMask = (1ull << kCountBits) - 1;

// Steps 3-9 of resolve_kernel (every thread of the block or cluster calls it).
template <typename S>
__device__ __forceinline__ void resolve_body(const ResolveParams &p, const Layout &L, int b,
                                          bool sorted, const S &sc, Arr<int32_t, S> keys,
                                          Arr<int32_t, S> first_in, Arr<uint8_t, S> jflags,
                                          Arr<int32_t, S> jslot, Arr<int32_t, S> jrank,
                                          Arr<int64_t, S> jhost, Arr<int64_t, S> jphys,
                                          Arr<unsigned long long, S> table, Arr<uint8_t, S> sflags,
                                          Arr<int32_t, S> lru_old, Arr<int32_t, S> victims,
                                          unsigned long long *scan_scratch) {
  const int tid = sc.tid(), nthreads = sc.nthreads();
  const int K = (int)p.count, H = (int)p.hot_rows;
  const int32_t *src_tab = p.source.at(b);
  const int32_t *res_tab = p.resident.at(b);
  const int32_t *hot_tab = p.hot.at(b);
  int32_t *tags = p.tags.at(b);
  int64_t *lru = p.lru.at(b);
  const int64_t length = p.lengths.at(b);
  const int P = p.page_size;
  int64_t *out_phys = p.out_physical + (int64_t)b * K;
  int64_t *out_mh = p.out_miss_host + (int64_t)b * K;
  int64_t *out_md = p.out_miss_device + (int64_t)b * K;
  int64_t *out_counts = p.out_counts + (int64_t)b * 3;
  const int per_k = (K + nthreads - 1) / nthreads;
  const int klo = min(K, tid * per_k), khi = min(K, klo + per_k);
  const int per_h = (H + nthreads - 1) / nthreads;
  const int hlo = min(H, tid * per_h), hhi = min(H, hlo + per_h);
  // ---- 3. per sorted entry: dedupe and page lookups; hash of the hot tags ------
  for (int j = tid; j < K; j += nthreads) {
    const int64_t v = keys[j];
    const bool causal = v < length;  // keys are normalised to [0, length] or INT32_MAX
    const bool unique = causal && (j == 0 || keys[j - 1] != keys[j]);
    // only causal keys read the tables: a request's tables cover its own pages
    // (ceil(length / P)), which may be fewer than table_pages
    int64_t page = causal ? v / P : 0;
    if (page > p.table_pages - 1) page = p.table_pages - 1;
    const int64_t offset = v % P;
    const int64_t source = causal ? (int64_t)src_tab[page] : -1;
    const int64_t resident = causal ? (int64_t)res_tab[page] : -1;
    uint8_t f = 0;
    int64_t phys = -1;
    if (unique && source >= 0) {
      f |= kValid;
      if (resident >= 0) {
        f |= kResidentHit;
        phys = resident * P + offset;
      } else {
        f |= kNeedsHot;
      }
    }
    jflags[j] = f;
    jhost[j] = source * P + offset;
    jphys[j] = phys;
  }
  for (int s = tid; s < H; s += nthreads) {
    const int32_t t = tags[s];
    if (t >= 0) hash_insert(table, L.ch, (uint32_t)t, (uint32_t)s);
  }
  sc.sync();
  // ---- 4. hot hits; tags wanted by this selection ---------------------------------
  for (int j = tid; j < K; j += nthreads) {
    uint8_t f = jflags[j];
    if (f & kNeedsHot) {
      const int64_t host = jhost[j];
      const int at = (host >= 0 && host <= INT32_MAX) ? hash_find(table, L.ch, (uint32_t)host)
                                                       : -1;
      if (at >= 0) {
        f |= kHotHit;
        jslot[j] = (int32_t)(table[at] & 0x7fffffffu);
        atomicOr(&table[at], kWantedBit);
      } else {
        f |= kMiss;
      }
      jflags[j] = f;
    }
  }
  sc.sync();
  // ---- 5. protected slots; packed counts and miss ranks (sorted logical order) ----
  for (int s = tid; s < H; s += nthreads) {
    const int32_t t = tags[s];
    if (t >= 0) {
      const int at = hash_find(table, L.ch, (uint32_t)t);
      if (at >= 0 && (table[at] & kWantedBit)) sflags[s] = kProtected;
    }
  }
  unsigned long long totals;
  {
    unsigned long long local = 0;
    for (int j = klo; j < khi; ++j) {
      const uint8_t f = jflags[j];
      local += (f & kMiss) ? 1ull : (f & kHotHit) ? (1ull << kCountBits)
               : (f & kResidentHit) ? (1ull << (2 * kCountBits)) : 0ull;
    }
    unsigned long long prefix = sc.template scan<unsigned long long>(local, scan_scratch,
                                                                        &totals);
    int rank = (int)(prefix & kCountMask);
    int ready = (int)(((prefix >> kCountBits) & kCountMask) + ((prefix >> (2 * kCountBits)) & kCountMask));
    for (int j = klo; j < khi; ++j) {
      const uint8_t f = jflags[j];
      if (f & kMiss) jrank[j] = rank++;
      else if (f & (kHotHit | kResidentHit)) jrank[j] = ready++;  // rank in the ready list
    }
  }
  const int misses = (int)(totals & kCountMask);
  // ---- 6. victims: unprotected slots in LRU order, then protected ---------------
  {
    unsigned long long local = 0;
    for (int i = hlo; i < hhi; ++i) local += !(sflags[lru_old[i]] & kProtected);
    unsigned long long unprotected;
    int pos = (int)sc.template scan<unsigned long long>(local, scan_scratch, &unprotected);
    for (int i = hlo; i < hhi; ++i) {
      const int32_t s = lru_old[i];
      if (!(sflags[s] & kProtected)) victims[pos++] = s;
      else victims[(int)unprotected + (i - pos)] = s;
    }
  }
  sc.sync();
  if (misses > H) {
    // only reachable with more positions than hot rows (the cache caps
    // positions at max_union_rows <= hot_rows)
    for (int i = tid; i < K; i += nthreads) out_phys[i] = out_mh[i] = out_md[i] = -1;
    if (p.out_ready)
      for (int i = tid; i < K; i += nthreads) p.out_ready[(int64_t)b * K + i] = -1;
    if (tid < 3) out_counts[tid] = 0;
    if (tid == 0) flag(p.status, HS_DEV_MISSES_EXCEED_HOT);
    return;
  }
  // ---- 7. slots, physical rows, miss plan, ready list, tag update --------------------
  int64_t *out_ready = p.out_ready ? p.out_ready + (int64_t)b * K : nullptr;
  for (int j = tid; j < K; j += nthreads) {
    const uint8_t f = jflags[j];
    if (out_ready && (f & kResidentHit)) out_ready[jrank[j]] = jphys[j];
    if (!(f & kNeedsHot)) continue;
    int32_t slot;
    if (f & kMiss) {
      slot = victims[jrank[j]];
      sflags[slot] |= kInserted;
    } else {
      slot = jslot[j];
    }
    const int64_t hot_phys = (int64_t)hot_tab[slot / P] * P + slot % P;
    jphys[j] = hot_phys;
    if (f & kMiss) {
      const int r = jrank[j];
      out_mh[r] = jhost[j];
      out_md[r] = hot_phys;
      tags[slot] = (int32_t)jhost[j];
    } else if (out_ready) {
      out_ready[jrank[j]] = hot_phys;
    }
  }
  for (int i = misses + tid; i < K; i += nthreads) out_mh[i] = out_md[i] = -1;
  if (out_ready) {
    const int ready = (int)(((totals >> kCountBits) & kCountMask) +
                            ((totals >> (2 * kCountBits)) & kCountMask));
    for (int i = ready + tid; i < K; i += nthreads) out_ready[i] = -1;
  }
  if (tid == 0) {
    out_counts[0] = (int64_t)((totals >> (2 * kCountBits)) & kCountMask);
    out_counts[1] = (int64_t)((totals >> kCountBits) & kCountMask);
    out_counts[2] = misses;
  }
  sc.sync();
  // ---- 8. new LRU: stable partition by category of the old order ------------------
  {
    // four 16-bit counters (hot_rows <= 65535, checked on the host)
    unsigned long long local = 0;
    for (int i = hlo; i < hhi; ++i) {
      const uint8_t f = sflags[lru_old[i]];
      const int cat = ((f & kInserted) ? 1 : 0) + ((f & kProtected) ? 2 : 0);
      local += 1ull << (16 * cat);
    }
    unsigned long long tot;
    const unsigned long long e = sc.template scan<unsigned long long>(local, scan_scratch, &tot);
    const int t0 = (int)(tot & 0xffff), t1 = (int)((tot >> 16) & 0xffff),
              t2 = (int)((tot >> 32) & 0xffff);
    int pos[4] = {(int)(e & 0xffff), t0 + (int)((e >> 16) & 0xffff),
                  t0 + t1 + (int)((e >> 32) & 0xffff), t0 + t1 + t2 + (int)((e >> 48) & 0xffff)};
    for (int i = hlo; i < hhi; ++i) {
      const int32_t s = lru_old[i];
      const uint8_t f = sflags[s];
      const int cat = ((f & kInserted) ? 1 : 0) + ((f & kProtected) ? 2 : 0);
      lru[pos[cat]++] = s;
    }
  }
  // ---- 9. results in input order ------------------------------------------------------
  if (sorted) {
    // input order is sorted order: the first occurrence is the unique entry
    for (int i = tid; i < K; i += nthreads) {
      const bool first = keys[i] < length && (i == 0 || keys[i - 1] != keys[i]);
      out_phys[i] = first ? jphys[i] : -1;
    }
  } else {
    for (int i = tid; i < K; i += nthreads) {
      const int64_t raw = load_position(p, b, i);
      int64_t r = -1;
      if (raw >= 0 && raw < length) {
        const int f = lower_bound(keys, K, raw);
        if (first_in[f] == i) r = jphys[f];
      }
      out_phys[i] = r;
    }
  }
}


// Steps 1-2, then the body, for request b (every thread of the block or cluster).
template <typename S>
__device__ __forceinline__ void resolve_run(const ResolveParams &p, int b, const S &sc,
                                         unsigned long long *scan_scratch) {
  const int tid = sc.tid(), nthreads = sc.nthreads();
  const Layout L(p.count, p.hot_rows);
  const int K = (int)p.count, H = (int)p.hot_rows, KP = (int)L.kp, CH = (int)L.ch;
  const Arr<int32_t, S> keys{sc, L.keys}, first_in{sc, L.first}, jslot{sc, L.slot},
      jrank{sc, L.rank}, lru_old{sc, L.lru_old}, victims{sc, L.victims};
  const Arr<uint8_t, S> jflags{sc, L.flags}, sflags{sc, L.sflags};
  const Arr<int64_t, S> jhost{sc, L.host}, jphys{sc, L.phys};
  const Arr<unsigned long long, S> table{sc, L.hash};

  int64_t *lru = p.lru.at(b);
  const int64_t length = p.lengths.at(b);
  int64_t *out_phys = p.out_physical + (int64_t)b * K;
  int64_t *out_mh = p.out_miss_host + (int64_t)b * K;
  int64_t *out_md = p.out_miss_device + (int64_t)b * K;
  int64_t *out_counts = p.out_counts + (int64_t)b * 3;

  // ---- 1. normalise positions; clear the hash; copy the LRU ---------------------
  for (int i = tid; i < KP; i += nthreads) {
    int32_t v = INT32_MAX;
    if (i < K) {
      const int64_t raw = load_position(p, b, i);
      v = (int32_t)((raw >= 0 && raw < length) ? raw : length);
    }
    keys[i] = v;
  }
  for (int s = tid; s < CH; s += nthreads) table[s] = kEmpty;
  sc.sync();
  int unsorted = 0, corrupt = 0;
  for (int i = tid; i + 1 < KP; i += nthreads) unsorted |= keys[i] > keys[i + 1];
  for (int s = tid; s < H; s += nthreads) {
    sflags[s] = 0;
    const int64_t v = lru[s];
    if (v < 0 || v >= H) corrupt = 1;
    lru_old[s] = (int32_t)v;
  }
  // ---- 2. sort (skipped for sorted input such as Quest's, whose -1 padding
  //         normalises past the end); first occurrence in input order --------
  const bool sorted = !sc.any(unsorted);
  const bool abort = sc.any(corrupt);
  if (!sorted) {
    for (int i = tid; i < K; i += nthreads) first_in[i] = K;
    for (int k = 2; k <= KP; k <<= 1) {
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = tid; i < KP; i += nthreads) {
          const int l = i ^ j;
          if (l > i) {
            const int32_t a = keys[i], c = keys[l];
            const bool up = (i & k) == 0;
            if ((a > c) == up) {
              keys[i] = c;
              keys[l] = a;
            }
          }
        }
        sc.sync();
      }
    }
    for (int i = tid; i < K; i += nthreads) {
      const int64_t raw = load_position(p, b, i);
      if (raw >= 0 && raw < length) atomicMin(&first_in[lower_bound(keys, K, raw)], i);
    }
  }
  if (abort) {
    // a corrupt LRU permutation cannot be resolved faithfully: tables stay
    // untouched and the plan is empty
    for (int i = tid; i < K; i += nthreads) out_phys[i] = out_mh[i] = out_md[i] = -1;
    if (p.out_ready)
      for (int i = tid; i < K; i += nthreads) p.out_ready[(int64_t)b * K + i] = -1;
    if (tid < 3) out_counts[tid] = 0;
    if (tid == 0) flag(p.status, HS_DEV_LRU_CORRUPT);
  } else {
    resolve_body(p, L, b, sorted, sc, keys, first_in, jflags, jslot, jrank, jhost, jphys, table,
                 sflags, lru_old, victims, scan_scratch);
  }
  if (p.head_columns != nullptr) {
    sc.sync();
    const int64_t n = p.head_count * p.head_width;
    for (int64_t i = tid; i < n; i += nthreads) {
      const int64_t c = p.head_columns[i];
      p.out_head_physical[i] = (c >= 0 && c < K) ? out_phys[c] : -1;
    }
  }
}

// One CTA per request; scratch in its shared memory or in the workspace.
__global__ void __launch_bounds__(kResolveThreads) resolve_kernel(ResolveParams p) {
  extern __shared__ __align__(16) char smem_raw[];
  __shared__ unsigned long long scan_scratch[33];
  const int b = blockIdx.x;
  const Layout L(p.count, p.hot_rows);
  const LocalScratch sc{p.workspace ? p.workspace + (size_t)b * L.total : smem_raw};
  resolve_run(p, b, sc, scan_scratch);
}

// One cluster of `size` CTAs per request; the scratch spread over their shared
// memory. Every thread of every CTA reaches the same cluster barriers (no path
// returns early), including one before any remote access and one before exit.
__global__ void __launch_bounds__(kResolveThreads, 1) resolve_cluster_kernel(ResolveParams p) {
  extern __shared__ __align__(16) char smem_raw[];
  __shared__ unsigned long long scan_scratch[33];
  __shared__ unsigned long long totals[kMaxCluster];
  unsigned size;
  asm volatile("mov.u32 %0, %%cluster_nctarank;\n" : "=r"(size));
  const unsigned rank = cluster_rank();
  const int b = (int)(blockIdx.x / size);
  const ClusterScratch sc{smem_raw, rank, size, (unsigned)(__ffs((int)size) - 1), totals};
  cluster_barrier();  // every CTA of the cluster runs before its shared memory is touched
  resolve_run(p, b, sc, scan_scratch);
  cluster_barrier();  // no CTA exits while another may still use its shared memory
}

// Shared memory of each CTA of a `size`-CTA cluster holding `total` bytes of
// scratch: its share of the 4 KiB granules dealt round-robin.
size_t cluster_part_bytes(size_t total, int size) {
  const size_t granules = (total + (size_t(1) << kGranuleShift) - 1) >> kGranuleShift;
  return ((granules + size - 1) / size) << kGranuleShift;
}

// Whether clusters of `size` resolver CTAs (1024 threads, `part` bytes of
// shared memory each) fit the device, asked once per device, size and part.
bool cluster_schedulable(int size, size_t part) {
  static std::mutex lock;
  static signed char known[64][kMaxCluster + 1][64];  // 0 unknown, 1 yes, -1 no
  int dev = 0;
  const size_t kib4 = part >> kGranuleShift;  // part in 4 KiB units (< 64: <= 200 KiB)
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || kib4 >= 64) return false;
  std::lock_guard<std::mutex> guard(lock);
  if (known[dev][size][kib4] != 0) return known[dev][size][kib4] > 0;
  bool ok = reserve_smem((const void *)resolve_cluster_kernel, part, "resolve") == HS_OK;
  if (ok && size > kPortableCluster)
    ok = cudaFuncSetAttribute((const void *)resolve_cluster_kernel,
                              cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
  if (ok) {
    cudaLaunchConfig_t config{};
    config.gridDim = dim3((unsigned)size);
    config.blockDim = dim3(kResolveThreads);
    config.dynamicSmemBytes = part;
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = (unsigned)size;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    config.attrs = &attr;
    config.numAttrs = 1;
    int clusters = 0;
    ok = cudaOccupancyMaxActiveClusters(&clusters, (const void *)resolve_cluster_kernel,
                                        &config) == cudaSuccess &&
         clusters > 0;
    cudaGetLastError();
  }
  known[dev][size][kib4] = ok ? 1 : -1;
  return ok;
}

int launch_cluster(const ResolveParams &p, int size, size_t part, cudaStream_t stream) {
  cudaLaunchConfig_t config{};
  config.gridDim = dim3((unsigned)(p.batch * size));
  config.blockDim = dim3(kResolveThreads);
  config.dynamicSmemBytes = part;
  config.stream = stream;
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = (unsigned)size;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  config.attrs = &attr;
  config.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&config, resolve_cluster_kernel, p);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return set_error(HS_ERR_CUDA, "resolve_cluster_kernel: launch failed: %s",
                     cudaGetErrorString(err));
  }
  return HS_OK;
}

int resolve_common(ResolveParams &p, size_t workspace_bytes, cudaStream_t stream) {
  if (p.batch < 1 || p.count < 1 || p.hot_rows < 1 || p.page_size < 1 || p.table_pages < 1)
    return set_error(HS_ERR_INVALID_ARGUMENT, "resolve: dimensions must be positive");
  if (p.count >= (1 << 21) || p.hot_rows > 65535)
    return set_error(HS_ERR_UNSUPPORTED,
                     "resolve: count must be < 2^21 and hot_rows <= 65535 (hot_rows is at "
                     "most 32768 in a cache)");
  if (p.hot_blocks * (int64_t)p.page_size < p.hot_rows)
    return set_error(HS_ERR_INVALID_ARGUMENT,
                     "resolve: hot table of %lld blocks cannot address %lld hot rows",
                     (long long)p.hot_blocks, (long long)p.hot_rows);
  if (!p.positions || !p.out_physical || !p.out_miss_host || !p.out_miss_device ||
      !p.out_counts)
    return set_error(HS_ERR_INVALID_ARGUMENT, "resolve: null tensor pointer");
  if (p.head_columns && (!p.out_head_physical || p.head_count < 1 || p.head_width < 1))
    return set_error(HS_ERR_INVALID_ARGUMENT, "resolve: invalid head columns");
  const Layout L(p.count, p.hot_rows);
  size_t smem = 0;
  if (L.total <= kResolveSmemLimit) {
    smem = L.total;
    p.workspace = nullptr;
  } else if (L.total <= ((size_t)kPortableCluster << kClusterShift)) {
    // too large for one SM: a cluster keeps the scratch in distributed shared
    // memory (no workspace read or written). Parts of at most 128 KiB (more
    // SMs per request) unless the batch's clusters would then need more than
    // one wave of SMs: then the fewest CTAs whose parts fit kResolveSmemLimit.
    int size = 2;  // a power of two: granules are dealt with masks and shifts
    while (((size_t)size << kClusterShift) < L.total) size <<= 1;
    int fewest = 2;
    while (fewest < size && cluster_part_bytes(L.total, fewest) > kResolveSmemLimit) fewest <<= 1;
    if ((int64_t)p.batch * size > sm_count() && fewest < size) size = fewest;
    // the largest scratch (clusters of 8) on few requests: 16 CTAs a request
    // where the device schedules them (one request's resolve is latency-bound,
    // and more CTAs shorten each of its passes)
    if (size == kPortableCluster && (int64_t)p.batch * kMaxCluster <= sm_count() &&
        cluster_schedulable(kMaxCluster, cluster_part_bytes(L.total, kMaxCluster)))
      size = kMaxCluster;
    const size_t part = cluster_part_bytes(L.total, size);
    if (cluster_schedulable(size, part)) return launch_cluster(p, size, part, stream);
    const size_t need = hs_resolve_workspace_bytes(p.batch, p.count, p.hot_rows);
    if (!p.workspace || workspace_bytes < need)
      return set_error(HS_ERR_WORKSPACE, "resolve: workspace of %zu bytes < required %zu",
                       workspace_bytes, need);
  } else {
    const size_t need = hs_resolve_workspace_bytes(p.batch, p.count, p.hot_rows);
    if (!p.workspace || workspace_bytes < need)
      return set_error(HS_ERR_WORKSPACE, "resolve: workspace of %zu bytes < required %zu",
                       workspace_bytes, need);
  }
  const int rc = reserve_smem((const void *)resolve_kernel, smem, "resolve");
  if (rc != HS_OK) return rc;
  resolve_kernel<<<p.batch, kResolveThreads, smem, stream>>>(p);
  return check_launch("resolve_kernel");
}

}  // namespace
}  // namespace hs

extern "C" size_t hs_resolve_workspace_bytes(int batch, int64_t count, int64_t hot_rows) {
  if (batch < 1 || count < 1 || hot_rows < 1) return 0;
  const hs::Layout L(count, hot_rows);
  if (L.total <= hs::kResolveSmemLimit) return 0;
  return (size_t)batch * L.total;
}

extern "C" int hs_resolve_rows(const void *positions, int positions_dtype, int64_t count,
                               const int32_t *source_table, const int32_t *resident_table,
                               int64_t table_pages, const int32_t *hot_table,
                               int64_t hot_blocks, int32_t *tags, int64_t *lru,
                               int64_t hot_rows, int64_t length, int page_size,
                               int64_t *out_physical, int64_t *out_miss_host,
                               int64_t *out_miss_device, int64_t *out_counts,
                               const int64_t *head_columns, int64_t head_count,
                               int64_t head_width, int64_t *out_head_physical,
                               void *workspace, size_t workspace_bytes,
                               int32_t *device_status, hs_stream stream) {
  if (positions_dtype != HS_INT32 && positions_dtype != HS_INT64)
    return hs::set_error(HS_ERR_INVALID_ARGUMENT, "resolve: positions must be int32 or int64");
  if (!source_table || !resident_table || !hot_table || !tags || !lru)
    return hs::set_error(HS_ERR_INVALID_ARGUMENT, "resolve: null table pointer");
  if (length < 0 || length > INT32_MAX)
    return hs::set_error(HS_ERR_INVALID_ARGUMENT, "resolve: length must be in [0, 2^31)");
  hs::ResolveParams p{};
  p.batch = 1;
  p.positions = positions;
  p.positions_i64 = positions_dtype == HS_INT64;
  p.count = count;
  p.source = {source_table, 0, nullptr};
  p.resident = {resident_table, 0, nullptr};
  p.hot = {hot_table, 0, nullptr};
  p.tags = {tags, 0, nullptr};
  p.lru = {lru, 0, nullptr};
  p.table_pages = table_pages;
  p.hot_blocks = hot_blocks;
  p.hot_rows = hot_rows;
  p.lengths = {nullptr, length};
  p.page_size = page_size;
  p.out_physical = out_physical;
  p.out_miss_host = out_miss_host;
  p.out_miss_device = out_miss_device;
  p.out_counts = out_counts;
  p.head_columns = head_columns;
  p.head_count = head_count;
  p.head_width = head_width;
  p.out_head_physical = out_head_physical;
  p.workspace = static_cast<char *>(workspace);
  p.status = device_status;
  return hs::resolve_common(p, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int hs_resolve_rows_batched(int batch, const int32_t *positions, int64_t count,
                                       const uint64_t *source_ptrs,
                                       const uint64_t *resident_ptrs, int64_t table_pages,
                                       const uint64_t *hot_ptrs, int64_t hot_blocks,
                                       const uint64_t *tags_ptrs, const uint64_t *lru_ptrs,
                                       int64_t hot_rows, const int32_t *lengths,
                                       int page_size, int64_t *out_physical,
                                       int64_t *out_miss_host, int64_t *out_miss_device,
                                       int64_t *out_counts, int64_t *out_ready,
                                       void *workspace, size_t workspace_bytes,
                                       int32_t *device_status, hs_stream stream) {
  if (!source_ptrs || !resident_ptrs || !hot_ptrs || !tags_ptrs || !lru_ptrs || !lengths)
    return hs::set_error(HS_ERR_INVALID_ARGUMENT, "resolve: null pointer array or lengths");
  hs::ResolveParams p{};
  p.batch = batch;
  p.positions = positions;
  p.positions_i64 = 0;
  p.count = count;
  p.source = {nullptr, 0, source_ptrs};
  p.resident = {nullptr, 0, resident_ptrs};
  p.hot = {nullptr, 0, hot_ptrs};
  p.tags = {nullptr, 0, tags_ptrs};
  p.lru = {nullptr, 0, lru_ptrs};
  p.table_pages = table_pages;
  p.hot_blocks = hot_blocks;
  p.hot_rows = hot_rows;
  p.lengths = {lengths, 0};
  p.page_size = page_size;
  p.out_physical = out_physical;
  p.out_miss_host = out_miss_host;
  p.out_miss_device = out_miss_device;
  p.out_counts = out_counts;
  p.out_ready = out_ready;
  p.workspace = static_cast<char *>(workspace);
  p.status = device_status;
  return hs::resolve_common(p, workspace_bytes, static_cast<cudaStream_t>(stream));
}
