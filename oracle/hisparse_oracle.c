/*
 * TEST INFRASTRUCTURE — NOT PART OF THE PRODUCT.
 *
 * CPU restatement of nano-hisparse's per-step sparse-decode hot path, used
 * only by tests/ (as the parity checker), __graft_entry__.smoke() (checker)
 * and bench.py's CPU-baseline arm. Nothing in nano-hisparse_b200/ links or
 * calls this code.
 *
 * Each function cites the reference code it restates (paths inside the
 * KiritoHugh/nano-hisparse tree). The algorithms are restated from their
 * semantics, not transcribed from the reference's tensor programs:
 *
 *   or_quest_scores   selection.py:69-91   Quest upper bound, head mean
 *   or_quest_head_sums                     the same, undivided, for one shard
 *                                          of a head-sharded selection
 *   or_quest_select   selection.py:86-91   forced tail/sink, top-k, and
 *                     selection.py:45-62   page -> token expansion
 *   or_resolve_rows   row_index.py:62-140  resolver + tag/LRU update
 *   or_gather_rows    hybrid.py:452-459    CPU gather loop (bytes)
 *   or_attend_rows    attention.py:26-35   masked softmax attention (fp64)
 *   or_append_rows    storage.py:296-321   one page chunk of HostStore.append:
 *                                          pool rows, host mirror, K min/max
 *                                          and mean-K summary
 *
 * The Quest score is a fp32 sum whose order the reference leaves to torch.
 * This oracle fixes the order that libhisparse's kernel uses (stated in
 * include/hisparse.h) so that scores and selections compare bit for bit;
 * selections are compared with the reference's own torch results separately,
 * where only near-ties at the k-th score may differ.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum { OR_F32 = 0, OR_F16 = 1, OR_BF16 = 2 };

/* ---- element conversion (IEEE binary16 / bfloat16 -> binary32) ---------- */
static float bits_to_float(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static uint32_t float_to_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

static float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
  if (exp == 0) {
    if (man == 0) return bits_to_float(sign);
    /* subnormal: value = man * 2^-24 */
    float v = (float)man * 5.9604644775390625e-08f;
    return sign ? -v : v;
  }
  if (exp == 31) return bits_to_float(sign | 0x7f800000u | (man << 13));
  return bits_to_float(sign | ((exp + 112u) << 23) | (man << 13));
}

static float load_elem(const void *base, int dtype, int64_t i) {
  switch (dtype) {
    case OR_F32: return ((const float *)base)[i];
    case OR_F16: return half_to_float(((const uint16_t *)base)[i]);
    default: return bits_to_float((uint32_t)((const uint16_t *)base)[i] << 16);
  }
}

/* xor-pairing tree over 32 values: (j, j^16), (j, j^8), ..., (j, j^1). */
static float xor_tree32(float x[32]) {
  float y[32];
  for (int o = 16; o > 0; o >>= 1) {
    for (int j = 0; j < 32; ++j) y[j] = x[j] + x[j ^ o];
    memcpy(x, y, sizeof(y));
  }
  return x[0];
}

/* ---- (1) Quest scores --------------------------------------------------- */
/* Lanes that share one head's row: the smallest power of two >= ceil(D / 8). */
static int quest_lanes(int D) {
  int L = 1;
  while (L * 8 < D) L *= 2;
  return L;
}

/* xor-pairing tree over L (a power of two) values: (j, j^(L/2)), ..., (j, j^1). */
static float xor_tree(float *x, int L) {
  float y[32];
  for (int o = L / 2; o > 0; o >>= 1) {
    for (int j = 0; j < L; ++j) y[j] = x[j] + x[j ^ o];
    memcpy(x, y, sizeof(float) * (size_t)L);
  }
  return x[0];
}

/* q: [Hq, D] (qdtype); mn/mx: [>= n, Hkv, D] (kvdtype); scores: [n].
 * divide = 0 leaves the head sum undivided: the partial score of one shard of a
 * head-sharded selection (heads indexed locally, same order).
 * Order (include/hisparse.h states it): lane j of L owns d = 8j .. 8j+7; it
 * adds the terms at even offsets left to right and those at odd offsets left
 * to right, then even + odd; the L lane values meet in the xor tree. */
static int quest_scores(const void *q, int qdtype, const void *mn, const void *mx, int kvdtype,
                        int Hq, int Hkv, int D, int64_t n, float *scores, int divide) {
  if (Hq < 1 || Hkv < 1 || D < 1 || D > 256 || Hq % Hkv) return 1;
  const int g = Hq / Hkv, L = quest_lanes(D);
  float *qf = (float *)malloc(sizeof(float) * (size_t)Hq * D);
  float *s = (float *)malloc(sizeof(float) * (size_t)Hq);
  float *lo = (float *)malloc(sizeof(float) * (size_t)D);
  float *hi = (float *)malloc(sizeof(float) * (size_t)D);
  if (!qf || !s || !lo || !hi) return 2;
  for (int64_t i = 0; i < (int64_t)Hq * D; ++i) qf[i] = load_elem(q, qdtype, i);
  for (int64_t p = 0; p < n; ++p) {
    for (int kh = 0; kh < Hkv; ++kh) {
      const int64_t row = (p * Hkv + kh) * (int64_t)D;
      for (int d = 0; d < D; ++d) {
        lo[d] = load_elem(mn, kvdtype, row + d);
        hi[d] = load_elem(mx, kvdtype, row + d);
      }
      for (int h = kh * g; h < kh * g + g; ++h) {
        float part[32];
        for (int j = 0; j < L; ++j) {
          float acc[2] = {0.f, 0.f};
          int have[2] = {0, 0};
          for (int e = 0; e < 8; ++e) {
            const int d = 8 * j + e;
            if (d >= D) break;
            const float qq = qf[h * D + d];
            const float t = fmaxf(qq * lo[d], qq * hi[d]);
            acc[e & 1] = have[e & 1] ? acc[e & 1] + t : t;
            have[e & 1] = 1;
          }
          part[j] = have[1] ? acc[0] + acc[1] : acc[0];
        }
        s[h] = xor_tree(part, L);
      }
    }
    /* lane j adds heads j, j+32, ... left to right; lanes meet in the xor tree */
    float u[32] = {0};
    for (int h = 0; h < Hq; ++h) u[h % 32] = u[h % 32] + s[h];
    scores[p] = divide ? xor_tree32(u) / (float)Hq : xor_tree32(u);
  }
  free(qf);
  free(s);
  free(lo);
  free(hi);
  return 0;
}

int or_quest_scores(const void *q, int qdtype, const void *mn, const void *mx, int kvdtype,
                    int Hq, int Hkv, int D, int64_t n, float *scores) {
  return quest_scores(q, qdtype, mn, mx, kvdtype, Hq, Hkv, D, n, scores, 1);
}

/* Head sums of one shard (hs_quest_partial_scores_batched); the shards' sums
 * are added in shard order and divided by the total heads by the caller. */
int or_quest_head_sums(const void *q, int qdtype, const void *mn, const void *mx, int kvdtype,
                       int Hq, int Hkv, int D, int64_t n, float *sums) {
  return quest_scores(q, qdtype, mn, mx, kvdtype, Hq, Hkv, D, n, sums, 0);
}

/* ---- (1) forced pages, top-k and token expansion -------------------------- */
static uint32_t score_key(float s) {
  if (isnan(s)) return 0xfffffffeu;
  if (s == 0.0f) s = 0.0f; /* fold -0 onto +0 */
  const uint32_t bits = float_to_bits(s);
  return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
}

typedef struct {
  uint32_t key;
  int64_t page;
} keyed_page;

static int by_key_desc_page_asc(const void *a, const void *b) {
  const keyed_page *x = (const keyed_page *)a, *y = (const keyed_page *)b;
  if (x->key != y->key) return x->key > y->key ? -1 : 1;
  return x->page < y->page ? -1 : (x->page > y->page);
}

int or_quest_select(const float *scores, int64_t length, int page_size, int top_pages,
                    int keep_sink, int32_t *out, int64_t capacity, int32_t *count) {
  if (length < 1 || page_size < 1 || top_pages < 1) return 1;
  const int64_t n = (length + page_size - 1) / page_size;
  for (int64_t i = 0; i < capacity; ++i) out[i] = -1;
  if (top_pages >= n) {
    if (length > capacity) return 3;
    for (int64_t t = 0; t < length; ++t) out[t] = (int32_t)t;
    *count = (int32_t)length;
    return 0;
  }
  keyed_page *kp = (keyed_page *)malloc(sizeof(keyed_page) * (size_t)n);
  unsigned char *chosen = (unsigned char *)calloc((size_t)n, 1);
  if (!kp || !chosen) return 2;
  const int sink = keep_sink && top_pages > 1 && n > 1;
  for (int64_t p = 0; p < n; ++p) {
    kp[p].page = p;
    kp[p].key = (p == n - 1 || (sink && p == 0)) ? 0xffffffffu : score_key(scores[p]);
  }
  qsort(kp, (size_t)n, sizeof(keyed_page), by_key_desc_page_asc);
  for (int i = 0; i < top_pages; ++i) chosen[kp[i].page] = 1;
  int64_t w = 0;
  for (int64_t p = 0; p < n; ++p) {
    if (!chosen[p]) continue;
    const int64_t first = p * page_size;
    const int64_t last = first + page_size < length ? first + page_size : length;
    for (int64_t t = first; t < last; ++t) {
      if (w >= capacity) {
        free(kp);
        free(chosen);
        return 3;
      }
      out[w++] = (int32_t)t;
    }
  }
  *count = (int32_t)w;
  free(kp);
  free(chosen);
  return 0;
}

/* ---- (2) resolver ---------------------------------------------------------- */
enum { ST_INVALID = 0, ST_RESIDENT = 1, ST_HOT_HIT = 2, ST_MISS = 3 };

static int cmp_i64(const void *a, const void *b) {
  const int64_t x = *(const int64_t *)a, y = *(const int64_t *)b;
  return x < y ? -1 : (x > y);
}

typedef struct {
  int64_t tag, slot;
} tag_slot;

static int by_tag_then_slot(const void *a, const void *b) {
  const tag_slot *x = (const tag_slot *)a, *y = (const tag_slot *)b;
  if (x->tag != y->tag) return x->tag < y->tag ? -1 : 1;
  return x->slot < y->slot ? -1 : (x->slot > y->slot);
}

/* Index of v in the sorted distinct array u[0, m), or -1. */
static int64_t find_sorted(const int64_t *u, int64_t m, int64_t v) {
  int64_t lo = 0, hi = m;
  while (lo < hi) {
    const int64_t mid = (lo + hi) / 2;
    if (u[mid] < v) lo = mid + 1; else hi = mid;
  }
  return (lo < m && u[lo] == v) ? lo : -1;
}

/*
 * Restates resolve_rows (row_index.py:62-140):
 *  - distinct valid logical positions (0 <= t < length), ascending;
 *  - page = min(t / P, table_pages - 1); host row = source*P + t%P;
 *    source < 0 -> invalid; resident >= 0 -> resident row resident*P + t%P;
 *  - other rows look up their host row among the nonnegative tags
 *    (hot hit) or miss;
 *  - every slot whose tag is a wanted host row is protected; victims are the
 *    unprotected slots in LRU order followed by the protected ones; the r-th
 *    miss (ascending position) takes victim r and its tag becomes its host
 *    row;
 *  - a hot row's physical row is hot[slot / P]*P + slot % P;
 *  - the new LRU keeps the old order within four groups: untouched,
 *    inserted, protected, inserted and protected;
 *  - the miss plan lists (host row, hot physical row) in ascending position
 *    order, -1 padded; outputs follow the input order, with -1 for invalid
 *    inputs and repeated inputs after their first occurrence.
 * tags/lru are int64 here and updated in place. Returns 4 when misses exceed
 * hot rows (the reference result is then undefined).
 */
int or_resolve_rows(const int64_t *positions, int64_t K, const int64_t *source,
                    const int64_t *resident, int64_t table_pages, const int64_t *hot,
                    int64_t hot_blocks, int64_t *tags, int64_t *lru, int64_t H, int64_t length,
                    int P, int64_t *out_physical, int64_t *miss_host, int64_t *miss_device,
                    int64_t *counts) {
  if (K < 1 || H < 1 || P < 1 || table_pages < 1 || hot_blocks * P < H) return 1;
  for (int64_t i = 0; i < H; ++i)
    if (lru[i] < 0 || lru[i] >= H) return 5;
  int64_t *u = (int64_t *)malloc(sizeof(int64_t) * (size_t)K);
  int64_t m = 0;
  for (int64_t i = 0; i < K; ++i)
    if (positions[i] >= 0 && positions[i] < length) u[m++] = positions[i];
  qsort(u, (size_t)m, sizeof(int64_t), cmp_i64);
  int64_t w = 0;
  for (int64_t i = 0; i < m; ++i)
    if (i == 0 || u[i] != u[i - 1]) u[w++] = u[i];
  m = w;
  int *state = (int *)calloc((size_t)(m ? m : 1), sizeof(int));
  int64_t *host = (int64_t *)calloc((size_t)(m ? m : 1), sizeof(int64_t));
  int64_t *phys = (int64_t *)calloc((size_t)(m ? m : 1), sizeof(int64_t));
  int64_t *slot = (int64_t *)calloc((size_t)(m ? m : 1), sizeof(int64_t));
  unsigned char *prot = (unsigned char *)calloc((size_t)H, 1);
  unsigned char *ins = (unsigned char *)calloc((size_t)H, 1);
  int64_t *victims = (int64_t *)malloc(sizeof(int64_t) * (size_t)H);
  int64_t *newlru = (int64_t *)malloc(sizeof(int64_t) * (size_t)H);
  int64_t c_res = 0, c_hot = 0, c_miss = 0;
  tag_slot *tagpairs = (tag_slot *)malloc(sizeof(tag_slot) * (size_t)H);
  int64_t nt = 0;
  for (int64_t s = 0; s < H; ++s)
    if (tags[s] >= 0) {
      tagpairs[nt].tag = tags[s];
      tagpairs[nt].slot = s;
      ++nt;
    }
  qsort(tagpairs, (size_t)nt, sizeof(tag_slot), by_tag_then_slot);
  for (int64_t j = 0; j < m; ++j) {
    int64_t page = u[j] / P;
    if (page > table_pages - 1) page = table_pages - 1;
    const int64_t off = u[j] % P, src = source[page], res = resident[page];
    host[j] = src * P + off;
    phys[j] = -1;
    if (src < 0) {
      state[j] = ST_INVALID;
    } else if (res >= 0) {
      state[j] = ST_RESIDENT;
      phys[j] = res * P + off;
      ++c_res;
    } else {
      /* lowest slot holding this host row, if any */
      int64_t found = -1;
      {
        int64_t lo2 = 0, hi2 = nt;
        while (lo2 < hi2) {
          const int64_t mid = (lo2 + hi2) / 2;
          if (tagpairs[mid].tag < host[j]) lo2 = mid + 1; else hi2 = mid;
        }
        if (lo2 < nt && tagpairs[lo2].tag == host[j]) found = tagpairs[lo2].slot;
      }
      if (found >= 0) {
        state[j] = ST_HOT_HIT;
        slot[j] = found;
        ++c_hot;
      } else {
        state[j] = ST_MISS;
        ++c_miss;
      }
    }
  }
  /* protected: nonnegative tag equal to some wanted (hot-needing) host row */
  {
    int64_t *wanted = (int64_t *)malloc(sizeof(int64_t) * (size_t)(m ? m : 1));
    int64_t nw = 0;
    for (int64_t j = 0; j < m; ++j)
      if (state[j] == ST_HOT_HIT || state[j] == ST_MISS) wanted[nw++] = host[j];
    qsort(wanted, (size_t)nw, sizeof(int64_t), cmp_i64);
    for (int64_t s = 0; s < H; ++s)
      if (tags[s] >= 0 && find_sorted(wanted, nw, tags[s]) >= 0) prot[s] = 1;
    free(wanted);
  }
  int rc = 0;
  if (c_miss > H) {
    rc = 4;
    goto done;
  }
  {
    int64_t nv = 0;
    for (int64_t i = 0; i < H; ++i)
      if (!prot[lru[i]]) victims[nv++] = lru[i];
    for (int64_t i = 0; i < H; ++i)
      if (prot[lru[i]]) victims[nv++] = lru[i];
  }
  {
    int64_t r = 0;
    for (int64_t i = 0; i < K; ++i) miss_host[i] = miss_device[i] = -1;
    for (int64_t j = 0; j < m; ++j) {
      if (state[j] == ST_MISS) slot[j] = victims[r++];
      if (state[j] == ST_HOT_HIT || state[j] == ST_MISS)
        phys[j] = hot[slot[j] / P] * P + slot[j] % P;
    }
    r = 0;
    for (int64_t j = 0; j < m; ++j) {
      if (state[j] != ST_MISS) continue;
      miss_host[r] = host[j];
      miss_device[r] = phys[j];
      ++r;
      ins[slot[j]] = 1;
      tags[slot[j]] = host[j];
    }
  }
  {
    int64_t n0 = 0;
    for (int cat = 0; cat < 4; ++cat)
      for (int64_t i = 0; i < H; ++i) {
        const int64_t s = lru[i];
        if (ins[s] + 2 * prot[s] == cat) newlru[n0++] = s;
      }
    memcpy(lru, newlru, sizeof(int64_t) * (size_t)H);
  }
  {
    /* first occurrence in input order */
    unsigned char *seen = (unsigned char *)calloc((size_t)(m ? m : 1), 1);
    for (int64_t i = 0; i < K; ++i) {
      out_physical[i] = -1;
      const int64_t t = positions[i];
      if (t < 0 || t >= length) continue;
      const int64_t j = find_sorted(u, m, t);
      if (!seen[j]) {
        seen[j] = 1;
        out_physical[i] = phys[j];
      }
    }
    free(seen);
  }
  counts[0] = c_res;
  counts[1] = c_hot;
  counts[2] = c_miss;
done:
  free(tagpairs);
  free(u);
  free(state);
  free(host);
  free(phys);
  free(slot);
  free(prot);
  free(ins);
  free(victims);
  free(newlru);
  return rc;
}

/* ---- (3) gather -------------------------------------------------------------- */
/* Copies both planes of every planned miss (hybrid.py:452-459). */
int or_gather_rows(const uint8_t *host, int64_t host_blocks, uint8_t *pool, int64_t pool_blocks,
                   const int64_t *miss_host, const int64_t *miss_device, int64_t count, int P,
                   int64_t row_bytes) {
  int rc = 0;
  for (int64_t i = 0; i < count; ++i) {
    const int64_t h = miss_host[i], d = miss_device[i];
    if (h < 0 || d < 0) continue;
    if (h / P >= host_blocks || d / P >= pool_blocks) {
      rc = 6;
      continue;
    }
    for (int plane = 0; plane < 2; ++plane) {
      const int64_t src = ((h / P) * 2 * P + plane * P + h % P) * row_bytes;
      const int64_t dst = ((d / P) * 2 * P + plane * P + d % P) * row_bytes;
      memcpy(pool + dst, host + src, (size_t)row_bytes);
    }
  }
  return rc;
}

/* ---- (5) append ---------------------------------------------------------------- */
/*
 * One page chunk of HostStore.append (storage.py:296-321): rows
 * within .. within+count-1 of the K and V planes of `block` (one pool block,
 * [2, P, E] elements, E = kv_heads*head_dim) take the count rows of k and v
 * ([count, E]); `host_block` (NULL: no mirror) receives the same rows; with
 * `block` NULL the chunk is host-only and `host_block` holds the page; then
 *   minimum[e] = min(minimum[e], min_i k[i][e]) and maximum likewise — exact
 *   in the KV dtype, NaN propagating, an equal new value replacing the old
 *   (torch.minimum / torch.maximum of old and new);
 *   summary[e] = (fp32) sum of K-plane rows 0 .. within+count-1, added in row
 *   order, divided by within+count (the mean of storage.py:309).
 * Element size is 4 (f32) or 2 (f16/bf16); min/max keep the winning element's
 * bits, so no conversion back to the KV dtype is needed.
 */
static int elem_less(float a, float b) { return a < b; }

int or_append_rows(const void *k, const void *v, int dtype, int64_t count, int64_t within,
                   void *block, void *host_block, void *minimum, void *maximum,
                   float *summary, int64_t elems, int P) {
  if (count < 0 || within < 0 || within + count > P || elems < 1) return 1;
  if (!block && !host_block) return 1;
  const int64_t es = dtype == OR_F32 ? 4 : 2;
  uint8_t *blk = (uint8_t *)(block ? block : host_block); /* the page's rows for the mean */
  const int64_t plane = (int64_t)P * elems * es, row = elems * es;
  for (int64_t i = 0; i < count; ++i) {
    if (block) {
      memcpy((uint8_t *)block + (within + i) * row, (const uint8_t *)k + i * row, (size_t)row);
      memcpy((uint8_t *)block + plane + (within + i) * row, (const uint8_t *)v + i * row,
             (size_t)row);
    }
    if (host_block) {
      memcpy((uint8_t *)host_block + (within + i) * row, (const uint8_t *)k + i * row, (size_t)row);
      memcpy((uint8_t *)host_block + plane + (within + i) * row, (const uint8_t *)v + i * row,
             (size_t)row);
    }
  }
  const int64_t valid = within + count;
  for (int64_t e = 0; e < elems; ++e) {
    if (count > 0) {
      int64_t lo = 0, hi = 0, nan_row = -1; /* rows of the chunk holding the min / max */
      for (int64_t i = 0; i < count; ++i) {
        const float x = load_elem(k, dtype, i * elems + e);
        if (isnan(x) && nan_row < 0) nan_row = i;
        if (elem_less(x, load_elem(k, dtype, lo * elems + e))) lo = i;
        if (elem_less(load_elem(k, dtype, hi * elems + e), x)) hi = i;
      }
      const float old_lo = load_elem(minimum, dtype, e), old_hi = load_elem(maximum, dtype, e);
      const float new_lo = load_elem(k, dtype, lo * elems + e);
      const float new_hi = load_elem(k, dtype, hi * elems + e);
      uint8_t *const mn = (uint8_t *)minimum + e * es, *const mx = (uint8_t *)maximum + e * es;
      const uint8_t *const kb = (const uint8_t *)k;
      /* torch.minimum(old, new): NaN if either is NaN, else the smaller, the new one on ties */
      if (isnan(old_lo)) {
      } else if (nan_row >= 0) {
        memcpy(mn, kb + (nan_row * elems + e) * es, (size_t)es);
      } else if (!elem_less(old_lo, new_lo)) {
        memcpy(mn, kb + (lo * elems + e) * es, (size_t)es);
      }
      if (isnan(old_hi)) {
      } else if (nan_row >= 0) {
        memcpy(mx, kb + (nan_row * elems + e) * es, (size_t)es);
      } else if (!elem_less(new_hi, old_hi)) {
        memcpy(mx, kb + (hi * elems + e) * es, (size_t)es);
      }
    }
    float sum = 0.f;
    for (int64_t r = 0; r < valid; ++r) sum += load_elem(blk, dtype, r * elems + e);
    summary[e] = valid > 0 ? sum / (float)valid : 0.f;
  }
  return 0;
}

/* ---- (4) attention ------------------------------------------------------------- */
/*
 * out[h] = softmax_r(q[h].K[r,kh]/sqrt(D)) V[r,kh] over rows r >= 0, in fp64;
 * zero if no valid row (attention.py:26-35; row_kernels.py:73-113).
 * rows[h*rows_head_stride + i], i < count. out: [Hq, D] fp64.
 */
int or_attend_rows(const void *q, int qdtype, const void *pool, int kvdtype, int64_t pool_blocks,
                   const int64_t *rows, int64_t rows_head_stride, int64_t count, int Hq,
                   int Hkv, int D, int P, double *out) {
  if (Hq < 1 || Hkv < 1 || D < 1 || Hq % Hkv || P < 1) return 1;
  const int g = Hq / Hkv;
  const double scale = 1.0 / sqrt((double)D);
  const int64_t row_elems = (int64_t)Hkv * D, plane = (int64_t)P * row_elems;
  double *scores = (double *)malloc(sizeof(double) * (size_t)(count ? count : 1));
  int rc = 0;
  for (int h = 0; h < Hq; ++h) {
    const int kh = h / g;
    const int64_t *hr = rows + h * rows_head_stride;
    double mx = -INFINITY;
    for (int64_t i = 0; i < count; ++i) {
      scores[i] = -INFINITY;
      const int64_t r = hr[i];
      if (r < 0) continue;
      if (r / P >= pool_blocks) {
        rc = 6;
        continue;
      }
      const int64_t base = ((r / P) * 2 * P + r % P) * row_elems + (int64_t)kh * D;
      double dot = 0.0;
      for (int d = 0; d < D; ++d)
        dot += (double)load_elem(q, qdtype, (int64_t)h * D + d) *
               (double)load_elem(pool, kvdtype, base + d);
      scores[i] = dot * scale;
      if (scores[i] > mx) mx = scores[i];
    }
    for (int d = 0; d < D; ++d) out[(int64_t)h * D + d] = 0.0;
    if (mx == -INFINITY) continue;
    double denom = 0.0;
    for (int64_t i = 0; i < count; ++i) {
      if (scores[i] == -INFINITY) continue;
      const double w = exp(scores[i] - mx);
      denom += w;
      const int64_t r = hr[i];
      const int64_t base = ((r / P) * 2 * P + r % P) * row_elems + plane + (int64_t)kh * D;
      for (int d = 0; d < D; ++d)
        out[(int64_t)h * D + d] += w * (double)load_elem(pool, kvdtype, base + d);
    }
    for (int d = 0; d < D; ++d) out[(int64_t)h * D + d] /= denom;
  }
  free(scores);
  return rc;
}

/* ---- one decode layer for a batch of requests (CPU baseline) ------------------- */
/*
 * Runs the whole per-(request, layer) hot path — Quest, resolver, gather,
 * attention — for `batch` requests, parallel over requests with OpenMP.
 * Per-request inputs are arrays of pointers; the pool and host store are
 * shared. Scratch (scores, tokens, plans) is allocated per request.
 */
int or_decode_layer_batched(int batch, const void *const *query, int qdtype,
                            const void *const *minimum, const void *const *maximum,
                            int kvdtype, const int64_t *lengths, int Hq, int Hkv, int D,
                            int P, int top_pages, int64_t max_pages,
                            const int64_t *const *source, const int64_t *const *resident,
                            const int64_t *const *hot, int64_t hot_blocks,
                            int64_t *const *tags, int64_t *const *lru, int64_t H,
                            const uint8_t *host_store, int64_t host_blocks, uint8_t *pool,
                            int64_t pool_blocks, double *const *out, int64_t *counts,
                            int threads) {
  const int64_t width = (int64_t)top_pages * P;
  const int64_t elem = kvdtype == OR_F32 ? 4 : 2;
  const int64_t row_bytes = (int64_t)Hkv * D * elem;
  int rc_all = 0;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(dynamic, 1) reduction(| : rc_all)
#endif
  for (int b = 0; b < batch; ++b) {
    const int64_t n = (lengths[b] + P - 1) / P;
    float *scores = (float *)malloc(sizeof(float) * (size_t)(n ? n : 1));
    int32_t *tokens = (int32_t *)malloc(sizeof(int32_t) * (size_t)width);
    int64_t *pos = (int64_t *)malloc(sizeof(int64_t) * (size_t)width);
    int64_t *phys = (int64_t *)malloc(sizeof(int64_t) * (size_t)width);
    int64_t *mh = (int64_t *)malloc(sizeof(int64_t) * (size_t)width);
    int64_t *md = (int64_t *)malloc(sizeof(int64_t) * (size_t)width);
    int32_t cnt = 0;
    int rc = or_quest_scores(query[b], qdtype, minimum[b], maximum[b], kvdtype, Hq, Hkv, D, n,
                             scores);
    rc |= or_quest_select(scores, lengths[b], P, top_pages, 1, tokens, width, &cnt);
    for (int64_t i = 0; i < width; ++i) pos[i] = tokens[i];
    rc |= or_resolve_rows(pos, width, source[b], resident[b], max_pages, hot[b], hot_blocks,
                          tags[b], lru[b], H, lengths[b], P, phys, mh, md, counts + 3 * b);
    rc |= or_gather_rows(host_store, host_blocks, pool, pool_blocks, mh, md, width, P,
                         row_bytes);
    rc |= or_attend_rows(query[b], qdtype, pool, kvdtype, pool_blocks, phys, 0, width, Hq, Hkv,
                         D, P, out[b]);
    rc_all |= rc;
    free(scores);
    free(tokens);
    free(pos);
    free(phys);
    free(mh);
    free(md);
  }
  return rc_all;
}
