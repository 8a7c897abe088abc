/*
 * hkv_oracle.c -- CPU restatement of the HierarchicalKV-ascend table rules.
 *
 * TEST INFRASTRUCTURE ONLY (see hkv_oracle.h). Each function cites the
 * reference file:line it restates; paths are relative to the reference
 * project's `include/` directory unless they start with tests/.
 *
 * Threading: every per-key rule touches one bucket only, so a batch is split
 * by bucket index over worker threads and each worker applies its keys in
 * index order. The result equals the single-threaded sequential result.
 */
#define _GNU_SOURCE
#include "hkv_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* Primitives                                                               */
/* ------------------------------------------------------------------------ */

/* Murmur3 64-bit finalizer, utils.h:53-61 (host) and :64-72 (device). */
uint64_t hkvo_murmur3(uint64_t k) {
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdull;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ull;
  k ^= k >> 33;
  return k;
}

/* get_digest / empty_digest / reclaim_digest, types.h:97-127. */
uint8_t hkvo_digest(uint64_t key) { return (uint8_t)(hkvo_murmur3(key) >> 32); }
uint8_t hkvo_empty_digest(void) { return hkvo_digest(HKVO_EMPTY_KEY); }
uint8_t hkvo_reclaim_digest(void) { return hkvo_digest(HKVO_RECLAIM_KEY); }

/* IS_RESERVED_KEY, types.h:153-156 with RESERVED_KEY_MASK types.h:67. */
int hkvo_is_reserved(uint64_t key) {
  return (key & HKVO_RESERVED_MASK) == HKVO_RESERVED_MASK;
}

/* precomputation_for_kernel_div, table.h:106-127 (round-up magic number
 * division, Granlund & Montgomery 1994). */
void hkvo_magic_div(uint64_t divisor, uint64_t* magic, uint64_t* shift) {
  unsigned __int128 one = 1;
  uint64_t s;
  for (s = 0; s < 64; s++) {
    if ((one << s) >= divisor) break;
  }
  unsigned __int128 m = ((one << 64) * ((one << s) - divisor)) / divisor + 1;
  *magic = (uint64_t)m;
  *shift = s - 1;
}

/* get_global_idx, utils.h:85-97. */
uint64_t hkvo_fast_mod(uint64_t x, uint64_t divisor, uint64_t magic,
                       uint64_t shift) {
  uint64_t q = (uint64_t)(((unsigned __int128)x * magic) >> 64);
  uint64_t t = ((x - q) >> 1) + q;
  uint64_t d = t >> shift;
  return x - d * divisor;
}

/* ------------------------------------------------------------------------ */
/* Score functors, score_functor.h                                          */
/* ------------------------------------------------------------------------ */
#define LOW32 0xFFFFFFFFull
#define HIGH32 0xFFFFFFFF00000000ull

/* make_epoch / make_nano, score_functor.h:35-43. */
static uint64_t make_epoch(uint64_t e) { return e << 32; }
static uint64_t make_nano(uint64_t c) { return LOW32 & (c >> 20); }

/* desired_when_missed: Lru :50-54, Lfu :116-120, EpochLru :215-223,
 * EpochLfu :286-293, Customized :410-414. */
uint64_t hkvo_desired_when_missed(int strategy, const uint64_t* in,
                                  size_t idx, uint64_t epoch, uint64_t cycle) {
  switch (strategy) {
    case HKVO_LRU:
      return cycle;
    case HKVO_LFU:
      return HKVO_MAX_SCORE;
    case HKVO_EPOCH_LRU:
      if (epoch == HKVO_IGNORED_EPOCH && in != NULL) return in[idx];
      return make_epoch(epoch) | make_nano(cycle);
    case HKVO_EPOCH_LFU:
      if (in == NULL) return 0; /* the reference dereferences NULL here */
      if (epoch == HKVO_IGNORED_EPOCH) return in[idx];
      return make_epoch(epoch) | (in[idx] & LOW32);
    default: /* Customized */
      return in ? in[idx] : 0;
  }
}

/* EpochLfu saturating low-32 add, score_functor.h:297-309. */
static uint64_t epoch_lfu_add(uint64_t old, uint64_t desired) {
  uint64_t s = old & LOW32;
  if (LOW32 - s > (desired & LOW32)) return s + desired;
  return (desired & HIGH32) | LOW32;
}

/* update_with_digest / update_score_only: Lru :56-84, Lfu :136-187,
 * EpochLru :241-268, EpochLfu :316-367, Customized :431-455. */
int hkvo_score_on_write(int strategy, uint64_t old, const uint64_t* in,
                        size_t idx, uint64_t desired, int new_insert,
                        uint64_t* out) {
  switch (strategy) {
    case HKVO_LFU:
      if (in == NULL) return 0;
      *out = new_insert ? in[idx] : in[idx] + old;
      return 1;
    case HKVO_EPOCH_LFU:
      *out = new_insert ? desired : epoch_lfu_add(old, desired);
      return 1;
    default: /* Lru, EpochLru, Customized store the desired score */
      *out = desired;
      return 1;
  }
}

/* update_without_missed (pointer form): Lru :99-111, Lfu :198-210,
 * EpochLru :270-281, EpochLfu :386-405, Customized :466-477. */
int hkvo_score_without_missed(int strategy, uint64_t old, const uint64_t* in,
                              size_t idx, uint64_t epoch, uint64_t cycle,
                              uint64_t* out) {
  switch (strategy) {
    case HKVO_LRU:
      *out = cycle;
      return 1;
    case HKVO_LFU:
      if (in == NULL) return 0;
      *out = in[idx] + old;
      return 1;
    case HKVO_EPOCH_LRU:
      *out = make_epoch(epoch) | make_nano(cycle);
      return 1;
    case HKVO_EPOCH_LFU: {
      if (in == NULL) return 0;
      uint64_t s = old & LOW32;
      if (LOW32 - s > (in[idx] & LOW32))
        *out = s + (make_epoch(epoch) | (in[idx] & LOW32));
      else
        *out = make_epoch(epoch) | LOW32;
      return 1;
    }
    default:
      if (in == NULL) return 0;
      *out = in[idx];
      return 1;
  }
}

/* ------------------------------------------------------------------------ */
/* Table                                                                    */
/* ------------------------------------------------------------------------ */
struct hkvo_table {
  uint64_t init_capacity, max_capacity, max_size;
  uint32_t B, bshift, dim, elem_bytes, value_bytes;
  int value_dtype, strategy;
  float max_load_factor;
  uint64_t capacity, num_buckets, magic, mshift;
  uint64_t* keys;
  uint64_t* scores;
  uint8_t* digests;
  int32_t* sizes;
  uint8_t* values;
  uint64_t epoch, clock;
  int reach_max, nthreads;
};

static uint32_t ilog2(uint64_t x) {
  uint32_t r = 0;
  while ((1ull << r) < x) r++;
  return r;
}

/* initialize_buckets key/digest/score fill, init_table_kernel.h:81-104. */
static void init_buckets(hkvo_table* t, uint64_t b0, uint64_t b1) {
  uint8_t ed = hkvo_empty_digest();
  for (uint64_t i = b0 * t->B; i < b1 * t->B; i++) {
    t->keys[i] = HKVO_EMPTY_KEY;
    t->scores[i] = 0;
    t->digests[i] = ed;
  }
  for (uint64_t b = b0; b < b1; b++) t->sizes[b] = 0;
  memset(t->values + b0 * t->B * t->value_bytes, 0,
         (b1 - b0) * t->B * t->value_bytes);
}

static void set_capacity(hkvo_table* t, uint64_t nb) {
  t->num_buckets = nb;
  t->capacity = nb * t->B;
  hkvo_magic_div(t->capacity, &t->magic, &t->mshift);
}

/* create_table bucket-count rule, table.h:279-332; reach_max_capacity_,
 * hkv_hashtable.h:1021. */
hkvo_table* hkvo_create(uint64_t init_capacity, uint64_t max_capacity,
                        uint32_t bucket_size, uint32_t dim, uint32_t elem_bytes,
                        int value_dtype, int strategy, float max_load_factor) {
  hkvo_table* t = (hkvo_table*)calloc(1, sizeof(hkvo_table));
  t->init_capacity = init_capacity;
  t->max_capacity = max_capacity;
  t->max_size = init_capacity > max_capacity ? init_capacity : max_capacity;
  t->B = bucket_size;
  t->bshift = ilog2(bucket_size);
  t->dim = dim;
  t->elem_bytes = elem_bytes;
  t->value_bytes = dim * elem_bytes;
  t->value_dtype = value_dtype;
  t->strategy = strategy;
  t->max_load_factor = max_load_factor;
  t->epoch = HKVO_IGNORED_EPOCH;
  t->nthreads = 1;
  uint64_t nb;
  if (init_capacity * 2 > t->max_size) {
    nb = 1 + (t->max_size - 1) / bucket_size;
  } else {
    nb = 1;
    while (nb * bucket_size < init_capacity) nb *= 2;
  }
  set_capacity(t, nb);
  size_t slots = (size_t)(nb * bucket_size);
  t->keys = (uint64_t*)malloc(slots * 8);
  t->scores = (uint64_t*)malloc(slots * 8);
  t->digests = (uint8_t*)malloc(slots);
  t->sizes = (int32_t*)malloc(nb * 4);
  t->values = (uint8_t*)malloc(slots * (size_t)t->value_bytes + 1);
  init_buckets(t, 0, nb);
  t->reach_max = init_capacity * 2 > max_capacity;
  return t;
}

void hkvo_destroy(hkvo_table* t) {
  if (!t) return;
  free(t->keys);
  free(t->scores);
  free(t->digests);
  free(t->sizes);
  free(t->values);
  free(t);
}

void hkvo_set_threads(hkvo_table* t, int n) { t->nthreads = n < 1 ? 1 : n; }
void hkvo_set_global_epoch(hkvo_table* t, uint64_t e) { t->epoch = e; }
void hkvo_set_clock(hkvo_table* t, uint64_t c) { t->clock = c; }
uint64_t hkvo_capacity(const hkvo_table* t) { return t->capacity; }
uint64_t hkvo_bucket_count(const hkvo_table* t) { return t->num_buckets; }
int hkvo_reach_max(const hkvo_table* t) { return t->reach_max; }

/* size(), hkv_hashtable.h:2792-2819: sum of per-bucket sizes. */
uint64_t hkvo_size(const hkvo_table* t) {
  int64_t s = 0;
  for (uint64_t b = 0; b < t->num_buckets; b++) s += t->sizes[b];
  return (uint64_t)s;
}

/* load_factor, hkv_hashtable.h:2945. */
float hkvo_load_factor(const hkvo_table* t) {
  return (float)((hkvo_size(t) * 1.0) / (t->capacity * 1.0));
}

/* ---- parallel helper: split key indices by bucket -------------------- */
typedef struct {
  void (*fn)(void* ctx, size_t i);
  void* ctx;
  const size_t* idx;
  size_t lo, hi;
} list_arg;

static void* list_worker(void* p) {
  list_arg* a = (list_arg*)p;
  for (size_t j = a->lo; j < a->hi; j++) a->fn(a->ctx, a->idx[j]);
  return NULL;
}

typedef struct {
  const hkvo_table* t;
  const uint64_t* keys;
  uint32_t* part;
  int nth;
  size_t lo, hi;
} part_arg;

static void* part_worker(void* p) {
  part_arg* a = (part_arg*)p;
  for (size_t i = a->lo; i < a->hi; i++) {
    uint64_t h = hkvo_murmur3(a->keys[i]);
    uint64_t bkt =
        hkvo_fast_mod(h, a->t->capacity, a->t->magic, a->t->mshift) >> a->t->bshift;
    a->part[i] = (uint32_t)(bkt % (uint64_t)a->nth);
  }
  return NULL;
}

/* Keys are grouped by bucket % nthreads (counting sort, stable), and every
 * worker applies its group in index order: a bucket is only ever touched by
 * one worker, in the batch's order. */
static void for_each_key(hkvo_table* t, size_t n, const uint64_t* keys,
                         void (*fn)(void*, size_t), void* ctx) {
  int nth = t->nthreads;
  if (nth <= 1 || n < 4096) {
    for (size_t i = 0; i < n; i++) fn(ctx, i);
    return;
  }
  if (nth > 256) nth = 256;
  uint32_t* part = (uint32_t*)malloc(n * sizeof(uint32_t));
  size_t* idx = (size_t*)malloc(n * sizeof(size_t));
  pthread_t th[256];
  part_arg pa[256];
  for (int i = 0; i < nth; i++) {
    pa[i] = (part_arg){t, keys, part, nth, n * (size_t)i / nth,
                       n * (size_t)(i + 1) / nth};
    pthread_create(&th[i], NULL, part_worker, &pa[i]);
  }
  for (int i = 0; i < nth; i++) pthread_join(th[i], NULL);
  size_t start[257];
  memset(start, 0, sizeof start);
  for (size_t i = 0; i < n; i++) start[part[i] + 1]++;
  for (int i = 0; i < nth; i++) start[i + 1] += start[i];
  size_t fill[256];
  for (int i = 0; i < nth; i++) fill[i] = start[i];
  for (size_t i = 0; i < n; i++) idx[fill[part[i]]++] = i;
  list_arg la[256];
  for (int i = 0; i < nth; i++) {
    la[i] = (list_arg){fn, ctx, idx, start[i], start[i + 1]};
    pthread_create(&th[i], NULL, list_worker, &la[i]);
  }
  for (int i = 0; i < nth; i++) pthread_join(th[i], NULL);
  free(part);
  free(idx);
}

typedef struct {
  void (*fn)(void*, uint64_t);
  void* ctx;
  uint64_t lo, hi;
} range_arg;

static void* range_worker(void* p) {
  range_arg* a = (range_arg*)p;
  for (uint64_t i = a->lo; i < a->hi; i++) a->fn(a->ctx, i);
  return NULL;
}

static void parallel_range(int nth, uint64_t n, void (*fn)(void*, uint64_t),
                           void* ctx) {
  if (nth <= 1 || n < 64) {
    for (uint64_t i = 0; i < n; i++) fn(ctx, i);
    return;
  }
  if (nth > 256) nth = 256;
  pthread_t th[256];
  range_arg args[256];
  for (int i = 0; i < nth; i++) {
    args[i] = (range_arg){fn, ctx, n * (uint64_t)i / nth,
                          n * (uint64_t)(i + 1) / nth};
    pthread_create(&th[i], NULL, range_worker, &args[i]);
  }
  for (int i = 0; i < nth; i++) pthread_join(th[i], NULL);
}

/* ---- addressing --------------------------------------------------------- */
typedef struct {
  uint64_t bkt;
  uint32_t pos;
  uint8_t digest;
} loc_t;

/* hash -> global_idx -> (bucket, start position), find_with_digest_kernel.h
 * :57-64. */
static loc_t locate(const hkvo_table* t, uint64_t key) {
  uint64_t h = hkvo_murmur3(key);
  uint64_t g = hkvo_fast_mod(h, t->capacity, t->magic, t->mshift);
  loc_t l;
  l.bkt = g >> t->bshift;
  l.pos = (uint32_t)(g & (t->B - 1));
  l.digest = (uint8_t)(h >> 32);
  return l;
}

static uint8_t* value_ptr(const hkvo_table* t, uint64_t slot) {
  return t->values + slot * (uint64_t)t->value_bytes;
}

/* find_without_lock, find_utils.h:31-86: groups of 4 digests from
 * align4(pos), wrapping once past the start; digest hits compare the key,
 * a digest-empty slot holding EMPTY_KEY ends the search (empties before pos
 * in the first group are skipped). Returns slot position or -1. */
static int find_pos(const hkvo_table* t, const loc_t* l, uint64_t key) {
  const uint32_t B = t->B;
  const uint64_t base = l->bkt * B;
  const uint8_t ed = hkvo_empty_digest();
  const uint32_t g0 = l->pos & ~3u;
  for (uint32_t off = 0; off < B + 4; off += 4) {
    uint32_t g = (g0 + off) & (B - 1);
    for (uint32_t j = 0; j < 4; j++) {
      uint32_t p = g + j;
      if (t->digests[base + p] == l->digest && t->keys[base + p] == key)
        return (int)p;
    }
    for (uint32_t j = 0; j < 4; j++) {
      uint32_t p = g + j;
      if (t->digests[base + p] != ed) continue;
      if (off == 0 && p < l->pos) continue;
      if (t->keys[base + p] == HKVO_EMPTY_KEY) return -1;
    }
  }
  return -1;
}

/* Probe of the unique-key insert kernels, insert_or_assign_kernel.h:105-183
 * (same in find_or_insert_kernel.h:100-179, insert_and_evict_kernel.h
 * :419-496): per group, digest hits first (key compare), then -- unless the
 * bucket size snapshot equals the bucket capacity -- the first digest-empty
 * slot holding EMPTY_KEY at or after pos. Returns DUPLICATE / OCCUPIED_EMPTY
 * with *slot, or 0 when the caller must evict. */
static int probe_insert(const hkvo_table* t, const loc_t* l, uint64_t key,
                        uint32_t* slot) {
  const uint32_t B = t->B;
  const uint64_t base = l->bkt * B;
  const uint8_t ed = hkvo_empty_digest();
  const uint32_t g0 = l->pos & ~3u;
  const int full = t->sizes[l->bkt] == (int32_t)B;
  for (uint32_t off = 0; off < B + 4; off += 4) {
    uint32_t g = (g0 + off) & (B - 1);
    for (uint32_t j = 0; j < 4; j++) {
      uint32_t p = g + j;
      if (t->digests[base + p] == l->digest && t->keys[base + p] == key) {
        *slot = p;
        return HKVO_R_DUPLICATE;
      }
    }
    if (full) continue;
    for (uint32_t j = 0; j < 4; j++) {
      uint32_t p = g + j;
      if (t->digests[base + p] != ed) continue;
      if (off == 0 && p < l->pos) continue;
      if (t->keys[base + p] == HKVO_EMPTY_KEY) {
        *slot = p;
        return HKVO_R_OCCUPIED_EMPTY;
      }
    }
  }
  return 0;
}

/* Victim choice of the unique-key kernels, insert_or_assign_kernel.h:193-238:
 * 16 lanes each take the first strictly-smallest score among non-EMPTY,
 * non-LOCKED slots at positions lane, lane+16, ...; an xor butterfly
 * (offsets 8,4,2,1) keeps the partner's candidate only when strictly smaller;
 * the key's own lane (kv_idx % 16) decides with the candidate it ends with. */
static void victim_unique(const hkvo_table* t, const loc_t* l, size_t kv_idx,
                          uint64_t* min_score, uint32_t* min_pos) {
  const uint32_t B = t->B;
  const uint64_t base = l->bkt * B;
  uint64_t sc[16], sc2[16];
  uint32_t ps[16], ps2[16];
  for (int c = 0; c < 16; c++) {
    sc[c] = HKVO_MAX_SCORE;
    ps[c] = l->pos;
    for (uint32_t p = (uint32_t)c; p < B; p += 16) {
      uint64_t s = t->scores[base + p];
      uint64_t k = t->keys[base + p];
      if (s < sc[c] && k != HKVO_LOCKED_KEY && k != HKVO_EMPTY_KEY) {
        sc[c] = s;
        ps[c] = p;
      }
    }
  }
  for (int o = 8; o > 0; o >>= 1) {
    for (int c = 0; c < 16; c++) {
      int x = c ^ o;
      if (sc[x] < sc[c]) {
        sc2[c] = sc[x];
        ps2[c] = ps[x];
      } else {
        sc2[c] = sc[c];
        ps2[c] = ps[c];
      }
    }
    memcpy(sc, sc2, sizeof sc);
    memcpy(ps, ps2, sizeof ps);
  }
  *min_score = sc[kv_idx & 15];
  *min_pos = ps[kv_idx & 15];
}

/* find_and_lock, find_utils.h:94-228 (used by accum_or_assign): 32-slot
 * windows starting at pos; a key hit wins, else the lowest lane holding
 * EMPTY_KEY is claimed; if the bucket has neither, each of 32 lanes takes the
 * first strictly-smallest score over its slots (pos+lane+32w) among non-EMPTY
 * keys, the global minimum is compared with the desired score (refuse iff
 * desired < min), and the lowest lane holding the minimum is the victim. */
static int probe_find_and_lock(const hkvo_table* t, const loc_t* l,
                               uint64_t key, uint64_t desired, uint32_t* slot,
                               uint64_t* evicted_key) {
  const uint32_t B = t->B;
  const uint64_t base = l->bkt * B;
  for (uint32_t w = 0; w < B; w += 32) {
    for (uint32_t lane = 0; lane < 32; lane++) {
      uint32_t p = (l->pos + w + lane) % B;
      if (t->keys[base + p] == key) {
        *slot = p;
        return HKVO_R_DUPLICATE;
      }
    }
    for (uint32_t lane = 0; lane < 32; lane++) {
      uint32_t p = (l->pos + w + lane) % B;
      if (t->keys[base + p] == HKVO_EMPTY_KEY) {
        *slot = p;
        return HKVO_R_OCCUPIED_EMPTY;
      }
    }
  }
  uint64_t lmin[32], gmin = HKVO_MAX_SCORE;
  uint32_t lpos[32];
  uint64_t lkey[32];
  for (uint32_t lane = 0; lane < 32; lane++) {
    lmin[lane] = HKVO_MAX_SCORE;
    lpos[lane] = 0;
    lkey[lane] = HKVO_EMPTY_KEY;
    for (uint32_t w = 0; w < B; w += 32) {
      uint32_t p = (l->pos + w + lane) % B;
      uint64_t s = t->scores[base + p];
      if (s < lmin[lane] && t->keys[base + p] != HKVO_EMPTY_KEY) {
        lmin[lane] = s;
        lpos[lane] = p;
        lkey[lane] = t->keys[base + p];
      }
    }
    if (lmin[lane] < gmin) gmin = lmin[lane];
  }
  if (desired < gmin) return HKVO_R_REFUSED;
  for (uint32_t lane = 0; lane < 32; lane++) {
    if (lmin[lane] <= gmin) {
      *slot = lpos[lane];
      *evicted_key = lkey[lane];
      return lkey[lane] == HKVO_RECLAIM_KEY ? HKVO_R_OCCUPIED_RECLAIMED
                                             : HKVO_R_EVICT;
    }
  }
  return HKVO_R_REFUSED;
}

/* check_evict_strategy, hkv_hashtable.h:3270-3298 is enforced by the caller;
 * `ignore_evict_strategy` runs the Customized functor, :1077-1091. */
static int eff_strategy(const hkvo_table* t, int ignore) {
  return ignore ? HKVO_CUSTOMIZED : t->strategy;
}

/* fast_load_factor, hkv_hashtable.h:3229-3268 (first min(buckets,1024)
 * bucket sizes), and the auto-grow loop, hkv_hashtable.h:1103-1106. */
static float fast_load_factor(const hkvo_table* t, size_t delta) {
  uint64_t N = t->num_buckets < 1024 ? t->num_buckets : 1024;
  int64_t s = 0;
  for (uint64_t b = 0; b < N; b++) s += t->sizes[b];
  return (float)((delta * 1.0) / (t->capacity * 1.0) +
                 (s * 1.0) / (t->B * N * 1.0));
}

static void auto_grow(hkvo_table* t, size_t n) {
  while (!t->reach_max && fast_load_factor(t, n) > t->max_load_factor)
    hkvo_reserve(t, t->capacity * 2);
}

/* Shared single-key upsert: returns the OccupyResult and the slot. */
typedef struct {
  hkvo_table* t;
  const uint64_t* keys;
  const uint8_t* in_values;
  uint8_t* io_values;
  const uint64_t* scores;
  int strategy;
  uint8_t* results;
  /* insert_and_evict per-key records */
  uint64_t* ev_key;
  uint64_t* ev_score;
  uint8_t* ev_value;
  uint8_t* ev_flag;
  const uint8_t* accum;
  int mode; /* 0 insert_or_assign, 1 find_or_insert, 2 insert_and_evict */
} up_ctx;

static void write_score(hkvo_table* t, int strategy, uint64_t slot,
                        const uint64_t* in, size_t idx, uint64_t desired,
                        int new_insert, uint8_t digest, int with_digest) {
  uint64_t s;
  if (!hkvo_score_on_write(strategy, t->scores[slot], in, idx, desired,
                           new_insert, &s))
    return; /* Lfu with NULL scores writes neither digest nor score */
  if (with_digest) t->digests[slot] = digest;
  t->scores[slot] = s;
}

/* Unique-key upsert, insert_or_assign_kernel.h:77-303,
 * find_or_insert_kernel.h:72-306, insert_and_evict_kernel.h:389-691. */
static void upsert_one(void* p, size_t i) {
  up_ctx* c = (up_ctx*)p;
  hkvo_table* t = c->t;
  const uint64_t key = c->keys[i];
  const uint32_t vb = t->value_bytes;
  if (hkvo_is_reserved(key)) {
    if (c->results) c->results[i] = HKVO_R_ILLEGAL;
    return;
  }
  const uint64_t desired =
      hkvo_desired_when_missed(c->strategy, c->scores, i, t->epoch, t->clock);
  loc_t l = locate(t, key);
  const uint64_t base = l.bkt * t->B;
  uint32_t slot = 0;
  int r = probe_insert(t, &l, key, &slot);
  uint64_t victim_key = 0, victim_score = 0;
  if (r == 0) {
    uint64_t mins;
    uint32_t minp;
    victim_unique(t, &l, i, &mins, &minp);
    if (desired < mins) {
      r = HKVO_R_REFUSED;
    } else {
      slot = minp;
      victim_key = t->keys[base + slot];
      victim_score = mins;
      r = victim_key == HKVO_RECLAIM_KEY ? HKVO_R_OCCUPIED_RECLAIMED
                                         : HKVO_R_EVICT;
    }
  }
  if (c->results) c->results[i] = (uint8_t)r;
  const uint8_t* in_v = c->in_values ? c->in_values + i * (size_t)vb : NULL;
  if (r == HKVO_R_REFUSED) {
    if (c->mode == 2) {
      /* insert_and_evict_kernel.h:553-557: the refused input is reported */
      c->ev_flag[i] = 1;
      c->ev_key[i] = key;
      c->ev_score[i] = desired;
      memcpy(c->ev_value + i * (size_t)vb, in_v, vb);
    }
    return;
  }
  const uint64_t s = base + slot;
  if (r == HKVO_R_DUPLICATE) {
    write_score(t, c->strategy, s, c->scores, i, desired, 0, l.digest, 0);
    if (c->mode == 1)
      memcpy(c->io_values + i * (size_t)vb, value_ptr(t, s), vb);
    else
      memcpy(value_ptr(t, s), in_v, vb);
    return;
  }
  if (r == HKVO_R_EVICT && c->mode == 2) {
    /* insert_and_evict_kernel.h:580-584, :654-661 */
    c->ev_flag[i] = 1;
    c->ev_key[i] = victim_key;
    c->ev_score[i] = victim_score;
    memcpy(c->ev_value + i * (size_t)vb, value_ptr(t, s), vb);
  }
  if (r == HKVO_R_OCCUPIED_EMPTY || r == HKVO_R_OCCUPIED_RECLAIMED)
    t->sizes[l.bkt]++;
  write_score(t, c->strategy, s, c->scores, i, desired, 1, l.digest, 1);
  const uint8_t* src = (c->mode == 1) ? c->io_values + i * (size_t)vb : in_v;
  memcpy(value_ptr(t, s), src, vb);
  t->keys[s] = key;
}

void hkvo_insert_or_assign(hkvo_table* t, size_t n, const uint64_t* keys,
                           const void* values, const uint64_t* scores,
                           int ignore, uint8_t* results) {
  if (n == 0) return;
  auto_grow(t, n);
  up_ctx c;
  memset(&c, 0, sizeof c);
  c.t = t;
  c.keys = keys;
  c.in_values = (const uint8_t*)values;
  c.scores = scores;
  c.strategy = eff_strategy(t, ignore);
  c.results = results;
  c.mode = 0;
  for_each_key(t, n, keys, upsert_one, &c);
}

void hkvo_find_or_insert(hkvo_table* t, size_t n, const uint64_t* keys,
                         void* values, const uint64_t* scores, int ignore,
                         uint8_t* results) {
  if (n == 0) return;
  auto_grow(t, n);
  up_ctx c;
  memset(&c, 0, sizeof c);
  c.t = t;
  c.keys = keys;
  c.io_values = (uint8_t*)values;
  c.scores = scores;
  c.strategy = eff_strategy(t, ignore);
  c.results = results;
  c.mode = 1;
  for_each_key(t, n, keys, upsert_one, &c);
}

size_t hkvo_insert_and_evict(hkvo_table* t, size_t n, const uint64_t* keys,
                             const void* values, const uint64_t* scores,
                             uint64_t* ev_keys, void* ev_values,
                             uint64_t* ev_scores, int ignore,
                             uint8_t* results) {
  if (n == 0) return 0;
  auto_grow(t, n);
  const uint32_t vb = t->value_bytes;
  up_ctx c;
  memset(&c, 0, sizeof c);
  c.t = t;
  c.keys = keys;
  c.in_values = (const uint8_t*)values;
  c.scores = scores;
  c.strategy = eff_strategy(t, ignore);
  c.results = results;
  c.mode = 2;
  c.ev_key = (uint64_t*)malloc(n * 8);
  c.ev_score = (uint64_t*)malloc(n * 8);
  c.ev_value = (uint8_t*)malloc(n * (size_t)vb + 1);
  c.ev_flag = (uint8_t*)calloc(n, 1);
  for_each_key(t, n, keys, upsert_one, &c);
  size_t cnt = 0;
  for (size_t i = 0; i < n; i++) {
    if (!c.ev_flag[i]) continue;
    ev_keys[cnt] = c.ev_key[i];
    if (ev_scores) ev_scores[cnt] = c.ev_score[i];
    memcpy((uint8_t*)ev_values + cnt * (size_t)vb, c.ev_value + i * (size_t)vb,
           vb);
    cnt++;
  }
  free(c.ev_key);
  free(c.ev_score);
  free(c.ev_value);
  free(c.ev_flag);
  return cnt;
}

/* ---- accum_or_assign, accum_or_assign_kernel.h:55-155 ------------------- */
static float h2f(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1F, man = h & 0x3FF, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      exp = 127 - 15 + 1;
      while ((man & 0x400) == 0) {
        man <<= 1;
        exp--;
      }
      man &= 0x3FF;
      bits = sign | (exp << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* float -> binary16, round to nearest even. */
static uint16_t f2h(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000;
  uint32_t ax = x & 0x7FFFFFFF;
  if (ax >= 0x7F800000) return (uint16_t)(sign | 0x7C00 | (ax > 0x7F800000 ? 0x200 : 0));
  if (ax >= 0x477FF000) return (uint16_t)(sign | 0x7C00); /* overflow */
  if (ax < 0x38800000) { /* subnormal or zero in half */
    float a;
    memcpy(&a, &ax, 4);
    /* scale so that 2^-24 is one unit, rint is round-half-even */
    float q = rintf(a * 16777216.0f);
    return (uint16_t)(sign | (uint32_t)q);
  }
  uint32_t e = (ax >> 23) - 127 + 15;
  uint32_t m = ax & 0x7FFFFF;
  uint32_t h = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1FFF;
  if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
  return (uint16_t)(sign | h);
}

static float bf2f(uint16_t b) {
  uint32_t bits = (uint32_t)b << 16;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static uint16_t f2bf(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  if ((x & 0x7FFFFFFF) > 0x7F800000) return (uint16_t)((x >> 16) | 0x40);
  uint32_t lsb = (x >> 16) & 1;
  x += 0x7FFF + lsb;
  return (uint16_t)(x >> 16);
}

/* accum_or_assign_vector, accum_or_assign_kernel.h:36-49: dst = src + dst
 * in the value type (two binary16/bfloat16 operands summed in binary32 and
 * rounded once more is correctly rounded, since 24 >= 2*11+2). */
static void accum_vec(const hkvo_table* t, uint8_t* dst, const uint8_t* src) {
  uint32_t d = t->dim;
  if (t->value_dtype == HKVO_F32) {
    float* o = (float*)dst;
    const float* s = (const float*)src;
    for (uint32_t i = 0; i < d; i++) o[i] = s[i] + o[i];
  } else if (t->value_dtype == HKVO_F16) {
    uint16_t* o = (uint16_t*)dst;
    const uint16_t* s = (const uint16_t*)src;
    for (uint32_t i = 0; i < d; i++) o[i] = f2h(h2f(s[i]) + h2f(o[i]));
  } else if (t->value_dtype == HKVO_BF16) {
    uint16_t* o = (uint16_t*)dst;
    const uint16_t* s = (const uint16_t*)src;
    for (uint32_t i = 0; i < d; i++) o[i] = f2bf(bf2f(s[i]) + bf2f(o[i]));
  }
}

static void accum_one(void* p, size_t i) {
  up_ctx* c = (up_ctx*)p;
  hkvo_table* t = c->t;
  const uint64_t key = c->keys[i];
  const uint32_t vb = t->value_bytes;
  if (hkvo_is_reserved(key)) {
    if (c->results) c->results[i] = HKVO_R_ILLEGAL;
    return;
  }
  const uint64_t desired =
      hkvo_desired_when_missed(c->strategy, c->scores, i, t->epoch, t->clock);
  const int is_accum = c->accum[i] != 0;
  loc_t l = locate(t, key);
  const uint64_t base = l.bkt * t->B;
  uint32_t slot = 0;
  uint64_t evk = 0;
  int r = probe_find_and_lock(t, &l, key, desired, &slot, &evk);
  if (c->results) c->results[i] = (uint8_t)r;
  if (r == HKVO_R_REFUSED) return;
  /* :114-128: mismatched accum/assign restores the slot and skips */
  if ((is_accum && r != HKVO_R_DUPLICATE) ||
      (!is_accum && r == HKVO_R_DUPLICATE)) {
    if (c->results) c->results[i] = HKVO_R_ILLEGAL;
    return;
  }
  const uint64_t s = base + slot;
  if (r == HKVO_R_OCCUPIED_EMPTY || r == HKVO_R_OCCUPIED_RECLAIMED)
    t->sizes[l.bkt]++;
  const uint8_t* src = c->in_values + i * (size_t)vb;
  if (is_accum)
    accum_vec(t, value_ptr(t, s), src);
  else
    memcpy(value_ptr(t, s), src, vb);
  write_score(t, c->strategy, s, c->scores, i, desired,
              r != HKVO_R_DUPLICATE, l.digest, 1);
  t->keys[s] = key;
}

void hkvo_accum_or_assign(hkvo_table* t, size_t n, const uint64_t* keys,
                          const void* values, const uint8_t* accum,
                          const uint64_t* scores, int ignore,
                          uint8_t* results) {
  if (n == 0) return;
  auto_grow(t, n);
  up_ctx c;
  memset(&c, 0, sizeof c);
  c.t = t;
  c.keys = keys;
  c.in_values = (const uint8_t*)values;
  c.scores = scores;
  c.accum = accum;
  c.strategy = eff_strategy(t, ignore);
  c.results = results;
  for_each_key(t, n, keys, accum_one, &c);
}

/* ---- read-only and score-only ops ------------------------------------- */
typedef struct {
  hkvo_table* t;
  const uint64_t* keys;
  uint8_t* values;
  uint8_t* founds;
  uint64_t* scores;
  const uint64_t* in_scores;
} ro_ctx;

/* find_with_digest_kernel.h:47-107: misses leave values and scores as they
 * were; founds is always written. */
static void find_one(void* p, size_t i) {
  ro_ctx* c = (ro_ctx*)p;
  const hkvo_table* t = c->t;
  const uint64_t key = c->keys[i];
  int found = 0;
  if (!hkvo_is_reserved(key)) {
    loc_t l = locate(t, key);
    int pos = find_pos(t, &l, key);
    if (pos >= 0) {
      found = 1;
      uint64_t s = l.bkt * t->B + (uint64_t)pos;
      if (c->scores) c->scores[i] = t->scores[s];
      if (c->values)
        memcpy(c->values + i * (size_t)t->value_bytes, value_ptr(t, s),
               t->value_bytes);
    }
  }
  if (c->founds) c->founds[i] = (uint8_t)found;
}

void hkvo_find(hkvo_table* t, size_t n, const uint64_t* keys, void* values,
               uint8_t* founds, uint64_t* scores) {
  ro_ctx c = {t, keys, (uint8_t*)values, founds, scores, NULL};
  for_each_key(t, n, keys, find_one, &c);
}

/* contains_kernel.h:31-64. */
void hkvo_contains(hkvo_table* t, size_t n, const uint64_t* keys,
                   uint8_t* founds) {
  ro_ctx c = {t, keys, NULL, founds, NULL, NULL};
  for_each_key(t, n, keys, find_one, &c);
}

/* assign_scores_kernel_with_filter.h:65-140: existing keys only, found with
 * the find stop rule, score = update_without_missed. */
static void assign_score_one(void* p, size_t i) {
  ro_ctx* c = (ro_ctx*)p;
  hkvo_table* t = c->t;
  const uint64_t key = c->keys[i];
  if (hkvo_is_reserved(key)) return;
  loc_t l = locate(t, key);
  int pos = find_pos(t, &l, key);
  if (pos < 0) return;
  uint64_t s = l.bkt * t->B + (uint64_t)pos, out;
  if (hkvo_score_without_missed(t->strategy, t->scores[s], c->in_scores, i,
                                t->epoch, t->clock, &out))
    t->scores[s] = out;
}

void hkvo_assign_scores(hkvo_table* t, size_t n, const uint64_t* keys,
                        const uint64_t* scores) {
  ro_ctx c = {t, keys, NULL, NULL, NULL, scores};
  for_each_key(t, n, keys, assign_score_one, &c);
}

/* remove_kernel.h:57-112: every digest hit whose key matches becomes a
 * RECLAIM tombstone with score 0 and the reclaim digest; size decrements.
 * The whole bucket is scanned (no stop rule). */
static void erase_one(void* p, size_t i) {
  ro_ctx* c = (ro_ctx*)p;
  hkvo_table* t = c->t;
  const uint64_t key = c->keys[i];
  if (hkvo_is_reserved(key)) return;
  loc_t l = locate(t, key);
  const uint32_t B = t->B;
  const uint64_t base = l.bkt * B;
  const uint32_t g0 = l.pos & ~3u;
  for (uint32_t off = 0; off < B + 4; off += 4) {
    uint32_t g = (g0 + off) & (B - 1);
    for (uint32_t j = 0; j < 4; j++) {
      uint64_t s = base + g + j;
      if (t->digests[s] == l.digest && t->keys[s] == key) {
        t->keys[s] = HKVO_RECLAIM_KEY;
        t->scores[s] = 0;
        t->digests[s] = hkvo_reclaim_digest();
        t->sizes[l.bkt]--;
        break;
      }
    }
  }
}

void hkvo_erase(hkvo_table* t, size_t n, const uint64_t* keys) {
  ro_ctx c = {t, keys, NULL, NULL, NULL, NULL};
  for_each_key(t, n, keys, erase_one, &c);
}

/* clear_kernel.h:29-60: keys EMPTY, digests empty, sizes 0; scores and
 * values are left as they were. */
void hkvo_clear(hkvo_table* t) {
  uint8_t ed = hkvo_empty_digest();
  for (uint64_t i = 0; i < t->capacity; i++) {
    t->keys[i] = HKVO_EMPTY_KEY;
    t->digests[i] = ed;
  }
  for (uint64_t b = 0; b < t->num_buckets; b++) t->sizes[b] = 0;
}

/* export_batch, hkv_hashtable.h:2519-2549 and dump_kernel.h:55-121: slots
 * [offset, offset + min(n, capacity - offset)) in slot order, reserved keys
 * skipped. (The device kernel's output order is not deterministic.) */
size_t hkvo_export_batch(hkvo_table* t, size_t n, size_t offset,
                         uint64_t* keys, void* values, uint64_t* scores) {
  if (offset >= t->capacity) return 0;
  if (n > t->capacity - offset) n = t->capacity - offset;
  size_t cnt = 0;
  for (size_t s = offset; s < offset + n; s++) {
    uint64_t k = t->keys[s];
    if (hkvo_is_reserved(k)) continue;
    keys[cnt] = k;
    if (scores) scores[cnt] = t->scores[s];
    if (values)
      memcpy((uint8_t*)values + cnt * (size_t)t->value_bytes, value_ptr(t, s),
             t->value_bytes);
    cnt++;
  }
  return cnt;
}

/* ---- reserve / rehash -------------------------------------------------- */
typedef struct {
  hkvo_table* t;
  uint64_t old_nb;
} rh_ctx;

/* copy_key_to_new_bucket, rehash_kernel.h:30-67: first EMPTY_KEY slot in
 * linear order from the key's start position in the new bucket. */
static void copy_to_new_bucket(hkvo_table* t, uint64_t key, uint64_t score,
                               const uint8_t* val, uint64_t nb, uint32_t npos) {
  const uint32_t B = t->B;
  for (uint32_t off = 0; off < B; off++) {
    uint32_t p = (npos + off) % B;
    uint64_t s = nb * B + p;
    if (t->keys[s] == HKVO_EMPTY_KEY) {
      t->keys[s] = key;
      t->scores[s] = score;
      t->digests[s] = hkvo_digest(key);
      t->sizes[nb]++;
      memcpy(value_ptr(t, s), val, t->value_bytes);
      return;
    }
  }
}

/* defragmentation_for_rehash, rehash_kernel.h:77-135: backward-shift the
 * run after a hole so every key stays reachable from its start position. */
static void defrag(hkvo_table* t, uint64_t b, uint32_t remove_pos,
                   uint64_t old_nb) {
  const uint32_t B = t->B;
  const uint64_t base = b * B;
  uint32_t off = 1;
  while (off < B) {
    uint32_t cur = (remove_pos + off) % B;
    uint64_t ck = t->keys[base + cur];
    if (ck == HKVO_EMPTY_KEY) break;
    uint64_t g = hkvo_murmur3(ck) % (old_nb * B);
    uint32_t start = (uint32_t)(g % B);
    if ((start <= remove_pos && remove_pos < cur) ||
        (cur < start && start <= remove_pos) ||
        (remove_pos < cur && cur < start)) {
      t->keys[base + remove_pos] = ck;
      t->scores[base + remove_pos] = t->scores[base + cur];
      t->digests[base + remove_pos] = hkvo_digest(ck);
      memcpy(value_ptr(t, base + remove_pos), value_ptr(t, base + cur),
             t->value_bytes);
      t->keys[base + cur] = HKVO_EMPTY_KEY;
      t->digests[base + cur] = hkvo_empty_digest();
      remove_pos = cur;
      off = 1;
    } else {
      off++;
    }
  }
}

/* rehash_kernel_vf, rehash_kernel.h:139-207 (one old bucket). */
static void rehash_bucket(void* p, uint64_t b) {
  rh_ctx* c = (rh_ctx*)p;
  hkvo_table* t = c->t;
  const uint32_t B = t->B;
  const uint64_t base = b * B;
  uint32_t kp = 0;
  while (kp < B) {
    uint64_t k = t->keys[base + kp];
    uint64_t sc = t->scores[base + kp];
    if (k == HKVO_EMPTY_KEY || k == HKVO_RECLAIM_KEY) {
      kp++;
      continue;
    }
    uint64_t g = hkvo_murmur3(k) % (t->num_buckets * B);
    uint64_t nb = g / B;
    if (nb == b) {
      kp++;
      continue;
    }
    copy_to_new_bucket(t, k, sc, value_ptr(t, base + kp), nb,
                       (uint32_t)(g % B));
    t->keys[base + kp] = HKVO_EMPTY_KEY;
    t->digests[base + kp] = hkvo_empty_digest();
    t->sizes[b]--;
    defrag(t, b, kp, c->old_nb);
    kp = 0;
  }
}

/* double_capacity, table.h:360-377. */
static void double_capacity(hkvo_table* t) {
  uint64_t nb = t->num_buckets, slots = nb * t->B;
  t->keys = (uint64_t*)realloc(t->keys, slots * 2 * 8);
  t->scores = (uint64_t*)realloc(t->scores, slots * 2 * 8);
  t->digests = (uint8_t*)realloc(t->digests, slots * 2);
  t->sizes = (int32_t*)realloc(t->sizes, nb * 2 * 4);
  t->values = (uint8_t*)realloc(t->values, slots * 2 * t->value_bytes + 1);
  init_buckets(t, nb, nb * 2);
  set_capacity(t, nb * 2);
}

/* reserve, hkv_hashtable.h:2873-2935. */
void hkvo_reserve(hkvo_table* t, uint64_t new_capacity) {
  if (t->reach_max || new_capacity > t->max_capacity) {
    t->reach_max = t->capacity * 2 > t->max_capacity;
    return;
  }
  while (t->capacity < new_capacity && t->capacity * 2 <= t->max_capacity) {
    uint64_t old_nb = t->num_buckets;
    double_capacity(t);
    rh_ctx c = {t, old_nb};
    parallel_range(t->nthreads, old_nb, rehash_bucket, &c);
  }
  t->reach_max = t->capacity * 2 > t->max_capacity;
}

/* ---- raw state --------------------------------------------------------- */
void hkvo_get_state(const hkvo_table* t, uint64_t* keys, uint64_t* scores,
                    uint8_t* digests, int32_t* sizes, void* values) {
  size_t slots = (size_t)t->capacity;
  if (keys) memcpy(keys, t->keys, slots * 8);
  if (scores) memcpy(scores, t->scores, slots * 8);
  if (digests) memcpy(digests, t->digests, slots);
  if (sizes) memcpy(sizes, t->sizes, t->num_buckets * 4);
  if (values) memcpy(values, t->values, slots * (size_t)t->value_bytes);
}

void hkvo_set_state(hkvo_table* t, const uint64_t* keys, const uint64_t* scores,
                    const uint8_t* digests, const int32_t* sizes,
                    const void* values) {
  size_t slots = (size_t)t->capacity;
  if (keys) memcpy(t->keys, keys, slots * 8);
  if (scores) memcpy(t->scores, scores, slots * 8);
  if (digests) memcpy(t->digests, digests, slots);
  if (sizes) memcpy(t->sizes, sizes, t->num_buckets * 4);
  if (values) memcpy(t->values, values, slots * (size_t)t->value_bytes);
}
