/*
 * hkv_oracle.h -- CPU restatement of the HierarchicalKV-ascend hash-table
 * rules (the reference's `include/` tree), used ONLY as a checker.
 *
 * TEST INFRASTRUCTURE. Nothing in the product (the CUDA library, the C++
 * HashTable mirror, the Python binding) links, loads or calls this code.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg do.
 *
 * Parity is pinned by the reference's own known-answer tests, restated in
 * tests/test_oracle_kat.py (score functors: tests/test_score_functor/
 * test_score_functor.cpp:162-380; strategy scores:
 * tests/test_find_or_insert_evict_strategies.cpp:576-623; admission and
 * eviction counts: tests/test_insert_and_evict.cpp:679-961, :1179-1438;
 * reserve: tests/test_reserve.cpp:37-170; export: tests/test_export_batch.cpp).
 * The reference itself cannot be built or run here (it needs Huawei CANN and
 * an Ascend NPU), so there is no compiled reference to diff against.
 *
 * Semantics are sequential: the keys of a batch are applied in index order.
 * Where the reference's outcome depends on thread interleaving (duplicate keys
 * in one batch, several misses racing for one bucket) the GPU result is one
 * valid serialisation and is compared through invariants, not bit-for-bit.
 */
#ifndef HKV_ORACLE_H_
#define HKV_ORACLE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Reserved keys, types.h:63-70. */
#define HKVO_EMPTY_KEY 0xFFFFFFFFFFFFFFFFull
#define HKVO_RECLAIM_KEY 0xFFFFFFFFFFFFFFFEull
#define HKVO_LOCKED_KEY 0xFFFFFFFFFFFFFFFDull
#define HKVO_RESERVED_MASK 0xFFFFFFFFFFFFFFFCull
#define HKVO_MAX_SCORE 0xFFFFFFFFFFFFFFFFull
#define HKVO_IGNORED_EPOCH 0xFFFFFFFFFFFFFFFFull

/* EvictStrategy, hkv_hashtable.h:111-119. */
enum {
  HKVO_LRU = 0,
  HKVO_LFU = 1,
  HKVO_EPOCH_LRU = 2,
  HKVO_EPOCH_LFU = 3,
  HKVO_CUSTOMIZED = 4
};

/* Element type of the value vectors; only matters for accum_or_assign. */
enum { HKVO_F32 = 0, HKVO_F16 = 1, HKVO_BF16 = 2, HKVO_F64 = 3, HKVO_RAW = 9 };

/* Outcome of one insert-like key, OccupyResult in types.h:250-259. */
enum {
  HKVO_R_ILLEGAL = 0,
  HKVO_R_DUPLICATE = 1,
  HKVO_R_OCCUPIED_EMPTY = 2,
  HKVO_R_OCCUPIED_RECLAIMED = 3,
  HKVO_R_EVICT = 4,
  HKVO_R_REFUSED = 5
};

typedef struct hkvo_table hkvo_table;

/* ---- primitives ------------------------------------------------------- */
uint64_t hkvo_murmur3(uint64_t key);
uint8_t hkvo_digest(uint64_t key);
uint8_t hkvo_empty_digest(void);
uint8_t hkvo_reclaim_digest(void);
int hkvo_is_reserved(uint64_t key);
void hkvo_magic_div(uint64_t divisor, uint64_t* magic, uint64_t* shift);
uint64_t hkvo_fast_mod(uint64_t x, uint64_t divisor, uint64_t magic,
                       uint64_t shift);

/* ---- score functors (score_functor.h:45-478) -------------------------- */
/* in_scores may be NULL; idx indexes it. */
uint64_t hkvo_desired_when_missed(int strategy, const uint64_t* in_scores,
                                  size_t idx, uint64_t epoch, uint64_t cycle);
/* Score stored by update_with_digest / update_score_only. `old` is the score
 * already in the slot; `new_insert` selects the insert rule. Returns 0 and
 * leaves *out untouched when the reference would not write (Lfu with NULL
 * input scores). */
int hkvo_score_on_write(int strategy, uint64_t old, const uint64_t* in_scores,
                        size_t idx, uint64_t desired, int new_insert,
                        uint64_t* out);
/* update_without_missed (assign_scores). Same return convention. */
int hkvo_score_without_missed(int strategy, uint64_t old,
                              const uint64_t* in_scores, size_t idx,
                              uint64_t epoch, uint64_t cycle, uint64_t* out);

/* ---- table ------------------------------------------------------------ */
hkvo_table* hkvo_create(uint64_t init_capacity, uint64_t max_capacity,
                        uint32_t bucket_size, uint32_t dim, uint32_t elem_bytes,
                        int value_dtype, int strategy, float max_load_factor);
void hkvo_destroy(hkvo_table* t);
void hkvo_set_threads(hkvo_table* t, int nthreads);
void hkvo_set_global_epoch(hkvo_table* t, uint64_t epoch);
/* Device-clock stand-in for Lru/EpochLru; the reference reads
 * GetSystemCycle() once per launch block. */
void hkvo_set_clock(hkvo_table* t, uint64_t clock);

uint64_t hkvo_capacity(const hkvo_table* t);
uint64_t hkvo_bucket_count(const hkvo_table* t);
uint64_t hkvo_size(const hkvo_table* t);
float hkvo_load_factor(const hkvo_table* t);
int hkvo_reach_max(const hkvo_table* t);

void hkvo_find(hkvo_table* t, size_t n, const uint64_t* keys, void* values,
               uint8_t* founds, uint64_t* scores);
void hkvo_contains(hkvo_table* t, size_t n, const uint64_t* keys,
                   uint8_t* founds);
/* `results` (may be NULL) receives one HKVO_R_* per input key. */
void hkvo_insert_or_assign(hkvo_table* t, size_t n, const uint64_t* keys,
                           const void* values, const uint64_t* scores,
                           int ignore_evict_strategy, uint8_t* results);
void hkvo_find_or_insert(hkvo_table* t, size_t n, const uint64_t* keys,
                         void* values, const uint64_t* scores,
                         int ignore_evict_strategy, uint8_t* results);
size_t hkvo_insert_and_evict(hkvo_table* t, size_t n, const uint64_t* keys,
                             const void* values, const uint64_t* scores,
                             uint64_t* ev_keys, void* ev_values,
                             uint64_t* ev_scores, int ignore_evict_strategy,
                             uint8_t* results);
void hkvo_accum_or_assign(hkvo_table* t, size_t n, const uint64_t* keys,
                          const void* values, const uint8_t* accum_or_assigns,
                          const uint64_t* scores, int ignore_evict_strategy,
                          uint8_t* results);
void hkvo_assign_scores(hkvo_table* t, size_t n, const uint64_t* keys,
                        const uint64_t* scores);
void hkvo_erase(hkvo_table* t, size_t n, const uint64_t* keys);
void hkvo_clear(hkvo_table* t);
size_t hkvo_export_batch(hkvo_table* t, size_t n, size_t offset,
                         uint64_t* keys, void* values, uint64_t* scores);
void hkvo_reserve(hkvo_table* t, uint64_t new_capacity);

/* Raw state, slot-major, for importing a GPU table and diffing slot by slot.
 * Any pointer may be NULL. */
void hkvo_get_state(const hkvo_table* t, uint64_t* keys, uint64_t* scores,
                    uint8_t* digests, int32_t* sizes, void* values);
void hkvo_set_state(hkvo_table* t, const uint64_t* keys, const uint64_t* scores,
                    const uint8_t* digests, const int32_t* sizes,
                    const void* values);

#ifdef __cplusplus
}
#endif
#endif /* HKV_ORACLE_H_ */
