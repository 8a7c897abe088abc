/*
 * hkv_b200.h -- C ABI of the B200 HierarchicalKV hash table.
 *
 * This is the drop-in boundary for the reference's HashTable<K,V,S,Strategy>
 * (yangzhen92/HierarchicalKV-ascend, include/hkv_hashtable.h). Every entry
 * point takes plain pointers and sizes; device pointers are CUDA device (or
 * mapped/managed) memory, `stream` is a cudaStream_t passed as void*. The C++
 * mirror in include/hkv_hashtable.h, the Python binding and any cgo/JNI/ctypes
 * caller bind exactly these symbols.
 *
 * Every function returns an hkv_status. On failure hkv_last_error() gives the
 * message of the calling thread's last error. Status codes mirror the
 * reference's exceptions: HKV_ERR_INVALID for HkvException (HKV_CHECK,
 * debug.h:53-74), HKV_ERR_CUDA for NpuException (NPU_CHECK, debug.h:30-51),
 * HKV_ERR_RUNTIME for std::runtime_error.
 *
 * Key type: 64-bit integers (uint64 or int64, same bit patterns). The four
 * reserved keys 0xFFFFFFFFFFFFFFFC..0xFFFFFFFFFFFFFFFF are ignored by every
 * operation (reference types.h:63-70, :153-156). Score type: uint64.
 * Values: rows of `dim` elements of `value_type`.
 */
#ifndef HKV_B200_H_
#define HKV_B200_H_

#include <stddef.h>
#include <stdint.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef enum {
  HKV_OK = 0,
  HKV_ERR_INVALID = 1,     /* bad argument or configuration (HkvException) */
  HKV_ERR_CUDA = 2,        /* CUDA runtime failure (NpuException) */
  HKV_ERR_TIMEOUT = 3,     /* a device lock wait ran out (device error word) */
  HKV_ERR_UNSUPPORTED = 4, /* valid in the reference, not supported here */
  HKV_ERR_RUNTIME = 5      /* std::runtime_error in the reference */
} hkv_status;

/* EvictStrategy::EvictStrategyEnum, hkv_hashtable.h:111-119. */
typedef enum {
  HKV_LRU = 0,
  HKV_LFU = 1,
  HKV_EPOCH_LRU = 2,
  HKV_EPOCH_LFU = 3,
  HKV_CUSTOMIZED = 4
} hkv_evict_strategy;

typedef enum { HKV_KEY_U64 = 0, HKV_KEY_I64 = 1 } hkv_key_type;

typedef enum {
  HKV_VALUE_F32 = 0,
  HKV_VALUE_F16 = 1,
  HKV_VALUE_BF16 = 2,
  HKV_VALUE_F64 = 3,
  HKV_VALUE_U32 = 4,
  HKV_VALUE_U16 = 5,
  HKV_VALUE_I8 = 6,
  HKV_VALUE_U64 = 7
} hkv_value_type;

/* HashTableOptions, hashtable_options.h:534-566 (field for field; the pool
 * options of MemoryPoolOptions are not needed by this build). */
typedef struct {
  uint64_t init_capacity;
  uint64_t max_capacity;
  uint64_t max_hbm_for_vectors; /* bytes of HBM for values; the rest goes to
                                   mapped pinned host memory */
  uint64_t max_bucket_size;     /* 128 */
  uint64_t dim;
  float max_load_factor;        /* 0.5 */
  int block_size;               /* accepted, unused */
  int io_block_size;            /* accepted, unused */
  int device_id;                /* -1: current device */
  int io_by_cpu;                /* must be 0 */
  int use_constant_memory;      /* reserved */
  int reserved_key_start_bit;   /* 0 only */
  uint64_t num_of_buckets_per_alloc;
  int api_lock;                 /* 1: calls from several host threads
                                   serialise as in the reference (readers
                                   share, updaters share, inserts and
                                   erases alone); each call then also
                                   synchronises its stream */
} hkv_options;

typedef struct hkv_table hkv_table;

/* Fills `o` with the reference's defaults (hashtable_options.h:535-562). */
void hkv_options_init(hkv_options* o);

/* Message of the calling thread's last failed call. */
const char* hkv_last_error(void);

/* HashTable::HashTable + init(options), hkv_hashtable.h:938-1042. */
int hkv_table_create(const hkv_options* options, int key_type, int value_type,
                     int evict_strategy, hkv_table** out);

/* ---- caller-provided allocator ----------------------------------------------
 * init(options, BaseAllocator*) (hkv_hashtable.h:962-978) takes every
 * allocation of the table from the caller's allocator, whose interface is
 * allocator.h:27-158: alloc / alloc_async / free / free_async of a
 * MemoryType (Device = HBM, Pinned = page-locked host memory, Host). Here the
 * allocator is a struct of callbacks on the caller's `user` object; each
 * returns 0 on success and non-zero on failure (the call then fails with
 * HKV_ERR_CUDA). The table takes from it:
 *  - Device: its bucket arrays (keys, scores, digests, sizes), the value
 *    slices that fit max_hbm_for_vectors, the slice table and its counters,
 *    at creation and at each doubling (reserve, auto-grow), the old arrays
 *    freed after the rehash;
 *  - Pinned, pinned_flags = cudaHostAllocMapped | cudaHostAllocPortable (3):
 *    the value slices beyond max_hbm_for_vectors; the memory must be mapped
 *    into the device address space (cudaHostGetDevicePointer must accept it);
 *  - Pinned, pinned_flags = 0: host staging for size() and save / load;
 *  - Device through alloc_async / free_async on the call's stream: per-call
 *    scratch (the duplicate-key merge, rehash rows, save / load chunks). When
 *    alloc_async / free_async are NULL, alloc is used, and free after the
 *    stream has drained.
 * Everything is freed through the same allocator by hkv_table_destroy. The
 * allocator must outlive the table. */
typedef enum {
  HKV_MEMORY_DEVICE = 0,
  HKV_MEMORY_PINNED = 1,
  HKV_MEMORY_HOST = 2
} hkv_memory_type;

typedef struct {
  void* user;
  int (*alloc)(void* user, int memory_type, void** ptr, size_t size,
               unsigned int pinned_flags);
  int (*alloc_async)(void* user, int memory_type, void** ptr, size_t size,
                     void* stream);
  int (*free)(void* user, int memory_type, void* ptr);
  int (*free_async)(void* user, int memory_type, void* ptr, void* stream);
} hkv_allocator;

/* HashTable::init(options, allocator), hkv_hashtable.h:962-978: as
 * hkv_table_create, with every allocation from `allocator` (copied; NULL
 * means the CUDA runtime, as hkv_table_create). */
int hkv_table_create_with_allocator(const hkv_options* options, int key_type,
                                    int value_type, int evict_strategy,
                                    const hkv_allocator* allocator,
                                    hkv_table** out);

/* HashTable::~HashTable, hkv_hashtable.h:944-960. */
int hkv_table_destroy(hkv_table* table);

/* set_max_capacity, hkv_hashtable.h:2955-2977: a power of two (else
 * HKV_ERR_INVALID) below the current capacity is ignored; otherwise it
 * becomes the capacity reserve and auto-grow may reach, and the table may
 * grow again. */
int hkv_set_max_capacity(hkv_table* table, size_t new_max_capacity);

/* insert_or_assign, hkv_hashtable.h:1077-1215. */
int hkv_insert_or_assign(hkv_table* table, size_t n, const void* keys,
                         const void* values, const uint64_t* scores,
                         void* stream, bool unique_key,
                         bool ignore_evict_strategy);

/* insert_and_evict (device counter), hkv_hashtable.h:1260-1310. The caller
 * zeroes *d_evicted_counter before the call. */
int hkv_insert_and_evict(hkv_table* table, size_t n, const void* keys,
                         const void* values, const uint64_t* scores,
                         void* evicted_keys, void* evicted_values,
                         uint64_t* evicted_scores, uint64_t* d_evicted_counter,
                         void* stream, bool unique_key,
                         bool ignore_evict_strategy);

/* insert_and_evict returning the count (synchronises the stream),
 * hkv_hashtable.h:1368-1396. */
int hkv_insert_and_evict_count(hkv_table* table, size_t n, const void* keys,
                               const void* values, const uint64_t* scores,
                               void* evicted_keys, void* evicted_values,
                               uint64_t* evicted_scores, void* stream,
                               bool unique_key, bool ignore_evict_strategy,
                               size_t* h_evicted_count);

/* accum_or_assign, hkv_hashtable.h:1438-1507. */
int hkv_accum_or_assign(hkv_table* table, size_t n, const void* keys,
                        const void* value_or_deltas,
                        const bool* accum_or_assigns, const uint64_t* scores,
                        void* stream, bool ignore_evict_strategy);

/* find_or_insert, hkv_hashtable.h:1526-1632. */
int hkv_find_or_insert(hkv_table* table, size_t n, const void* keys,
                       void* values, const uint64_t* scores, void* stream,
                       bool unique_key, bool ignore_evict_strategy);

/* assign_scores (and its alias assign), hkv_hashtable.h:1943-1995. */
int hkv_assign_scores(hkv_table* table, size_t n, const void* keys,
                      const uint64_t* scores, void* stream, bool unique_key);

/* find, hkv_hashtable.h:2113-2152. Misses leave values/scores untouched. */
int hkv_find(hkv_table* table, size_t n, const void* keys, void* values,
             bool* founds, uint64_t* scores, void* stream);

/* find* (pointer-returning find), hkv_hashtable.h:2244-2264: values[i] is
 * the device address of key i's value row in the table (a mapped host
 * address for rows in host memory), NULL for a missed or reserved key;
 * founds and scores (nullable) as in find. The addresses stay valid until
 * the next call that can move or evict rows (insert-like calls, erase,
 * clear, reserve). */
int hkv_find_ptr(hkv_table* table, size_t n, const void* keys, void** values,
                 bool* founds, uint64_t* scores, void* stream);

/* find_or_insert* (pointer-returning), hkv_hashtable.h:1658-1727: finds or
 * inserts each key as find_or_insert does (same placement, eviction and
 * score rules) but copies no value: values[i] is the address of the key's
 * row (for an inserted key the row still holds the previous occupant's
 * bytes; the caller writes it), NULL for a refused or reserved key;
 * founds[i] tells whether the key was there before. As in the reference, a
 * later key of the same batch may evict a key placed earlier in it and then
 * owns that row. With repeated keys
 * (unique_key = false) every occurrence gets the same address and only the
 * first can report a new key. With locked_key_ptrs (unique_key = true only,
 * HKV_ERR_UNSUPPORTED otherwise) every placed or found key stays locked for
 * the caller and locked_key_ptrs[i] is the address of its key word (NULL
 * where values[i] is NULL); release them with hkv_unlock_keys. */
int hkv_find_or_insert_ptr(hkv_table* table, size_t n, const void* keys,
                           void** values, bool* founds, const uint64_t* scores,
                           void* stream, bool unique_key,
                           bool ignore_evict_strategy, void** locked_key_ptrs);

/* lock_keys, hkv_hashtable.h:1744-1768: each present key is locked, its
 * score set by the hit rule (scores as in find_or_insert; NULL for Lru),
 * and the address of its key word written to locked_key_ptrs[i]; absent or
 * reserved keys get NULL and succeededs[i] = false. A locked key is not
 * found by find / contains / assign_scores / erase / accum_or_assign (its
 * key word holds a lock marker, as in the reference) and its slot is never
 * chosen as an eviction victim. Deviations from the reference: the marker is
 * 0xFFFFFFFFFFFFFFFC (the fourth reserved key; the reference writes
 * LOCKED_KEY, 0xFFFFFFFFFFFFFFFD), and the table cannot grow (reserve,
 * auto-grow) while keys are locked: HKV_ERR_RUNTIME. As in the reference, an
 * insert-like call of a key that is locked does not see it and places a
 * second copy. */
int hkv_lock_keys(hkv_table* table, size_t n, const void* keys, void** locked_key_ptrs,
                  bool* succeededs, void* stream, const uint64_t* scores);

/* unlock_keys, hkv_hashtable.h:1788-1806: puts keys[i] back into the key
 * word at locked_key_ptrs[i] if that word is still locked by the caller;
 * succeededs[i] tells whether it was (false for NULL, for an address outside
 * this table's keys, or for a word that is not locked). While keys may be
 * locked, insert-like calls run kernels that pass locked slots by; to learn
 * when none is left, this call recounts the locks and so synchronises the
 * stream. */
int hkv_unlock_keys(hkv_table* table, size_t n, void** locked_key_ptrs, const void* keys,
                    bool* succeededs, void* stream);

/* contains, hkv_hashtable.h:2330-2348. */
int hkv_contains(hkv_table* table, size_t n, const void* keys, bool* founds,
                 void* stream);

/* erase, hkv_hashtable.h:2358-2376. */
int hkv_erase(hkv_table* table, size_t n, const void* keys, void* stream);

/* clear, hkv_hashtable.h:2482-2493. */
int hkv_clear(hkv_table* table, void* stream);

/* export_batch (device counter, set not accumulated), hkv_hashtable.h
 * :2519-2549. */
int hkv_export_batch(hkv_table* table, size_t n, size_t offset,
                     uint64_t* d_counter, void* keys, void* values,
                     uint64_t* scores, void* stream);

/* export_batch returning the count (synchronises), hkv_hashtable.h
 * :2557-2577. */
int hkv_export_batch_count(hkv_table* table, size_t n, size_t offset,
                           void* keys, void* values, uint64_t* scores,
                           void* stream, size_t* h_count);

/* size / empty / capacity / load_factor / dim / max_bucket_size /
 * bucket_count / is_pure_hbm_mode, hkv_hashtable.h:2784-2819, :2849, :2945,
 * :2984-3008. size and load_factor synchronise the stream. */
int hkv_size(hkv_table* table, void* stream, size_t* out);
int hkv_capacity(hkv_table* table, size_t* out);
int hkv_load_factor(hkv_table* table, void* stream, float* out);
int hkv_dim(hkv_table* table, size_t* out);
int hkv_max_bucket_size(hkv_table* table, size_t* out);
int hkv_bucket_count(hkv_table* table, size_t* out);
int hkv_is_pure_hbm_mode(hkv_table* table, bool* out);

/* reserve, hkv_hashtable.h:2873-2935. */
int hkv_reserve(hkv_table* table, size_t new_capacity, void* stream);

/* set_global_epoch, hkv_hashtable.h:3197. */
int hkv_set_global_epoch(hkv_table* table, uint64_t epoch);

/* ---- slot scans with predicates ---------------------------------------------
 * The reference's erase_if / export_batch_if / size_if take a device
 * functor as a template argument (hkv_hashtable.h:2409-2476, :2623-2731,
 * :2829-2846) and for_each an execution functor (:2754-2775). C++ callers
 * compiled with nvcc get those member templates from include/hkv_scan.cuh
 * through include/hkv_hashtable.h. Other callers pass this built-in
 * predicate: a live slot matches when (key & key_mask) == key_value and
 * score <cmp> threshold. It covers the predicates of the reference's tests
 * (score thresholds, key bit patterns, both). */
typedef enum {
  HKV_CMP_ANY = 0,
  HKV_CMP_LT = 1,
  HKV_CMP_LE = 2,
  HKV_CMP_GT = 3,
  HKV_CMP_GE = 4,
  HKV_CMP_EQ = 5
} hkv_score_cmp;

typedef struct {
  uint64_t key_mask;
  uint64_t key_value;
  int score_cmp; /* hkv_score_cmp */
  uint64_t threshold;
} hkv_predicate;

/* erase_if: matching slots become tombstones; the count erased returns on
 * the host (synchronises `stream`). */
int hkv_erase_if(hkv_table* table, const hkv_predicate* pred, void* stream,
                 size_t* out_count);
/* export_batch_if: matching slots of [offset, offset + n) compacted to the
 * outputs (order not specified), *d_counter set to their number. */
int hkv_export_batch_if(hkv_table* table, const hkv_predicate* pred, size_t n,
                        size_t offset, uint64_t* d_counter, void* keys,
                        void* values, uint64_t* scores, void* stream);
/* size_if: number of matching slots into *d_counter (device). */
int hkv_size_if(hkv_table* table, const hkv_predicate* pred,
                uint64_t* d_counter, void* stream);

/* No reference counterpart: the table's raw device arrays, for the scan
 * kernels of include/hkv_scan.cuh. Slot g lives in bucket g / bucket_size;
 * its value row is slices[b >> slice_shift] + ((b & (2^slice_shift - 1)) *
 * bucket_size + g % bucket_size) * value_bytes. Valid until the next call
 * that can reallocate the table (reserve, auto-grow). */
typedef struct {
  uint64_t* keys;
  uint64_t* scores;
  uint8_t* digests;
  int32_t* sizes;   /* per bucket: live slots in the low 16 bits (keys held
                      * by hkv_lock_keys are counted from bit 16) */
  uint8_t** slices; /* device array of slice base addresses */
  uint64_t capacity;
  uint64_t num_buckets;
  uint32_t bucket_size;
  uint32_t slice_shift;
  uint32_t value_bytes;
  uint32_t dim;
  uint8_t reclaim_digest;
} hkv_table_view;
int hkv_table_get_view(hkv_table* table, hkv_table_view* out);

/* ---- save / load, hkv_hashtable.h:3021-3195 --------------------------------
 * The reference takes a BaseKVFile (types.h:291-334) whose read/write move
 * n (key, vector, score) tuples between host buffers and a file. Here that
 * object is a pair of callbacks on HOST buffers, returning the number of
 * tuples moved. Both functions synchronise `stream`. */
typedef size_t (*hkv_kv_write_fn)(void* user, size_t n, size_t dim,
                                  const void* keys, const void* values,
                                  const uint64_t* scores);
typedef size_t (*hkv_kv_read_fn)(void* user, size_t n, size_t dim, void* keys,
                                 void* values, uint64_t* scores);

/* save, hkv_hashtable.h:3021-3112: walks the slots in chunks of
 * max_workspace_size / (sizeof key + sizeof score + dim * sizeof value)
 * tuples (the export of each chunk), hands each chunk to `write`. */
int hkv_save(hkv_table* table, hkv_kv_write_fn write, void* user,
             size_t max_workspace_size, void* stream, size_t* out_count);

/* load, hkv_hashtable.h:3125-3195: reads chunks of the same size with `read`
 * until it returns 0 and inserts each with insert_or_assign(unique_key =
 * true, ignore_evict_strategy = true) after setting the global epoch to
 * IGNORED_GLOBAL_EPOCH (which it stays at, as in the reference). */
int hkv_load(hkv_table* table, hkv_kv_read_fn read, void* user,
             size_t max_workspace_size, void* stream, size_t* out_count);

/* save / load through the reference's LocalKVFile format (types.h:349-464):
 * three files of raw keys, raw value rows and raw uint64 scores, written
 * ("wb") or read ("rb") in the same order. */
int hkv_save_files(hkv_table* table, const char* keys_path,
                   const char* values_path, const char* scores_path,
                   size_t max_workspace_size, void* stream, size_t* out_count);
int hkv_load_files(hkv_table* table, const char* keys_path,
                   const char* values_path, const char* scores_path,
                   size_t max_workspace_size, void* stream, size_t* out_count);

/* No reference counterpart. find_or_insert for a batch that may repeat
 * keys (as with unique_key = false) that allocates no device memory, for
 * callers that cannot call cudaMalloc while serving, such as a service whose
 * GPU memory is all handed to a fixed arena at start-up. The duplicate-key
 * merge uses one file-scope device array of 2 MiB instead of per-call
 * scratch, so a call takes at most 16384 keys; larger calls fail with
 * HKV_ERR_INVALID. The table
 * never grows in this call: a batch that would trigger auto-grow fails with
 * HKV_ERR_RUNTIME (call hkv_reserve first); to tell, a call on a table that
 * has not reached its maximum capacity reads the sampled bucket sizes back
 * and so synchronises `stream`, as the reference's auto-grow check does. The
 * first call on a device looks up the array's device address, so make that
 * first call before any stream capture; the address is kept for the life of
 * the process, so after cudaDeviceReset on that device this entry point must
 * not be called again. Every call in the process shares the array and finds the last
 * call's contents in it (what must start empty is cleared at the start of
 * each call); calls that overlap on the GPU race on it and must be ordered
 * by the caller. Results are those of hkv_find_or_insert with
 * unique_key = false. */
int hkv_find_or_insert_noalloc(hkv_table* table, size_t n, const void* keys,
                               void* values, const uint64_t* scores,
                               void* stream, bool ignore_evict_strategy);

/* No reference counterpart: synchronises `stream` and reports a device lock
 * wait that ran out during earlier calls (HKV_ERR_TIMEOUT), then clears it.
 * The reference's device waits have no bound (find_utils.h:169-173). */
int hkv_check_device_error(hkv_table* table, void* stream);

/* No reference counterpart (instrumentation): number of kernels this library
 * has enqueued in this process so far, on every table and stream. */
int hkv_kernel_launches(uint64_t* out);

/* No reference counterpart (test support): copies the raw slot state to /
 * from HOST buffers, slot-major (capacity entries; sizes has bucket_count
 * entries; values capacity*dim elements). Any pointer may be NULL. */
int hkv_debug_get_state(hkv_table* table, uint64_t* keys, uint64_t* scores,
                        uint8_t* digests, int32_t* sizes, void* values);
int hkv_debug_set_state(hkv_table* table, const uint64_t* keys,
                        const uint64_t* scores, const uint8_t* digests,
                        const int32_t* sizes, const void* values);

/* ---- sharded table (no reference counterpart: the reference is one device)
 * One table shard per GPU; keys are routed to shard owner(key) =
 * (Murmur3(key) >> 40) % world_size. Two transports move the keys and rows:
 *  - peer memory (HKV_TRANSPORT_PEER): each rank maps the others' receive
 *    windows over NVLink (CUDA IPC); requesters write keys straight into the
 *    owner's window, owners write results straight back, device flags order
 *    the steps, no host synchronisation. Used when max_batch > 0, the shards
 *    never grow (init_capacity * 2 > max_capacity) and every rank could map
 *    every peer; each rank's window holds world_size * max_batch entries.
 *  - NCCL grouped send/recv (HKV_TRANSPORT_NCCL) otherwise, with one host
 *    synchronisation per call to size the receive buffers. ---------------- */
typedef struct hkv_sharded hkv_sharded;

typedef enum { HKV_TRANSPORT_NCCL = 0, HKV_TRANSPORT_PEER = 1 } hkv_transport;

/* NCCL unique id (128 bytes) for rank 0 to broadcast to the others. */
int hkv_nccl_unique_id(uint8_t out[128]);

/* Collective. max_batch: the largest n any rank passes to one call of the
 * peer transport (every rank must pass the same value; 0 selects NCCL). */
int hkv_sharded_create(const hkv_options* local_options, int key_type,
                       int value_type, int evict_strategy,
                       const uint8_t nccl_id[128], int rank, int world_size,
                       size_t max_batch, hkv_sharded** out);
int hkv_sharded_destroy(hkv_sharded* s);
hkv_table* hkv_sharded_local(hkv_sharded* s);
/* The transport in use (hkv_transport). */
int hkv_sharded_transport(hkv_sharded* s, int* out);

/* Collective: every rank calls with its own batch (sizes may differ; with
 * the peer transport each n must be at most max_batch). Semantics per key
 * are those of the local op on the owner shard. unique_key = true promises
 * that a rank's batch holds no repeated key (as the reference's unique_key);
 * with false, repeated keys are merged as the local unique_key = false
 * calls do. The same key sent by several ranks in one call is applied in
 * rank order. A peer wait that runs out (a rank that never
 * joins the call) is reported by hkv_check_device_error on the local table
 * as HKV_ERR_TIMEOUT; the table is then in an undefined state. */
int hkv_sharded_find_or_insert(hkv_sharded* s, size_t n, const void* keys,
                               void* values, const uint64_t* scores,
                               void* stream, bool unique_key);
int hkv_sharded_find(hkv_sharded* s, size_t n, const void* keys, void* values,
                     bool* founds, uint64_t* scores, void* stream);
int hkv_sharded_insert_or_assign(hkv_sharded* s, size_t n, const void* keys,
                                 const void* values, const uint64_t* scores,
                                 void* stream, bool unique_key);
/* Collective sum of the shard sizes. */
int hkv_sharded_size(hkv_sharded* s, void* stream, size_t* out);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif /* HKV_B200_H_ */
