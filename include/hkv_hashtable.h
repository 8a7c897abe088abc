/*
 * hkv_hashtable.h -- C++ drop-in for the reference's HashTable API
 * (yangzhen92/HierarchicalKV-ascend, include/hkv_hashtable.h), implemented
 * over the C ABI of include/hkv_b200.h (libhkv_b200.so).
 *
 * Same class template, method names, argument order and defaults as the
 * reference for the hot path: init, insert_or_assign, insert_and_evict (both
 * overloads), accum_or_assign, find_or_insert, assign_scores / assign, find,
 * contains, erase, clear, export_batch (both overloads), size, empty,
 * capacity, load_factor, reserve, dim, max_bucket_size, bucket_count,
 * is_pure_hbm_mode, set_global_epoch. Streams are cudaStream_t where the
 * reference takes aclrtStream. Errors throw HkvException (reference HKV_CHECK,
 * debug.h:53-74), CudaException (reference NpuException, debug.h:30-51) or
 * std::runtime_error, as the reference does.
 *
 * `namespace npu::hkv` is an alias of `hkv_b200`, so code written against the
 * reference compiles unchanged apart from the stream type.
 */
#ifndef HKV_B200_HASHTABLE_H_
#define HKV_B200_HASHTABLE_H_

#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <type_traits>

#include "hkv_b200.h"
#ifdef __CUDACC__
#include "hkv_scan.cuh"
#endif

namespace hkv_b200 {

/* EvictStrategy, reference hkv_hashtable.h:111-119. */
struct EvictStrategy {
  enum EvictStrategyEnum {
    kLru = HKV_LRU,
    kLfu = HKV_LFU,
    kEpochLru = HKV_EPOCH_LRU,
    kEpochLfu = HKV_EPOCH_LFU,
    kCustomized = HKV_CUSTOMIZED,
  };
};

/* HashTableOptions, reference hashtable_options.h:534-566 (the memory-pool
 * options are not needed: scratch is stream-ordered). */
struct HashTableOptions {
  size_t init_capacity = 0;
  size_t max_capacity = 0;
  size_t max_hbm_for_vectors = 0;
  size_t max_bucket_size = 128;
  size_t dim = 64;
  float max_load_factor = 0.5f;
  int block_size = 128;
  int io_block_size = 1024;
  int device_id = -1;
  bool io_by_cpu = false;
  bool use_constant_memory = false;
  int reserved_key_start_bit = 0;
  size_t num_of_buckets_per_alloc = 1;
  bool api_lock = false;
};

constexpr uint64_t IGNORED_GLOBAL_EPOCH = UINT64_C(0xFFFFFFFFFFFFFFFF);

class HkvException : public std::runtime_error {
 public:
  explicit HkvException(const std::string& m) : std::runtime_error(m) {}
};
class CudaException : public std::runtime_error {
 public:
  explicit CudaException(const std::string& m) : std::runtime_error(m) {}
};
class HkvTimeout : public std::runtime_error {
 public:
  explicit HkvTimeout(const std::string& m) : std::runtime_error(m) {}
};

namespace detail {
inline void check(int status) {
  if (status == HKV_OK) return;
  const std::string m = hkv_last_error();
  switch (status) {
    case HKV_ERR_INVALID:
      throw HkvException(m);
    case HKV_ERR_CUDA:
      throw CudaException(m);
    case HKV_ERR_TIMEOUT:
      throw HkvTimeout(m);
    default:
      throw std::runtime_error(m);
  }
}
inline void cuda(cudaError_t e) {
  if (e != cudaSuccess) throw CudaException(cudaGetErrorString(e));
}
template <class V>
constexpr int value_code() {
  return std::is_same<V, float>::value      ? HKV_VALUE_F32
         : std::is_same<V, double>::value   ? HKV_VALUE_F64
         : std::is_same<V, uint32_t>::value ? HKV_VALUE_U32
         : std::is_same<V, uint64_t>::value ? HKV_VALUE_U64
         : std::is_same<V, int8_t>::value   ? HKV_VALUE_I8
         : (sizeof(V) == 2)                 ? HKV_VALUE_F16
                                            : -1;
}
inline void* st(cudaStream_t s) { return reinterpret_cast<void*>(s); }
}  // namespace detail

/* MemoryType and BaseAllocator, reference allocator.h:27-84: the interface
 * of a caller's allocator, from which HashTable::init(options, allocator)
 * takes every allocation of the table (see hkv_allocator in hkv_b200.h for
 * which memory comes from where). Pinned memory given for value rows must be
 * mapped into the device address space (pinned_flags carries
 * cudaHostAllocMapped). The allocator must outlive the table. */
enum MemoryType {
  Device,  // HBM
  Pinned,  // page-locked host memory
  Host,    // host memory
};

class BaseAllocator {
 public:
  BaseAllocator(const BaseAllocator&) = delete;
  BaseAllocator(BaseAllocator&&) = delete;
  BaseAllocator& operator=(const BaseAllocator&) = delete;
  BaseAllocator& operator=(BaseAllocator&&) = delete;
  BaseAllocator() = default;
  virtual ~BaseAllocator() = default;

  virtual void alloc(const MemoryType type, void** ptr, size_t size,
                     unsigned int pinned_flags = 0) = 0;
  virtual void alloc_async(const MemoryType type, void** ptr, size_t size,
                           cudaStream_t stream) = 0;
  virtual void free(const MemoryType type, void* ptr) = 0;
  virtual void free_async(const MemoryType type, void* ptr, cudaStream_t stream) = 0;

  template <typename T>
  void alloc(const MemoryType type, T** ptr, size_t size, unsigned int pinned_flags = 0) {
    void* p = nullptr;
    alloc(type, &p, size, pinned_flags);
    *ptr = static_cast<T*>(p);
  }
  template <typename T>
  void alloc_async(const MemoryType type, T** ptr, size_t size, cudaStream_t stream) {
    void* p = nullptr;
    alloc_async(type, &p, size, stream);
    *ptr = static_cast<T*>(p);
  }
};

/* DefaultAllocator, reference allocator.h:86-158, on the CUDA runtime. */
class DefaultAllocator : public virtual BaseAllocator {
 public:
  using BaseAllocator::alloc;
  using BaseAllocator::alloc_async;
  void alloc(const MemoryType type, void** ptr, size_t size,
             unsigned int pinned_flags = 0) override {
    switch (type) {
      case Device:
        detail::cuda(cudaMalloc(ptr, size));
        break;
      case Pinned:
        detail::cuda(cudaHostAlloc(ptr, size, pinned_flags));
        break;
      case Host:
        *ptr = std::malloc(size);
        break;
    }
  }
  void alloc_async(const MemoryType type, void** ptr, size_t size,
                   cudaStream_t stream) override {
    if (type != Device)
      throw HkvException("[DefaultAllocator] alloc_async is only support for MemoryType::Device!");
    detail::cuda(cudaMallocAsync(ptr, size, stream));
  }
  void free(const MemoryType type, void* ptr) override {
    if (ptr == nullptr) return;
    switch (type) {
      case Device:
        detail::cuda(cudaFree(ptr));
        break;
      case Pinned:
        detail::cuda(cudaFreeHost(ptr));
        break;
      case Host:
        std::free(ptr);
        break;
    }
  }
  void free_async(const MemoryType type, void* ptr, cudaStream_t stream) override {
    if (ptr == nullptr) return;
    if (type != Device)
      throw HkvException("[DefaultAllocator] free_async is only support for MemoryType::Device!");
    detail::cuda(cudaFreeAsync(ptr, stream));
  }
};

namespace detail {
/* hkv_allocator callbacks over a BaseAllocator: exceptions stay on this side
 * of the C ABI and become a non-zero status. */
inline int alloc_cb(void* u, int type, void** ptr, size_t size, unsigned int flags) {
  try {
    static_cast<BaseAllocator*>(u)->alloc(static_cast<MemoryType>(type), ptr, size, flags);
    return 0;
  } catch (...) {
    return 1;
  }
}
inline int alloc_async_cb(void* u, int type, void** ptr, size_t size, void* stream) {
  try {
    static_cast<BaseAllocator*>(u)->alloc_async(static_cast<MemoryType>(type), ptr, size,
                                                static_cast<cudaStream_t>(stream));
    return 0;
  } catch (...) {
    return 1;
  }
}
inline int free_cb(void* u, int type, void* ptr) {
  try {
    static_cast<BaseAllocator*>(u)->free(static_cast<MemoryType>(type), ptr);
    return 0;
  } catch (...) {
    return 1;
  }
}
inline int free_async_cb(void* u, int type, void* ptr, void* stream) {
  try {
    static_cast<BaseAllocator*>(u)->free_async(static_cast<MemoryType>(type), ptr,
                                               static_cast<cudaStream_t>(stream));
    return 0;
  } catch (...) {
    return 1;
  }
}
}  // namespace detail

/* BaseKVFile / LocalKVFile, reference types.h:291-464: save() and load()
 * move (key, vector, score) tuples between the table and a file through
 * these. LocalKVFile keeps the reference's on-disk format: three files of
 * raw keys, raw vectors and raw scores in the same order. */
template <class K, class V, class S>
class BaseKVFile {
 public:
  virtual ~BaseKVFile() {}
  virtual size_t read(const size_t n, const size_t dim, K* keys, V* vectors,
                      S* scores) = 0;
  virtual size_t write(const size_t n, const size_t dim, const K* keys,
                       const V* vectors, const S* scores) = 0;
};

template <class K, class V, class S>
class LocalKVFile : public BaseKVFile<K, V, S> {
 public:
  LocalKVFile() = default;
  ~LocalKVFile() { close(); }
  bool open(const std::string& keys_path, const std::string& values_path,
            const std::string& scores_path, const char* mode) {
    close();
    fp_[0] = std::fopen(keys_path.c_str(), mode);
    fp_[1] = fp_[0] ? std::fopen(values_path.c_str(), mode) : nullptr;
    fp_[2] = fp_[1] ? std::fopen(scores_path.c_str(), mode) : nullptr;
    if (!fp_[2]) close();
    return fp_[2] != nullptr;
  }
  void close() noexcept {
    for (auto& f : fp_)
      if (f) {
        std::fclose(f);
        f = nullptr;
      }
  }
  size_t read(const size_t n, const size_t dim, K* keys, V* vectors,
              S* scores) override {
    const size_t a = std::fread(keys, sizeof(K), n, fp_[0]);
    const size_t b = std::fread(vectors, sizeof(V) * dim, n, fp_[1]);
    const size_t c = std::fread(scores, sizeof(S), n, fp_[2]);
    return (a == b && a == c) ? a : 0;
  }
  size_t write(const size_t n, const size_t dim, const K* keys,
               const V* vectors, const S* scores) override {
    const size_t a = std::fwrite(keys, sizeof(K), n, fp_[0]);
    const size_t b = std::fwrite(vectors, sizeof(V) * dim, n, fp_[1]);
    const size_t c = std::fwrite(scores, sizeof(S), n, fp_[2]);
    return (a == b && a == c) ? a : 0;
  }

 private:
  std::FILE* fp_[3] = {nullptr, nullptr, nullptr};
};

/* HashTableBase<K, V, S>, reference hkv_hashtable.h:171-871: the abstract
 * interface a caller may hold the table through. HashTable implements every
 * method; assign with values, assign_values, find with missed keys and
 * find_and_update are outside this build's scope and throw HkvException. */
template <typename K, typename V, typename S = uint64_t>
class HashTableBase {
 public:
  using size_type = size_t;
  using key_type = K;
  using value_type = V;
  using score_type = S;
  using allocator_type = BaseAllocator;

  virtual ~HashTableBase() {}
  virtual void init(const HashTableOptions& options, allocator_type* allocator = nullptr) = 0;
  virtual void insert_or_assign(const size_type n, const key_type* keys,
                                const value_type* values, const score_type* scores = nullptr,
                                cudaStream_t stream = 0, bool unique_key = true,
                                bool ignore_evict_strategy = false) = 0;
  virtual void insert_and_evict(const size_type n, const key_type* keys,
                                const value_type* values, const score_type* scores,
                                key_type* evicted_keys, value_type* evicted_values,
                                score_type* evicted_scores, size_type* d_evicted_counter,
                                cudaStream_t stream = 0, bool unique_key = true,
                                bool ignore_evict_strategy = false) = 0;
  virtual size_type insert_and_evict(const size_type n, const key_type* keys,
                                     const value_type* values, const score_type* scores,
                                     key_type* evicted_keys, value_type* evicted_values,
                                     score_type* evicted_scores, cudaStream_t stream = 0,
                                     bool unique_key = true,
                                     bool ignore_evict_strategy = false) = 0;
  virtual void accum_or_assign(const size_type n, const key_type* keys,
                               const value_type* value_or_deltas, const bool* accum_or_assigns,
                               const score_type* scores = nullptr, cudaStream_t stream = 0,
                               bool ignore_evict_strategy = false) = 0;
  virtual void find_or_insert(const size_type n, const key_type* keys, value_type* values,
                              score_type* scores = nullptr, cudaStream_t stream = 0,
                              bool unique_key = true, bool ignore_evict_strategy = false) = 0;
  virtual void find_or_insert(const size_type n, const key_type* keys, value_type** values,
                              bool* founds, score_type* scores = nullptr,
                              cudaStream_t stream = 0, bool unique_key = true,
                              bool ignore_evict_strategy = false,
                              key_type** locked_key_ptrs = nullptr) = 0;
  virtual void lock_keys(const size_type n, key_type const* keys, key_type** locked_key_ptrs,
                         bool* succeededs = nullptr, cudaStream_t stream = 0,
                         score_type const* scores = nullptr) = 0;
  virtual void unlock_keys(const size_type n, key_type** locked_key_ptrs,
                           const key_type* keys, bool* succeededs = nullptr,
                           cudaStream_t stream = 0) = 0;
  virtual void assign(const size_type n, const key_type* keys, const value_type* values,
                      const score_type* scores = nullptr, cudaStream_t stream = 0,
                      bool unique_key = true) = 0;
  virtual void assign_scores(const size_type n, const key_type* keys,
                             const score_type* scores = nullptr, cudaStream_t stream = 0,
                             bool unique_key = true) = 0;
  virtual void assign(const size_type n, const key_type* keys,
                      const score_type* scores = nullptr, cudaStream_t stream = 0,
                      bool unique_key = true) = 0;
  virtual void assign_values(const size_type n, const key_type* keys,
                             const value_type* values, cudaStream_t stream = 0,
                             bool unique_key = true) = 0;
  virtual void find(const size_type n, const key_type* keys, value_type* values,
                    bool* founds, score_type* scores = nullptr,
                    cudaStream_t stream = 0) const = 0;
  virtual void find(const size_type n, const key_type* keys, value_type* values,
                    key_type* missed_keys, int* missed_indices, int* missed_size,
                    score_type* scores = nullptr, cudaStream_t stream = 0) const = 0;
  virtual void find(const size_type n, const key_type* keys, value_type** values,
                    bool* founds, score_type* scores = nullptr, cudaStream_t stream = 0,
                    bool unique_key = true) const = 0;
  virtual void find_and_update(const size_type n, const key_type* keys, value_type** values,
                               bool* founds, score_type* scores = nullptr,
                               cudaStream_t stream = 0, bool unique_key = true) = 0;
  virtual void contains(const size_type n, const key_type* keys, bool* founds,
                        cudaStream_t stream = 0) const = 0;
  virtual void erase(const size_type n, const key_type* keys, cudaStream_t stream = 0) = 0;
  virtual void clear(cudaStream_t stream = 0) = 0;
  virtual void export_batch(size_type n, const size_type offset, size_type* d_counter,
                            key_type* keys, value_type* values,
                            score_type* scores = nullptr,
                            cudaStream_t stream = 0) const = 0;
  virtual size_type export_batch(const size_type n, const size_type offset, key_type* keys,
                                 value_type* values, score_type* scores = nullptr,
                                 cudaStream_t stream = 0) const = 0;
  virtual bool empty(cudaStream_t stream = 0) const = 0;
  virtual size_type size(cudaStream_t stream = 0) const = 0;
  virtual size_type capacity() const = 0;
  virtual void reserve(const size_type new_capacity, cudaStream_t stream = 0) = 0;
  virtual float load_factor(cudaStream_t stream = 0) const = 0;
  virtual void set_max_capacity(size_type new_max_capacity) = 0;
  virtual size_type dim() const noexcept = 0;
  virtual size_type max_bucket_size() const noexcept = 0;
  virtual size_type bucket_count() const noexcept = 0;
  virtual bool is_pure_hbm_mode() const noexcept = 0;
  virtual size_type save(BaseKVFile<K, V, S>* file,
                         const size_t max_workspace_size = 1L * 1024 * 1024,
                         cudaStream_t stream = 0) const = 0;
  virtual size_type load(BaseKVFile<K, V, S>* file,
                         const size_t max_workspace_size = 1L * 1024 * 1024,
                         cudaStream_t stream = 0) = 0;
  virtual void set_global_epoch(const uint64_t epoch) = 0;
};

/* HashTable<K, V, S, Strategy>, reference hkv_hashtable.h:895-3485.
 * K: uint64_t or int64_t; S: uint64_t; V: the element type of the vectors
 * (float, double, uint32_t, uint64_t, int8_t, or a 2-byte half type; for a
 * 2-byte type define HKV_B200_VALUE_BF16 before including this header to
 * select bfloat16 arithmetic in accum_or_assign). */
template <typename K, typename V, typename S = uint64_t,
          int Strategy = EvictStrategy::kLru>
class HashTable : public HashTableBase<K, V, S> {
 public:
  using size_type = size_t;
  using key_type = K;
  using value_type = V;
  using score_type = S;
  using allocator_type = BaseAllocator;
  static constexpr int evict_strategy = Strategy;

  HashTable() {
    static_assert(std::is_same<K, int64_t>::value || std::is_same<K, uint64_t>::value,
                  "The key_type must be int64_t or uint64_t.");
    static_assert(std::is_same<S, uint64_t>::value, "The score_type must be uint64_t.");
  }
  ~HashTable() override {
    if (t_) hkv_table_destroy(t_);
  }
  HashTable(const HashTable&) = delete;
  HashTable& operator=(const HashTable&) = delete;
  HashTable(HashTable&&) = delete;
  HashTable& operator=(HashTable&&) = delete;

  /* init, reference hkv_hashtable.h:962-1042: every allocation of the table
   * comes from `allocator` (the CUDA runtime when it is null), which must
   * outlive the table. */
  void init(const HashTableOptions& options, allocator_type* allocator = nullptr) override {
    if (t_) return;
    hkv_options o;
    hkv_options_init(&o);
    o.init_capacity = options.init_capacity;
    o.max_capacity = options.max_capacity;
    o.max_hbm_for_vectors = options.max_hbm_for_vectors;
    o.max_bucket_size = options.max_bucket_size;
    o.dim = options.dim;
    o.max_load_factor = options.max_load_factor;
    o.block_size = options.block_size;
    o.io_block_size = options.io_block_size;
    o.device_id = options.device_id;
    o.io_by_cpu = options.io_by_cpu;
    o.use_constant_memory = options.use_constant_memory;
    o.reserved_key_start_bit = options.reserved_key_start_bit;
    o.num_of_buckets_per_alloc = options.num_of_buckets_per_alloc;
    o.api_lock = options.api_lock;
    int vc = detail::value_code<V>();
#ifdef HKV_B200_VALUE_BF16
    if (sizeof(V) == 2) vc = HKV_VALUE_BF16;
#endif
    if (vc < 0) throw HkvException("unsupported value_type");
    hkv_allocator a{allocator, &detail::alloc_cb, &detail::alloc_async_cb, &detail::free_cb,
                    &detail::free_async_cb};
    detail::check(hkv_table_create_with_allocator(
        &o, std::is_same<K, int64_t>::value ? HKV_KEY_I64 : HKV_KEY_U64, vc,
        Strategy, allocator != nullptr ? &a : nullptr, &t_));
    options_ = options;
  }

  void insert_or_assign(const size_type n, const key_type* keys,
                        const value_type* values,
                        const score_type* scores = nullptr,
                        cudaStream_t stream = 0, bool unique_key = true,
                        bool ignore_evict_strategy = false) {
    detail::check(hkv_insert_or_assign(t_, n, keys, values, scores,
                                       detail::st(stream), unique_key,
                                       ignore_evict_strategy));
  }

  void insert_and_evict(const size_type n, const key_type* keys,
                        const value_type* values, const score_type* scores,
                        key_type* evicted_keys, value_type* evicted_values,
                        score_type* evicted_scores,
                        size_type* d_evicted_counter, cudaStream_t stream = 0,
                        bool unique_key = true,
                        bool ignore_evict_strategy = false) {
    detail::check(hkv_insert_and_evict(
        t_, n, keys, values, scores, evicted_keys, evicted_values,
        evicted_scores, reinterpret_cast<uint64_t*>(d_evicted_counter),
        detail::st(stream), unique_key, ignore_evict_strategy));
  }

  size_type insert_and_evict(const size_type n, const key_type* keys,
                             const value_type* values,
                             const score_type* scores, key_type* evicted_keys,
                             value_type* evicted_values,
                             score_type* evicted_scores,
                             cudaStream_t stream = 0, bool unique_key = true,
                             bool ignore_evict_strategy = false) {
    size_t c = 0;
    detail::check(hkv_insert_and_evict_count(
        t_, n, keys, values, scores, evicted_keys, evicted_values,
        evicted_scores, detail::st(stream), unique_key, ignore_evict_strategy,
        &c));
    return c;
  }

  void accum_or_assign(const size_type n, const key_type* keys,
                       const value_type* value_or_deltas,
                       const bool* accum_or_assigns,
                       const score_type* scores = nullptr,
                       cudaStream_t stream = 0,
                       bool ignore_evict_strategy = false) {
    detail::check(hkv_accum_or_assign(t_, n, keys, value_or_deltas,
                                      accum_or_assigns, scores,
                                      detail::st(stream),
                                      ignore_evict_strategy));
  }

  void find_or_insert(const size_type n, const key_type* keys,
                      value_type* values, score_type* scores = nullptr,
                      cudaStream_t stream = 0, bool unique_key = true,
                      bool ignore_evict_strategy = false) {
    detail::check(hkv_find_or_insert(t_, n, keys, values, scores,
                                     detail::st(stream), unique_key,
                                     ignore_evict_strategy));
  }

  void assign_scores(const size_type n, const key_type* keys,
                     const score_type* scores = nullptr,
                     cudaStream_t stream = 0, bool unique_key = true) {
    detail::check(hkv_assign_scores(t_, n, keys, scores, detail::st(stream),
                                    unique_key));
  }
  void assign(const size_type n, const key_type* keys,
              const score_type* scores = nullptr, cudaStream_t stream = 0,
              bool unique_key = true) {
    assign_scores(n, keys, scores, stream, unique_key);
  }

  void find(const size_type n, const key_type* keys, value_type* values,
            bool* founds, score_type* scores = nullptr,
            cudaStream_t stream = 0) const {
    detail::check(
        hkv_find(t_, n, keys, values, founds, scores, detail::st(stream)));
  }

  /* find* (addresses of the value rows), reference hkv_hashtable.h:2244-2264. */
  void find(const size_type n, const key_type* keys, value_type** values,
            bool* founds, score_type* scores = nullptr, cudaStream_t stream = 0,
            bool unique_key = true) const {
    (void)unique_key;
    detail::check(hkv_find_ptr(t_, n, keys, reinterpret_cast<void**>(values),
                               founds, scores, detail::st(stream)));
  }

  /* find_or_insert* (addresses of the value rows), reference
   * hkv_hashtable.h:1658-1727; with locked_key_ptrs (unique_key only) the
   * keys stay locked until unlock_keys. */
  void find_or_insert(const size_type n, const key_type* keys, value_type** values,
                      bool* founds, score_type* scores = nullptr,
                      cudaStream_t stream = 0, bool unique_key = true,
                      bool ignore_evict_strategy = false,
                      key_type** locked_key_ptrs = nullptr) {
    detail::check(hkv_find_or_insert_ptr(
        t_, n, keys, reinterpret_cast<void**>(values), founds, scores,
        detail::st(stream), unique_key, ignore_evict_strategy,
        reinterpret_cast<void**>(locked_key_ptrs)));
  }

  /* lock_keys / unlock_keys, reference hkv_hashtable.h:1744-1806 (see
   * hkv_lock_keys in hkv_b200.h for the lock marker and the bounded wait). */
  void lock_keys(const size_type n, key_type const* keys, key_type** locked_key_ptrs,
                 bool* succeededs = nullptr, cudaStream_t stream = 0,
                 score_type const* scores = nullptr) {
    detail::check(hkv_lock_keys(t_, n, keys, reinterpret_cast<void**>(locked_key_ptrs),
                                succeededs, detail::st(stream), scores));
  }
  void unlock_keys(const size_type n, key_type** locked_key_ptrs, const key_type* keys,
                   bool* succeededs = nullptr, cudaStream_t stream = 0) {
    detail::check(hkv_unlock_keys(t_, n, reinterpret_cast<void**>(locked_key_ptrs), keys,
                                  succeededs, detail::st(stream)));
  }

  void contains(const size_type n, const key_type* keys, bool* founds,
                cudaStream_t stream = 0) const {
    detail::check(hkv_contains(t_, n, keys, founds, detail::st(stream)));
  }

  void erase(const size_type n, const key_type* keys, cudaStream_t stream = 0) {
    detail::check(hkv_erase(t_, n, keys, detail::st(stream)));
  }

  void clear(cudaStream_t stream = 0) {
    detail::check(hkv_clear(t_, detail::st(stream)));
  }

  void export_batch(size_type n, const size_type offset, size_type* d_counter,
                    key_type* keys, value_type* values,
                    score_type* scores = nullptr,
                    cudaStream_t stream = 0) const {
    detail::check(hkv_export_batch(t_, n, offset,
                                   reinterpret_cast<uint64_t*>(d_counter), keys,
                                   values, scores, detail::st(stream)));
  }

  size_type export_batch(const size_type n, const size_type offset,
                         key_type* keys, value_type* values,
                         score_type* scores = nullptr,
                         cudaStream_t stream = 0) const {
    size_t c = 0;
    detail::check(hkv_export_batch_count(t_, n, offset, keys, values, scores,
                                         detail::st(stream), &c));
    return c;
  }

  bool empty(cudaStream_t stream = 0) const { return size(stream) == 0; }

  size_type size(cudaStream_t stream = 0) const {
    size_t s = 0;
    detail::check(hkv_size(t_, detail::st(stream), &s));
    return s;
  }

  size_type capacity() const {
    size_t c = 0;
    detail::check(hkv_capacity(t_, &c));
    return c;
  }

  void reserve(const size_type new_capacity, cudaStream_t stream = 0) {
    detail::check(hkv_reserve(t_, new_capacity, detail::st(stream)));
  }

  float load_factor(cudaStream_t stream = 0) const {
    float f = 0;
    detail::check(hkv_load_factor(t_, detail::st(stream), &f));
    return f;
  }

  size_type dim() const noexcept { return options_.dim; }
  size_type max_bucket_size() const noexcept { return options_.max_bucket_size; }
  size_type bucket_count() const noexcept override {
    size_t c = 0;
    return hkv_bucket_count(t_, &c) == HKV_OK ? c : 0;
  }
  bool is_pure_hbm_mode() const noexcept override {
    bool b = true;
    return hkv_is_pure_hbm_mode(t_, &b) == HKV_OK ? b : true;
  }

  /* set_max_capacity, reference hkv_hashtable.h:2955-2977. */
  void set_max_capacity(size_type new_max_capacity) override {
    detail::check(hkv_set_max_capacity(t_, new_max_capacity));
    if (new_max_capacity >= capacity()) options_.max_capacity = new_max_capacity;
  }

  /* Outside this build's scope (HashTableBase declares them): each throws. */
  void assign(const size_type, const key_type*, const value_type*,
              const score_type* = nullptr, cudaStream_t = 0, bool = true) override {
    throw HkvException("assign with values is not supported by this build");
  }
  void assign_values(const size_type, const key_type*, const value_type*,
                     cudaStream_t = 0, bool = true) override {
    throw HkvException("assign_values is not supported by this build");
  }
  void find(const size_type, const key_type*, value_type*, key_type*, int*, int*,
            score_type* = nullptr, cudaStream_t = 0) const override {
    throw HkvException("find with missed keys is not supported by this build");
  }
  void find_and_update(const size_type, const key_type*, value_type**, bool*,
                       score_type* = nullptr, cudaStream_t = 0, bool = true) override {
    throw HkvException("find_and_update is not supported by this build");
  }

#ifdef __CUDACC__
  /* Slot scans with caller functors (nvcc translation units only; the
   * kernels are in hkv_scan.cuh): erase_if / erase_if_v2, reference
   * hkv_hashtable.h:2409-2476; export_batch_if / export_batch_if_v2,
   * :2623-2731; size_if, :2829-2846; for_each, :2754-2775. */
  template <template <typename, typename> class PredFunctor>
  size_type erase_if(const key_type& pattern, const score_type& threshold,
                     cudaStream_t stream = 0) {
    scan::PredV1<K, V, S, PredFunctor> p{pattern, threshold};
    return erase_if_impl(p, stream);
  }
  template <typename PredFunctor>
  size_type erase_if_v2(PredFunctor& pred, cudaStream_t stream = 0) {
    return erase_if_impl(pred, stream);
  }
  template <template <typename, typename> class PredFunctor>
  void export_batch_if(const key_type& pattern, const score_type& threshold,
                       size_type n, const size_type offset, size_type* d_counter,
                       key_type* keys, value_type* values,
                       score_type* scores = nullptr, cudaStream_t stream = 0) const {
    scan::PredV1<K, V, S, PredFunctor> p{pattern, threshold};
    export_if_impl(p, n, offset, d_counter, keys, values, scores, stream);
  }
  template <typename PredFunctor>
  void export_batch_if_v2(PredFunctor& pred, size_type n, const size_type offset,
                          size_type* d_counter, key_type* keys, value_type* values,
                          score_type* scores = nullptr, cudaStream_t stream = 0) const {
    export_if_impl(pred, n, offset, d_counter, keys, values, scores, stream);
  }
  template <template <typename, typename> class PredFunctor>
  void size_if(const key_type& pattern, const score_type& threshold,
               size_type* d_counter, cudaStream_t stream = 0) const {
    scan::PredV1<K, V, S, PredFunctor> p{pattern, threshold};
    const hkv_table_view v = view();
    detail::cuda(cudaMemsetAsync(d_counter, 0, sizeof(size_type), stream));
    scan::size_if_kernel<K, V, S><<<scan::grid_for(v.capacity), 256, 0, stream>>>(
        v, p, reinterpret_cast<unsigned long long*>(d_counter));
    detail::cuda(cudaGetLastError());
  }
  template <typename ExecutionFunc>
  void for_each(const size_type first, const size_type last, ExecutionFunc& f,
                cudaStream_t stream = 0) {
    const hkv_table_view v = view();
    if (first >= v.capacity || last > v.capacity || first >= last) return;
    scan::for_each_kernel<K, V, S><<<scan::grid_for(last - first), 256, 0, stream>>>(
        v, first, last - first, f);
    detail::cuda(cudaGetLastError());
  }
#endif

  /* save / load, reference hkv_hashtable.h:3021-3195 (synchronous). */
  size_type save(BaseKVFile<K, V, S>* file,
                 const size_t max_workspace_size = 1L * 1024 * 1024,
                 cudaStream_t stream = 0) const {
    size_t n = 0;
    detail::check(hkv_save(t_, &write_trampoline, file, max_workspace_size,
                           detail::st(stream), &n));
    return n;
  }
  size_type load(BaseKVFile<K, V, S>* file,
                 const size_t max_workspace_size = 1L * 1024 * 1024,
                 cudaStream_t stream = 0) {
    size_t n = 0;
    detail::check(hkv_load(t_, &read_trampoline, file, max_workspace_size,
                           detail::st(stream), &n));
    return n;
  }

  void set_global_epoch(const uint64_t epoch) {
    detail::check(hkv_set_global_epoch(t_, epoch));
  }

  /* No reference counterpart: reports a device lock wait that ran out. */
  void check_device_error(cudaStream_t stream = 0) {
    detail::check(hkv_check_device_error(t_, detail::st(stream)));
  }

  hkv_table* handle() const noexcept { return t_; }

 private:
#ifdef __CUDACC__
  hkv_table_view view() const {
    hkv_table_view v;
    detail::check(hkv_table_get_view(t_, &v));
    return v;
  }
  template <class P>
  size_type erase_if_impl(P& p, cudaStream_t stream) {
    const hkv_table_view v = view();
    unsigned long long* d = nullptr;
    detail::cuda(cudaMallocAsync(reinterpret_cast<void**>(&d), 8, stream));
    detail::cuda(cudaMemsetAsync(d, 0, 8, stream));
    scan::erase_if_kernel<K, V, S><<<scan::grid_for(v.capacity), 256, 0, stream>>>(
        v, p, v.reclaim_digest, d);
    detail::cuda(cudaGetLastError());
    unsigned long long h = 0;
    detail::cuda(cudaMemcpyAsync(&h, d, 8, cudaMemcpyDeviceToHost, stream));
    detail::cuda(cudaFreeAsync(d, stream));
    detail::cuda(cudaStreamSynchronize(stream));
    return static_cast<size_type>(h);
  }
  template <class P>
  void export_if_impl(P& p, size_type n, size_type offset, size_type* d_counter,
                      key_type* keys, value_type* values, score_type* scores,
                      cudaStream_t stream) const {
    const hkv_table_view v = view();
    detail::cuda(cudaMemsetAsync(d_counter, 0, sizeof(size_type), stream));
    if (offset >= v.capacity) return;
    n = n < v.capacity - offset ? n : v.capacity - offset;
    if (n == 0) return;
    scan::export_if_kernel<K, V, S><<<scan::grid_for(n), 256, 0, stream>>>(
        v, p, offset, n, reinterpret_cast<unsigned long long*>(d_counter), keys,
        values, scores);
    detail::cuda(cudaGetLastError());
  }
#endif
  static size_t write_trampoline(void* u, size_t n, size_t dim, const void* k,
                                 const void* v, const uint64_t* sc) {
    return static_cast<BaseKVFile<K, V, S>*>(u)->write(
        n, dim, static_cast<const K*>(k), static_cast<const V*>(v), sc);
  }
  static size_t read_trampoline(void* u, size_t n, size_t dim, void* k, void* v,
                                uint64_t* sc) {
    return static_cast<BaseKVFile<K, V, S>*>(u)->read(
        n, dim, static_cast<K*>(k), static_cast<V*>(v), sc);
  }
  hkv_table* t_ = nullptr;
  HashTableOptions options_;
};

}  // namespace hkv_b200

namespace npu {
namespace hkv = ::hkv_b200;
}  // namespace npu

#endif /* HKV_B200_HASHTABLE_H_ */
