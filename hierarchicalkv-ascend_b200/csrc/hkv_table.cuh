// hkv_table.cuh -- host-side table object behind the C ABI.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <condition_variable>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/hkv_b200.h"
#include "hkv_device.cuh"

namespace hkvb {

struct HkvError {
  int code;
  std::string msg;
};

// Kernels enqueued by this library in this process; every launch passes its
// stream through counted().
extern std::atomic<uint64_t> g_kernel_launches;
inline cudaStream_t counted(cudaStream_t s) {
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return s;
}

#define HKV_REQUIRE(cond, code, msg)              \
  do {                                            \
    if (!(cond)) throw ::hkvb::HkvError{(code), (msg)}; \
  } while (0)

#define CUDA_TRY(expr)                                                     \
  do {                                                                     \
    cudaError_t e_ = (expr);                                               \
    if (e_ != cudaSuccess)                                                 \
      throw ::hkvb::HkvError{HKV_ERR_CUDA, std::string(#expr) + ": " +     \
                                               cudaGetErrorString(e_)};    \
  } while (0)

struct Slice {
  uint8_t* dev;   // device-visible address
  uint8_t* host;  // host address when the slice is pinned host memory
  size_t bytes;
};

// Where a table's memory comes from: the CUDA runtime, or the caller's
// allocator (the reference's BaseAllocator, allocator.h:27-158, taken by
// init, hkv_hashtable.h:962-978) through the callbacks of hkv_allocator.
class MemSource {
 public:
  MemSource() = default;
  explicit MemSource(const hkv_allocator* a) {
    if (a == nullptr) return;
    HKV_REQUIRE(a->alloc != nullptr && a->free != nullptr, HKV_ERR_INVALID,
                "the allocator needs alloc and free");
    a_ = *a;
    custom_ = true;
  }
  bool custom() const { return custom_; }
  void* device(size_t bytes) {
    void* p = nullptr;
    if (!custom_) {
      CUDA_TRY(cudaMalloc(&p, bytes));
      return p;
    }
    const int rc = a_.alloc(a_.user, HKV_MEMORY_DEVICE, &p, bytes, 0);
    take(rc, p, bytes, "device");
    return p;
  }
  void free_device(void* p) noexcept {
    if (p == nullptr) return;
    if (custom_)
      a_.free(a_.user, HKV_MEMORY_DEVICE, p);
    else
      cudaFree(p);
  }
  void* pinned(size_t bytes, unsigned int flags) {
    void* p = nullptr;
    if (!custom_) {
      CUDA_TRY(cudaHostAlloc(&p, bytes, flags));
      return p;
    }
    const int rc = a_.alloc(a_.user, HKV_MEMORY_PINNED, &p, bytes, flags);
    take(rc, p, bytes, "pinned");
    return p;
  }
  void free_pinned(void* p) noexcept {
    if (p == nullptr) return;
    if (custom_)
      a_.free(a_.user, HKV_MEMORY_PINNED, p);
    else
      cudaFreeHost(p);
  }
  // per-call scratch of a custom allocator (the pool otherwise)
  void* device_async(size_t bytes, cudaStream_t s) {
    void* p = nullptr;
    // (the call completes before p is read: argument order is unspecified)
    const int rc = a_.alloc_async != nullptr
                       ? a_.alloc_async(a_.user, HKV_MEMORY_DEVICE, &p, bytes, s)
                       : a_.alloc(a_.user, HKV_MEMORY_DEVICE, &p, bytes, 0);
    take(rc, p, bytes, "device");
    return p;
  }
  void free_device_async(void* p, cudaStream_t s) noexcept {
    if (p == nullptr) return;
    if (a_.free_async != nullptr) {
      a_.free_async(a_.user, HKV_MEMORY_DEVICE, p, s);
    } else {
      cudaStreamSynchronize(s);  // the scratch may still be in use on s
      a_.free(a_.user, HKV_MEMORY_DEVICE, p);
    }
  }

 private:
  static void take(int rc, void* p, size_t bytes, const char* what) {
    if (rc != 0 || (p == nullptr && bytes != 0))
      throw HkvError{HKV_ERR_CUDA, std::string("the caller's allocator failed to allocate ") +
                                       std::to_string(bytes) + " bytes of " + what +
                                       " memory"};
  }
  hkv_allocator a_{};
  bool custom_ = false;
};

// Stream-ordered scratch for one call: from the table's own memory pool,
// whose freed blocks stay reserved (a steady stream of same-sized calls maps
// device memory once instead of at every call), or from the caller's
// allocator when the table has one.
class Workspace {
 public:
  Workspace(cudaStream_t s, cudaMemPool_t pool, MemSource* mem = nullptr)
      : stream_(s), pool_(pool), mem_(mem != nullptr && mem->custom() ? mem : nullptr) {}
  ~Workspace() {
    for (void* p : ptrs_) {
      if (mem_)
        mem_->free_device_async(p, stream_);
      else
        cudaFreeAsync(p, stream_);
    }
  }
  template <class T>
  T* get(size_t count) {
    void* p = nullptr;
    const size_t bytes = count * sizeof(T) + 16;
    if (mem_)
      p = mem_->device_async(bytes, stream_);
    else
      CUDA_TRY(cudaMallocFromPoolAsync(&p, bytes, pool_, stream_));
    ptrs_.push_back(p);
    return static_cast<T*>(p);
  }

 private:
  cudaStream_t stream_;
  cudaMemPool_t pool_;
  MemSource* mem_;
  std::vector<void*> ptrs_;
};

// Duplicate-key merge of one batch (hkv_dedup.cuh). All arrays live in the
// workspace; `dm` is the device-side count of representatives.
struct DedupResult {
  uint64_t* ukeys;
  uint32_t* rep_first;
  uint32_t* rep_last;
  uint32_t* uid_of;
  uint64_t* uscores;  // merged scores, nullptr when scores == nullptr
  uint32_t* dm;
};
// need_last: the caller uses rep_last (rows from each key's last
// occurrence); without it rep_last is nullptr unless the scores need it
DedupResult dedup_batch(size_t n, const uint64_t* keys, const uint64_t* scores,
                        int strategy, Workspace& ws, cudaStream_t s,
                        int sm_count, int* d_error, bool need_last = true);

// The reference's api_lock (group_lock.h:45-406): readers share it
// (find, contains, export, size), updaters share it (assign_scores), and
// inserts / erases / clear / reserve / scans that modify / save take it
// alone. A holder keeps it until its stream has drained, so the lock covers
// the kernels it launched. Host-side only: the reference's device counters
// serve waits on the device, which this build does not do across streams.
class GroupMutex {
 public:
  enum Mode { kRead = 0, kUpdate = 1, kUnique = 2 };
  void lock(Mode m) {
    std::unique_lock<std::mutex> lk(mu_);
    if (m == kRead) {
      cv_.wait(lk, [&] { return updaters_ == 0 && !unique_; });
      readers_++;
    } else if (m == kUpdate) {
      cv_.wait(lk, [&] { return readers_ == 0 && !unique_; });
      updaters_++;
    } else {
      cv_.wait(lk, [&] { return !unique_; });
      unique_ = true;  // no new reader or updater from here on
      cv_.wait(lk, [&] { return readers_ == 0 && updaters_ == 0; });
    }
  }
  void unlock(Mode m) {
    {
      std::lock_guard<std::mutex> lk(mu_);
      if (m == kRead)
        readers_--;
      else if (m == kUpdate)
        updaters_--;
      else
        unique_ = false;
    }
    cv_.notify_all();
  }

 private:
  std::mutex mu_;
  std::condition_variable cv_;
  int readers_ = 0, updaters_ = 0;
  bool unique_ = false;
};

class TableImpl {
 public:
  // allocator: the caller's (reference BaseAllocator), nullptr for the CUDA
  // runtime; copied
  TableImpl(const hkv_options& o, int key_type, int value_type, int strategy,
            const hkv_allocator* allocator = nullptr);
  ~TableImpl();

  TableView view() const;
  hkv_table_view public_view() const;

  void insert_or_assign(size_t n, const uint64_t* keys, const uint8_t* values,
                        const uint64_t* scores, cudaStream_t s, bool unique,
                        bool ignore);
  void insert_and_evict(size_t n, const uint64_t* keys, const uint8_t* values,
                        const uint64_t* scores, uint64_t* ev_keys,
                        uint8_t* ev_values, uint64_t* ev_scores,
                        uint64_t* d_counter, cudaStream_t s, bool unique,
                        bool ignore);
  void find_or_insert(size_t n, const uint64_t* keys, uint8_t* values,
                      const uint64_t* scores, cudaStream_t s, bool unique,
                      bool ignore, uint8_t* status = nullptr);
  void accum_or_assign(size_t n, const uint64_t* keys, const uint8_t* values,
                       const bool* accum, const uint64_t* scores,
                       cudaStream_t s, bool ignore);
  void assign_scores(size_t n, const uint64_t* keys, const uint64_t* scores,
                     cudaStream_t s);
  void find(size_t n, const uint64_t* keys, uint8_t* values, bool* founds,
            uint64_t* scores, cudaStream_t s);
  // find over nseg key arrays (segment k: counts[k] keys, at most bound);
  // result j of segment k goes to the strided slots described in seg
  void find_segments(const FindSegments& seg, uint32_t nseg, const uint32_t* counts,
                     uint64_t bound, cudaStream_t s);
  // unique-key insert_or_assign / find_or_insert of up to n_bound keys
  // (device count *dn), per-key Occupy result at status[i * status_stride];
  // no auto-grow. find_or_insert given values_in reads an input row there
  // only for a key it inserts and writes values_io only for a key it finds.
  void upsert_counted(int mode, size_t n_bound, const uint32_t* dn,
                      const uint64_t* keys, const uint8_t* values_in,
                      uint8_t* values_io, const uint64_t* scores,
                      uint8_t* status, uint32_t status_stride, cudaStream_t s);
  // find_or_insert of a merged batch, last step: every later occurrence of
  // a key copies the row its representative left at rep_first[uid_of[i]]
  // (skipped where ustatus says the key was refused)
  void scatter_found_rows(uint8_t* values, const uint32_t* uid_of,
                          const uint32_t* rep_first, const uint8_t* ustatus, size_t n,
                          cudaStream_t s);
  // find* / find_or_insert*: addresses of the value rows instead of copies
  void find_ptr(size_t n, const uint64_t* keys, uint8_t** value_ptrs, bool* founds,
                uint64_t* scores, cudaStream_t s);
  void find_or_insert_ptr(size_t n, const uint64_t* keys, uint8_t** value_ptrs,
                          bool* founds, const uint64_t* scores, cudaStream_t s,
                          bool unique, bool ignore,
                          uint64_t** locked_key_ptrs = nullptr);
  // keys held locked by the caller across calls (lock_keys / unlock_keys)
  void lock_keys(size_t n, const uint64_t* keys, uint64_t** locked_key_ptrs,
                 bool* succeeded, const uint64_t* scores, cudaStream_t s);
  void unlock_keys(size_t n, uint64_t* const* locked_key_ptrs, const uint64_t* keys,
                   bool* succeeded, cudaStream_t s);
  void contains(size_t n, const uint64_t* keys, bool* founds, cudaStream_t s);
  void erase(size_t n, const uint64_t* keys, cudaStream_t s);
  void clear(cudaStream_t s);
  void export_batch(size_t n, size_t offset, uint64_t* d_counter,
                    uint64_t* keys, uint8_t* values, uint64_t* scores,
                    cudaStream_t s);
  size_t size(cudaStream_t s);
  float load_factor(cudaStream_t s);
  void reserve(size_t new_capacity, cudaStream_t s);
  void set_max_capacity(size_t new_max_capacity);
  void check_device_error(cudaStream_t s);
  // save / load through BaseKVFile-style callbacks (synchronous)
  size_t save(hkv_kv_write_fn write, void* user, size_t max_ws, cudaStream_t s);
  size_t load(hkv_kv_read_fn read, void* user, size_t max_ws, cudaStream_t s);
  void get_state(uint64_t* keys, uint64_t* scores, uint8_t* digests,
                 int32_t* sizes, uint8_t* values);
  void set_state(const uint64_t* keys, const uint64_t* scores,
                 const uint8_t* digests, const int32_t* sizes,
                 const uint8_t* values);

  uint64_t capacity() const { return capacity_; }
  uint64_t bucket_count() const { return num_buckets_; }
  uint64_t dim() const { return opt_.dim; }
  uint32_t value_bytes() const { return value_bytes_; }
  bool pure_hbm() const { return pure_hbm_; }
  int strategy() const { return strategy_; }
  int value_type() const { return value_type_; }
  int device() const { return device_; }
  cudaMemPool_t pool() const { return pool_; }
  // scratch for one call on stream s (the caller's allocator, if any)
  Workspace workspace(cudaStream_t s) { return Workspace(s, pool_, &mem_); }
  MemSource& mem() { return mem_; }
  int* error_word() const { return d_error_; }
  int value_width(std::initializer_list<const void*> ptrs) const;
  void set_global_epoch(uint64_t e) { epoch_ = e; }
  uint64_t global_epoch() const { return epoch_; }

  // grid size for kernels that use one 8-lane tile per key
  int tile_grid(size_t n) const;
  int existing_grid(size_t n) const;
  int find_grid(size_t n) const;
  int upsert_grid(size_t n, int mode = -1) const;
  int warp_grid(size_t nwarps) const;

  // find_or_insert for batches that may repeat keys, with every scratch
  // buffer carved out of caller-provided device memory `scratch` (no
  // allocation). Defined next to the static scratch array in hkv_table.cu.
  void find_or_insert_in_scratch(size_t n, const uint64_t* keys,
                                 uint8_t* values, const uint64_t* scores,
                                 cudaStream_t s, bool ignore, uint8_t* scratch,
                                 size_t scratch_bytes);

  // throws as the reference does when scores / epoch do not fit the strategy
  void check_strategy(const uint64_t* scores, bool ignore) const;
  // init_capacity * 2 > max_capacity: the table never grows
  bool at_max_capacity() const { return reach_max_; }
  // the api_lock group mutex, nullptr when options.api_lock is false
  GroupMutex* api_mutex() { return api_mutex_.get(); }

 private:
  void auto_grow(size_t n, cudaStream_t s);
  float fast_load_factor(size_t delta, cudaStream_t s);
  uint64_t sum_sizes(uint64_t nb, cudaStream_t s);
  // sum over buckets of (size word >> shift) & kSizeMask
  uint64_t sum_counts(uint64_t nb, int shift, cudaStream_t s);
  void allocate_slices(uint64_t b0, uint64_t b1);
  // frees every table allocation (destructor, failed construction)
  void release() noexcept;
  void upload_slices();
  // doubles the bucket count until it reaches final_nb (a power of two
  // times the current count), rehashing after each doubling
  void grow(uint64_t final_nb, cudaStream_t s);
  void upsert(int mode, size_t n, const uint64_t* keys,
              const uint8_t* values_in, uint8_t* values_io,
              const uint64_t* scores, uint64_t* ev_keys, uint8_t* ev_values,
              uint64_t* ev_scores, uint64_t* d_counter, cudaStream_t s,
              bool unique, bool ignore, uint8_t* status,
              const uint32_t* dn = nullptr, uint32_t status_stride = 1,
              uint8_t** value_ptrs = nullptr, bool* founds = nullptr,
              uint64_t** locked_key_ptrs = nullptr);

  hkv_options opt_;
  MemSource mem_;  // every table allocation goes through it
  int key_type_, value_type_, strategy_;
  uint32_t elem_bytes_, value_bytes_;
  int device_ = 0;
  int sm_count_ = 148;
  cudaMemPool_t pool_ = nullptr;
  std::unique_ptr<GroupMutex> api_mutex_;
  uint64_t* keys_ = nullptr;
  uint64_t* scores_ = nullptr;
  uint8_t* digests_ = nullptr;
  int32_t* sizes_ = nullptr;  // live slots, caller locks from bit kLockShift
  int* d_error_ = nullptr;
  unsigned long long* d_scratch_ = nullptr;  // small device counters
  unsigned long long* h_scratch_ = nullptr;  // pinned host mirror
  std::vector<Slice> slices_;
  uint8_t** d_slices_ = nullptr;
  size_t d_slices_cap_ = 0;
  uint64_t capacity_ = 0, num_buckets_ = 0, max_size_ = 0;
  uint64_t div_magic_ = 0;
  uint32_t div_shift_ = 0;
  uint32_t slice_shift_ = 0;
  uint64_t remaining_hbm_ = 0;
  bool reach_max_ = false;
  bool pure_hbm_ = true;
  uint64_t epoch_ = kIgnoredEpoch;
  // keys may be held locked by the caller (set by lock calls, cleared by an
  // unlock that leaves none): upserts then use the lock-passing kernels
  bool maybe_locked_ = false;
};

}  // namespace hkvb

struct hkv_table {
  hkvb::TableImpl* impl;
};
