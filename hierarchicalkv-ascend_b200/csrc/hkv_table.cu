// hkv_table.cu -- host logic of the B200 HierarchicalKV table and its C ABI.
//
// Mirrors the reference host class (include/hkv_hashtable.h) and table core
// (include/table.h): option checks, bucket-count rule, value slices split
// between HBM and mapped pinned host memory, auto-grow before insert-like
// calls, reserve by doubling plus rehash. All device work is in
// hkv_kernels.cuh / hkv_dedup.cuh; there is no CPU fallback.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "hkv_dedup.cuh"
#include "hkv_kernels.cuh"

#include "../../include/hkv_scan.cuh"
#include "hkv_table.cuh"

namespace hkvb {

std::atomic<uint64_t> g_kernel_launches{0};

namespace {

thread_local std::string g_last_error;

uint32_t elem_size(int vt) {
  switch (vt) {
    case HKV_VALUE_F32: return 4;
    case HKV_VALUE_F16: return 2;
    case HKV_VALUE_BF16: return 2;
    case HKV_VALUE_F64: return 8;
    case HKV_VALUE_U32: return 4;
    case HKV_VALUE_U16: return 2;
    case HKV_VALUE_I8: return 1;
    case HKV_VALUE_U64: return 8;
    default: return 0;
  }
}

bool is_pow2(uint64_t x) { return x && !(x & (x - 1)); }

uint32_t log2_floor(uint64_t x) {
  uint32_t r = 0;
  while ((2ull << r) <= x) r++;
  return r;
}

uint64_t ceil_div(uint64_t a, uint64_t b) { return (a + b - 1) / b; }

constexpr uint64_t MB(uint64_t n) { return n << 20; }
constexpr uint64_t GB(uint64_t n) { return n << 30; }

// get_slice_size, reference table.h:244-268.
uint64_t slice_size_rule(uint64_t max_size, uint32_t value_bytes) {
  const uint64_t min_slice = kBucket * static_cast<uint64_t>(value_bytes);
  const uint64_t max_table = max_size * value_bytes;
  uint64_t s;
  if (max_table >= GB(128))
    s = GB(16);
  else if (max_table >= GB(16))
    s = GB(2);
  else if (max_table >= GB(2))
    s = MB(128);
  else if (max_table >= MB(128))
    s = MB(16);
  else if (max_table >= MB(16))
    s = MB(1);
  else
    s = min_slice;
  return std::max(std::max(min_slice, s), MB(2));
}

// precomputation_for_kernel_div, reference table.h:106-127.
void magic_for(uint64_t d, uint64_t* magic, uint32_t* shift) {
  unsigned __int128 one = 1;
  uint64_t s = 0;
  for (; s < 64; s++)
    if ((one << s) >= d) break;
  const unsigned __int128 m = ((one << 64) * ((one << s) - d)) / d + 1;
  *magic = static_cast<uint64_t>(m);
  *shift = static_cast<uint32_t>(s - 1);
}

}  // namespace

// ---------------------------------------------------------------------------
TableImpl::TableImpl(const hkv_options& o, int key_type, int value_type,
                     int strategy, const hkv_allocator* allocator)
    : opt_(o), mem_(allocator), key_type_(key_type), value_type_(value_type),
      strategy_(strategy) {
  // option checks, reference hkv_hashtable.h:962-1042
  HKV_REQUIRE(key_type == HKV_KEY_U64 || key_type == HKV_KEY_I64,
              HKV_ERR_INVALID, "The key_type must be int64_t or uint64_t.");
  HKV_REQUIRE(strategy >= HKV_LRU && strategy <= HKV_CUSTOMIZED,
              HKV_ERR_INVALID, "unknown evict strategy");
  elem_bytes_ = elem_size(value_type);
  HKV_REQUIRE(elem_bytes_ != 0, HKV_ERR_INVALID, "unknown value type");
  HKV_REQUIRE(o.dim > 0, HKV_ERR_INVALID, "dim must be positive");
  HKV_REQUIRE(o.reserved_key_start_bit >= 0 && o.reserved_key_start_bit <= 62,
              HKV_ERR_INVALID,
              "options.reserved_key_start_bit should >= 0 and <= 62.");
  HKV_REQUIRE(o.reserved_key_start_bit == 0, HKV_ERR_UNSUPPORTED,
              "only the default reserved keys (reserved_key_start_bit = 0) "
              "are supported");
  HKV_REQUIRE(o.max_bucket_size >= 16, HKV_ERR_INVALID,
              "Bucket size should be greater than or equal to 16");
  HKV_REQUIRE(is_pow2(o.max_bucket_size), HKV_ERR_INVALID,
              "Bucket size should be the pow of 2");
  HKV_REQUIRE(o.max_bucket_size == kBucket, HKV_ERR_UNSUPPORTED,
              "this build supports max_bucket_size = 128 only");
  HKV_REQUIRE(is_pow2(o.num_of_buckets_per_alloc), HKV_ERR_INVALID,
              "Then `num_of_buckets_per_alloc` should be the pow of 2");
  HKV_REQUIRE(o.init_capacity >= o.num_of_buckets_per_alloc * o.max_bucket_size,
              HKV_ERR_INVALID,
              "Then `num_of_buckets_per_alloc` must be equal or less than "
              "initial required buckets number");
  HKV_REQUIRE(!(o.io_by_cpu && o.max_hbm_for_vectors != 0), HKV_ERR_INVALID,
              "[HierarchicalKV] `io_by_cpu` should not be true when "
              "`max_hbm_for_vectors` is not 0!");
  HKV_REQUIRE(!o.io_by_cpu, HKV_ERR_UNSUPPORTED,
              "io_by_cpu is not supported: values are read zero-copy");
  if (o.api_lock) api_mutex_.reset(new GroupMutex);
  value_bytes_ = static_cast<uint32_t>(o.dim * elem_bytes_);

  if (o.device_id >= 0) {
    CUDA_TRY(cudaSetDevice(o.device_id));
    device_ = o.device_id;
  } else {
    CUDA_TRY(cudaGetDevice(&device_));
    opt_.device_id = device_;
  }
  CUDA_TRY(cudaDeviceGetAttribute(&sm_count_, cudaDevAttrMultiProcessorCount,
                                  device_));
  // Per-call scratch comes from a pool owned by this table whose freed blocks
  // stay reserved (a release threshold of 0 would return them to the driver
  // at every synchronisation and map them again on the next call).
  {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.handleTypes = cudaMemHandleTypeNone;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = device_;
    CUDA_TRY(cudaMemPoolCreate(&pool_, &props));
    uint64_t keep = UINT64_MAX;
    CUDA_TRY(cudaMemPoolSetAttribute(pool_, cudaMemPoolAttrReleaseThreshold, &keep));
  }

  // bucket count rule, reference table.h:299-309
  max_size_ = std::max(o.init_capacity, o.max_capacity);
  if (o.init_capacity * 2 > max_size_) {
    num_buckets_ = 1 + (max_size_ - 1) / kBucket;
  } else {
    num_buckets_ = 1;
    while (num_buckets_ * kBucket < o.init_capacity) num_buckets_ *= 2;
  }
  capacity_ = num_buckets_ * kBucket;
  magic_for(capacity_, &div_magic_, &div_shift_);
  reach_max_ = o.init_capacity * 2 > o.max_capacity;  // hkv_hashtable.h:1021
  remaining_hbm_ = o.max_hbm_for_vectors;

  // slice geometry: 2^slice_shift buckets per slice, never more than the
  // initial bucket count so that doubling appends whole slices.
  const uint64_t bucket_bytes = kBucket * static_cast<uint64_t>(value_bytes_);
  const uint64_t rule = std::max<uint64_t>(
      1, slice_size_rule(max_size_, value_bytes_) / bucket_bytes);
  slice_shift_ = std::min(log2_floor(rule), log2_floor(num_buckets_));

  const size_t slots = capacity_;
  // every allocation from mem_ (the caller's allocator, if any); a failure
  // part way frees what was taken
  try {
    keys_ = static_cast<uint64_t*>(mem_.device(slots * 8));
    scores_ = static_cast<uint64_t*>(mem_.device(slots * 8));
    digests_ = static_cast<uint8_t*>(mem_.device(slots));
    sizes_ = static_cast<int32_t*>(mem_.device(num_buckets_ * 4));
    d_error_ = static_cast<int*>(mem_.device(2 * sizeof(int)));
    CUDA_TRY(cudaMemset(d_error_, 0, 2 * sizeof(int)));
    d_scratch_ = static_cast<unsigned long long*>(mem_.device(4 * sizeof(unsigned long long)));
    h_scratch_ = static_cast<unsigned long long*>(
        mem_.pinned(4 * sizeof(unsigned long long), cudaHostAllocDefault));
    const uint64_t max_buckets = std::max<uint64_t>(
        num_buckets_, ceil_div(std::max<uint64_t>(max_size_, capacity_), kBucket));
    d_slices_cap_ = ceil_div(max_buckets, 1ull << slice_shift_) + 1;
    d_slices_ = static_cast<uint8_t**>(mem_.device(d_slices_cap_ * sizeof(uint8_t*)));
    allocate_slices(0, num_buckets_);
  } catch (...) {
    release();
    throw;
  }
  upload_slices();
  const TableView v = view();
  init_buckets_kernel<<<std::max(1, warp_grid(num_buckets_)), 256, 0, counted(0)>>>(
      v, 0, num_buckets_, 1);
  CUDA_TRY(cudaGetLastError());
  CUDA_TRY(cudaDeviceSynchronize());
}

TableImpl::~TableImpl() {
  cudaDeviceSynchronize();
  release();
}

void TableImpl::release() noexcept {
  for (auto& s : slices_) {
    if (s.host)
      mem_.free_pinned(s.host);
    else
      mem_.free_device(s.dev);
  }
  slices_.clear();
  mem_.free_device(keys_);
  mem_.free_device(scores_);
  mem_.free_device(digests_);
  mem_.free_device(sizes_);
  mem_.free_device(d_error_);
  mem_.free_device(d_scratch_);
  mem_.free_device(d_slices_);
  mem_.free_pinned(h_scratch_);
  keys_ = scores_ = nullptr;
  digests_ = nullptr;
  sizes_ = nullptr;
  d_error_ = nullptr;
  d_scratch_ = h_scratch_ = nullptr;
  d_slices_ = nullptr;
  if (pool_) cudaMemPoolDestroy(pool_);
  pool_ = nullptr;
}

// initialize_buckets slice placement, reference table.h:143-184: slices go to
// HBM while the remaining budget holds a whole slice, then to pinned host
// memory mapped into the device address space.
void TableImpl::allocate_slices(uint64_t b0, uint64_t b1) {
  const uint64_t bps = 1ull << slice_shift_;
  const uint64_t bucket_bytes = kBucket * static_cast<uint64_t>(value_bytes_);
  for (uint64_t b = b0; b < b1; b += bps) {
    const uint64_t cnt = std::min(bps, b1 - b);
    const size_t bytes = cnt * bucket_bytes;
    Slice s{nullptr, nullptr, bytes};
    if (remaining_hbm_ >= bytes) {
      s.dev = static_cast<uint8_t*>(mem_.device(bytes));
      remaining_hbm_ -= bytes;
    } else {
      pure_hbm_ = false;
      s.host = static_cast<uint8_t*>(
          mem_.pinned(bytes, cudaHostAllocMapped | cudaHostAllocPortable));
      const cudaError_t e =
          cudaHostGetDevicePointer(reinterpret_cast<void**>(&s.dev), s.host, 0);
      if (e != cudaSuccess) {
        mem_.free_pinned(s.host);
        throw HkvError{HKV_ERR_CUDA,
                       std::string("a host value slice is not mapped into the device "
                                   "address space (cudaHostGetDevicePointer: ") +
                           cudaGetErrorString(e) + ")"};
      }
    }
    slices_.push_back(s);
  }
}

void TableImpl::upload_slices() {
  HKV_REQUIRE(slices_.size() <= d_slices_cap_, HKV_ERR_RUNTIME,
              "slice table overflow");
  std::vector<uint8_t*> p(slices_.size());
  for (size_t i = 0; i < slices_.size(); i++) p[i] = slices_[i].dev;
  CUDA_TRY(cudaMemcpy(d_slices_, p.data(), p.size() * sizeof(uint8_t*),
                      cudaMemcpyHostToDevice));
}

hkv_table_view TableImpl::public_view() const {
  hkv_table_view v;
  v.keys = keys_;
  v.scores = scores_;
  v.digests = digests_;
  v.sizes = sizes_;
  v.slices = d_slices_;
  v.capacity = capacity_;
  v.num_buckets = num_buckets_;
  v.bucket_size = kBucket;
  v.slice_shift = slice_shift_;
  v.value_bytes = value_bytes_;
  v.dim = static_cast<uint32_t>(opt_.dim);
  v.reclaim_digest = kReclaimDigest;
  return v;
}

TableView TableImpl::view() const {
  TableView v;
  v.keys = keys_;
  v.scores = scores_;
  v.digests = digests_;
  v.sizes = sizes_;
  v.slices = d_slices_;
  v.values0 = slices_.empty() ? nullptr : slices_[0].dev;
  v.error = d_error_;
  v.capacity = capacity_;
  v.num_buckets = num_buckets_;
  v.div_magic = div_magic_;
  v.div_shift = div_shift_;
  v.cap_pow2 = is_pow2(capacity_) ? 1 : 0;
  v.slice_shift = slice_shift_;
  v.single_slice = slices_.size() == 1 ? 1 : 0;
  v.value_bytes = value_bytes_;
  v.num_slices = static_cast<uint32_t>(slices_.size());
  return v;
}

int TableImpl::tile_grid(size_t n) const {
  const uint64_t blocks = ceil_div(std::max<size_t>(n, 1), 256 / kTile);
  return static_cast<int>(std::min<uint64_t>(blocks, sm_count_ * 64ull));
}

// assign_scores / erase / lock_keys blocks: 256 / kExistTile keys per block
// pass, at most HKV_EXIST_BLOCKS_PER_SM blocks per SM. 8 stay resident; a
// grid of many short blocks measured faster than one resident wave
// (assign_scores 148 -> 129 us, erase 166 -> 156 us per 1 Mi keys)
#ifndef HKV_EXIST_BLOCKS_PER_SM
#define HKV_EXIST_BLOCKS_PER_SM 64
#endif
int TableImpl::existing_grid(size_t n) const {
  const uint64_t blocks = ceil_div(std::max<size_t>(n, 1), 256 / kExistTile);
  return static_cast<int>(
      std::min<uint64_t>(blocks, sm_count_ * uint64_t{HKV_EXIST_BLOCKS_PER_SM}));
}

// Find blocks; each tile walks its keys with the next key loaded ahead.
int TableImpl::find_grid(size_t n) const {
  const uint64_t blocks = ceil_div(std::max<size_t>(n, 1), 256 / kFindTile);
  return static_cast<int>(std::min<uint64_t>(blocks, sm_count_ * uint64_t{kFindBlocksPerSm}));
}

#ifndef HKV_UPSERT_BLOCKS_PER_SM
#define HKV_UPSERT_BLOCKS_PER_SM HKV_UPSERT_MIN_BLOCKS
#endif
// insert_and_evict: many short blocks measured faster than one resident wave
// (727 -> 652 us per 1 Mi keys); insert_or_assign / find_or_insert measured
// the other way (359 -> 366, 378 -> 384 us) and keep the resident grid
#ifndef HKV_EVICT_BLOCKS_PER_SM
#define HKV_EVICT_BLOCKS_PER_SM 64
#endif
int TableImpl::upsert_grid(size_t n, int mode) const {
  const uint64_t blocks = ceil_div(std::max<size_t>(n, 1), 256 / kUpsertTile);
  const uint64_t per_sm =
      mode == kModeInsertAndEvict ? HKV_EVICT_BLOCKS_PER_SM : HKV_UPSERT_BLOCKS_PER_SM;
  return static_cast<int>(std::min<uint64_t>(blocks, sm_count_ * per_sm));
}

int TableImpl::warp_grid(size_t nwarps) const {
  const uint64_t blocks = ceil_div(std::max<size_t>(nwarps, 1), 8);
  return static_cast<int>(std::min<uint64_t>(blocks, sm_count_ * 64ull));
}

// Vector width for value rows: the largest of 16/4/1 bytes dividing the row
// size and the alignment of every row base pointer.
int TableImpl::value_width(std::initializer_list<const void*> ptrs) const {
  int w = 16;
  auto fits = [&](int x) {
    if (value_bytes_ % x) return false;
    for (const void* p : ptrs)
      if (p && reinterpret_cast<uintptr_t>(p) % x) return false;
    return true;
  };
  while (w > 1 && !fits(w)) w = (w == 16) ? 4 : 1;
  return w;
}

#define DISPATCH_VW(vw, ...)            \
  do {                                  \
    if ((vw) == 16) {                   \
      constexpr int VW = 16;            \
      __VA_ARGS__;                      \
    } else if ((vw) == 4) {             \
      constexpr int VW = 4;             \
      __VA_ARGS__;                      \
    } else {                            \
      constexpr int VW = 1;             \
      __VA_ARGS__;                      \
    }                                   \
  } while (0)

#define DISPATCH_STRATEGY(st, ...)      \
  do {                                  \
    switch (st) {                       \
      case kLru: {                      \
        constexpr int S = kLru;         \
        __VA_ARGS__;                    \
        break;                          \
      }                                 \
      case kLfu: {                      \
        constexpr int S = kLfu;         \
        __VA_ARGS__;                    \
        break;                          \
      }                                 \
      case kEpochLru: {                 \
        constexpr int S = kEpochLru;    \
        __VA_ARGS__;                    \
        break;                          \
      }                                 \
      case kEpochLfu: {                 \
        constexpr int S = kEpochLfu;    \
        __VA_ARGS__;                    \
        break;                          \
      }                                 \
      default: {                        \
        constexpr int S = kCustomized;  \
        __VA_ARGS__;                    \
        break;                          \
      }                                 \
    }                                   \
  } while (0)

// check_evict_strategy, reference hkv_hashtable.h:3270-3298.
void TableImpl::check_strategy(const uint64_t* scores, bool ignore) const {
  if (ignore) return;
  if (strategy_ == kLru || strategy_ == kEpochLru)
    HKV_REQUIRE(scores == nullptr, HKV_ERR_INVALID,
                "the scores should not be specified when running on LRU or "
                "Epoch LRU mode.");
  if (strategy_ == kLfu || strategy_ == kEpochLfu)
    HKV_REQUIRE(scores != nullptr, HKV_ERR_INVALID,
                "the scores should be specified when running on LFU or Epoch "
                "LFU mode.");
  if (strategy_ == kCustomized)
    HKV_REQUIRE(scores != nullptr, HKV_ERR_INVALID,
                "the scores should be specified when running on customized "
                "mode.");
  if (strategy_ == kEpochLru || strategy_ == kEpochLfu)
    HKV_REQUIRE(epoch_ != kIgnoredEpoch, HKV_ERR_INVALID,
                "the global_epoch is invalid and should be assigned by calling "
                "`set_global_epoch` when running on Epoch LRU or Epoch LFU "
                "mode.");
}

uint64_t TableImpl::sum_sizes(uint64_t nb, cudaStream_t s) {
  return sum_counts(nb, 0, s);
}

uint64_t TableImpl::sum_counts(uint64_t nb, int shift, cudaStream_t s) {
  CUDA_TRY(cudaMemsetAsync(d_scratch_, 0, sizeof(unsigned long long), s));
  const int blocks = static_cast<int>(
      std::min<uint64_t>(ceil_div(nb, 256 * 4), sm_count_ * 4ull));
  sum_sizes_kernel<<<std::max(blocks, 1), 256, 0, counted(s)>>>(sizes_, nb, d_scratch_,
                                                                 shift);
  CUDA_TRY(cudaGetLastError());
  CUDA_TRY(cudaMemcpyAsync(h_scratch_, d_scratch_, sizeof(unsigned long long),
                           cudaMemcpyDeviceToHost, s));
  CUDA_TRY(cudaStreamSynchronize(s));
  return h_scratch_[0];
}

// fast_load_factor, reference hkv_hashtable.h:3229-3268.
float TableImpl::fast_load_factor(size_t delta, cudaStream_t s) {
  const uint64_t N = std::min<uint64_t>(num_buckets_, 1024);
  const uint64_t total = sum_sizes(N, s);
  return static_cast<float>((delta * 1.0) / (capacity_ * 1.0) +
                            (total * 1.0) / (opt_.max_bucket_size * N * 1.0));
}

// auto-grow before insert-like calls, reference hkv_hashtable.h:1103-1106.
void TableImpl::auto_grow(size_t n, cudaStream_t s) {
  while (!reach_max_ && fast_load_factor(n, s) > opt_.max_load_factor)
    reserve(capacity_ * 2, s);
}

size_t TableImpl::size(cudaStream_t s) { return sum_sizes(num_buckets_, s); }

float TableImpl::load_factor(cudaStream_t s) {
  return static_cast<float>((size(s) * 1.0) / (capacity_ * 1.0));
}

// ---------------------------------------------------------------------------
// Upsert family
// ---------------------------------------------------------------------------
// The upsert kernel of MODE for the enclosing S and VW: the variant whose
// evictions pass caller-held locks by while the caller may hold some.
#define LAUNCH_UPSERT(MODE, VWIDTH, grid, s, v, a)                                   \
  do {                                                                              \
    if (maybe_locked_)                                                              \
      upsert_kernel<MODE, S, VWIDTH, true><<<(grid), 256, 0, counted(s)>>>(v, a);   \
    else                                                                            \
      upsert_kernel<MODE, S, VWIDTH, false><<<(grid), 256, 0, counted(s)>>>(v, a);  \
  } while (0)
void TableImpl::upsert(int mode, size_t n, const uint64_t* keys,
                       const uint8_t* values_in, uint8_t* values_io,
                       const uint64_t* scores, uint64_t* ev_keys,
                       uint8_t* ev_values, uint64_t* ev_scores,
                       uint64_t* d_counter, cudaStream_t s, bool unique,
                       bool ignore, uint8_t* status, const uint32_t* dn,
                       uint32_t status_stride, uint8_t** value_ptrs,
                       bool* founds, uint64_t** locked_key_ptrs) {
  const int st = ignore ? kCustomized : strategy_;
  const TableView v = view();
  UpsertArgs a;
  std::memset(&a, 0, sizeof a);
  a.epoch = epoch_;
  a.ev_keys = ev_keys;
  a.ev_values = ev_values;
  a.ev_scores = ev_scores;
  a.ev_counter = reinterpret_cast<unsigned long long*>(d_counter);
  a.report_refused = 1;
  a.status = status;
  a.status_stride = status_stride;
  a.value_ptrs = value_ptrs;
  a.founds = founds;
  a.locked_key_ptrs = locked_key_ptrs;
  const uint8_t* rows = mode == kModeFindOrInsert ? values_io : values_in;

  if (unique) {
    a.keys = keys;
    a.values_in = values_in;
    a.values_io = values_io;
    a.scores = scores;
    a.n = n;
    a.dn = dn;
    const int vw = value_width({rows, values_in, ev_values});
    const int grid = upsert_grid(n, mode);
    DISPATCH_STRATEGY(st, DISPATCH_VW(vw, {
      if (mode == kModeInsertOrAssign)
        LAUNCH_UPSERT(kModeInsertOrAssign, VW, grid, s, v, a);
      else if (mode == kModeFindOrInsert)
        LAUNCH_UPSERT(kModeFindOrInsert, VW, grid, s, v, a);
      else if (mode == kModeFindOrInsertPtr)
        LAUNCH_UPSERT(kModeFindOrInsertPtr, VW, grid, s, v, a);
      else
        LAUNCH_UPSERT(kModeInsertAndEvict, VW, grid, s, v, a);
    }));
    CUDA_TRY(cudaGetLastError());
    return;
  }

  if (mode == kModeFindOrInsertPtr) {
    // repeated keys: the representatives get addresses, every occurrence
    // then takes its representative's
    Workspace ws(s, pool_, &mem_);
    const DedupResult d =
        dedup_batch(n, keys, scores, st, ws, s, sm_count_, d_error_, false);
    uint8_t** uptrs = ws.get<uint8_t*>(n);
    bool* ufound = ws.get<bool>(n);
    a.keys = d.ukeys;
    a.scores = d.uscores;
    a.n = n;
    a.dn = d.dm;
    a.value_ptrs = uptrs;
    a.founds = ufound;
    const int grid = upsert_grid(n);
    DISPATCH_STRATEGY(st, {
      LAUNCH_UPSERT(kModeFindOrInsertPtr, 16, grid, s, v, a);
    });
    CUDA_TRY(cudaGetLastError());
    scatter_ptrs_kernel<<<static_cast<int>(std::min<uint64_t>(ceil_div(n, 256),
                                                             sm_count_ * 32ull)),
                          256, 0, counted(s)>>>(value_ptrs, founds, uptrs, ufound,
                                                d.uid_of, d.rep_first, n);
    CUDA_TRY(cudaGetLastError());
    return;
  }

  // ---- duplicate keys: merge to one representative per key ---------------
  Workspace ws(s, pool_, &mem_);
  const DedupResult d = dedup_batch(n, keys, scores, st, ws, s, sm_count_, d_error_,
                                    mode != kModeFindOrInsert);
  uint8_t* ustatus = ws.get<uint8_t>(n);
  const uint32_t* uid_of = d.uid_of;
  // Each representative works on the caller's row of one of its
  // occurrences, in place: the last (insert_or_assign, insert_and_evict:
  // each later duplicate overwrites) or the first (find_or_insert: the first
  // inserts, the rest hit and read it back).
  a.keys = d.ukeys;
  a.values_in = values_in;
  a.values_io = values_io;
  a.row_index = mode == kModeFindOrInsert ? d.rep_first : d.rep_last;
  a.scores = d.uscores;
  a.n = n;
  a.dn = d.dm;
  a.status = ustatus;
  a.report_refused = 0;
  CUDA_TRY(cudaMemsetAsync(ustatus, kIllegal, n, s));
  const int vwr = value_width({rows});
  const int vw = value_width({rows, ev_values});
  const int grid = upsert_grid(n, mode);
  DISPATCH_STRATEGY(st, DISPATCH_VW(vw, {
    if (mode == kModeInsertOrAssign)
      LAUNCH_UPSERT(kModeInsertOrAssign, VW, grid, s, v, a);
    else if (mode == kModeFindOrInsert)
      LAUNCH_UPSERT(kModeFindOrInsert, VW, grid, s, v, a);
    else
      LAUNCH_UPSERT(kModeInsertAndEvict, VW, grid, s, v, a);
  }));
  CUDA_TRY(cudaGetLastError());
  if (mode == kModeFindOrInsert) {
    DISPATCH_VW(vwr, scatter_found_rows_kernel<VW><<<tile_grid(n), 256, 0, counted(s)>>>(
                         values_io, uid_of, d.rep_first, ustatus, n, value_bytes_));
  } else if (mode == kModeInsertAndEvict) {
    const int vwe = value_width({rows, ev_values});
    DISPATCH_STRATEGY(st, DISPATCH_VW(vwe, {
      scatter_refused_kernel<S, VW><<<tile_grid(n), 256, 0, counted(s)>>>(
          keys, rows, scores, uid_of, ustatus, n, value_bytes_, epoch_,
          ev_keys, ev_values, ev_scores,
          reinterpret_cast<unsigned long long*>(d_counter));
    }));
  }
  if (status != nullptr) {
    // per-input status: each occurrence reports its representative's result
    expand_status_kernel<<<static_cast<int>(std::min<uint64_t>(
                               ceil_div(n, 256), sm_count_ * 32ull)), 256, 0, counted(s)>>>(ustatus, uid_of, n, status);
  }
  CUDA_TRY(cudaGetLastError());
}

// The merge stages on a set d whose arrays this resets; every other array
// is written before it is read.
void dedup_stages(const DedupView& d, size_t n, const uint64_t* keys,
                  const uint64_t* scores, int score_mode, uint32_t* slot_of,
                  uint32_t* rank, uint32_t* sums, uint32_t* dm, uint64_t* ukeys,
                  uint32_t* rep_first, uint32_t* rep_last, uint32_t* uid_of,
                  uint64_t* uscores, cudaStream_t s, int sm_count, int* d_error) {
  CUDA_TRY(cudaMemsetAsync(d.set_keys, 0xFF, d.cap * 8, s));
  CUDA_TRY(cudaMemsetAsync(d.set_first, 0xFF, d.cap * 4, s));
  if (d.set_last != nullptr) CUDA_TRY(cudaMemsetAsync(d.set_last, 0, d.cap * 4, s));
  if (score_mode >= kScoreSum) CUDA_TRY(cudaMemsetAsync(d.set_sum, 0, d.cap * 8, s));
  const uint64_t ntiles = ceil_div(n, kScanTile);
  const int g1 = static_cast<int>(
      std::min<uint64_t>(ceil_div(n, 256), sm_count * 32ull));
  const int gi = static_cast<int>(
      std::min<uint64_t>(ceil_div(n, kDedupChunk), sm_count * 4ull));
  dedup_insert_kernel<<<gi, kDedupThreads, 0, counted(s)>>>(d, keys, n, scores, score_mode,
                                                            slot_of, d_error);
  scan_first_tiles_kernel<<<static_cast<int>(ntiles), kScanThreads, 0, counted(s)>>>(
      d, slot_of, n, rank, sums);
  scan_sums_kernel<<<1, kScanThreads, 0, counted(s)>>>(sums, ntiles, dm);
  scan_add_kernel<<<static_cast<int>(ntiles), kScanThreads, 0, counted(s)>>>(rank, n,
                                                                             sums);
  dedup_emit_kernel<<<g1, 256, 0, counted(s)>>>(d, keys, slot_of, rank, n, ukeys, rep_first,
                                                rep_last, scores, score_mode, uscores, uid_of);
  CUDA_TRY(cudaGetLastError());
}

DedupResult dedup_batch(size_t n, const uint64_t* keys, const uint64_t* scores,
                        int strategy, Workspace& ws, cudaStream_t s,
                        int sm_count, int* d_error, bool need_last) {
  uint64_t cap = 1024;
  while (cap < 2 * static_cast<uint64_t>(n)) cap <<= 1;
  const int score_mode = dedup_score_mode(strategy, scores != nullptr);
  // the last occurrence: its row (insert_or_assign, insert_and_evict) or its
  // score (score_mode kScoreLast)
  need_last = need_last || score_mode == kScoreLast;
  DedupView d;
  d.cap = cap;
  d.set_keys = ws.get<uint64_t>(cap);
  d.set_first = ws.get<uint32_t>(cap);
  d.set_last = need_last ? ws.get<uint32_t>(cap) : nullptr;
  d.set_sum = score_mode >= kScoreSum ? ws.get<unsigned long long>(cap) : nullptr;
  DedupResult r;
  uint32_t* slot_of = ws.get<uint32_t>(n);
  uint32_t* rank = ws.get<uint32_t>(n);
  r.uid_of = ws.get<uint32_t>(n);
  uint32_t* sums = ws.get<uint32_t>(ceil_div(n, kScanTile) + 1);
  r.dm = ws.get<uint32_t>(1);
  r.ukeys = ws.get<uint64_t>(n);
  r.rep_first = ws.get<uint32_t>(n);
  r.rep_last = need_last ? ws.get<uint32_t>(n) : nullptr;
  r.uscores = scores ? ws.get<uint64_t>(n) : nullptr;
  dedup_stages(d, n, keys, scores, score_mode, slot_of, rank, sums, r.dm, r.ukeys,
               r.rep_first, r.rep_last, r.uid_of, r.uscores, s, sm_count, d_error);
  return r;
}

void TableImpl::insert_or_assign(size_t n, const uint64_t* keys,
                                 const uint8_t* values, const uint64_t* scores,
                                 cudaStream_t s, bool unique, bool ignore) {
  if (n == 0) return;
  auto_grow(n, s);
  check_strategy(scores, ignore);
  HKV_REQUIRE(keys != nullptr && values != nullptr, HKV_ERR_INVALID,
              "keys and values must not be null");
  upsert(kModeInsertOrAssign, n, keys, values, nullptr, scores, nullptr,
         nullptr, nullptr, nullptr, s, unique, ignore, nullptr);
}

void TableImpl::insert_and_evict(size_t n, const uint64_t* keys,
                                 const uint8_t* values, const uint64_t* scores,
                                 uint64_t* ev_keys, uint8_t* ev_values,
                                 uint64_t* ev_scores, uint64_t* d_counter,
                                 cudaStream_t s, bool unique, bool ignore) {
  if (n == 0) return;
  // reference hkv_hashtable.h:1273-1276: null buffers return silently
  if (keys == nullptr || values == nullptr || ev_keys == nullptr ||
      ev_values == nullptr || d_counter == nullptr)
    return;
  auto_grow(n, s);
  check_strategy(scores, ignore);
  if (!pure_hbm_)
    throw HkvError{HKV_ERR_RUNTIME,
                   "Only allow insert_and_evict in pure HBM mode."};
  upsert(kModeInsertAndEvict, n, keys, values, nullptr, scores, ev_keys,
         ev_values, ev_scores, d_counter, s, unique, ignore, nullptr);
}

void TableImpl::find_or_insert(size_t n, const uint64_t* keys, uint8_t* values,
                               const uint64_t* scores, cudaStream_t s,
                               bool unique, bool ignore, uint8_t* status) {
  if (n == 0) return;
  auto_grow(n, s);
  check_strategy(scores, ignore);
  HKV_REQUIRE(keys != nullptr && values != nullptr, HKV_ERR_INVALID,
              "keys and values must not be null");
  // the input rows are passed as values_in too: the kernel then reads a
  // key's input row only when it inserts the key, instead of loading every
  // row before the probe (a found key's row replaces it)
  upsert(kModeFindOrInsert, n, keys, values, values, scores, nullptr, nullptr,
         nullptr, nullptr, s, unique, ignore, status);
}

void TableImpl::accum_or_assign(size_t n, const uint64_t* keys,
                                const uint8_t* values, const bool* accum,
                                const uint64_t* scores, cudaStream_t s,
                                bool ignore) {
  // reference hkv_hashtable.h:1445-1450
  if (value_type_ == HKV_VALUE_F64 || value_type_ == HKV_VALUE_U16 ||
      value_type_ == HKV_VALUE_U32)
    throw HkvError{HKV_ERR_RUNTIME,
                   "[accum_or_assign] Does not support double/uint16_t/"
                   "uint32_t value_type."};
  HKV_REQUIRE(value_type_ == HKV_VALUE_F32 || value_type_ == HKV_VALUE_F16 ||
                  value_type_ == HKV_VALUE_BF16,
              HKV_ERR_UNSUPPORTED,
              "accum_or_assign supports float, half and bfloat16 values");
  if (n == 0) return;
  auto_grow(n, s);
  check_strategy(scores, ignore);
  if (keys == nullptr || values == nullptr || accum == nullptr) return;
  const int st = ignore ? kCustomized : strategy_;
  const TableView v = view();
  AccumArgs a{keys, values, accum, scores, n, epoch_, nullptr,
              value_type_ == HKV_VALUE_F32 && value_width({values}) == 16 ? 1u : 0u};
  const uint64_t blocks = ceil_div(std::max<size_t>(n, 1), 256 / kAccumTile);
  const int grid = static_cast<int>(
      std::min<uint64_t>(blocks, sm_count_ * uint64_t{HKV_ACCUM_BLOCKS_PER_SM}));
  DISPATCH_STRATEGY(st, {
    if (value_type_ == HKV_VALUE_F32)
      accum_kernel<S, float><<<grid, 256, 0, counted(s)>>>(v, a);
    else if (value_type_ == HKV_VALUE_F16)
      accum_kernel<S, __half><<<grid, 256, 0, counted(s)>>>(v, a);
    else
      accum_kernel<S, __nv_bfloat16><<<grid, 256, 0, counted(s)>>>(v, a);
  });
  CUDA_TRY(cudaGetLastError());
}

void TableImpl::assign_scores(size_t n, const uint64_t* keys,
                              const uint64_t* scores, cudaStream_t s) {
  if (n == 0) return;
  check_strategy(scores, false);
  const TableView v = view();
  DISPATCH_STRATEGY(strategy_, {
    existing_key_kernel<S, false><<<existing_grid(n), 256, 0, counted(s)>>>(v, keys, scores,
                                                                   n, epoch_);
  });
  CUDA_TRY(cudaGetLastError());
}

void TableImpl::find(size_t n, const uint64_t* keys, uint8_t* values,
                     bool* founds, uint64_t* scores, cudaStream_t s) {
  if (n == 0) return;
  // reference find_with_digest_kernel.h:42-44: null values -> nothing written
  if (keys == nullptr || values == nullptr) return;
  const TableView v = view();
  const int vw = value_width({values});
  DISPATCH_VW(vw, find_kernel<VW><<<find_grid(n), 256, 0, counted(s)>>>(
                      v, keys, values, founds, scores, n, nullptr, nullptr));
  CUDA_TRY(cudaGetLastError());
}

void TableImpl::find_ptr(size_t n, const uint64_t* keys, uint8_t** value_ptrs,
                         bool* founds, uint64_t* scores, cudaStream_t s) {
  if (n == 0) return;
  // reference find_ptr_with_digest_kernel.h:21-23: null keys or outputs ->
  // nothing written
  if (keys == nullptr || value_ptrs == nullptr) return;
  find_ptr_kernel<<<find_grid(n), 256, 0, counted(s)>>>(view(), keys, value_ptrs,
                                                        founds, scores, n);
  CUDA_TRY(cudaGetLastError());
}

void TableImpl::find_or_insert_ptr(size_t n, const uint64_t* keys,
                                   uint8_t** value_ptrs, bool* founds,
                                   const uint64_t* scores, cudaStream_t s,
                                   bool unique, bool ignore,
                                   uint64_t** locked_key_ptrs) {
  if (n == 0) return;
  // a repeated key cannot be held locked by two of its occurrences
  HKV_REQUIRE(locked_key_ptrs == nullptr || unique, HKV_ERR_UNSUPPORTED,
              "locked_key_ptrs needs unique_key = true");
  auto_grow(n, s);
  if (!ignore) check_strategy(scores, false);
  HKV_REQUIRE(keys != nullptr && value_ptrs != nullptr && founds != nullptr,
              HKV_ERR_INVALID, "keys, values and founds must not be null");
  if (locked_key_ptrs != nullptr) maybe_locked_ = true;
  upsert(kModeFindOrInsertPtr, n, keys, nullptr, nullptr, scores, nullptr,
         nullptr, nullptr, nullptr, s, unique, ignore, nullptr, nullptr, 1,
         value_ptrs, founds, locked_key_ptrs);
}

void TableImpl::lock_keys(size_t n, const uint64_t* keys, uint64_t** locked_key_ptrs,
                          bool* succeeded, const uint64_t* scores, cudaStream_t s) {
  if (n == 0) return;
  // reference lock_keys_kernel.h:23-25: null keys or outputs -> nothing done
  if (keys == nullptr || locked_key_ptrs == nullptr) return;
  check_strategy(scores, false);
  maybe_locked_ = true;
  const TableView v = view();
  DISPATCH_STRATEGY(strategy_, {
    lock_keys_kernel<S><<<existing_grid(n), 256, 0, counted(s)>>>(v, keys, locked_key_ptrs,
                                                              succeeded, scores, n, epoch_);
  });
  CUDA_TRY(cudaGetLastError());
}

void TableImpl::unlock_keys(size_t n, uint64_t* const* locked_key_ptrs,
                            const uint64_t* keys, bool* succeeded, cudaStream_t s) {
  if (n == 0) return;
  // reference unlock_keys_kernel.h:21-23: null inputs -> nothing done
  if (keys == nullptr || locked_key_ptrs == nullptr) return;
  unlock_keys_kernel<<<static_cast<int>(std::min<uint64_t>(ceil_div(n, 256), sm_count_ * 16ull)),
                       256, 0, counted(s)>>>(view(), n, locked_key_ptrs, keys, succeeded);
  CUDA_TRY(cudaGetLastError());
  // the last lock released: later upserts go back to the kernels without the
  // lock-passing scan (a recount, so this call synchronises the stream)
  if (maybe_locked_) maybe_locked_ = sum_counts(num_buckets_, kLockShift, s) != 0;
}

void TableImpl::find_segments(const FindSegments& seg, uint32_t nseg,
                              const uint32_t* counts, uint64_t bound,
                              cudaStream_t s) {
  HKV_REQUIRE(nseg >= 1 && nseg <= kMaxSegments, HKV_ERR_INVALID, "bad segment count");
  if (bound == 0) return;
  int vw = 16;
  for (uint32_t k = 0; k < nseg; k++)
    if (seg.values[k]) vw = std::min(vw, value_width({seg.values[k]}));
  while (vw > 1 && seg.row_stride % vw) vw = vw == 16 ? 4 : 1;
  const TableView v = view();
#ifndef HKV_SEG_BLOCKS_PER_SM
#define HKV_SEG_BLOCKS_PER_SM 64
#endif
  // a multiple of nseg blocks: block b serves segment b % nseg
  const uint64_t per_seg = std::max<uint64_t>(
      1, std::min<uint64_t>(ceil_div(bound, 256 / kFindTile),
                            sm_count_ * uint64_t{HKV_SEG_BLOCKS_PER_SM} / nseg));
  const int grid = static_cast<int>(per_seg * nseg);
  DISPATCH_VW(vw, find_segments_kernel<VW><<<grid, 256, 0, counted(s)>>>(
                      v, seg, nseg, counts, bound));
  CUDA_TRY(cudaGetLastError());
}

void TableImpl::upsert_counted(int mode, size_t n_bound, const uint32_t* dn,
                               const uint64_t* keys, const uint8_t* values_in,
                               uint8_t* values_io, const uint64_t* scores,
                               uint8_t* status, uint32_t status_stride,
                               cudaStream_t s) {
  if (n_bound == 0) return;
  upsert(mode, n_bound, keys, values_in, values_io, scores, nullptr, nullptr,
         nullptr, nullptr, s, true, false, status, dn, status_stride);
}

void TableImpl::scatter_found_rows(uint8_t* values, const uint32_t* uid_of,
                                   const uint32_t* rep_first, const uint8_t* ustatus,
                                   size_t n, cudaStream_t s) {
  if (n == 0 || values == nullptr) return;
  const int vw = value_width({values});
  DISPATCH_VW(vw, scatter_found_rows_kernel<VW><<<tile_grid(n), 256, 0, counted(s)>>>(
                      values, uid_of, rep_first, ustatus, n, value_bytes_));
  CUDA_TRY(cudaGetLastError());
}

void TableImpl::contains(size_t n, const uint64_t* keys, bool* founds,
                         cudaStream_t s) {
  if (n == 0) return;
  if (keys == nullptr || founds == nullptr) return;
  const TableView v = view();
  find_kernel<16><<<find_grid(n), 256, 0, counted(s)>>>(v, keys, nullptr, founds,
                                               nullptr, n, nullptr, nullptr);
  CUDA_TRY(cudaGetLastError());
}

void TableImpl::erase(size_t n, const uint64_t* keys, cudaStream_t s) {
  if (n == 0 || keys == nullptr) return;
  existing_key_kernel<kLru, true><<<existing_grid(n), 256, 0, counted(s)>>>(view(), keys,
                                                                   nullptr, n, 0);
  CUDA_TRY(cudaGetLastError());
}

void TableImpl::clear(cudaStream_t s) {
  init_buckets_kernel<<<warp_grid(num_buckets_), 256, 0, counted(s)>>>(
      view(), 0, num_buckets_, 0);
  CUDA_TRY(cudaGetLastError());
  maybe_locked_ = false;  // every key word and lock count is reset
}

void TableImpl::export_batch(size_t n, size_t offset, uint64_t* d_counter,
                             uint64_t* keys, uint8_t* values, uint64_t* scores,
                             cudaStream_t s) {
  HKV_REQUIRE(d_counter != nullptr, HKV_ERR_INVALID, "d_counter is null");
  CUDA_TRY(cudaMemsetAsync(d_counter, 0, sizeof(uint64_t), s));
  if (offset >= capacity_) return;
  n = std::min<size_t>(capacity_ - offset, n);
  if (n == 0) return;
  const int vw = value_width({values});
  DISPATCH_VW(vw, export_kernel<VW><<<warp_grid(ceil_div(n, 32)), 256, 0, counted(s)>>>(
                      view(), offset, n,
                      reinterpret_cast<unsigned long long*>(d_counter), keys,
                      values, scores));
  CUDA_TRY(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// save / load, reference hkv_hashtable.h:3021-3195
// ---------------------------------------------------------------------------
namespace {
// pinned host staging for one chunk of tuples: keys | scores | values
struct HostChunk {
  MemSource& mem;
  uint8_t* p = nullptr;
  HostChunk(MemSource& m, size_t bytes) : mem(m) {
    p = static_cast<uint8_t*>(mem.pinned(std::max<size_t>(bytes, 1), cudaHostAllocDefault));
  }
  ~HostChunk() { mem.free_pinned(p); }
};
}  // namespace

size_t TableImpl::save(hkv_kv_write_fn write, void* user, size_t max_ws,
                       cudaStream_t s) {
  const size_t tuple = 8 + 8 + value_bytes_;
  HKV_REQUIRE(max_ws >= tuple, HKV_ERR_INVALID,
              "[HierarchicalKV] max_workspace_size is smaller than a single "
              "`key + score + value` tuple! Please set a larger value!");
  const size_t total = capacity_;
  const size_t n = std::min(max_ws / tuple, total);
  HostChunk h(mem_, n * tuple);
  uint64_t* hk = reinterpret_cast<uint64_t*>(h.p);
  uint64_t* hs = hk + n;
  uint8_t* hv = reinterpret_cast<uint8_t*>(hs + n);
  Workspace ws(s, pool_, &mem_);
  uint64_t* dcount = ws.get<uint64_t>(1);
  uint64_t* dk = ws.get<uint64_t>(n);
  uint64_t* dsc = ws.get<uint64_t>(n);
  uint8_t* dv = ws.get<uint8_t>(n * value_bytes_);
  size_t saved = 0;
  for (size_t i = 0; i < total; i += n) {
    export_batch(std::min(total - i, n), i, dcount, dk, dv, dsc, s);
    uint64_t c = 0;
    CUDA_TRY(cudaMemcpyAsync(&c, dcount, 8, cudaMemcpyDeviceToHost, s));
    CUDA_TRY(cudaStreamSynchronize(s));
    if (c == 0) continue;
    CUDA_TRY(cudaMemcpyAsync(hk, dk, c * 8, cudaMemcpyDeviceToHost, s));
    CUDA_TRY(cudaMemcpyAsync(hs, dsc, c * 8, cudaMemcpyDeviceToHost, s));
    CUDA_TRY(cudaMemcpyAsync(hv, dv, c * value_bytes_, cudaMemcpyDeviceToHost, s));
    CUDA_TRY(cudaStreamSynchronize(s));
    write(user, c, opt_.dim, hk, hv, hs);
    saved += c;
  }
  return saved;
}

size_t TableImpl::load(hkv_kv_read_fn read, void* user, size_t max_ws,
                       cudaStream_t s) {
  const size_t tuple = 8 + 8 + value_bytes_;
  HKV_REQUIRE(max_ws >= tuple, HKV_ERR_INVALID,
              "[HierarchicalKV] max_workspace_size is smaller than a single "
              "`key + score + value` tuple! Please set a larger value!");
  const size_t n = max_ws / tuple;
  HostChunk h(mem_, n * tuple);
  uint64_t* hk = reinterpret_cast<uint64_t*>(h.p);
  uint64_t* hs = hk + n;
  uint8_t* hv = reinterpret_cast<uint8_t*>(hs + n);
  size_t c = read(user, n, opt_.dim, hk, hv, hs);
  if (c == 0) return 0;
  Workspace ws(s, pool_, &mem_);
  uint64_t* dk = ws.get<uint64_t>(n);
  uint64_t* dsc = ws.get<uint64_t>(n);
  uint8_t* dv = ws.get<uint8_t>(n * value_bytes_);
  size_t loaded = 0;
  do {
    c = std::min(c, n);
    CUDA_TRY(cudaMemcpyAsync(dk, hk, c * 8, cudaMemcpyHostToDevice, s));
    CUDA_TRY(cudaMemcpyAsync(dsc, hs, c * 8, cudaMemcpyHostToDevice, s));
    CUDA_TRY(cudaMemcpyAsync(dv, hv, c * value_bytes_, cudaMemcpyHostToDevice, s));
    // the reference sets the epoch to IGNORED_GLOBAL_EPOCH and leaves it there
    epoch_ = kIgnoredEpoch;
    insert_or_assign(c, dk, dv, dsc, s, true, true);
    loaded += c;
    CUDA_TRY(cudaStreamSynchronize(s));
    c = read(user, n, opt_.dim, hk, hv, hs);
  } while (c > 0);
  return loaded;
}

// ---------------------------------------------------------------------------
// reserve, reference hkv_hashtable.h:2873-2935 and table.h:360-377
// ---------------------------------------------------------------------------
void TableImpl::grow(uint64_t final_nb, cudaStream_t s) {
  // a rehash would move a key a caller holds locked away from the address
  // the caller was given
  HKV_REQUIRE(sum_counts(num_buckets_, kLockShift, s) == 0, HKV_ERR_RUNTIME,
              "the table cannot grow while keys are locked (lock_keys or "
              "find_or_insert with locked_key_ptrs): unlock them first");
  const uint64_t start_nb = num_buckets_;
  const size_t final_slots = final_nb * kBucket;
  // pass 2 runs one warp per old bucket, each with kBucket scratch rows for
  // the rows that change slot inside their bucket (at most 512 MB of scratch)
  const uint64_t row_block = uint64_t{kBucket} * value_bytes_;
  const uint64_t max_warps = std::max<uint64_t>(
      8, std::min<uint64_t>(sm_count_ * 64ull, (512ull << 20) / row_block));
  const int grid = static_cast<int>(std::max<uint64_t>(
      1, std::min<uint64_t>(ceil_div(final_nb / 2, 8), max_warps / 8)));
  // every allocation first, once for all the doublings: a failure leaves the
  // table as it was
  Workspace ws(s, pool_, &mem_);
  uint64_t *nk = nullptr, *ns = nullptr;
  uint8_t* nd = nullptr;
  int32_t* nz = nullptr;
  uint8_t *maps = nullptr, *scratch = nullptr;
  try {
    nk = static_cast<uint64_t*>(mem_.device(final_slots * 8));
    ns = static_cast<uint64_t*>(mem_.device(final_slots * 8));
    nd = static_cast<uint8_t*>(mem_.device(final_slots));
    nz = static_cast<int32_t*>(mem_.device(final_nb * 4));
    // 2 x kBucket bytes of slot maps per old bucket of the last doubling
    maps = ws.get<uint8_t>(final_nb / 2 * 2 * kBucket);
    scratch = ws.get<uint8_t>(uint64_t{static_cast<uint32_t>(grid)} * 8 * row_block);
  } catch (...) {
    mem_.free_device(nk);
    mem_.free_device(ns);
    mem_.free_device(nd);
    mem_.free_device(nz);
    throw;
  }
  const size_t had_slices = slices_.size();
  const size_t had_hbm = remaining_hbm_;
  const bool was_pure = pure_hbm_;
  try {
    allocate_slices(start_nb, final_nb);
    upload_slices();
  } catch (...) {
    // give back the slices this call added, then the new arrays
    for (size_t i = had_slices; i < slices_.size(); i++) {
      if (slices_[i].host != nullptr)
        mem_.free_pinned(slices_[i].host);
      else
        mem_.free_device(slices_[i].dev);
    }
    slices_.resize(had_slices);
    remaining_hbm_ = had_hbm;
    pure_hbm_ = was_pure;
    mem_.free_device(nk);
    mem_.free_device(ns);
    mem_.free_device(nd);
    mem_.free_device(nz);
    throw;
  }
  // The two passes read the key and score arrays of the previous size and
  // write every slot of both halves of the doubled size (keys, scores,
  // digests), so neither a copy of the old metadata nor a clear of the new
  // buckets is needed; the sizes start from the old ones. The first doubling
  // reads the old arrays, each later one the new arrays in place (pass 2
  // stages an old bucket in shared memory before it rewrites it).
  CUDA_TRY(cudaMemcpyAsync(nz, sizes_, start_nb * 4, cudaMemcpyDeviceToDevice, s));
  uint64_t* const ok = keys_;
  uint64_t* const os = scores_;
  uint8_t* const od = digests_;
  int32_t* const oz = sizes_;
  keys_ = nk;
  scores_ = ns;
  digests_ = nd;
  sizes_ = nz;
  CUDA_TRY(cudaFuncSetAttribute(rehash_replay_kernel,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(kReplaySmem)));
  const int vw = value_width({});
  const uint64_t* src_keys = ok;
  const uint64_t* src_scores = os;
  for (uint64_t old_nb = start_nb; old_nb < final_nb; old_nb *= 2) {
    num_buckets_ = old_nb * 2;
    capacity_ = num_buckets_ * kBucket;
    magic_for(capacity_, &div_magic_, &div_shift_);
    const TableView v = view();
    const int rgrid = static_cast<int>(std::max<uint64_t>(
        1, std::min<uint64_t>(ceil_div(old_nb, kReplayBuckets), sm_count_ * 64ull)));
    rehash_replay_kernel<<<rgrid, kReplayBuckets, kReplaySmem, counted(s)>>>(v, old_nb,
                                                                            src_keys, maps);
    CUDA_TRY(cudaGetLastError());
    DISPATCH_VW(vw, rehash_apply_kernel<VW><<<grid, 256, 0, counted(s)>>>(
                        v, old_nb, src_keys, src_scores, maps, scratch));
    CUDA_TRY(cudaGetLastError());
    src_keys = keys_;
    src_scores = scores_;
  }
  CUDA_TRY(cudaStreamSynchronize(s));
  mem_.free_device(ok);
  mem_.free_device(os);
  mem_.free_device(od);
  mem_.free_device(oz);
}

void TableImpl::reserve(size_t new_capacity, cudaStream_t s) {
  if (reach_max_ || new_capacity > opt_.max_capacity) {
    reach_max_ = capacity_ * 2 > opt_.max_capacity;
    return;
  }
  CUDA_TRY(cudaStreamSynchronize(s));
  // the reference doubles until the capacity covers the request
  // (hkv_hashtable.h:2873-2935); here the arrays grow once to the final size
  // and the doublings' rehashes run one after another
  uint64_t target = capacity_;
  while (target < new_capacity && target * 2 <= opt_.max_capacity) target *= 2;
  if (target > capacity_) grow(target / kBucket, s);
  reach_max_ = capacity_ * 2 > opt_.max_capacity;
}

// set_max_capacity, reference hkv_hashtable.h:2955-2977.
void TableImpl::set_max_capacity(size_t new_max) {
  HKV_REQUIRE(is_pow2(new_max), HKV_ERR_INVALID,
              "None power-of-2 new_max_capacity is not supported.");
  if (new_max < capacity_) return;
  // the slice table must hold the slices of the new maximum
  const uint64_t need = ceil_div(ceil_div(new_max, kBucket), 1ull << slice_shift_) + 1;
  if (need > d_slices_cap_) {
    uint8_t** grown = static_cast<uint8_t**>(mem_.device(need * sizeof(uint8_t*)));
    CUDA_TRY(cudaDeviceSynchronize());  // kernels in flight may read the old table
    mem_.free_device(d_slices_);
    d_slices_ = grown;
    d_slices_cap_ = need;
    upload_slices();
  }
  reach_max_ = false;
  opt_.max_capacity = new_max;
  max_size_ = std::max<uint64_t>(max_size_, new_max);
}

void TableImpl::check_device_error(cudaStream_t s) {
  CUDA_TRY(cudaStreamSynchronize(s));
  int e[2] = {0, 0};
  CUDA_TRY(cudaMemcpy(e, d_error_, sizeof(e), cudaMemcpyDeviceToHost));
  if (e[0]) {
    CUDA_TRY(cudaMemset(d_error_, 0, sizeof(e)));
    if (e[0] & kErrBounds)
      throw HkvError{HKV_ERR_RUNTIME, "device index check failed at site " +
                                          std::to_string(e[1])};
    if (e[0] & kErrPeerOverflow)
      throw HkvError{HKV_ERR_INVALID,
                     "a sharded call sent more keys to one shard than its "
                     "receive area holds (every rank must keep n <= max_batch)"};
    throw HkvError{HKV_ERR_TIMEOUT,
                   "a device lock wait exceeded its time limit (site " +
                       std::to_string(e[1]) +
                       "); the keys involved were not processed"};
  }
}

void TableImpl::get_state(uint64_t* keys, uint64_t* scores, uint8_t* digests,
                          int32_t* sizes, uint8_t* values) {
  CUDA_TRY(cudaDeviceSynchronize());
  if (keys) CUDA_TRY(cudaMemcpy(keys, keys_, capacity_ * 8, cudaMemcpyDeviceToHost));
  if (scores) CUDA_TRY(cudaMemcpy(scores, scores_, capacity_ * 8, cudaMemcpyDeviceToHost));
  if (digests) CUDA_TRY(cudaMemcpy(digests, digests_, capacity_, cudaMemcpyDeviceToHost));
  if (sizes) {
    CUDA_TRY(cudaMemcpy(sizes, sizes_, num_buckets_ * 4, cudaMemcpyDeviceToHost));
    for (uint64_t b = 0; b < num_buckets_; b++) sizes[b] &= kSizeMask;  // live slots only
  }
  if (values) {
    size_t off = 0;
    for (auto& sl : slices_) {
      CUDA_TRY(cudaMemcpy(values + off, sl.dev, sl.bytes, cudaMemcpyDefault));
      off += sl.bytes;
    }
  }
}

void TableImpl::set_state(const uint64_t* keys, const uint64_t* scores,
                          const uint8_t* digests, const int32_t* sizes,
                          const uint8_t* values) {
  CUDA_TRY(cudaDeviceSynchronize());
  if (keys) CUDA_TRY(cudaMemcpy(keys_, keys, capacity_ * 8, cudaMemcpyHostToDevice));
  if (scores) CUDA_TRY(cudaMemcpy(scores_, scores, capacity_ * 8, cudaMemcpyHostToDevice));
  if (digests) CUDA_TRY(cudaMemcpy(digests_, digests, capacity_, cudaMemcpyHostToDevice));
  if (sizes) CUDA_TRY(cudaMemcpy(sizes_, sizes, num_buckets_ * 4, cudaMemcpyHostToDevice));
  if (values) {
    size_t off = 0;
    for (auto& sl : slices_) {
      CUDA_TRY(cudaMemcpy(sl.dev, values + off, sl.bytes, cudaMemcpyDefault));
      off += sl.bytes;
    }
  }
  CUDA_TRY(cudaDeviceSynchronize());
}

void set_last_error(const std::string& m) { g_last_error = m; }
const char* last_error() { return g_last_error.c_str(); }

}  // namespace hkvb

// ===========================================================================
// find_or_insert without allocation (no reference counterpart).
//
// Some callers cannot allocate device memory while they serve lookups: an
// embedding service that hands all of its GPU memory to a fixed arena at
// start-up, or code running where a cudaMalloc would stall or fail. The
// duplicate-key merge normally allocates O(n) scratch per call; this
// variant takes it from one file-scope device array instead. The array is
// shared by every call in the process on that device and keeps the last
// call's contents; everything the merge needs zeroed is cleared at the start
// of each call. Two calls that overlap on the GPU (different streams, or
// different tables on one device) race on the array and must be ordered by
// the caller.
// ===========================================================================
namespace hkvb {

constexpr size_t kNoAllocMaxKeys = 16384;   // keys per call
constexpr size_t kNoAllocSetSlots = 2 * kNoAllocMaxKeys;
constexpr size_t kNoAllocScratchBytes = 2u << 20;  // 2 MiB, checked by ScratchArena

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

// Bump allocator over a fixed buffer (256-byte aligned pieces).
class ScratchArena {
 public:
  ScratchArena(uint8_t* base, size_t bytes) : base_(base), bytes_(bytes) {}
  template <class T>
  T* get(size_t count) {
    const size_t b = (count * sizeof(T) + 255) & ~size_t(255);
    HKV_REQUIRE(used_ + b <= bytes_, HKV_ERR_RUNTIME,
                "static scratch layout exceeds its array");
    T* p = reinterpret_cast<T*>(base_ + used_);
    used_ += b;
    return p;
  }

 private:
  uint8_t* base_;
  size_t bytes_;
  size_t used_ = 0;
};

}  // namespace

void TableImpl::find_or_insert_in_scratch(size_t n, const uint64_t* keys,
                                          uint8_t* values,
                                          const uint64_t* scores,
                                          cudaStream_t s, bool ignore,
                                          uint8_t* scratch,
                                          size_t scratch_bytes) {
  if (n == 0) return;
  HKV_REQUIRE(keys != nullptr && values != nullptr, HKV_ERR_INVALID,
              "keys and values must not be null");
  HKV_REQUIRE(n <= kNoAllocMaxKeys, HKV_ERR_INVALID,
              "hkv_find_or_insert_noalloc: at most 16384 keys per call");
  // Growing the table allocates, so this variant refuses a call that would
  // trigger the reference's auto-grow (hkv_hashtable.h:1103-1106).
  HKV_REQUIRE(reach_max_ || fast_load_factor(n, s) <= opt_.max_load_factor,
              HKV_ERR_RUNTIME,
              "hkv_find_or_insert_noalloc: this batch would grow the table, "
              "which allocates; call hkv_reserve first");
  check_strategy(scores, ignore);
  const int st = ignore ? kCustomized : strategy_;
  ScratchArena ws(scratch, scratch_bytes);
  const int score_mode = dedup_score_mode(st, scores != nullptr);
  DedupView d;
  d.cap = kNoAllocSetSlots;
  d.set_keys = ws.get<uint64_t>(d.cap);
  d.set_first = ws.get<uint32_t>(d.cap);
  // find_or_insert takes the first occurrence's row; the last matters only
  // for its score under score_mode kScoreLast
  d.set_last = score_mode == kScoreLast ? ws.get<uint32_t>(d.cap) : nullptr;
  d.set_sum = ws.get<unsigned long long>(d.cap);
  uint32_t* slot_of = ws.get<uint32_t>(n);
  uint32_t* rank = ws.get<uint32_t>(n);
  uint32_t* uid_of = ws.get<uint32_t>(n);
  uint32_t* sums = ws.get<uint32_t>(ceil_div(n, kScanTile) + 1);
  uint32_t* dm = ws.get<uint32_t>(1);
  uint64_t* ukeys = ws.get<uint64_t>(n);
  uint32_t* rep_first = ws.get<uint32_t>(n);
  uint32_t* rep_last = d.set_last != nullptr ? ws.get<uint32_t>(n) : nullptr;
  uint64_t* uscores = scores ? ws.get<uint64_t>(n) : nullptr;
  uint8_t* ustatus = ws.get<uint8_t>(n);
  // the array keeps the previous call's contents: reset what starts empty
  CUDA_TRY(cudaMemsetAsync(ustatus, kIllegal, n, s));
  dedup_stages(d, n, keys, scores, score_mode, slot_of, rank, sums, dm, ukeys, rep_first,
               rep_last, uid_of, uscores, s, sm_count_, d_error_);
  // representatives find or insert in place at their first occurrence's row
  UpsertArgs a;
  std::memset(&a, 0, sizeof a);
  a.keys = ukeys;
  a.values_in = values;  // input rows read only for inserted keys
  a.values_io = values;
  a.row_index = rep_first;
  a.scores = uscores;
  a.n = n;
  a.dn = dm;
  a.epoch = epoch_;
  a.status = ustatus;
  const TableView v = view();
  const int vw = value_width({values});
  const int grid = upsert_grid(n);
  DISPATCH_STRATEGY(st, DISPATCH_VW(vw, {
    LAUNCH_UPSERT(kModeFindOrInsert, VW, grid, s, v, a);
  }));
  DISPATCH_VW(vw, scatter_found_rows_kernel<VW><<<tile_grid(n), 256, 0, counted(s)>>>(
                      values, uid_of, rep_first, ustatus, n, value_bytes_));
  CUDA_TRY(cudaGetLastError());
}

namespace {

// Device address of g_noalloc_scratch, looked up once per device with that
// device current. In host code the array's name is only a host-side stand-in
// for the symbol, so kernels must be given this address.
std::mutex g_noalloc_mu;
uint8_t* g_noalloc_ptr[64] = {nullptr};

uint8_t* noalloc_scratch_for(int device) {
  HKV_REQUIRE(device >= 0 && device < 64, HKV_ERR_INVALID, "device id");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[device] == nullptr) {
    int cur = 0;
    CUDA_TRY(cudaGetDevice(&cur));
    if (cur != device) CUDA_TRY(cudaSetDevice(device));
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (cur != device) cudaSetDevice(cur);
    if (e != cudaSuccess)
      throw HkvError{HKV_ERR_CUDA,
                     std::string("cudaGetSymbolAddress(g_noalloc_scratch): ") +
                         cudaGetErrorString(e)};
    g_noalloc_ptr[device] = static_cast<uint8_t*>(p);
  }
  return g_noalloc_ptr[device];
}

}  // namespace
}  // namespace hkvb

// ===========================================================================
// C ABI
// ===========================================================================
using hkvb::HkvError;
using hkvb::TableImpl;

#define HKV_API_BEGIN try {
#define HKV_API_END                                     \
  return HKV_OK;                                        \
  }                                                     \
  catch (const HkvError& e) {                           \
    hkvb::set_last_error(e.msg);                        \
    return e.code;                                      \
  }                                                     \
  catch (const std::exception& e) {                     \
    hkvb::set_last_error(e.what());                     \
    return HKV_ERR_RUNTIME;                             \
  }

#define HKV_TABLE(t)                                                      \
  HKV_REQUIRE((t) != nullptr && (t)->impl != nullptr, HKV_ERR_INVALID,    \
              "null table");                                              \
  TableImpl* T = (t)->impl

static inline cudaStream_t as_stream(void* s) {
  return reinterpret_cast<cudaStream_t>(s);
}

// Takes the table's api_lock (when it has one) for the rest of a C ABI call
// and gives it back after the call's stream has drained.
class ApiLock {
 public:
  ApiLock(TableImpl* t, hkvb::GroupMutex::Mode m, void* stream)
      : mu_(t->api_mutex()), mode_(m), stream_(as_stream(stream)) {
    if (mu_) mu_->lock(mode_);
  }
  ~ApiLock() {
    if (!mu_) return;
    cudaStreamSynchronize(stream_);
    mu_->unlock(mode_);
  }
  ApiLock(const ApiLock&) = delete;
  ApiLock& operator=(const ApiLock&) = delete;

 private:
  hkvb::GroupMutex* mu_;
  hkvb::GroupMutex::Mode mode_;
  cudaStream_t stream_;
};

#define HKV_LOCK(mode, stream) ApiLock api_lock_guard_(T, hkvb::GroupMutex::mode, stream)

extern "C" {

void hkv_options_init(hkv_options* o) {
  std::memset(o, 0, sizeof(*o));
  o->max_bucket_size = 128;
  o->dim = 64;
  o->max_load_factor = 0.5f;
  o->block_size = 128;
  o->io_block_size = 1024;
  o->device_id = -1;
  o->num_of_buckets_per_alloc = 1;
}

const char* hkv_last_error(void) { return hkvb::last_error(); }

int hkv_table_create(const hkv_options* options, int key_type, int value_type,
                     int evict_strategy, hkv_table** out) {
  return hkv_table_create_with_allocator(options, key_type, value_type, evict_strategy,
                                         nullptr, out);
}

int hkv_table_create_with_allocator(const hkv_options* options, int key_type,
                                    int value_type, int evict_strategy,
                                    const hkv_allocator* allocator, hkv_table** out) {
  HKV_API_BEGIN
  HKV_REQUIRE(options != nullptr && out != nullptr, HKV_ERR_INVALID,
              "null argument");
  *out = nullptr;
  auto* t = new hkv_table;
  try {
    t->impl = new TableImpl(*options, key_type, value_type, evict_strategy, allocator);
  } catch (...) {
    delete t;
    throw;
  }
  *out = t;
  HKV_API_END
}

int hkv_set_max_capacity(hkv_table* table, size_t new_max_capacity) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUpdate, nullptr);
  T->set_max_capacity(new_max_capacity);
  HKV_API_END
}

int hkv_table_destroy(hkv_table* table) {
  HKV_API_BEGIN
  if (table) {
    delete table->impl;
    delete table;
  }
  HKV_API_END
}

int hkv_insert_or_assign(hkv_table* table, size_t n, const void* keys,
                         const void* values, const uint64_t* scores,
                         void* stream, bool unique_key,
                         bool ignore_evict_strategy) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUnique, stream);
  T->insert_or_assign(n, static_cast<const uint64_t*>(keys),
                      static_cast<const uint8_t*>(values), scores,
                      as_stream(stream), unique_key, ignore_evict_strategy);
  HKV_API_END
}

int hkv_insert_and_evict(hkv_table* table, size_t n, const void* keys,
                         const void* values, const uint64_t* scores,
                         void* evicted_keys, void* evicted_values,
                         uint64_t* evicted_scores, uint64_t* d_evicted_counter,
                         void* stream, bool unique_key,
                         bool ignore_evict_strategy) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUnique, stream);
  T->insert_and_evict(n, static_cast<const uint64_t*>(keys),
                      static_cast<const uint8_t*>(values), scores,
                      static_cast<uint64_t*>(evicted_keys),
                      static_cast<uint8_t*>(evicted_values), evicted_scores,
                      d_evicted_counter, as_stream(stream), unique_key,
                      ignore_evict_strategy);
  HKV_API_END
}

int hkv_insert_and_evict_count(hkv_table* table, size_t n, const void* keys,
                               const void* values, const uint64_t* scores,
                               void* evicted_keys, void* evicted_values,
                               uint64_t* evicted_scores, void* stream,
                               bool unique_key, bool ignore_evict_strategy,
                               size_t* h_evicted_count) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUnique, stream);
  HKV_REQUIRE(h_evicted_count != nullptr, HKV_ERR_INVALID, "null count");
  *h_evicted_count = 0;
  if (n == 0) return HKV_OK;
  cudaStream_t s = as_stream(stream);
  uint64_t* d = nullptr;
  CUDA_TRY(cudaMallocFromPoolAsync(&d, sizeof(uint64_t), T->pool(), s));
  CUDA_TRY(cudaMemsetAsync(d, 0, sizeof(uint64_t), s));
  try {
    T->insert_and_evict(n, static_cast<const uint64_t*>(keys),
                        static_cast<const uint8_t*>(values), scores,
                        static_cast<uint64_t*>(evicted_keys),
                        static_cast<uint8_t*>(evicted_values), evicted_scores,
                        d, s, unique_key, ignore_evict_strategy);
  } catch (...) {
    cudaFreeAsync(d, s);
    throw;
  }
  uint64_t h = 0;
  CUDA_TRY(cudaMemcpyAsync(&h, d, sizeof(uint64_t), cudaMemcpyDeviceToHost, s));
  CUDA_TRY(cudaFreeAsync(d, s));
  CUDA_TRY(cudaStreamSynchronize(s));
  *h_evicted_count = h;
  HKV_API_END
}

int hkv_accum_or_assign(hkv_table* table, size_t n, const void* keys,
                        const void* value_or_deltas,
                        const bool* accum_or_assigns, const uint64_t* scores,
                        void* stream, bool ignore_evict_strategy) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUnique, stream);
  T->accum_or_assign(n, static_cast<const uint64_t*>(keys),
                     static_cast<const uint8_t*>(value_or_deltas),
                     accum_or_assigns, scores, as_stream(stream),
                     ignore_evict_strategy);
  HKV_API_END
}

int hkv_find_or_insert(hkv_table* table, size_t n, const void* keys,
                       void* values, const uint64_t* scores, void* stream,
                       bool unique_key, bool ignore_evict_strategy) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUnique, stream);
  T->find_or_insert(n, static_cast<const uint64_t*>(keys),
                    static_cast<uint8_t*>(values), scores, as_stream(stream),
                    unique_key, ignore_evict_strategy);
  HKV_API_END
}

int hkv_assign_scores(hkv_table* table, size_t n, const void* keys,
                      const uint64_t* scores, void* stream, bool unique_key) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUpdate, stream);
  (void)unique_key;  // duplicates serialise on the key lock either way
  T->assign_scores(n, static_cast<const uint64_t*>(keys), scores,
                   as_stream(stream));
  HKV_API_END
}

int hkv_find(hkv_table* table, size_t n, const void* keys, void* values,
             bool* founds, uint64_t* scores, void* stream) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kRead, stream);
  T->find(n, static_cast<const uint64_t*>(keys), static_cast<uint8_t*>(values),
          founds, scores, as_stream(stream));
  HKV_API_END
}

int hkv_contains(hkv_table* table, size_t n, const void* keys, bool* founds,
                 void* stream) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kRead, stream);
  T->contains(n, static_cast<const uint64_t*>(keys), founds, as_stream(stream));
  HKV_API_END
}

int hkv_erase(hkv_table* table, size_t n, const void* keys, void* stream) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUnique, stream);
  T->erase(n, static_cast<const uint64_t*>(keys), as_stream(stream));
  HKV_API_END
}

int hkv_clear(hkv_table* table, void* stream) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUnique, stream);
  T->clear(as_stream(stream));
  HKV_API_END
}

int hkv_export_batch(hkv_table* table, size_t n, size_t offset,
                     uint64_t* d_counter, void* keys, void* values,
                     uint64_t* scores, void* stream) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kRead, stream);
  T->export_batch(n, offset, d_counter, static_cast<uint64_t*>(keys),
                  static_cast<uint8_t*>(values), scores, as_stream(stream));
  HKV_API_END
}

int hkv_export_batch_count(hkv_table* table, size_t n, size_t offset,
                           void* keys, void* values, uint64_t* scores,
                           void* stream, size_t* h_count) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kRead, stream);
  HKV_REQUIRE(h_count != nullptr, HKV_ERR_INVALID, "null count");
  cudaStream_t s = as_stream(stream);
  uint64_t* d = nullptr;
  CUDA_TRY(cudaMallocFromPoolAsync(&d, sizeof(uint64_t), T->pool(), s));
  try {
    T->export_batch(n, offset, d, static_cast<uint64_t*>(keys),
                    static_cast<uint8_t*>(values), scores, s);
  } catch (...) {
    cudaFreeAsync(d, s);
    throw;
  }
  uint64_t h = 0;
  CUDA_TRY(cudaMemcpyAsync(&h, d, sizeof(uint64_t), cudaMemcpyDeviceToHost, s));
  CUDA_TRY(cudaFreeAsync(d, s));
  CUDA_TRY(cudaStreamSynchronize(s));
  *h_count = h;
  HKV_API_END
}

namespace {
// the C ABI's built-in predicate (hkv_predicate)
struct BuiltinPred {
  uint64_t key_mask, key_value, threshold;
  int cmp;
  __device__ __forceinline__ bool operator()(const uint64_t& key, const uint8_t*,
                                             const uint64_t& score, int) const {
    if ((key & key_mask) != key_value) return false;
    switch (cmp) {
      case HKV_CMP_LT: return score < threshold;
      case HKV_CMP_LE: return score <= threshold;
      case HKV_CMP_GT: return score > threshold;
      case HKV_CMP_GE: return score >= threshold;
      case HKV_CMP_EQ: return score == threshold;
      default: return true;
    }
  }
};
BuiltinPred builtin(const hkv_predicate* p) {
  HKV_REQUIRE(p != nullptr, HKV_ERR_INVALID, "null predicate");
  HKV_REQUIRE(p->score_cmp >= HKV_CMP_ANY && p->score_cmp <= HKV_CMP_EQ, HKV_ERR_INVALID,
              "bad score comparison");
  return BuiltinPred{p->key_mask, p->key_value, p->threshold, p->score_cmp};
}
}  // namespace

int hkv_table_get_view(hkv_table* table, hkv_table_view* out) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_REQUIRE(out != nullptr, HKV_ERR_INVALID, "null argument");
  *out = T->public_view();
  HKV_API_END
}

int hkv_erase_if(hkv_table* table, const hkv_predicate* pred, void* stream,
                 size_t* out_count) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUnique, stream);
  HKV_REQUIRE(out_count != nullptr, HKV_ERR_INVALID, "null count");
  const BuiltinPred p = builtin(pred);
  cudaStream_t s = as_stream(stream);
  const hkv_table_view v = T->public_view();
  unsigned long long* d = nullptr;
  CUDA_TRY(cudaMallocFromPoolAsync(reinterpret_cast<void**>(&d), 8, T->pool(), s));
  CUDA_TRY(cudaMemsetAsync(d, 0, 8, s));
  hkv_b200::scan::erase_if_kernel<uint64_t, uint8_t, uint64_t>
      <<<hkv_b200::scan::grid_for(v.capacity), 256, 0, hkvb::counted(s)>>>(
          v, p, v.reclaim_digest, d);
  CUDA_TRY(cudaGetLastError());
  unsigned long long h = 0;
  CUDA_TRY(cudaMemcpyAsync(&h, d, 8, cudaMemcpyDeviceToHost, s));
  CUDA_TRY(cudaFreeAsync(d, s));
  CUDA_TRY(cudaStreamSynchronize(s));
  *out_count = h;
  HKV_API_END
}

int hkv_export_batch_if(hkv_table* table, const hkv_predicate* pred, size_t n,
                        size_t offset, uint64_t* d_counter, void* keys,
                        void* values, uint64_t* scores, void* stream) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kRead, stream);
  HKV_REQUIRE(d_counter != nullptr, HKV_ERR_INVALID, "d_counter is null");
  const BuiltinPred p = builtin(pred);
  cudaStream_t s = as_stream(stream);
  CUDA_TRY(cudaMemsetAsync(d_counter, 0, 8, s));
  const hkv_table_view v = T->public_view();
  if (offset >= v.capacity) return HKV_OK;
  n = std::min<size_t>(n, v.capacity - offset);
  if (n == 0) return HKV_OK;
  HKV_REQUIRE(keys != nullptr, HKV_ERR_INVALID, "keys must not be null");
  hkv_b200::scan::export_if_kernel<uint64_t, uint8_t, uint64_t>
      <<<hkv_b200::scan::grid_for(n), 256, 0, hkvb::counted(s)>>>(
          v, p, offset, n, reinterpret_cast<unsigned long long*>(d_counter),
          static_cast<uint64_t*>(keys), static_cast<uint8_t*>(values), scores);
  CUDA_TRY(cudaGetLastError());
  HKV_API_END
}

int hkv_size_if(hkv_table* table, const hkv_predicate* pred, uint64_t* d_counter,
                void* stream) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kRead, stream);
  HKV_REQUIRE(d_counter != nullptr, HKV_ERR_INVALID, "d_counter is null");
  const BuiltinPred p = builtin(pred);
  cudaStream_t s = as_stream(stream);
  CUDA_TRY(cudaMemsetAsync(d_counter, 0, 8, s));
  const hkv_table_view v = T->public_view();
  hkv_b200::scan::size_if_kernel<uint64_t, uint8_t, uint64_t>
      <<<hkv_b200::scan::grid_for(v.capacity), 256, 0, hkvb::counted(s)>>>(
          v, p, reinterpret_cast<unsigned long long*>(d_counter));
  CUDA_TRY(cudaGetLastError());
  HKV_API_END
}

int hkv_find_ptr(hkv_table* table, size_t n, const void* keys, void** values,
                 bool* founds, uint64_t* scores, void* stream) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kRead, stream);
  T->find_ptr(n, static_cast<const uint64_t*>(keys),
              reinterpret_cast<uint8_t**>(values), founds, scores, as_stream(stream));
  HKV_API_END
}

int hkv_find_or_insert_ptr(hkv_table* table, size_t n, const void* keys,
                           void** values, bool* founds, const uint64_t* scores,
                           void* stream, bool unique_key,
                           bool ignore_evict_strategy, void** locked_key_ptrs) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUnique, stream);
  T->find_or_insert_ptr(n, static_cast<const uint64_t*>(keys),
                        reinterpret_cast<uint8_t**>(values), founds, scores,
                        as_stream(stream), unique_key, ignore_evict_strategy,
                        reinterpret_cast<uint64_t**>(locked_key_ptrs));
  HKV_API_END
}

int hkv_lock_keys(hkv_table* table, size_t n, const void* keys, void** locked_key_ptrs,
                  bool* succeededs, void* stream, const uint64_t* scores) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUnique, stream);
  T->lock_keys(n, static_cast<const uint64_t*>(keys),
               reinterpret_cast<uint64_t**>(locked_key_ptrs), succeededs, scores,
               as_stream(stream));
  HKV_API_END
}

int hkv_unlock_keys(hkv_table* table, size_t n, void** locked_key_ptrs, const void* keys,
                    bool* succeededs, void* stream) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUnique, stream);
  T->unlock_keys(n, reinterpret_cast<uint64_t* const*>(locked_key_ptrs),
                 static_cast<const uint64_t*>(keys), succeededs, as_stream(stream));
  HKV_API_END
}

int hkv_save(hkv_table* table, hkv_kv_write_fn write, void* user,
             size_t max_workspace_size, void* stream, size_t* out_count) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUnique, stream);
  HKV_REQUIRE(write != nullptr && out_count != nullptr, HKV_ERR_INVALID,
              "null argument");
  *out_count = T->save(write, user, max_workspace_size, as_stream(stream));
  HKV_API_END
}

int hkv_load(hkv_table* table, hkv_kv_read_fn read, void* user,
             size_t max_workspace_size, void* stream, size_t* out_count) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUnique, stream);
  HKV_REQUIRE(read != nullptr && out_count != nullptr, HKV_ERR_INVALID,
              "null argument");
  *out_count = T->load(read, user, max_workspace_size, as_stream(stream));
  HKV_API_END
}

namespace {
// LocalKVFile (reference types.h:349-464): three stdio streams.
struct KVFiles {
  FILE* f[3] = {nullptr, nullptr, nullptr};
  size_t kb, vb;  // key bytes, value bytes per element
  ~KVFiles() {
    for (FILE* x : f)
      if (x) std::fclose(x);
  }
  bool open(const char* k, const char* v, const char* sc, const char* mode) {
    f[0] = std::fopen(k, mode);
    f[1] = f[0] ? std::fopen(v, mode) : nullptr;
    f[2] = f[1] ? std::fopen(sc, mode) : nullptr;
    return f[2] != nullptr;
  }
  static size_t write(void* u, size_t n, size_t dim, const void* keys,
                      const void* values, const uint64_t* scores) {
    auto* F = static_cast<KVFiles*>(u);
    const size_t a = std::fwrite(keys, F->kb, n, F->f[0]);
    const size_t b = std::fwrite(values, F->vb * dim, n, F->f[1]);
    const size_t c = std::fwrite(scores, sizeof(uint64_t), n, F->f[2]);
    return (a == b && a == c) ? a : 0;
  }
  static size_t read(void* u, size_t n, size_t dim, void* keys, void* values,
                     uint64_t* scores) {
    auto* F = static_cast<KVFiles*>(u);
    const size_t a = std::fread(keys, F->kb, n, F->f[0]);
    const size_t b = std::fread(values, F->vb * dim, n, F->f[1]);
    const size_t c = std::fread(scores, sizeof(uint64_t), n, F->f[2]);
    return (a == b && a == c) ? a : 0;
  }
};
}  // namespace

int hkv_save_files(hkv_table* table, const char* keys_path,
                   const char* values_path, const char* scores_path,
                   size_t max_workspace_size, void* stream, size_t* out_count) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUnique, stream);
  HKV_REQUIRE(keys_path && values_path && scores_path && out_count,
              HKV_ERR_INVALID, "null argument");
  KVFiles F;
  F.kb = 8;
  F.vb = T->value_bytes() / T->dim();
  HKV_REQUIRE(F.open(keys_path, values_path, scores_path, "wb"), HKV_ERR_RUNTIME,
              "cannot open the key, value or score file for writing");
  *out_count = T->save(&KVFiles::write, &F, max_workspace_size, as_stream(stream));
  HKV_API_END
}

int hkv_load_files(hkv_table* table, const char* keys_path,
                   const char* values_path, const char* scores_path,
                   size_t max_workspace_size, void* stream, size_t* out_count) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUnique, stream);
  HKV_REQUIRE(keys_path && values_path && scores_path && out_count,
              HKV_ERR_INVALID, "null argument");
  KVFiles F;
  F.kb = 8;
  F.vb = T->value_bytes() / T->dim();
  HKV_REQUIRE(F.open(keys_path, values_path, scores_path, "rb"), HKV_ERR_RUNTIME,
              "cannot open the key, value or score file for reading");
  *out_count = T->load(&KVFiles::read, &F, max_workspace_size, as_stream(stream));
  HKV_API_END
}

int hkv_size(hkv_table* table, void* stream, size_t* out) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kRead, stream);
  *out = T->size(as_stream(stream));
  HKV_API_END
}

int hkv_capacity(hkv_table* table, size_t* out) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  *out = T->capacity();
  HKV_API_END
}

int hkv_load_factor(hkv_table* table, void* stream, float* out) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kRead, stream);
  *out = T->load_factor(as_stream(stream));
  HKV_API_END
}

int hkv_dim(hkv_table* table, size_t* out) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  *out = T->dim();
  HKV_API_END
}

int hkv_max_bucket_size(hkv_table* table, size_t* out) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  *out = T->bucket_count() > 0 ? hkvb::kBucket : 0;
  HKV_API_END
}

int hkv_bucket_count(hkv_table* table, size_t* out) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  *out = T->bucket_count();
  HKV_API_END
}

int hkv_is_pure_hbm_mode(hkv_table* table, bool* out) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  *out = T->pure_hbm();
  HKV_API_END
}

int hkv_reserve(hkv_table* table, size_t new_capacity, void* stream) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUnique, stream);
  T->reserve(new_capacity, as_stream(stream));
  HKV_API_END
}

int hkv_set_global_epoch(hkv_table* table, uint64_t epoch) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  T->set_global_epoch(epoch);
  HKV_API_END
}

int hkv_kernel_launches(uint64_t* out) {
  HKV_API_BEGIN
  HKV_REQUIRE(out != nullptr, HKV_ERR_INVALID, "null argument");
  *out = hkvb::g_kernel_launches.load(std::memory_order_relaxed);
  HKV_API_END
}

int hkv_check_device_error(hkv_table* table, void* stream) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  T->check_device_error(as_stream(stream));
  HKV_API_END
}

int hkv_debug_get_state(hkv_table* table, uint64_t* keys, uint64_t* scores,
                        uint8_t* digests, int32_t* sizes, void* values) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  T->get_state(keys, scores, digests, sizes, static_cast<uint8_t*>(values));
  HKV_API_END
}

int hkv_find_or_insert_noalloc(hkv_table* table, size_t n, const void* keys,
                               void* values, const uint64_t* scores,
                               void* stream, bool ignore_evict_strategy) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  HKV_LOCK(kUnique, stream);
  uint8_t* scratch = hkvb::noalloc_scratch_for(T->device());
  T->find_or_insert_in_scratch(n, static_cast<const uint64_t*>(keys),
                               static_cast<uint8_t*>(values), scores,
                               as_stream(stream), ignore_evict_strategy,
                               scratch, hkvb::kNoAllocScratchBytes);
  HKV_API_END
}

int hkv_debug_set_state(hkv_table* table, const uint64_t* keys,
                        const uint64_t* scores, const uint8_t* digests,
                        const int32_t* sizes, const void* values) {
  HKV_API_BEGIN
  HKV_TABLE(table);
  T->set_state(keys, scores, digests, sizes,
               static_cast<const uint8_t*>(values));
  HKV_API_END
}

}  // extern "C"
