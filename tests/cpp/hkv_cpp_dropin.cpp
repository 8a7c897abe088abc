// Drop-in check of include/hkv_hashtable.h: code written against the
// reference's npu::hkv::HashTable API (include/hkv_hashtable.h of the
// reference) compiles against this build and behaves the same way. Mirrors
// the pattern of the reference's tests/test_find_or_insert_evict_strategies.cpp
// (two find_or_insert calls, Lfu scores double) and tests/test_insert_and_evict.cpp
// (refused low-score keys are reported).
#include <cuda_runtime.h>

#include <cstdio>
#include <string>
#include <vector>

#include "hkv_hashtable.h"

using namespace npu::hkv;
using K = uint64_t;
using V = float;
using S = uint64_t;

#define CK(x)                                                      \
  do {                                                             \
    cudaError_t e = (x);                                           \
    if (e != cudaSuccess) {                                        \
      std::printf("CUDA error %s at %d\n", cudaGetErrorString(e), __LINE__); \
      return 2;                                                    \
    }                                                              \
  } while (0)
#define EXPECT(c)                                                  \
  do {                                                             \
    if (!(c)) {                                                    \
      std::printf("FAILED: %s at line %d\n", #c, __LINE__);        \
      return 1;                                                    \
    }                                                              \
  } while (0)

// A caller's allocator (reference allocator.h BaseAllocator) that records
// every block it hands out, so the test can tell where the table's memory
// came from.
class CountingAllocator : public DefaultAllocator {
 public:
  struct Block {
    void* p;
    size_t size;
    MemoryType type;
    unsigned flags;
  };
  std::vector<Block> live;
  size_t allocs = 0, async_allocs = 0, frees = 0;

  void alloc(const MemoryType type, void** ptr, size_t size, unsigned int flags = 0) override {
    DefaultAllocator::alloc(type, ptr, size, flags);
    live.push_back({*ptr, size, type, flags});
    allocs++;
  }
  void alloc_async(const MemoryType type, void** ptr, size_t size, cudaStream_t s) override {
    DefaultAllocator::alloc_async(type, ptr, size, s);
    live.push_back({*ptr, size, type, 0});
    async_allocs++;
  }
  void free(const MemoryType type, void* ptr) override {
    forget(ptr);
    DefaultAllocator::free(type, ptr);
  }
  void free_async(const MemoryType type, void* ptr, cudaStream_t s) override {
    forget(ptr);
    DefaultAllocator::free_async(type, ptr, s);
  }
  size_t bytes(MemoryType t) const {
    size_t b = 0;
    for (const auto& x : live)
      if (x.type == t) b += x.size;
    return b;
  }
  // [p, p + len) inside one live block of type t
  bool owns(const void* p, size_t len, MemoryType t) const {
    const char* c = static_cast<const char*>(p);
    for (const auto& x : live) {
      const char* b = static_cast<const char*>(x.p);
      if (x.type == t && c >= b && c + len <= b + x.size) return true;
    }
    return false;
  }

 private:
  void forget(void* p) {
    for (size_t i = 0; i < live.size(); i++)
      if (live[i].p == p) {
        live.erase(live.begin() + i);
        frees++;
        return;
      }
  }
};

// init(options, allocator) and the HashTableBase interface (reference
// hkv_hashtable.h:171-871, :962-978).
static int allocator_and_base_checks() {
  constexpr size_t dim = 16, n = 2048;
  CountingAllocator alloc;
  HashTableOptions options;
  options.init_capacity = 128 * 64;
  options.max_capacity = 128 * 256;
  options.max_hbm_for_vectors = 1ull << 30;
  options.dim = dim;
  options.max_load_factor = 1.0f;
  {
    auto* concrete = new HashTable<K, V, S, EvictStrategy::kLru>();
    HashTableBase<K, V, S>* base = concrete;
    base->init(options, &alloc);
    const size_t slots = 128 * 64;
    // every table array lies in a block of the caller's allocator
    hkv_table_view v;
    if (hkv_table_get_view(concrete->handle(), &v) != HKV_OK) return 3;
    EXPECT(alloc.owns(v.keys, slots * 8, Device));
    EXPECT(alloc.owns(v.scores, slots * 8, Device));
    EXPECT(alloc.owns(v.digests, slots, Device));
    EXPECT(alloc.owns(v.sizes, 64 * 4, Device));
    EXPECT(alloc.owns(v.slices, sizeof(void*), Device));
    std::vector<uint8_t*> sl(1);
    CK(cudaMemcpy(sl.data(), v.slices, sizeof(void*), cudaMemcpyDeviceToHost));
    EXPECT(alloc.owns(sl[0], slots * dim * sizeof(V), Device));
    EXPECT(alloc.bytes(Device) >= slots * (8 + 8 + 1 + dim * sizeof(V)));
    EXPECT(alloc.bytes(Pinned) > 0);  // host staging of size()
    // the table works through the base interface
    std::vector<K> hk(n);
    std::vector<V> hv(n * dim);
    for (size_t i = 0; i < n; i++) {
      hk[i] = 1000 + i * 7919;
      for (size_t j = 0; j < dim; j++) hv[i * dim + j] = float(i) + 0.25f * j;
    }
    K* dk;
    V* dv;
    bool* df;
    CK(cudaMalloc(&dk, n * sizeof(K)));
    CK(cudaMalloc(&dv, n * dim * sizeof(V)));
    CK(cudaMalloc(&df, n));
    CK(cudaMemcpy(dk, hk.data(), n * sizeof(K), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dv, hv.data(), n * dim * sizeof(V), cudaMemcpyHostToDevice));
    base->insert_or_assign(n, dk, dv, nullptr, 0, false);  // merge scratch
    CK(cudaDeviceSynchronize());
    EXPECT(alloc.async_allocs > 0);  // per-call scratch came from the allocator
    EXPECT(base->size() == n);
    const size_t before = alloc.live.size();
    base->reserve(128 * 128);  // the doubled arrays too
    EXPECT(base->capacity() == 128 * 128);
    if (hkv_table_get_view(concrete->handle(), &v) != HKV_OK) return 3;
    EXPECT(alloc.owns(v.keys, 2 * slots * 8, Device));
    EXPECT(alloc.live.size() > before);
    CK(cudaMemset(dv, 0, n * dim * sizeof(V)));
    base->find(n, dk, dv, df);
    std::vector<V> got(n * dim);
    std::vector<char> hf(n);
    CK(cudaMemcpy(got.data(), dv, n * dim * sizeof(V), cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(hf.data(), df, n, cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < n; i++) EXPECT(hf[i]);
    EXPECT(got == hv);
    // set_max_capacity lets the table grow past its first maximum
    base->set_max_capacity(128 * 1024);
    base->reserve(128 * 512);
    EXPECT(base->capacity() == 128 * 512);
    bool threw = false;
    try {
      base->assign_values(n, dk, dv);
    } catch (const HkvException&) {
      threw = true;
    }
    EXPECT(threw);
    delete base;  // destroys the table through the interface
    CK(cudaFree(dk));
    CK(cudaFree(dv));
    CK(cudaFree(df));
  }
  CK(cudaDeviceSynchronize());
  EXPECT(alloc.live.empty());  // every block went back to the allocator
  // value slices beyond max_hbm_for_vectors come as mapped pinned memory
  {
    HashTableOptions o2 = options;
    o2.max_hbm_for_vectors = 0;
    HashTable<K, V, S> t;
    t.init(o2, &alloc);
    EXPECT(!t.is_pure_hbm_mode());
    bool mapped = false;
    for (const auto& b : alloc.live)
      if (b.type == Pinned && (b.flags & cudaHostAllocMapped) && b.size >= 128 * 64 * dim * sizeof(V))
        mapped = true;
    EXPECT(mapped);
  }
  EXPECT(alloc.live.empty());
  return 0;
}

int main(int argc, char** argv) {
  if (int rc = allocator_and_base_checks()) return rc;
  constexpr size_t dim = 16, n = 4096;
  HashTableOptions options;
  options.init_capacity = 128 * 256;
  options.max_capacity = 128 * 256;
  options.max_hbm_for_vectors = 1ull << 30;
  options.dim = dim;
  HashTable<K, V, S, EvictStrategy::kLfu> table;
  table.init(options);
  EXPECT(table.size() == 0 && table.capacity() == 128 * 256);

  std::vector<K> hk(n);
  std::vector<V> hv(n * dim);
  std::vector<S> hs(n);
  for (size_t i = 0; i < n; i++) {
    hk[i] = 1000 + i * 7;
    hs[i] = 1 + i % 100;
    for (size_t j = 0; j < dim; j++) hv[i * dim + j] = static_cast<V>(hk[i] * 0.00001);
  }
  K* dk;
  V* dv;
  S* ds;
  bool* df;
  CK(cudaMalloc(&dk, n * sizeof(K)));
  CK(cudaMalloc(&dv, n * dim * sizeof(V)));
  CK(cudaMalloc(&ds, n * sizeof(S)));
  CK(cudaMalloc(&df, n * sizeof(bool)));
  CK(cudaMemcpy(dk, hk.data(), n * sizeof(K), cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dv, hv.data(), n * dim * sizeof(V), cudaMemcpyHostToDevice));
  CK(cudaMemcpy(ds, hs.data(), n * sizeof(S), cudaMemcpyHostToDevice));

  table.find_or_insert(n, dk, dv, ds);
  table.find_or_insert(n, dk, dv, ds);
  S* out_s;
  CK(cudaMalloc(&out_s, n * sizeof(S)));
  table.find(n, dk, dv, df, out_s);
  CK(cudaDeviceSynchronize());
  std::vector<S> got(n);
  std::vector<char> found(n);
  CK(cudaMemcpy(got.data(), out_s, n * sizeof(S), cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(found.data(), df, n * sizeof(bool), cudaMemcpyDeviceToHost));
  for (size_t i = 0; i < n; i++) {
    EXPECT(found[i]);
    EXPECT(got[i] == 2 * hs[i]);  // Lfu: a hit adds the input score
  }
  EXPECT(table.size() == n);

  // export_batch returns every key
  K* ek;
  V* ev;
  CK(cudaMalloc(&ek, table.capacity() * sizeof(K)));
  CK(cudaMalloc(&ev, table.capacity() * dim * sizeof(V)));
  EXPECT(table.export_batch(table.capacity(), 0, ek, ev) == n);

  // argument checks throw like the reference's HKV_CHECK
  bool threw = false;
  try {
    table.insert_or_assign(n, dk, dv, nullptr);  // Lfu needs scores
  } catch (const HkvException&) {
    threw = true;
  }
  EXPECT(threw);
  // save to the LocalKVFile format, load into a second table (reference
  // hkv_hashtable.h:3021-3195; small workspace: several chunks)
  const std::string base = std::string(argc > 1 ? argv[1] : "/tmp") + "/dropin";
  {
    LocalKVFile<K, V, S> f;
    EXPECT(f.open(base + "_keys", base + "_values", base + "_scores", "wb"));
    EXPECT(table.save(&f, 64 * 1024) == n);
  }
  HashTable<K, V, S, EvictStrategy::kLfu> copy;
  copy.init(options);
  {
    LocalKVFile<K, V, S> f;
    EXPECT(f.open(base + "_keys", base + "_values", base + "_scores", "rb"));
    EXPECT(copy.load(&f, 64 * 1024) == n);
  }
  EXPECT(copy.size() == n);
  copy.find(n, dk, dv, df, out_s);
  CK(cudaDeviceSynchronize());
  CK(cudaMemcpy(got.data(), out_s, n * sizeof(S), cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(found.data(), df, n * sizeof(bool), cudaMemcpyDeviceToHost));
  for (size_t i = 0; i < n; i++) EXPECT(found[i] && got[i] == 2 * hs[i]);

  // lock_keys / unlock_keys (reference hkv_hashtable.h:1744-1806 and
  // tests/test_lock_unlock_keys.cpp): locked keys are hidden from find until
  // they are unlocked; a second unlock fails
  constexpr size_t nl = 64;
  K** lp;
  bool* lok;
  CK(cudaMalloc(&lp, nl * sizeof(K*)));
  CK(cudaMalloc(&lok, nl * sizeof(bool)));
  std::vector<char> ok(nl);
  table.lock_keys(nl, dk, lp, lok, 0, ds);  // Lfu: the lock adds the score
  CK(cudaMemcpy(ok.data(), lok, nl * sizeof(bool), cudaMemcpyDeviceToHost));
  for (size_t i = 0; i < nl; i++) EXPECT(ok[i]);
  table.find(n, dk, dv, df, out_s);
  CK(cudaMemcpy(found.data(), df, n * sizeof(bool), cudaMemcpyDeviceToHost));
  for (size_t i = 0; i < n; i++) EXPECT(static_cast<bool>(found[i]) == (i >= nl));
  table.unlock_keys(nl, lp, dk, lok);
  CK(cudaMemcpy(ok.data(), lok, nl * sizeof(bool), cudaMemcpyDeviceToHost));
  for (size_t i = 0; i < nl; i++) EXPECT(ok[i]);
  table.find(n, dk, dv, df, out_s);
  CK(cudaMemcpy(got.data(), out_s, n * sizeof(S), cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(found.data(), df, n * sizeof(bool), cudaMemcpyDeviceToHost));
  for (size_t i = 0; i < n; i++) EXPECT(found[i] && got[i] == (i < nl ? 3 : 2) * hs[i]);
  table.unlock_keys(nl, lp, dk, lok);
  CK(cudaMemcpy(ok.data(), lok, nl * sizeof(bool), cudaMemcpyDeviceToHost));
  for (size_t i = 0; i < nl; i++) EXPECT(!ok[i]);

  table.erase(n / 2, dk);
  EXPECT(table.size() == n - n / 2);
  table.clear();
  EXPECT(table.empty());
  std::printf("cpp drop-in ok\n");
  return 0;
}
