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

int main(int argc, char** argv) {
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
