// Drop-in check of the functor scans of include/hkv_hashtable.h (nvcc
// translation unit): erase_if, erase_if_v2, export_batch_if,
// export_batch_if_v2, size_if and for_each with caller functors shaped like
// the reference's (include/hkv_hashtable.h:130-170 and the predicates of
// tests/test_size_if.cpp, tests/test_export_batch_if_v2.cpp,
// tests/test_accum_or_assign.cpp), checked against the same predicates on
// the host over a table whose contents are known.
#include <cuda_runtime.h>

#include <cstdio>
#include <vector>

#include "hkv_hashtable.h"

using namespace npu::hkv;
using K = uint64_t;
using V = float;
using S = uint64_t;

#define CK(x)                                                                \
  do {                                                                       \
    cudaError_t e = (x);                                                     \
    if (e != cudaSuccess) {                                                  \
      std::printf("CUDA error %s at %d\n", cudaGetErrorString(e), __LINE__); \
      return 2;                                                              \
    }                                                                        \
  } while (0)
#define EXPECT(c)                                             \
  do {                                                        \
    if (!(c)) {                                               \
      std::printf("FAILED: %s at line %d\n", #c, __LINE__);   \
      return 1;                                               \
    }                                                         \
  } while (0)

template <class K_, class S_>
struct ScoreGtePred {
  __device__ bool operator()(const K_& key, S_& score, const K_& pattern,
                             const S_& threshold) {
    (void)key;
    (void)pattern;
    return score >= threshold;
  }
};

template <class K_, class S_>
struct OddKeyScoreLtPred {
  __device__ bool operator()(const K_& key, S_& score, const K_& pattern,
                             const S_& threshold) {
    (void)pattern;
    return (key & 0x1u) == 0x1u && score < threshold;
  }
};

template <class K_, class S_>
struct KeyMatchPred {
  __device__ bool operator()(const K_& key, S_& score, const K_& pattern,
                             const S_& threshold) {
    (void)score;
    (void)threshold;
    return (key & pattern) == pattern;
  }
};

// v2 with the group size as a template parameter (export_batch_if_v2 test)
struct ScoreLtV2 {
  S threshold;
  template <int GroupSize>
  __device__ bool operator()(const K& key, const V* value, const S& score) const {
    (void)key;
    (void)value;
    return score < threshold;
  }
};

// v2 with the group size as an argument, reading the value row
struct FirstElemNegativeV2 {
  __device__ bool operator()(const K& key, const V* value, const S& score, int g) const {
    (void)key;
    (void)score;
    (void)g;
    return value[0] < 0.0f;
  }
};

struct ScaleBy2 {
  __device__ void operator()(const K& key, V* value, S* score, int g) const {
    (void)score;
    (void)g;
    if (key < 0xFFFFFFFFFFFFFFFCull) value[0] *= 2.0f;
  }
};

int main() {
  constexpr size_t dim = 4, n = 3000;
  HashTableOptions options;
  options.init_capacity = 128 * 64;
  options.max_capacity = 128 * 64;
  options.max_hbm_for_vectors = 1ull << 30;
  options.dim = dim;
  HashTable<K, V, S, EvictStrategy::kCustomized> table;
  table.init(options);

  std::vector<K> hk(n);
  std::vector<V> hv(n * dim);
  std::vector<S> hs(n);
  for (size_t i = 0; i < n; i++) {
    hk[i] = 1 + i * 2654435761ull % 1000003ull * 16 + (i & 1);  // distinct
    hs[i] = 1 + i;
    for (size_t j = 0; j < dim; j++) hv[i * dim + j] = (i % 3 == 0 ? -1.0f : 1.0f) * (j + 1);
  }
  K* dk;
  V* dv;
  S* ds;
  CK(cudaMalloc(&dk, n * sizeof(K)));
  CK(cudaMalloc(&dv, n * dim * sizeof(V)));
  CK(cudaMalloc(&ds, n * sizeof(S)));
  CK(cudaMemcpy(dk, hk.data(), n * sizeof(K), cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dv, hv.data(), n * dim * sizeof(V), cudaMemcpyHostToDevice));
  CK(cudaMemcpy(ds, hs.data(), n * sizeof(S), cudaMemcpyHostToDevice));
  table.insert_or_assign(n, dk, dv, ds);
  CK(cudaDeviceSynchronize());
  EXPECT(table.size() == n);  // 3000 keys in 8192 slots: no bucket overflows here

  auto count_host = [&](auto pred) {
    size_t c = 0;
    for (size_t i = 0; i < n; i++) c += pred(i) ? 1 : 0;
    return c;
  };
  size_t* d_counter;
  CK(cudaMalloc(&d_counter, sizeof(size_t)));
  size_t h_counter = 0;

  // size_if
  table.size_if<ScoreGtePred>(0, 1001, d_counter);
  CK(cudaMemcpy(&h_counter, d_counter, sizeof(size_t), cudaMemcpyDeviceToHost));
  EXPECT(h_counter == count_host([&](size_t i) { return hs[i] >= 1001; }));
  table.size_if<KeyMatchPred>(0x11, 0, d_counter);
  CK(cudaMemcpy(&h_counter, d_counter, sizeof(size_t), cudaMemcpyDeviceToHost));
  EXPECT(h_counter == count_host([&](size_t i) { return (hk[i] & 0x11) == 0x11; }));

  // export_batch_if over the whole table
  K* ek;
  V* ev;
  S* es;
  const size_t cap = table.capacity();
  CK(cudaMalloc(&ek, cap * sizeof(K)));
  CK(cudaMalloc(&ev, cap * dim * sizeof(V)));
  CK(cudaMalloc(&es, cap * sizeof(S)));
  table.export_batch_if<ScoreGtePred>(0, 2001, cap, 0, d_counter, ek, ev, es);
  CK(cudaMemcpy(&h_counter, d_counter, sizeof(size_t), cudaMemcpyDeviceToHost));
  EXPECT(h_counter == count_host([&](size_t i) { return hs[i] >= 2001; }));
  std::vector<S> got_s(h_counter);
  CK(cudaMemcpy(got_s.data(), es, h_counter * sizeof(S), cudaMemcpyDeviceToHost));
  for (S sc : got_s) EXPECT(sc >= 2001);

  ScoreLtV2 lt{100};
  table.export_batch_if_v2(lt, cap, 0, d_counter, ek, ev, es);
  CK(cudaMemcpy(&h_counter, d_counter, sizeof(size_t), cudaMemcpyDeviceToHost));
  EXPECT(h_counter == count_host([&](size_t i) { return hs[i] < 100; }));

  // for_each doubles element 0 of every live row
  ScaleBy2 f2;
  table.for_each(0, cap, f2);
  bool* df;
  CK(cudaMalloc(&df, n * sizeof(bool)));
  table.find(n, dk, dv, df);
  std::vector<V> after(n * dim);
  CK(cudaMemcpy(after.data(), dv, n * dim * sizeof(V), cudaMemcpyDeviceToHost));
  for (size_t i = 0; i < n; i++) EXPECT(after[i * dim] == 2.0f * hv[i * dim]);

  // erase_if_v2 on the value row, then erase_if on key bits and score
  FirstElemNegativeV2 neg;
  const size_t negs = count_host([&](size_t i) { return hv[i * dim] < 0.0f; });
  EXPECT(table.erase_if_v2(neg) == negs);
  EXPECT(table.size() == n - negs);
  const size_t odd_low = count_host(
      [&](size_t i) { return hv[i * dim] >= 0.0f && (hk[i] & 1) == 1 && hs[i] < 1500; });
  EXPECT(table.erase_if<OddKeyScoreLtPred>(0, 1500) == odd_low);
  EXPECT(table.size() == n - negs - odd_low);
  std::printf("cpp scan drop-in ok\n");
  return 0;
}
