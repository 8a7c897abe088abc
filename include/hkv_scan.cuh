/*
 * hkv_scan.cuh -- slot scans of the B200 HierarchicalKV table with caller
 * functors: erase_if, export_batch_if, size_if (reference
 * include/hkv_hashtable.h:2409-2476, :2623-2731, :2829-2846) and for_each
 * (:2754-2775). A CUDA header: a translation unit compiled by nvcc
 * instantiates these kernels with its own device functors, exactly as the
 * reference's member templates do; the library instantiates them with its
 * built-in predicate for the C ABI (hkv_erase_if and friends).
 *
 * The kernels work on the table's raw arrays, described by hkv_table_view
 * (hkv_table_get_view). Like the reference, a scan is not synchronised with
 * other calls on other streams; calls on one stream are ordered.
 *
 * Functor shapes (as in the reference):
 *   v1 predicate  PredFunctor<K, S>: bool operator()(const K& key, S& score,
 *                 const K& pattern, const S& threshold)
 *   v2 predicate  bool operator()(const K& key, const V* value,
 *                 const S& score, int group_size)
 *   for_each      void operator()(const K& key, V* value, S* score,
 *                 int group_size)
 * group_size is 1 here: one thread per slot.
 */
#ifndef HKV_B200_SCAN_CUH_
#define HKV_B200_SCAN_CUH_

#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>
#include <utility>

#include "hkv_b200.h"

namespace hkv_b200 {
namespace scan {

constexpr uint64_t kReservedMin = 0xFFFFFFFFFFFFFFFCull;  // 4 reserved keys
constexpr uint64_t kReclaimKey = 0xFFFFFFFFFFFFFFFEull;

__device__ __forceinline__ bool reserved(uint64_t k) { return k >= kReservedMin; }

__device__ __forceinline__ uint8_t* row_of(const hkv_table_view& v, uint64_t slot) {
  const uint64_t b = slot / v.bucket_size;
  const uint64_t in_slice = ((b & ((uint64_t{1} << v.slice_shift) - 1)) * v.bucket_size +
                             slot % v.bucket_size);
  return v.slices[b >> v.slice_shift] + in_slice * v.value_bytes;
}

// A v2 predicate or for_each functor is called as f(key, value, score,
// group_size), or as f.template operator()<group_size>(key, value, score)
// when it declares the group size as a template parameter (both shapes occur
// in the reference's tests).
template <class F, class K, class V, class S, class = void>
struct HasTemplatedCall : std::false_type {};
template <class F, class K, class V, class S>
struct HasTemplatedCall<F, K, V, S,
                        decltype((void)std::declval<F&>().template operator()<1>(
                            std::declval<const K&>(), std::declval<V>(),
                            std::declval<S>()))> : std::true_type {};

template <class F, class K, class V, class S>
__device__ __forceinline__ auto call_v2(F& f, const K& key, V value, S score) {
  if constexpr (HasTemplatedCall<F, K, V, S>::value)
    return f.template operator()<1>(key, value, score);
  else
    return f(key, value, score, 1);
}

// Adaptors giving every predicate the v2 call shape.
template <class K, class V, class S, template <typename, typename> class Pred>
struct PredV1 {
  K pattern;
  S threshold;
  __device__ __forceinline__ bool operator()(const K& key, const V*, const S& score,
                                             int) const {
    Pred<K, S> p;
    S s = score;
    return p(key, s, pattern, threshold);
  }
};

// erase_if (reference remove_kernel.h:114-203): a matching live slot becomes
// a RECLAIM tombstone with score 0 and the reclaim digest; its bucket's size
// drops by one. *count accumulates the number erased.
template <class K, class V, class S, class Pred>
__global__ void erase_if_kernel(hkv_table_view v, Pred pred, uint8_t reclaim_digest,
                                unsigned long long* count) {
  const uint64_t nthreads = uint64_t{gridDim.x} * blockDim.x;
  unsigned long long mine = 0;
  for (uint64_t slot = uint64_t{blockIdx.x} * blockDim.x + threadIdx.x; slot < v.capacity;
       slot += nthreads) {
    const uint64_t key = v.keys[slot];
    bool hit = false;
    if (!reserved(key)) {
      const S score = static_cast<S>(v.scores[slot]);
      hit = call_v2(pred, static_cast<K>(key), reinterpret_cast<const V*>(row_of(v, slot)),
                    score);
    }
    if (hit) {
      v.keys[slot] = kReclaimKey;
      v.scores[slot] = 0;
      v.digests[slot] = reclaim_digest;
      atomicSub(v.sizes + slot / v.bucket_size, 1);
      mine++;
    }
  }
  for (int o = 16; o > 0; o >>= 1) mine += __shfl_xor_sync(0xFFFFFFFFu, mine, o);
  if ((threadIdx.x & 31) == 0 && mine) atomicAdd(count, mine);
}

// export_batch_if (reference dump_kernel_if.h, dump_kernel_if_v2.h): the
// matching live slots of [offset, offset + n) compacted to the outputs; a
// block takes blockDim.x consecutive slots, reserves its output range with
// one atomic and each warp's lanes then copy the matching rows' 16-byte (or
// 4-byte, or 1-byte, by alignment) pieces. *counter (zeroed by the caller)
// receives the total.
template <class U>
__device__ __forceinline__ void copy_rows_of_vote(const hkv_table_view& v, uint32_t vote,
                                                  uint64_t first_slot, uint8_t* out,
                                                  uint32_t lane) {
  const uint32_t n = v.value_bytes / sizeof(U);
  const uint32_t total = __popc(vote) * n;
  for (uint32_t x = lane; x < total; x += 32) {
    const uint32_t rank = x / n;
    const uint32_t e = x - rank * n;
    const uint64_t slot = first_slot + __fns(vote, 0, static_cast<int>(rank) + 1);
    reinterpret_cast<U*>(out + rank * uint64_t{v.value_bytes})[e] =
        reinterpret_cast<const U*>(row_of(v, slot))[e];
  }
}

template <class K, class V, class S, class Pred>
__global__ void export_if_kernel(hkv_table_view v, Pred pred, uint64_t offset, uint64_t n,
                                 unsigned long long* counter, K* keys, V* values,
                                 S* scores) {
  __shared__ uint32_t warp_cnt[32];
  __shared__ unsigned long long block_base;
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t wi = threadIdx.x >> 5;
  const uint64_t end = n;  // n is already clamped to the capacity
  // the loop runs block-uniformly so that the ballots and barriers see every
  // thread
  for (uint64_t c0 = uint64_t{blockIdx.x} * blockDim.x; c0 < end;
       c0 += uint64_t{gridDim.x} * blockDim.x) {
    const uint64_t i = c0 + threadIdx.x;
    bool hit = false;
    uint64_t slot = 0, key = 0;
    if (i < end) {
      slot = offset + i;
      key = v.keys[slot];
      if (!reserved(key))
        hit = call_v2(pred, static_cast<K>(key), reinterpret_cast<const V*>(row_of(v, slot)),
                      static_cast<S>(v.scores[slot]));
    }
    const uint32_t mask = __ballot_sync(0xFFFFFFFFu, hit);
    if (lane == 0) warp_cnt[wi] = __popc(mask);
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t total = 0;
      for (uint32_t j = 0; j < blockDim.x / 32; j++) total += warp_cnt[j];
      block_base = total ? atomicAdd(counter, static_cast<unsigned long long>(total)) : 0;
    }
    __syncthreads();
    unsigned long long at = block_base;
    for (uint32_t j = 0; j < wi; j++) at += warp_cnt[j];
    if (hit) {
      const uint64_t o = at + __popc(mask & ((1u << lane) - 1));
      keys[o] = static_cast<K>(key);
      if (scores != nullptr) scores[o] = static_cast<S>(v.scores[slot]);
    }
    if (values != nullptr && mask) {
      uint8_t* out = reinterpret_cast<uint8_t*>(values) + at * v.value_bytes;
      const uint64_t first = offset + c0 + wi * 32;
      // rows sit at value_bytes strides from allocation-aligned slice bases
      const uintptr_t al = reinterpret_cast<uintptr_t>(values) | v.value_bytes;
      if ((al & 15) == 0)
        copy_rows_of_vote<uint4>(v, mask, first, out, lane);
      else if ((al & 3) == 0)
        copy_rows_of_vote<uint32_t>(v, mask, first, out, lane);
      else
        copy_rows_of_vote<uint8_t>(v, mask, first, out, lane);
    }
    __syncthreads();  // warp_cnt and block_base are rewritten next chunk
  }
}

// size_if (reference size_if_kernel.h): matching live slots counted into
// *counter (zeroed by the caller).
template <class K, class V, class S, class Pred>
__global__ void size_if_kernel(hkv_table_view v, Pred pred, unsigned long long* counter) {
  const uint64_t nthreads = uint64_t{gridDim.x} * blockDim.x;
  unsigned long long mine = 0;
  for (uint64_t slot = uint64_t{blockIdx.x} * blockDim.x + threadIdx.x; slot < v.capacity;
       slot += nthreads) {
    const uint64_t key = v.keys[slot];
    if (!reserved(key) &&
        call_v2(pred, static_cast<K>(key), reinterpret_cast<const V*>(row_of(v, slot)),
                static_cast<S>(v.scores[slot])))
      mine++;
  }
  for (int o = 16; o > 0; o >>= 1) mine += __shfl_xor_sync(0xFFFFFFFFu, mine, o);
  if ((threadIdx.x & 31) == 0 && mine) atomicAdd(counter, mine);
}

// for_each (reference traverse_kernel.h): f(key, value row, score) on every
// slot of [first, first + n), reserved keys included (the functor decides).
template <class K, class V, class S, class F>
__global__ void for_each_kernel(hkv_table_view v, uint64_t first, uint64_t n, F f) {
  const uint64_t nthreads = uint64_t{gridDim.x} * blockDim.x;
  for (uint64_t i = uint64_t{blockIdx.x} * blockDim.x + threadIdx.x; i < n; i += nthreads) {
    const uint64_t slot = first + i;
    call_v2(f, static_cast<K>(v.keys[slot]), reinterpret_cast<V*>(row_of(v, slot)),
            reinterpret_cast<S*>(v.scores + slot));
  }
}

inline int grid_for(uint64_t work) {
  const uint64_t g = (work + 255) / 256;
  return static_cast<int>(g < 148 * 16 ? (g ? g : 1) : 148 * 16);
}

}  // namespace scan
}  // namespace hkv_b200

#endif /* HKV_B200_SCAN_CUH_ */
