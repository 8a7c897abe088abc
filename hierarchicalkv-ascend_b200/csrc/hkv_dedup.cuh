// hkv_dedup.cuh -- merging duplicate keys of one batch.
//
// Insert-like calls with unique_key=false, and the sharded table, first
// collapse each batch to one representative per distinct key. The scratch
// is an open-addressing set of 2^k >= 2n slots (key, smallest input index).
// Representatives are numbered in order of first occurrence (a prefix sum),
// so the merged batch is deterministic.
#pragma once

#include "hkv_device.cuh"

namespace hkvb {

constexpr uint32_t kNoIndex = 0xFFFFFFFFu;

struct DedupView {
  uint64_t* set_keys;   // [cap] EMPTY_KEY when free
  uint32_t* set_first;  // [cap] smallest input index holding that key
  uint32_t* set_last;   // [cap] largest input index holding that key (nullptr:
                        // not needed, the last occurrence is never used)
  unsigned long long* set_sum;  // [cap] summed scores (score_mode kScoreSum*)
  uint64_t cap;         // power of two
};

// How the scores of one key's occurrences merge: Lfu sums them (a hit adds
// every occurrence's score, score_functor.h:157-160); EpochLfu sums their
// low 32 bits and saturates (:297-309); the other rules keep the last
// occurrence's score (each later occurrence overwrites, :431-455).
enum DedupScoreMode : int { kScoreNone = 0, kScoreLast = 1, kScoreSum = 2, kScoreSumLow32 = 3 };

__host__ __device__ inline int dedup_score_mode(int strategy, bool has_scores) {
  if (!has_scores) return kScoreNone;
  if (strategy == kLfu) return kScoreSum;
  if (strategy == kEpochLfu) return kScoreSumLow32;
  return kScoreLast;
}

// Stage 1 merges each block's chunk of the batch in shared memory first, so
// a key repeated across the batch (a hot key of a power-law stream) costs one
// global set update per block instead of one per occurrence; then every
// distinct key of the chunk is entered in the global set with the chunk's
// smallest and largest index (and its summed score). slot_of[i] = the key's
// global set slot (kNoIndex for reserved keys, which the table ignores).
constexpr int kDedupThreads = 256;
constexpr int kDedupPerThread = 4;
constexpr int kDedupChunk = kDedupThreads * kDedupPerThread;
constexpr int kDedupLocal = 2 * kDedupChunk;  // local set at load factor <= 0.5

__device__ __forceinline__ uint64_t dedup_hash(uint64_t key) {
  return murmur3(key ^ 0x9E3779B97F4A7C15ull);
}

__global__ void __launch_bounds__(kDedupThreads)
dedup_insert_kernel(DedupView d, const uint64_t* __restrict__ keys, uint64_t n,
                    const uint64_t* __restrict__ scores, int score_mode,
                    uint32_t* __restrict__ slot_of, int* error) {
  __shared__ uint64_t lkey[kDedupLocal];
  __shared__ uint32_t lfirst[kDedupLocal];  // after the global phase: global slot
  __shared__ uint32_t llast[kDedupLocal];
  __shared__ unsigned long long lsum[kDedupLocal];
  const bool sum = score_mode >= kScoreSum;
  for (uint64_t c0 = uint64_t{blockIdx.x} * kDedupChunk; c0 < n;
       c0 += uint64_t{gridDim.x} * kDedupChunk) {
    for (int l = threadIdx.x; l < kDedupLocal; l += kDedupThreads) {
      lkey[l] = kEmptyKey;
      lfirst[l] = kNoIndex;
      llast[l] = 0;
      lsum[l] = 0;
    }
    __syncthreads();
    uint32_t mine[kDedupPerThread];
#pragma unroll
    for (int j = 0; j < kDedupPerThread; j++) {
      const uint64_t i = c0 + static_cast<uint64_t>(j) * kDedupThreads + threadIdx.x;
      mine[j] = kNoIndex;
      if (i >= n) continue;
      const uint64_t key = keys[i];
      if (is_reserved(key)) continue;
      uint32_t l = static_cast<uint32_t>(dedup_hash(key)) & (kDedupLocal - 1);
      // at most kDedupChunk distinct keys in 2x slots: a free or matching
      // slot is always found within kDedupLocal probes
      for (int probe = 0; probe < kDedupLocal; probe++) {
        const unsigned long long old = atomicCAS(
            reinterpret_cast<unsigned long long*>(lkey + l), kEmptyKey, key);
        if (old == kEmptyKey || old == key) break;
        l = (l + 1) & (kDedupLocal - 1);
      }
      mine[j] = l;
      atomicMin(lfirst + l, static_cast<uint32_t>(i));
      atomicMax(llast + l, static_cast<uint32_t>(i));
      if (sum) {
        const uint64_t sc = score_mode == kScoreSumLow32 ? (scores[i] & 0xFFFFFFFFull)
                                                         : scores[i];
        atomicAdd(lsum + l, static_cast<unsigned long long>(sc));
      }
    }
    __syncthreads();
    for (int l = threadIdx.x; l < kDedupLocal; l += kDedupThreads) {
      const uint64_t key = lkey[l];
      if (key == kEmptyKey) continue;
      uint64_t g = dedup_hash(key) & (d.cap - 1);
      uint32_t res = kNoIndex;
      for (uint64_t probe = 0; probe < d.cap; probe++) {
        // a plain L2 read first: a key already entered by another block
        // needs no CAS (a stale EMPTY only costs the CAS below)
        uint64_t cur = __ldcg(d.set_keys + g);
        if (cur == kEmptyKey) cur = cas_u64(d.set_keys + g, kEmptyKey, key);
        if (cur == kEmptyKey || cur == key) {
          res = static_cast<uint32_t>(g);
          break;
        }
        g = (g + 1) & (d.cap - 1);
      }
      if (res == kNoIndex) {
        atomicOr(error, kErrSpinTimeout);  // set full: cannot happen at 2x
      } else {
        atomicMin(d.set_first + res, lfirst[l]);
        if (d.set_last != nullptr) atomicMax(d.set_last + res, llast[l]);
        if (sum) atomicAdd(d.set_sum + res, lsum[l]);
      }
      lfirst[l] = res;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kDedupPerThread; j++) {
      const uint64_t i = c0 + static_cast<uint64_t>(j) * kDedupThreads + threadIdx.x;
      if (i < n) slot_of[i] = mine[j] == kNoIndex ? kNoIndex : lfirst[mine[j]];
    }
    __syncthreads();  // the next chunk re-initialises the local set
  }
}

// ---- Stage 2: exclusive prefix count of first occurrences (three passes) ---
constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;

__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v,
                                                         uint32_t* total) {
  __shared__ uint32_t warp_sums[kScanThreads / 32];
  const uint32_t lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, o);
    if (lane >= static_cast<uint32_t>(o)) x += y;
  }
  if (lane == 31) warp_sums[w] = x;
  __syncthreads();
  if (w == 0) {
    uint32_t s = lane < kScanThreads / 32 ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, s, o);
      if (lane >= static_cast<uint32_t>(o)) s += y;
    }
    if (lane < kScanThreads / 32) warp_sums[lane] = s;
  }
  __syncthreads();
  const uint32_t before = (w > 0 ? warp_sums[w - 1] : 0) + x - v;
  *total = warp_sums[kScanThreads / 32 - 1];
  __syncthreads();
  return before;
}

// pass 1 of the merge's scan with the flags computed in place: input i
// counts 1 iff it is its key's first occurrence (the set holds the key's
// smallest index); rank[i] = the exclusive count before i within the tile
__global__ void __launch_bounds__(kScanThreads)
    scan_first_tiles_kernel(DedupView d, const uint32_t* __restrict__ slot_of, uint64_t n,
                            uint32_t* __restrict__ rank, uint32_t* __restrict__ sums) {
  const uint64_t base = blockIdx.x * (uint64_t)kScanTile + threadIdx.x * kScanItems;
  uint32_t v[kScanItems], acc = 0;
#pragma unroll
  for (int j = 0; j < kScanItems; j++) {
    const uint64_t i = base + j;
    uint32_t f = 0;
    if (i < n) {
      const uint32_t s = slot_of[i];
      f = (s != kNoIndex && d.set_first[s] == static_cast<uint32_t>(i)) ? 1u : 0u;
    }
    v[j] = f;
    acc += f;
  }
  uint32_t total;
  uint32_t run = block_exclusive_scan(acc, &total);
#pragma unroll
  for (int j = 0; j < kScanItems; j++) {
    if (base + j < n) rank[base + j] = run;
    run += v[j];
  }
  if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

// pass 2: exclusive scan of the tile totals (one block); grand total in *total
__global__ void __launch_bounds__(kScanThreads)
    scan_sums_kernel(uint32_t* __restrict__ sums, uint64_t nt,
                     uint32_t* __restrict__ total_out) {
  uint32_t carry = 0;
  for (uint64_t b = 0; b < nt; b += kScanThreads) {
    const uint64_t i = b + threadIdx.x;
    const uint32_t v = i < nt ? sums[i] : 0u;
    uint32_t tot;
    const uint32_t ex = block_exclusive_scan(v, &tot);
    if (i < nt) sums[i] = carry + ex;
    carry += tot;
  }
  if (threadIdx.x == 0) *total_out = carry;
}

// pass 3: add tile offsets
__global__ void __launch_bounds__(kScanThreads)
    scan_add_kernel(uint32_t* __restrict__ data, uint64_t n,
                    const uint32_t* __restrict__ sums) {
  const uint64_t base = blockIdx.x * (uint64_t)kScanTile;
  const uint32_t add = sums[blockIdx.x];
  for (int j = threadIdx.x; j < kScanTile; j += kScanThreads)
    if (base + j < n) data[base + j] += add;
}

// Stage 3: representatives and the inverse map. Every input i gets
// uid_of[i] = the representative number of its key, which is the scanned
// rank of the key's first occurrence (kNoIndex for reserved inputs); for a
// first occurrence i with rank u: ukeys[u] = key, rep_first[u] = i,
// rep_last[u] = the key's last index, uscores[u] = its merged score
// (score_mode).
__global__ void dedup_emit_kernel(DedupView d, const uint64_t* __restrict__ keys,
                                  const uint32_t* __restrict__ slot_of,
                                  const uint32_t* __restrict__ rank, uint64_t n,
                                  uint64_t* __restrict__ ukeys,
                                  uint32_t* __restrict__ rep_first,
                                  uint32_t* __restrict__ rep_last,
                                  const uint64_t* __restrict__ scores, int score_mode,
                                  uint64_t* __restrict__ uscores,
                                  uint32_t* __restrict__ uid_of) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t s = slot_of[i];
    if (s == kNoIndex) {
      uid_of[i] = kNoIndex;
      continue;
    }
    const uint32_t f = d.set_first[s];
    const uint32_t u = rank[f];
    uid_of[i] = u;
    if (f != static_cast<uint32_t>(i)) continue;
    const uint32_t last = d.set_last != nullptr ? d.set_last[s] : 0u;
    ukeys[u] = keys[i];
    rep_first[u] = static_cast<uint32_t>(i);
    if (rep_last) rep_last[u] = last;
    if (score_mode == kScoreLast) {
      uscores[u] = scores[last];
    } else if (score_mode == kScoreSum) {
      uscores[u] = d.set_sum[s];
    } else if (score_mode == kScoreSumLow32) {
      const uint64_t t = d.set_sum[s];
      uscores[u] = t > 0xFFFFFFFFull ? 0xFFFFFFFFull : t;
    }
  }
}

// find_or_insert scatter: the representatives found or inserted their keys
// in place (at their first occurrence's row); every later occurrence reads
// its representative's row. values is both source and destination (a source
// row is a first occurrence, never a destination). A warp resolves 32
// consecutive occurrences at once, lists the ones that copy, and moves their
// rows 32 / nv at a time (nv vectors per row), four rows in flight per lane.
template <int VW>
__global__ void __launch_bounds__(256)
    scatter_found_rows_kernel(uint8_t* values, const uint32_t* __restrict__ uid_of,
                              const uint32_t* __restrict__ rep_first,
                              const uint8_t* __restrict__ ustatus, uint64_t n, uint32_t vb) {
  using V = typename VecOf<VW>::T;
  __shared__ uint8_t lst[8][32];  // blockDim.x == 256: 8 warps
  const uint32_t nv = vb / VW;
  const uint32_t lane = threadIdx.x & 31, wi = threadIdx.x >> 5;
  const uint64_t warp = (blockIdx.x * uint64_t{blockDim.x} + threadIdx.x) >> 5;
  const uint64_t nwarps = uint64_t{gridDim.x} * (blockDim.x >> 5);
  for (uint64_t base = warp * 32; base < n; base += nwarps * 32) {
    const uint64_t i = base + lane;
    uint32_t src = kNoIndex;
    if (i < n) {
      const uint32_t u = uid_of[i];
      if (u != kNoIndex) {
        const uint32_t f = rep_first[u];
        const uint8_t st = ustatus[u];
        if (f != static_cast<uint32_t>(i) && st != kRefused && st != kIllegal &&
            st != kTimedOut)
          src = f;
      }
    }
    const uint32_t todo = __ballot_sync(0xFFFFFFFFu, src != kNoIndex);
    if (src != kNoIndex) lst[wi][__popc(todo & ((1u << lane) - 1))] = static_cast<uint8_t>(lane);
    __syncwarp();
    const uint32_t cnt = __popc(todo);
    if (nv <= 32) {
      const uint32_t rpi = 32 / nv, lq = lane / nv, lv = lane - lq * nv;
      for (uint32_t k0 = 0; k0 < cnt; k0 += 4 * rpi) {
        V x[4];
        uint32_t rr[4];
        bool ok[4];
#pragma unroll
        for (uint32_t u = 0; u < 4; u++) {
          const uint32_t k = k0 + u * rpi + lq;
          ok[u] = lq < rpi && k < cnt;
          rr[u] = ok[u] ? lst[wi][k] : 0u;
          const uint32_t sr = __shfl_sync(0xFFFFFFFFu, src, rr[u]);
          if (ok[u]) x[u] = reinterpret_cast<const V*>(values + uint64_t{sr} * vb)[lv];
        }
#pragma unroll
        for (uint32_t u = 0; u < 4; u++)
          if (ok[u]) reinterpret_cast<V*>(values + (base + rr[u]) * vb)[lv] = x[u];
      }
    } else {
      for (uint32_t k = 0; k < cnt; k++) {
        const uint32_t r = lst[wi][k];
        const uint32_t sr = __shfl_sync(0xFFFFFFFFu, src, r);
        const V* sp = reinterpret_cast<const V*>(values + uint64_t{sr} * vb);
        V* dp = reinterpret_cast<V*>(values + (base + r) * vb);
        for (uint32_t v = lane; v < nv; v += 32) dp[v] = sp[v];
      }
    }
    __syncwarp();  // the next pass rewrites the list
  }
}

// insert_and_evict scatter: every occurrence of a refused representative is
// reported with its own key, value and desired score (each duplicate is
// refused on its own in the reference, insert_and_evict_kernel.h:291-303).
template <int S, int VW>
__global__ void scatter_refused_kernel(const uint64_t* __restrict__ keys,
                                       const uint8_t* __restrict__ values,
                                       const uint64_t* __restrict__ scores,
                                       const uint32_t* __restrict__ uid_of,
                                       const uint8_t* __restrict__ ustatus,
                                       uint64_t n, uint32_t vb, uint64_t epoch,
                                       uint64_t* __restrict__ ev_keys,
                                       uint8_t* __restrict__ ev_values,
                                       uint64_t* __restrict__ ev_scores,
                                       unsigned long long* __restrict__ counter) {
  __shared__ uint64_t s_clock;
  if (threadIdx.x == 0) s_clock = global_timer_ns();
  __syncthreads();
  const Tile tile;
  const uint64_t ntiles = (uint64_t)gridDim.x * (blockDim.x / kTile);
  for (uint64_t i = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) / kTile;
       i < n; i += ntiles) {
    const uint32_t u = uid_of[i];
    if (u == kNoIndex || ustatus[u] != kRefused) continue;
    unsigned long long o = 0;
    if (tile.lane == 0) {
      o = atomicAdd(counter, 1ull);
      ev_keys[o] = keys[i];
      if (ev_scores)
        ev_scores[o] = desired_when_missed<S>(scores, i, epoch, s_clock);
    }
    o = tile.shfl(o, 0);
    copy_row<VW>(ev_values + o * vb, values + i * vb, vb, tile.lane, kTile);
  }
}

// status[i] = ustatus[uid_of[i]] (kIllegal for reserved inputs).
__global__ void expand_status_kernel(const uint8_t* __restrict__ ustatus,
                                     const uint32_t* __restrict__ uid_of,
                                     uint64_t n, uint8_t* __restrict__ status) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t u = uid_of[i];
    status[i] = u == kNoIndex ? static_cast<uint8_t>(kIllegal) : ustatus[u];
  }
}

// find_or_insert* with repeated keys: every occurrence gets its
// representative's row address; the first occurrence reports whether the
// key was there before, later ones find it if the first got a slot.
__global__ void scatter_ptrs_kernel(uint8_t** __restrict__ value_ptrs,
                                    bool* __restrict__ founds,
                                    uint8_t* const* __restrict__ uptrs,
                                    const bool* __restrict__ ufound,
                                    const uint32_t* __restrict__ uid_of,
                                    const uint32_t* __restrict__ rep_first,
                                    uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t u = uid_of[i];
    uint8_t* p = u != 0xFFFFFFFFu ? uptrs[u] : nullptr;
    value_ptrs[i] = p;
    if (founds != nullptr)
      founds[i] = u != 0xFFFFFFFFu && (rep_first[u] == i ? ufound[u] : p != nullptr);
  }
}

}  // namespace hkvb
