// hkv_device.cuh -- device-side primitives of the B200 HierarchicalKV table.
//
// HBM layout (slot s = bucket * 128 + position):
//   digests [buckets][128] u8   one 128-byte line per bucket
//   keys    [buckets][128] u64  1 KiB per bucket
//   scores  [buckets][128] u64  1 KiB per bucket
//   sizes   [buckets]      i32
//   values  slices of 2^slice_shift buckets, [bucket][128][value_bytes]; a
//           slice is HBM or mapped pinned host memory.
// A key's bucket, start position and digest come from the Murmur3 finalizer
// (reference utils.h:64-72, types.h:97-136, find_with_digest_kernel.h:57-64).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace hkvb {

constexpr uint32_t kBucket = 128;       // slots per bucket
constexpr uint32_t kTile = 8;           // lanes cooperating on one key
constexpr uint32_t kDigestsPerLane = kBucket / kTile;  // 16 -> one uint4
constexpr uint32_t kBucketShift = 7;

// Reserved keys, reference types.h:63-70.
constexpr uint64_t kEmptyKey = 0xFFFFFFFFFFFFFFFFull;
constexpr uint64_t kReclaimKey = 0xFFFFFFFFFFFFFFFEull;
constexpr uint64_t kLockedKey = 0xFFFFFFFFFFFFFFFDull;
// A key word a caller holds locked across calls (lock_keys, find_or_insert*
// with locked_key_ptrs): the fourth reserved value, so that the kernels can
// tell a caller's lock from the short lock of an operation in flight.
constexpr uint64_t kUserLockedKey = 0xFFFFFFFFFFFFFFFCull;
// A bucket's size word: live slots in the low 16 bits, the slots a caller
// holds locked above them (read together, so the probe pays nothing for it).
constexpr int32_t kSizeMask = 0xFFFF;
constexpr int kLockShift = 16;
constexpr uint64_t kReservedMask = 0xFFFFFFFFFFFFFFFCull;
constexpr uint64_t kMaxScore = 0xFFFFFFFFFFFFFFFFull;
constexpr uint64_t kIgnoredEpoch = 0xFFFFFFFFFFFFFFFFull;

enum Strategy : int { kLru = 0, kLfu = 1, kEpochLru = 2, kEpochLfu = 3, kCustomized = 4 };

// Outcome of an insert-like key (reference OccupyResult, types.h:250-259).
enum Occupy : int {
  kIllegal = 0,
  kDuplicate = 1,
  kOccupiedEmpty = 2,
  kOccupiedReclaimed = 3,
  kEvict = 4,
  kRefused = 5,
  kTimedOut = 6,
};

// Device error word bits.
// Up to kMaxSegments key arrays looked up in one launch (the sharded table's
// per-requester regions), each with its own outputs. Result j of segment k
// goes to values[k] + j * row_stride, founds[k] + j * flag_stride (one
// byte, 0/1) and scores[k] + j * score_stride (8 bytes), so results can be
// packed as records.
constexpr uint32_t kMaxSegments = 64;
struct FindSegments {
  const uint64_t* keys[kMaxSegments];
  uint8_t* values[kMaxSegments];
  uint8_t* founds[kMaxSegments];
  uint8_t* scores[kMaxSegments];
  uint32_t row_stride, flag_stride, score_stride;
};

enum UpsertMode : int {
  kModeInsertOrAssign = 0,
  kModeFindOrInsert = 1,
  kModeInsertAndEvict = 2,
  kModeFindOrInsertPtr = 3  // find_or_insert* : row addresses, no value copy
};

constexpr int kErrSpinTimeout = 1;
constexpr int kErrBounds = 2;  // only raised by builds with HKV_CHECK_BOUNDS
constexpr int kErrPeerOverflow = 4;  // a sharded batch overflowed a peer inbox

// Murmur3 64-bit finalizer (reference utils.h:64-72).
__host__ __device__ constexpr uint64_t murmur3(uint64_t k) {
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdull;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ull;
  k ^= k >> 33;
  return k;
}

__host__ __device__ constexpr uint8_t digest_of_hash(uint64_t h) {
  return static_cast<uint8_t>(h >> 32);
}

// empty_digest / reclaim_digest (reference types.h:97-107) are constants.
constexpr uint8_t kEmptyDigest = digest_of_hash(murmur3(kEmptyKey));
constexpr uint8_t kReclaimDigest = digest_of_hash(murmur3(kReclaimKey));

__host__ __device__ __forceinline__ bool is_reserved(uint64_t k) {
  return (k & kReservedMask) == kReservedMask;
}

// POD view of one table handed to every kernel by value.
struct TableView {
  uint64_t* keys;
  uint64_t* scores;
  uint8_t* digests;
  int32_t* sizes;          // per bucket: live slots (low 16 bits) and slots a
                           // caller holds locked (bits 16 and up)
  uint8_t* const* slices;  // device array of slice base pointers
  uint8_t* values0;        // slice 0 (used directly when single_slice)
  int* error;              // device error word
  uint64_t capacity;       // buckets * 128
  uint64_t num_buckets;
  uint64_t div_magic;      // capacity division (reference table.h:106-127)
  uint32_t div_shift;
  uint32_t cap_pow2;       // capacity is a power of two: mod is a mask
  uint32_t slice_shift;    // log2(buckets per slice)
  uint32_t single_slice;
  uint32_t value_bytes;    // dim * sizeof(V)
  uint32_t num_slices;
};

// Self-checking builds (-DHKV_CHECK_BOUNDS) verify every table index before
// use; a bad index raises kErrBounds, records a site code in error[1] and the
// access is redirected to slot 0 of bucket 0 instead of faulting.
#ifdef HKV_CHECK_BOUNDS
#define HKV_BOUND(t, cond, site)                   \
  ((cond) ? true                                   \
          : (atomicOr((t).error, kErrBounds),      \
             atomicExch((t).error + 1, (site)), false))
#else
#define HKV_BOUND(t, cond, site) true
#endif

// hashed % capacity by the round-up magic-number method the reference uses
// (Granlund & Montgomery; reference utils.h:85-97, table.h:106-127).
__device__ __forceinline__ uint64_t global_index(const TableView& t,
                                                 uint64_t h) {
  if (t.cap_pow2) return h & (t.capacity - 1);
  uint64_t q = __umul64hi(h, t.div_magic);
  uint64_t x = ((h - q) >> 1) + q;
  return h - (x >> t.div_shift) * t.capacity;
}

__device__ __forceinline__ uint8_t* value_ptr(const TableView& t, uint64_t bkt,
                                              uint32_t pos) {
  if (!HKV_BOUND(t, bkt < t.num_buckets && pos < kBucket, 11)) {
    bkt = 0;
    pos = 0;
  }
  if (!t.single_slice &&
      !HKV_BOUND(t, (bkt >> t.slice_shift) < t.num_slices, 12))
    bkt = 0;
  uint8_t* base;
  uint64_t local;
  if (t.single_slice) {
    base = t.values0;
    local = bkt;
  } else {
    base = t.slices[bkt >> t.slice_shift];
    local = bkt & ((1ull << t.slice_shift) - 1);
  }
  return base + (local * kBucket + pos) * static_cast<uint64_t>(t.value_bytes);
}

// ---- clocks and bounded waits ---------------------------------------------
__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Every spin on a lock gives up after this long and raises kErrSpinTimeout.
constexpr uint64_t kSpinLimitNs = 1000000000ull;  // 1 s

__device__ __forceinline__ void backoff(int round) {
  __nanosleep(round < 8 ? 32u : 256u);
}

// ---- relaxed global loads that bypass L1 (tables change under us) --------
__device__ __forceinline__ uint64_t ld_cg_u64(const uint64_t* p) {
  return __ldcg(reinterpret_cast<const unsigned long long*>(p));
}
// Output position for a counter shared by the whole grid: the lanes of a
// warp that call this together take consecutive positions with one atomic
// (one per warp instead of one per lane on a single hot word).
__device__ __forceinline__ unsigned long long warp_claim(unsigned long long* counter) {
  const uint32_t act = __activemask();
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t leader = __ffs(act) - 1;
  unsigned long long base = 0;
  if (lane == leader) base = atomicAdd(counter, static_cast<unsigned long long>(__popc(act)));
  base = __shfl_sync(act, base, leader);
  return base + __popc(act & ((1u << lane) - 1));
}

// A strong load at GPU scope (table words are only written by kernels on
// the table's own GPU). A C++ volatile load would be relaxed at system scope,
// which after an acquire on the same slot measured ~10x slower per key.
__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t cas_u64(uint64_t* p, uint64_t expect,
                                            uint64_t desired) {
  return atomicCAS(reinterpret_cast<unsigned long long*>(p), expect, desired);
}
__device__ __forceinline__ uint64_t exch_u64(uint64_t* p, uint64_t v) {
  return atomicExch(reinterpret_cast<unsigned long long*>(p), v);
}
// Flags written and read across GPUs (peer memory over NVLink): system scope.
__device__ __forceinline__ uint64_t ld_acquire_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Exchange with acquire semantics at GPU scope (victim locking: swapping
// LOCKED_KEY in returns the key that was there in the same round trip).
__device__ __forceinline__ uint64_t exch_acquire_u64(uint64_t* p, uint64_t v) {
  uint64_t old;
  asm volatile("atom.acquire.gpu.global.exch.b64 %0, [%1], %2;"
               : "=l"(old)
               : "l"(p), "l"(v)
               : "memory");
  return old;
}
// Lock acquisition: CAS with acquire semantics at GPU scope, so the slot's
// contents written before its last release are visible to the winner.
__device__ __forceinline__ uint64_t cas_acquire_u64(uint64_t* p, uint64_t expect,
                                                    uint64_t desired) {
  uint64_t old;
  asm volatile("atom.acquire.gpu.global.cas.b64 %0, [%1], %2, %3;"
               : "=l"(old)
               : "l"(p), "l"(expect), "l"(desired)
               : "memory");
  return old;
}
// Lock release: store of the final key word with release semantics at GPU
// scope. Writes of the other lanes of the tile are ordered before it by the
// tile's __syncwarp (which orders memory among its participants) and the
// release is cumulative over them.
__device__ __forceinline__ void store_release_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v)
               : "memory");
}

// ---- byte compare of 16 digests: bit j set when byte j equals d ----------
// Exact zero-byte test of x = w ^ d4 ("determine if a word has a zero byte",
// the carry-free form from Sean Anderson's Bit Twiddling Hacks): bit 7 of
// each byte of z is set iff that byte of x is zero. The multiply by
// 2^0 + 2^7 + 2^14 + 2^21 moves bits 7, 15, 23, 31 to bits 28..31 without
// carries, giving the byte-order mask in four bits.
__device__ __forceinline__ uint32_t bytes_eq4(uint32_t w, uint32_t d4) {
  const uint32_t x = w ^ d4;
  const uint32_t z = ~(((x & 0x7F7F7F7Fu) + 0x7F7F7F7Fu) | x | 0x7F7F7F7Fu);
  return (z * 0x00204081u) >> 28;
}
__device__ __forceinline__ uint32_t bytes_eq16(uint4 v, uint32_t d4) {
  return bytes_eq4(v.x, d4) | (bytes_eq4(v.y, d4) << 4) |
         (bytes_eq4(v.z, d4) << 8) | (bytes_eq4(v.w, d4) << 12);
}

// ---- tile helpers (8 consecutive lanes of a warp) ---------------------------
struct Tile {
  uint32_t lane;   // 0..7
  uint32_t mask;   // warp mask of this tile
  uint32_t shift;  // bit offset of this tile in a warp ballot
  __device__ __forceinline__ Tile() {
    uint32_t wl = threadIdx.x & 31;
    lane = wl & (kTile - 1);
    shift = wl & ~(kTile - 1);
    mask = 0xFFu << shift;
  }
  __device__ __forceinline__ uint32_t ballot(bool p) const {
    return (__ballot_sync(mask, p) >> shift) & 0xFFu;
  }
  template <class T>
  __device__ __forceinline__ T shfl(T v, int src) const {
    return __shfl_sync(mask, v, src, kTile);
  }
  template <class T>
  __device__ __forceinline__ T shfl_xor(T v, int o) const {
    return __shfl_xor_sync(mask, v, o, kTile);
  }
  __device__ __forceinline__ void sync() const { __syncwarp(mask); }
};

// A tile of W consecutive lanes (W = 2, 4 or 8) sharing one key; each lane
// holds kBucket / W of the bucket's digests.
template <uint32_t W>
struct TileW {
  static constexpr uint32_t kWidth = W;
  static constexpr uint32_t kDigests = kBucket / W;
  uint32_t lane, mask, shift;
  __device__ __forceinline__ TileW() {
    const uint32_t wl = threadIdx.x & 31;
    lane = wl & (W - 1);
    shift = wl & ~(W - 1);
    mask = ((1u << W) - 1) << shift;
  }
  __device__ __forceinline__ uint32_t ballot(bool p) const {
    return (__ballot_sync(mask, p) >> shift) & ((1u << W) - 1);
  }
  template <class T>
  __device__ __forceinline__ T shfl(T v, int src) const {
    return __shfl_sync(mask, v, src, W);
  }
  template <class T>
  __device__ __forceinline__ T shfl_xor(T v, int o) const {
    return __shfl_xor_sync(mask, v, o, W);
  }
  __device__ __forceinline__ void sync() const { __syncwarp(mask); }
};

// ---- probe order ------------------------------------------------------------
// The reference walks a bucket in groups of 4 slots starting at the group of
// the key's start position `pos` (find_utils.h:40-84). Within a group digest
// hits are examined before empty slots; an empty slot before `pos` in the
// first group is only examined after the walk wraps around. These ranks give
// that order: a digest hit at p precedes an empty slot at e iff
// hit_rank(p) < empty_rank(e).
__device__ __forceinline__ uint32_t group_index(uint32_t p, uint32_t pos) {
  return ((p >> 2) - (pos >> 2)) & (kBucket / 4 - 1);
}
__device__ __forceinline__ uint32_t hit_rank(uint32_t p, uint32_t pos) {
  return group_index(p, pos) * 2;
}
__device__ __forceinline__ uint32_t empty_rank(uint32_t p, uint32_t pos) {
  uint32_t g = group_index(p, pos);
  if (g == 0 && p < pos) g = kBucket / 4;
  return g * 2 + 1;
}
// Linear order from pos (claiming empty slots): rank = (p - pos) mod B.
__device__ __forceinline__ uint32_t linear_rank(uint32_t p, uint32_t pos) {
  return (p - pos) & (kBucket - 1);
}

// Bits j of the kD slots [lo, lo + kD) held by one lane whose slot lo + j
// has linear rank from pos below L (0 <= L <= kBucket). The ranks of the
// window rise by one per slot and wrap to 0 once, after w = kBucket - a
// slots, a being the rank of slot lo.
template <class M, uint32_t kD>
__device__ __forceinline__ M linear_below(uint32_t lo, uint32_t pos, uint32_t L) {
  auto low = [](uint32_t c) -> uint64_t { return c >= 64 ? ~0ull : ((1ull << c) - 1); };
  const uint32_t a = (lo - pos) & (kBucket - 1);
  const uint32_t w = kBucket - a;
  const uint32_t c1 = L > a ? min(L - a, w) : 0u;
  const uint64_t m = low(c1) | (low(min(w + L, kD)) & ~low(w));
  return static_cast<M>(m & low(kD));
}

// Linear rank bound of the empty slots the group walk reaches before a digest
// hit at p: the slots from pos up to p's group, none when p is in the start
// group (hits of a group come before its empties, find_utils.h:40-84 and
// insert_or_assign_kernel.h:105-183). empty_rank(q) < hit_rank(p) exactly
// when q's linear rank is below this bound.
__device__ __forceinline__ uint32_t walk_bound(uint32_t p, uint32_t pos) {
  return group_index(p, pos) == 0 ? 0u : linear_rank(p & ~3u, pos);
}

// ---- score rules (reference score_functor.h) --------------------------------
__device__ __forceinline__ uint64_t make_epoch(uint64_t e) { return e << 32; }
__device__ __forceinline__ uint64_t make_nano(uint64_t c) {
  return 0xFFFFFFFFull & (c >> 20);
}

// desired_when_missed, score_functor.h:50, :116, :215, :286, :410.
template <int S>
__device__ __forceinline__ uint64_t desired_when_missed(const uint64_t* in,
                                                        uint64_t idx,
                                                        uint64_t epoch,
                                                        uint64_t clk) {
  if constexpr (S == kLru) {
    return clk;
  } else if constexpr (S == kLfu) {
    return kMaxScore;
  } else if constexpr (S == kEpochLru) {
    if (epoch == kIgnoredEpoch && in != nullptr) return in[idx];
    return make_epoch(epoch) | make_nano(clk);
  } else if constexpr (S == kEpochLfu) {
    if (in == nullptr) return 0;
    if (epoch == kIgnoredEpoch) return in[idx];
    return make_epoch(epoch) | (in[idx] & 0xFFFFFFFFull);
  } else {
    return in != nullptr ? in[idx] : 0;
  }
}

// Score written on a hit (new_insert=false) or an insert (new_insert=true);
// update_score_only / update_with_digest, score_functor.h:56-84, :136-187,
// :241-268, :316-367, :431-455. Returns false when the reference writes
// nothing (Lfu without input scores).
template <int S>
__device__ __forceinline__ bool score_on_write(uint64_t old, const uint64_t* in,
                                               uint64_t idx, uint64_t desired,
                                               bool new_insert, uint64_t* out) {
  if constexpr (S == kLfu) {
    if (in == nullptr) return false;
    *out = new_insert ? in[idx] : in[idx] + old;
    return true;
  } else if constexpr (S == kEpochLfu) {
    if (new_insert) {
      *out = desired;
    } else {
      uint64_t s = old & 0xFFFFFFFFull;
      *out = (0xFFFFFFFFull - s > (desired & 0xFFFFFFFFull))
                 ? s + desired
                 : ((desired & 0xFFFFFFFF00000000ull) | 0xFFFFFFFFull);
    }
    return true;
  } else {
    *out = desired;
    return true;
  }
}

// update_without_missed (assign_scores), score_functor.h:99, :198, :270,
// :386, :466.
template <int S>
__device__ __forceinline__ bool score_without_missed(uint64_t old,
                                                     const uint64_t* in,
                                                     uint64_t idx,
                                                     uint64_t epoch,
                                                     uint64_t clk,
                                                     uint64_t* out) {
  if constexpr (S == kLru) {
    *out = clk;
    return true;
  } else if constexpr (S == kLfu) {
    if (in == nullptr) return false;
    *out = in[idx] + old;
    return true;
  } else if constexpr (S == kEpochLru) {
    *out = make_epoch(epoch) | make_nano(clk);
    return true;
  } else if constexpr (S == kEpochLfu) {
    if (in == nullptr) return false;
    uint64_t s = old & 0xFFFFFFFFull;
    uint64_t v = in[idx] & 0xFFFFFFFFull;
    *out = (0xFFFFFFFFull - s > v) ? s + (make_epoch(epoch) | v)
                                   : (make_epoch(epoch) | 0xFFFFFFFFull);
    return true;
  } else {
    if (in == nullptr) return false;
    *out = in[idx];
    return true;
  }
}

// ---- value movement -----------------------------------------------------------
// A value row is value_bytes long; VW (16, 8, 4, 2 or 1) divides value_bytes
// and the alignment of every row. `lane`/`nlanes` split the row.
template <int VW>
struct VecOf;
template <> struct VecOf<16> { using T = uint4; };
template <> struct VecOf<8> { using T = uint2; };
template <> struct VecOf<4> { using T = uint32_t; };
template <> struct VecOf<2> { using T = uint16_t; };
template <> struct VecOf<1> { using T = uint8_t; };

template <int VW>
__device__ __forceinline__ void copy_row(uint8_t* __restrict__ dst,
                                         const uint8_t* __restrict__ src,
                                         uint32_t bytes, uint32_t lane,
                                         uint32_t nlanes) {
  using V = typename VecOf<VW>::T;
  const uint32_t nv = bytes / VW;
  V* d = reinterpret_cast<V*>(dst);
  const V* s = reinterpret_cast<const V*>(src);
  for (uint32_t i = lane; i < nv; i += nlanes) d[i] = s[i];
}

// Read-only source (table rows during find, inputs) and streaming stores.
template <int VW>
__device__ __forceinline__ void copy_row_nc_cs(uint8_t* __restrict__ dst,
                                               const uint8_t* __restrict__ src,
                                               uint32_t bytes, uint32_t lane,
                                               uint32_t nlanes) {
  using V = typename VecOf<VW>::T;
  const uint32_t nv = bytes / VW;
  V* d = reinterpret_cast<V*>(dst);
  const V* s = reinterpret_cast<const V*>(src);
  for (uint32_t i = lane; i < nv; i += nlanes) __stcs(d + i, __ldg(s + i));
}

}  // namespace hkvb
