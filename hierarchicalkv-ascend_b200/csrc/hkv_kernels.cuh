// hkv_kernels.cuh -- sm_100a kernels of the HierarchicalKV hot path.
//
// One key is handled by a tile of W lanes (4 for find and the upsert family,
// 8 for the others). Each lane loads 128 / W of the bucket's 128 digests in
// 16-byte loads (the tile reads the whole 128-byte line), compares them with
// a carry-free zero-byte test, and the tile picks slots with ballots and
// shuffles. Values move in VW-byte vectors (16 bytes for float rows whose
// byte size is a multiple of 16). Locks are the key words themselves: a slot
// is owned by whoever swapped its key to LOCKED_KEY (reference types.h:65).
#pragma once

#include <cuda_bf16.h>
#include <type_traits>
#include <cuda_fp16.h>

#include "hkv_device.cuh"

namespace hkvb {

// ============================================================================
// Table initialisation and clear
// ============================================================================

// initialize_buckets key/digest/score fill (reference init_table_kernel.h
// :81-104), one launch for any bucket range. Each thread owns 16 slots.
__global__ void init_buckets_kernel(TableView t, uint64_t b0, uint64_t b1,
                                    int reset_scores) {
  const uint64_t chunks = (b1 - b0) * (kBucket / 16);
  const uint4 ek = make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu,
                              0xFFFFFFFFu);
  const uint32_t ed = kEmptyDigest * 0x01010101u;
  const uint4 ed4 = make_uint4(ed, ed, ed, ed);
  for (uint64_t c = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; c < chunks;
       c += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t s = b0 * kBucket + c * 16;
    reinterpret_cast<uint4*>(t.digests + s)[0] = ed4;
    uint4* k4 = reinterpret_cast<uint4*>(t.keys + s);
#pragma unroll
    for (int j = 0; j < 8; j++) k4[j] = ek;
    if (reset_scores) {
      uint4* s4 = reinterpret_cast<uint4*>(t.scores + s);
#pragma unroll
      for (int j = 0; j < 8; j++) s4[j] = make_uint4(0, 0, 0, 0);
    }
    if ((s & (kBucket - 1)) == 0) t.sizes[s >> kBucketShift] = 0;
  }
}

// ============================================================================
// Reductions for size() and fast_load_factor()
// ============================================================================
// Sum of sizes[0, nb) into *out (out zeroed by the caller).
// shift 0 sums the live slots, kLockShift the slots callers hold locked.
__global__ void sum_sizes_kernel(const int32_t* __restrict__ sizes, uint64_t nb,
                                 unsigned long long* out, int shift) {
  int64_t s = 0;
  for (uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; b < nb;
       b += (uint64_t)gridDim.x * blockDim.x)
    s += (sizes[b] >> shift) & kSizeMask;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  __shared__ int64_t part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    int64_t v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    if (threadIdx.x == 0) atomicAdd(out, static_cast<unsigned long long>(v));
  }
}

// ============================================================================
// Digest probe shared by the lookup kernels
// ============================================================================
struct Locate {
  uint64_t bkt;
  uint32_t pos;
  uint32_t d4;  // digest replicated into 4 bytes
};

__device__ __forceinline__ Locate locate(const TableView& t, uint64_t key) {
  const uint64_t h = murmur3(key);
  const uint64_t g = global_index(t, h);
  Locate l;
  l.bkt = g >> kBucketShift;
  if (!HKV_BOUND(t, l.bkt < t.num_buckets, 1)) l.bkt = 0;
  l.pos = static_cast<uint32_t>(g & (kBucket - 1));
  l.d4 = static_cast<uint32_t>(digest_of_hash(h)) * 0x01010101u;
  return l;
}

// ============================================================================
// find / contains (reference find_with_digest_kernel.h:33-108,
// contains_kernel.h:31-64)
//
// A tile of kFindTile lanes handles one key; each lane compares
// kBucket / kFindTile digests (one to four 16-byte loads). The key of a
// tile's next iteration is loaded one iteration ahead. Per key the tile then
// makes three dependent trips: the digest line, the keys of the digest hits
// (with the keys of the digest-empty slots ranked before the first hit),
// and the value row.
// ============================================================================
#ifndef HKV_FIND_TILE
#define HKV_FIND_TILE 4
#endif
#ifndef HKV_FIND_MIN_BLOCKS
#define HKV_FIND_MIN_BLOCKS 8
#endif
#ifndef HKV_FIND_BLOCKS_PER_SM
#define HKV_FIND_BLOCKS_PER_SM 64
#endif
constexpr uint32_t kFindBlocksPerSm = HKV_FIND_BLOCKS_PER_SM;
constexpr uint32_t kFindTile = HKV_FIND_TILE;

template <class M>
__device__ __forceinline__ uint32_t low_bit(M m) {
  if constexpr (sizeof(M) == 8)
    return static_cast<uint32_t>(__ffsll(static_cast<long long>(m)) - 1);
  else
    return static_cast<uint32_t>(__ffs(static_cast<int>(m)) - 1);
}

// The find rule of the reference (find_utils.h:31-86) for one key on one
// tile: the slot of the first digest hit holding the key in the group walk,
// unless a digest-empty slot holding EMPTY_KEY comes before it; -1 if none.
template <uint32_t W>
__device__ __forceinline__ int find_probe(const TableView& t, const TileW<W>& tile,
                                          uint64_t key, uint64_t& bkt) {
  constexpr uint32_t kD = TileW<W>::kDigests;  // digests per lane
  constexpr uint32_t kDV = kD / 16;            // 16-byte digest loads per lane
  using M = typename std::conditional<(kD > 32), uint64_t, uint32_t>::type;
  bkt = 0;
  if (is_reserved(key)) return -1;
  const Locate l = locate(t, key);
  bkt = l.bkt;
  const uint32_t lo = tile.lane * kD;
  const uint64_t* bk = t.keys + l.bkt * kBucket;
  const uint4* dl =
      reinterpret_cast<const uint4*>(t.digests + l.bkt * kBucket) + tile.lane * kDV;
  // the bucket's size word, read beside the digest line: a full bucket holds
  // no EMPTY_KEY slot, so the stop rule below cannot apply to it
  const int32_t bword = __ldg(t.sizes + l.bkt);
  M hits = 0, empt = 0;
#pragma unroll
  for (uint32_t j = 0; j < kDV; j++) {
    const uint4 dv = __ldg(dl + j);
    hits |= static_cast<M>(bytes_eq16(dv, l.d4)) << (16 * j);
    empt |= static_cast<M>(bytes_eq16(dv, kEmptyDigest * 0x01010101u)) << (16 * j);
  }
  if ((bword & kSizeMask) >= static_cast<int32_t>(kBucket)) empt = 0;
  // digest hits holding the key, best = first in the reference's walk
  uint32_t best = 0xFFFFFFFFu;
  for (M h = hits; h; h &= h - 1) {
    const uint32_t q = lo + low_bit(h);
    if (__ldg(bk + q) == key) best = min(best, (hit_rank(q, l.pos) << 8) | q);
  }
#pragma unroll
  for (int o = W / 2; o > 0; o >>= 1) best = min(best, tile.shfl_xor(best, o));
  if (best == 0xFFFFFFFFu) return -1;
  // an empty slot holding EMPTY_KEY ranked before the hit ends the walk
  // (find_utils.h:58-66)
  const uint32_t p = best & 0xFF;
  bool stop = false;
  if (empt) {  // none at all in a full bucket
    for (M e = empt & linear_below<M, kD>(lo, l.pos, walk_bound(p, l.pos)); e; e &= e - 1)
      if (__ldg(bk + lo + low_bit(e)) == kEmptyKey) stop = true;
  }
  return tile.ballot(stop) ? -1 : static_cast<int>(p);
}

// Writes one find result at position o: flag, and for a hit the score and
// the value row (byte strides between consecutive results).
template <int VW, uint32_t W>
__device__ __forceinline__ void find_output(const TableView& t, const TileW<W>& tile,
                                            int p, uint64_t bkt, uint64_t o,
                                            uint8_t* __restrict__ values,
                                            uint8_t* __restrict__ founds,
                                            uint8_t* __restrict__ scores,
                                            uint32_t row_stride, uint32_t flag_stride,
                                            uint32_t score_stride) {
  using V = typename VecOf<VW>::T;
  if (tile.lane == 0 && founds != nullptr) founds[o * flag_stride] = p >= 0;
  if (p < 0) return;
  if (scores != nullptr && tile.lane == 0)
    *reinterpret_cast<uint64_t*>(scores + o * score_stride) =
        __ldg(t.scores + bkt * kBucket + p);
  if (values != nullptr) {
    const uint32_t vb = t.value_bytes;
    V* dst = reinterpret_cast<V*>(values + o * row_stride);
    const V* src = reinterpret_cast<const V*>(value_ptr(t, bkt, p));
    for (uint32_t v = tile.lane; v < vb / VW; v += W) __stcs(dst + v, __ldg(src + v));
  }
}

template <int VW>
__global__ void __launch_bounds__(256, HKV_FIND_MIN_BLOCKS)
    find_kernel(TableView t, const uint64_t* __restrict__ keys,
                uint8_t* __restrict__ values, bool* __restrict__ founds,
                uint64_t* __restrict__ scores, uint64_t n,
                const uint32_t* __restrict__ dn,
                const uint32_t* __restrict__ out_index) {
  // dn: optional device-side key count (at most n); out_index: optional
  // output position of each key (results of key i go to out_index[i])
  if (dn != nullptr) n = min(n, static_cast<uint64_t>(*dn));
  constexpr uint32_t W = kFindTile;
  const TileW<W> tile;
  const uint64_t ntiles = (uint64_t)gridDim.x * (blockDim.x / W);
  uint64_t i = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) / W;
  uint64_t next = i < n ? __ldg(keys + i) : 0;
  for (; i < n; i += ntiles) {
    const uint64_t key = next;
    if (i + ntiles < n) next = __ldg(keys + i + ntiles);
    uint64_t bkt;
    const int p = find_probe(t, tile, key, bkt);
    const uint64_t o = out_index != nullptr ? __ldg(out_index + i) : i;
    find_output<VW>(t, tile, p, bkt, o, values, reinterpret_cast<uint8_t*>(founds),
                    reinterpret_cast<uint8_t*>(scores), t.value_bytes, 1, 8);
  }
}

// find* (reference find_ptr_with_digest_kernel.h:33-160): the address of
// each found key's value row (and its score), nullptr for a missed key.
__global__ void __launch_bounds__(256, HKV_FIND_MIN_BLOCKS)
    find_ptr_kernel(TableView t, const uint64_t* __restrict__ keys,
                    uint8_t** __restrict__ value_ptrs, bool* __restrict__ founds,
                    uint64_t* __restrict__ scores, uint64_t n) {
  constexpr uint32_t W = kFindTile;
  const TileW<W> tile;
  const uint64_t ntiles = (uint64_t)gridDim.x * (blockDim.x / W);
  for (uint64_t i = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) / W; i < n;
       i += ntiles) {
    uint64_t bkt;
    const int p = find_probe(t, tile, __ldg(keys + i), bkt);
    if (tile.lane == 0) {
      value_ptrs[i] = p >= 0 ? value_ptr(t, bkt, p) : nullptr;
      if (founds != nullptr) founds[i] = p >= 0;
      if (p >= 0 && scores != nullptr) scores[i] = __ldg(t.scores + bkt * kBucket + p);
    }
  }
}

// find over several key arrays at once (segment s has counts[s] keys, at
// most `bound`). The host launches a multiple of nseg blocks: block b works on
// segment b % nseg, so neighbouring blocks keep every segment in flight,
// while the tiles of one block take consecutive keys of their segment, so a
// warp's key loads (which may cross NVLink) are one contiguous read.
template <int VW>
__global__ void __launch_bounds__(256, HKV_FIND_MIN_BLOCKS)
    find_segments_kernel(TableView t, FindSegments seg, uint32_t nseg,
                         const uint32_t* __restrict__ counts, uint64_t bound) {
  constexpr uint32_t W = kFindTile;
  constexpr uint32_t kTilesPerBlock = 256 / W;
  const TileW<W> tile;
  const uint32_t k = blockIdx.x % nseg;
  const uint64_t step = uint64_t{gridDim.x / nseg} * kTilesPerBlock;
  const uint64_t cnt = min(static_cast<uint64_t>(counts[k]), bound);
  // keys may live in a peer's memory (and change between calls: no
  // non-coherent cache); each tile loads its next key one iteration ahead
  const uint64_t* keys = seg.keys[k];
  uint8_t* values = seg.values[k];
  uint8_t* founds = seg.founds[k];
  uint8_t* scores = seg.scores[k];
  uint64_t j = uint64_t{blockIdx.x / nseg} * kTilesPerBlock + threadIdx.x / W;
  uint64_t next = j < cnt ? __ldcg(keys + j) : 0;
  for (; j < cnt; j += step) {
    const uint64_t key = next;
    if (j + step < cnt) next = __ldcg(keys + j + step);
    uint64_t bkt;
    const int p = find_probe(t, tile, key, bkt);
    find_output<VW>(t, tile, p, bkt, j, values, founds, scores, seg.row_stride,
                    seg.flag_stride, seg.score_stride);
  }
}

// ============================================================================
// Upsert family: insert_or_assign, find_or_insert, insert_and_evict
// ============================================================================

struct UpsertArgs {
  const uint64_t* keys;
  const uint8_t* values_in;  // insert_or_assign / insert_and_evict input rows;
                             // find_or_insert: input rows apart (optional)
  uint8_t* values_io;        // find_or_insert rows (in on a miss, out on a hit;
                             // out on a hit only when values_in is set)
  const uint64_t* scores;    // input scores (nullable per strategy)
  uint64_t n;
  uint64_t epoch;
  uint64_t* ev_keys;         // insert_and_evict outputs
  uint8_t* ev_values;
  uint64_t* ev_scores;
  unsigned long long* ev_counter;
  uint8_t* status;           // optional Occupy code per key
  uint32_t status_stride;    // bytes between two keys' codes (0 means 1)
  const uint32_t* dn;        // optional device-side key count (overrides n)
  int report_refused;        // insert_and_evict: report refused inputs
  uint8_t** value_ptrs;      // find_or_insert*: address of each key's row
  bool* founds;              // find_or_insert*: the key was already there
  const uint32_t* row_index; // optional: key i's input/output row is row_index[i]
  uint64_t** locked_key_ptrs;  // find_or_insert*: keep each slot locked for the caller
};

// Row of key i in the caller's value array: a merged batch of repeated keys
// keeps each representative's row where its chosen occurrence has it.
__device__ __forceinline__ uint64_t key_row(const UpsertArgs& a, uint64_t i) {
  return a.row_index != nullptr ? a.row_index[i] : i;
}

// ---------------------------------------------------------------------------
// Lock discipline. A slot is owned by whoever swapped its key word to
// LOCKED_KEY. The four tiles of a warp work in warp-uniform rounds: in a
// round each tile takes its decision with plain loads while holding
// nothing, makes one CAS attempt, and if it wins it writes the slot and
// releases it before the round ends; a tile that meets a lock simply tries
// again next round. No tile therefore ever waits, inside a round, for a
// lock held by a tile of its own warp (whose release could sit behind a
// reconvergence point), and tiles of other warps always finish the round
// that holds their lock. A key gives up after kSpinLimitNs of failed rounds
// and raises kErrSpinTimeout.
// ---------------------------------------------------------------------------
constexpr int kRetry = 7;  // a round's result when a lock was in the way

// Victim of a full bucket with the reference's 16-lane scan and xor
// butterfly (insert_or_assign_kernel.h:193-238), so ties resolve exactly as
// there: virtual lane c takes the first strictly smallest score among
// positions c, c+16, ..., then the 16 virtual lanes exchange (score,
// position) across xor offsets 8, 4, 2, 1, each keeping its own pair unless
// the partner's score is strictly smaller; the key's own virtual lane is
// owner_idx % 16. Here lane L of a W-lane tile reads 16-byte score pairs at
// positions 2L + 2Wj (one coalesced 2W*8-byte run per load), so it holds
// the complete virtual lanes c = 2L + e + 2W*h (e in {0,1}, h < 8/W),
// stored at r = e + 2h. Exchanges between two virtual lanes of one lane
// stay in registers; the others are tile shuffles.
template <uint32_t W, bool kSkipUser = false>
__device__ __forceinline__ void min_score_butterfly(const TileW<W>& tile,
                                                    const uint64_t* bs,
                                                    uint32_t pos,
                                                    uint64_t owner_idx,
                                                    uint64_t& ms, uint32_t& mp,
                                                    const uint64_t* bk = nullptr) {
  constexpr uint32_t R = 16 / W;  // virtual lanes per lane
  constexpr uint32_t H = 8 / W;   // pair loads per virtual-lane pair and k
  uint64_t sv[R];
  uint32_t pv[R];
#pragma unroll
  for (uint32_t r = 0; r < R; r++) {
    sv[r] = kMaxScore;
    pv[r] = pos;
  }
  const uint4* b4 = reinterpret_cast<const uint4*>(bs);
#pragma unroll
  for (uint32_t j = 0; j < kBucket / (2 * W); j++) {
    const uint32_t q = 2 * tile.lane + 2 * W * j;
    const uint4 v = __ldcg(b4 + q / 2);
    uint64_t s0 = (static_cast<uint64_t>(v.y) << 32) | v.x;
    uint64_t s1 = (static_cast<uint64_t>(v.w) << 32) | v.z;
    if constexpr (kSkipUser) {
      // a bucket holding caller locks: their slots are never victims (the
      // reference's scan skips locked key words, insert_or_assign_kernel.h:214)
      if (ld_relaxed_u64(bk + q) == kUserLockedKey) s0 = kMaxScore;
      if (ld_relaxed_u64(bk + q + 1) == kUserLockedKey) s1 = kMaxScore;
    }
    const uint32_t r = 2 * (j % H);
    if (s0 < sv[r]) { sv[r] = s0; pv[r] = q; }
    if (s1 < sv[r + 1]) { sv[r + 1] = s1; pv[r + 1] = q + 1; }
  }
#pragma unroll
  for (uint32_t o = 8; o > 0; o >>= 1) {
    if (o == 1 || o >= 2 * W) {
      const uint32_t d = o == 1 ? 1 : o / W;
      uint64_t ns[R];
      uint32_t np[R];
#pragma unroll
      for (uint32_t r = 0; r < R; r++) {
        const bool take = sv[r ^ d] < sv[r];
        ns[r] = take ? sv[r ^ d] : sv[r];
        np[r] = take ? pv[r ^ d] : pv[r];
      }
#pragma unroll
      for (uint32_t r = 0; r < R; r++) {
        sv[r] = ns[r];
        pv[r] = np[r];
      }
    } else {
#pragma unroll
      for (uint32_t r = 0; r < R; r++) {
        const uint64_t os = tile.shfl_xor(sv[r], o / 2);
        const uint32_t op = tile.shfl_xor(pv[r], o / 2);
        if (os < sv[r]) { sv[r] = os; pv[r] = op; }
      }
    }
  }
  const uint32_t c = static_cast<uint32_t>(owner_idx & 15);
  const uint32_t src = (c & (2 * W - 1)) >> 1;
  const uint32_t rc = (c & 1) | ((c / (2 * W)) << 1);
  uint64_t s_out = sv[0];
  uint32_t p_out = pv[0];
#pragma unroll
  for (uint32_t r = 1; r < R; r++)
    if (r == rc) { s_out = sv[r]; p_out = pv[r]; }
  ms = tile.shfl(s_out, src);
  mp = tile.shfl(p_out, src);
}

// The first kHead * W vectors of a value row, vector lane + k*W in v[k]:
// an input row is loaded into registers before the probe starts.
template <int VW, uint32_t W>
struct RowHead {
  using V = typename VecOf<VW>::T;
  static constexpr uint32_t kHead = W >= 8 ? 1 : 8 / W;
  V v[kHead];
  __device__ __forceinline__ void load(const uint8_t* __restrict__ src,
                                       uint32_t nv, uint32_t lane) {
    const V* sp = reinterpret_cast<const V*>(src);
#pragma unroll
    for (uint32_t k = 0; k < kHead; k++)
      v[k] = lane + k * W < nv ? sp[lane + k * W] : V{};
  }
  // the whole row: head from registers, the rest from src. Streaming
  // (evict-first) stores: the kernel never reads the row back, and its
  // write-back then happens inside this launch instead of the next one's
  __device__ __forceinline__ void store(uint8_t* __restrict__ dst,
                                        const uint8_t* __restrict__ src,
                                        uint32_t nv, uint32_t lane) const {
    V* d = reinterpret_cast<V*>(dst);
    const V* sp = reinterpret_cast<const V*>(src);
#pragma unroll
    for (uint32_t k = 0; k < kHead; k++)
      if (lane + k * W < nv) __stcs(d + lane + k * W, v[k]);
    for (uint32_t x = lane + kHead * W; x < nv; x += W) __stcs(d + x, sp[x]);
  }
};

// Holds the lock of `slot`: score/digest/size (the reference writes them
// right after winning the slot, insert_or_assign_kernel.h:146-149, :170-174,
// :241-252), outputs, value rows, then the release.
template <int Mode, int S, int VW, uint32_t W>
__device__ __forceinline__ void upsert_locked(const TableView& t,
                                              const TileW<W>& tile,
                                              const UpsertArgs& a, uint64_t i,
                                              const Locate& l, uint64_t key,
                                              uint64_t desired, int res,
                                              uint32_t slot, uint64_t vkey,
                                              uint64_t vscore,
                                              const RowHead<VW, W>& head) {
  const uint32_t vb = t.value_bytes;
  const uint32_t nv = vb / VW;
  const uint64_t s = l.bkt * kBucket + slot;
  unsigned long long ev_idx = 0;
  if (tile.lane == 0) {
    const bool ins = res != kDuplicate;
    uint64_t ns;
    // only the Lfu rules add to the stored score
    const uint64_t old =
        (ins || (S != kLfu && S != kEpochLfu)) ? 0 : ld_relaxed_u64(t.scores + s);
    if (score_on_write<S>(old, a.scores, i, desired, ins, &ns)) {
      if (ins) t.digests[s] = static_cast<uint8_t>(l.d4);
      t.scores[s] = ns;
    }
    if (res == kOccupiedEmpty || res == kOccupiedReclaimed)
      atomicAdd(t.sizes + l.bkt, 1);
    if constexpr (Mode == kModeInsertAndEvict) {
      if (res == kEvict) {
        ev_idx = warp_claim(a.ev_counter);
        if (!HKV_BOUND(t, ev_idx < a.n, 3)) ev_idx = 0;
        a.ev_keys[ev_idx] = vkey;
        if (a.ev_scores) a.ev_scores[ev_idx] = vscore;
      }
    }
  }
  uint8_t* row = value_ptr(t, l.bkt, slot);
  if constexpr (Mode == kModeFindOrInsertPtr) {
    // the caller reads or writes the row through its address
    // (find_or_insert_ptr_kernel_v2.h:275-286)
    if (tile.lane == 0) {
      a.value_ptrs[i] = row;
      if (a.founds != nullptr) a.founds[i] = res == kDuplicate;
    }
  }
  if constexpr (Mode == kModeInsertAndEvict) {
    if (res == kEvict) {
      ev_idx = tile.shfl(ev_idx, 0);
      copy_row<VW>(a.ev_values + ev_idx * vb, row, vb, tile.lane, W);
    }
  }
  if constexpr (Mode == kModeFindOrInsert) {
    if (res == kDuplicate)
      copy_row<VW>(a.values_io + key_row(a, i) * vb, row, vb, tile.lane, W);
    else if (a.values_in != nullptr)  // input rows apart, read only here
      copy_row<VW>(row, a.values_in + key_row(a, i) * vb, vb, tile.lane, W);
    else
      head.store(row, a.values_io + key_row(a, i) * vb, nv, tile.lane);
  } else if constexpr (Mode != kModeFindOrInsertPtr) {
    head.store(row, a.values_in + key_row(a, i) * vb, nv, tile.lane);
  }
  tile.sync();
  if (tile.lane == 0) {
    if (Mode == kModeFindOrInsertPtr && a.locked_key_ptrs != nullptr) {
      // the slot stays locked for the caller (find_or_insert_ptr_kernel_v2.h:
      // locked_key_ptrs), counted per bucket so that evictions pass it by
      atomicAdd(t.sizes + l.bkt, 1 << kLockShift);
      store_release_u64(t.keys + s, kUserLockedKey);
      a.locked_key_ptrs[i] = t.keys + s;
    } else {
      store_release_u64(t.keys + s, key);
    }
  }
}

// One round for one key of insert_or_assign / find_or_insert /
// insert_and_evict (reference insert_or_assign_kernel.h:77-303,
// find_or_insert_kernel.h:72-306, insert_and_evict_kernel.h:389-691):
//  1. digest hits: a slot holding the key -> update it (DUPLICATE); a
//     locked hit slot may be this key being evicted -> retry;
//  2. bucket not full: the first EMPTY_KEY slot in linear order from pos
//     (the order the reference's group walk visits empty slots) is claimed
//     with CAS(EMPTY -> LOCKED), trying the next candidate on failure;
//  3. otherwise the minimum-score slot (butterfly above); refuse iff
//     desired < min; CAS(victim -> LOCKED) and re-check its score.
// Returns the Occupy result, or kRetry.
//
// phase kPhaseProbe stops before step 3 when the bucket is full and returns
// kDeferred; phase kPhaseEvict is step 3 alone, for a key such a probe
// deferred (absent from a full bucket: a unique-key batch places a key only
// through its own tile, and bucket sizes only grow during an upsert).
enum UpsertPhase : int { kPhaseFull = 0, kPhaseProbe = 1, kPhaseEvict = 2 };
constexpr int kDeferred = 8;  // a round's result: the key waits for an evict round
template <int Mode, int S, int VW, uint32_t W, bool kLocks>
__device__ __forceinline__ int upsert_round(const TableView& t, const TileW<W>& tile,
                                            const UpsertArgs& a, uint64_t i,
                                            uint64_t key, uint64_t desired,
                                            const Locate& l,
                                            const RowHead<VW, W>& head,
                                            int phase = kPhaseFull) {
  constexpr uint32_t kD = TileW<W>::kDigests;  // digests per lane
  constexpr uint32_t kDV = kD / 16;
  using M = typename std::conditional<(kD > 32), uint64_t, uint32_t>::type;
  uint64_t* bk = t.keys + l.bkt * kBucket;
  const uint64_t* bs = t.scores + l.bkt * kBucket;
  const uint32_t lo = tile.lane * kD;
  const uint4* dl = reinterpret_cast<const uint4*>(t.digests + l.bkt * kBucket) + tile.lane * kDV;
  M hits = 0, empt = 0;
  if (phase != kPhaseEvict) {
#pragma unroll
    for (uint32_t j = 0; j < kDV; j++) {
      const uint4 dv = __ldcg(dl + j);
      hits |= static_cast<M>(bytes_eq16(dv, l.d4)) << (16 * j);
      empt |= static_cast<M>(bytes_eq16(dv, kEmptyDigest * 0x01010101u)) << (16 * j);
    }
  }
  const int32_t bword = __ldcg(t.sizes + l.bkt);  // size, caller locks above it
  // ---- 1. is the key here? (a digest hit that holds it is locked at once)
  // Each lane locks its first digest hit holding the key in walk order, the
  // tile keeps the first in walk order. A key has one slot, so normally one
  // lane finds it and the index-order loop below is the walk order; only on
  // layouts where a second copy was placed in front of the key do the two
  // rare branches matter: a match in the start group's lane before the start
  // group comes last in the walk (the lane keeps looking), and two lanes
  // holding the key leave it to the walk rank.
  int mine = -1;
  bool busy = false;
  {
    const uint32_t g0 = l.pos & ~3u;
    const uint32_t rot = (g0 >= lo && g0 < lo + kD) ? g0 - lo : 0;
    int late = -1;  // a match before the start group, in that group's lane
    while (hits) {
      const uint32_t j = low_bit(hits);
      hits &= hits - 1;
      const uint64_t k = cas_acquire_u64(bk + lo + j, key, kLockedKey);
      if (k == key) {
        if (j >= rot) {
          mine = static_cast<int>(lo + j);
          break;
        }
        if (late < 0) late = static_cast<int>(lo + j);
        else store_release_u64(bk + lo + j, key);
        continue;
      }
      // an operation in flight may hold the key: retry. A caller's lock says
      // nothing about which key it hides (a digest hit may belong to another
      // key): like the reference, which compares the word with the key
      // itself (insert_or_assign_kernel.h:128-140), such a slot is not it.
      busy |= (k == kLockedKey);
    }
    if (late >= 0) {
      if (mine < 0)
        mine = late;
      else
        store_release_u64(bk + late, key);
    }
  }
  int res = kRetry;
  bool got = false;
  uint32_t slot = 0;
  uint64_t vkey = 0, vscore = 0;
  const bool not_full =
      phase != kPhaseEvict && (bword & kSizeMask) < static_cast<int32_t>(kBucket);
  const uint32_t fm = tile.ballot(mine >= 0);
  // the key is in the bucket, but the reference's group walk reaches an
  // EMPTY slot first: it claims that slot instead
  bool to_empty = false;
  if (fm) {
    slot = tile.shfl(static_cast<uint32_t>(mine), __ffs(fm) - 1);
    if (__builtin_expect(__popc(fm) > 1, 0)) {
      uint32_t first = mine >= 0 ? (hit_rank(mine, l.pos) << 8) | static_cast<uint32_t>(mine)
                                 : 0xFFFFFFFFu;
#pragma unroll
      for (int o = W / 2; o > 0; o >>= 1) first = min(first, tile.shfl_xor(first, o));
      slot = first & 0xFF;
    }
    const bool holder = mine == static_cast<int>(slot);
    if (mine >= 0 && !holder) store_release_u64(bk + mine, key);
    // The walk (insert_or_assign_kernel.h:105-183) examines a group's digest
    // hits, then, below a full bucket, that group's EMPTY slots, group by
    // group from pos: an EMPTY slot in a group before the key's takes the
    // key (a second copy). Only a layout with a slot emptied in front of a
    // placed key has one; the candidates are empty digests, rarely any.
    bool before = false;
    if (not_full) {
      empt &= linear_below<M, kD>(lo, l.pos, walk_bound(slot, l.pos));
      for (M e = empt; e; e &= e - 1)
        if (ld_relaxed_u64(bk + lo + low_bit(e)) == kEmptyKey) before = true;
    }
    if (tile.ballot(before)) {
      if (holder) store_release_u64(bk + slot, key);
      to_empty = true;
    } else {
      got = true;
      res = kDuplicate;
    }
  }
  if (!got && (to_empty || !tile.ballot(busy))) {
    // ---- 2. first EMPTY slot in linear order from pos (with to_empty, only
    // those ahead of the key's group)
    if (not_full) {
      const uint32_t sh = (l.pos >= lo && l.pos < lo + kD) ? l.pos - lo : 0;
      while (true) {
        uint32_t best = 0xFFFFFFFFu;
        if (empt) {
          const M hi = empt & (~static_cast<M>(0) << sh);
          const uint32_t q = lo + low_bit(hi ? hi : empt);
          best = (linear_rank(q, l.pos) << 8) | q;
        }
#pragma unroll
        for (int o = W / 2; o > 0; o >>= 1) best = min(best, tile.shfl_xor(best, o));
        if (best == 0xFFFFFFFFu) break;
        const uint32_t q = best & 0xFF;
        const uint32_t owner = q / kD;
        bool ok = false;
        if (tile.lane == owner) {
          ok = cas_acquire_u64(bk + q, kEmptyKey, kLockedKey) == kEmptyKey;
          empt &= ~(static_cast<M>(1) << (q - lo));
        }
        if (tile.shfl(ok, owner)) {
          slot = q;
          got = true;
          res = kOccupiedEmpty;
          break;
        }
      }
    }
    // ---- 3. evict the minimum score (a key in the bucket whose EMPTY slots
    // ahead were all taken meanwhile is retried: the walk then hits it)
    if (!got && !to_empty && phase == kPhaseProbe && !not_full) return kDeferred;
    if (!got && !to_empty) {
      uint64_t ms;
      uint32_t mp;
      // kernels launched while the caller may hold locks pass them by; the
      // others carry no trace of that scan
      if (kLocks && (bword >> kLockShift) > 0)
        min_score_butterfly<W, kLocks>(tile, bs, l.pos, i, ms, mp, bk);
      else
        min_score_butterfly<W, false>(tile, bs, l.pos, i, ms, mp);
      if (desired < ms) {
        res = kRefused;
      } else {
        uint64_t k = 0;
        int r = 0;
        if (tile.lane == 0) {
          // Swapping LOCKED_KEY in locks the victim and returns its key in
          // one round trip. A slot another tile holds stays LOCKED_KEY (its
          // owner's release writes the final key); an EMPTY_KEY slot is put
          // back; a victim whose score rose since the scan is put back.
          k = exch_acquire_u64(bk + mp, kLockedKey);
          if (k == kEmptyKey || k == kUserLockedKey) {
            // put back an empty slot, or a caller's lock taken after the scan
            store_release_u64(bk + mp, k);
          } else if (k != kLockedKey) {
            if (ld_relaxed_u64(bs + mp) <= ms)
              r = (k == kReclaimKey) ? kOccupiedReclaimed : kEvict;
            else
              store_release_u64(bk + mp, k);
          }
        }
        r = tile.shfl(r, 0);
        if (r) {
          got = true;
          res = r;
          slot = mp;
          vkey = tile.shfl(k, 0);
          vscore = ms;
        }
      }
    }
  }
  if (got) {
    if (!HKV_BOUND(t, slot < kBucket, 2)) slot = 0;
    upsert_locked<Mode, S, VW, W>(t, tile, a, i, l, key, desired, res, slot, vkey,
                                  vscore, head);
  }
  return res;
}

// lane 0 of a tile: true once the key has been retried for kSpinLimitNs
template <class Tl>
__device__ __forceinline__ bool retry_expired(const TableView& t, const Tl& tile,
                                              uint64_t& t0, int site) {
  int expired = 0;
  if (tile.lane == 0) {
    const uint64_t now = global_timer_ns();
    if (t0 == 0) t0 = now;
    expired = now - t0 > kSpinLimitNs;
    if (expired) {
      atomicOr(t.error, kErrSpinTimeout);
      atomicExch(t.error + 1, site);
    }
  }
  return tile.shfl(expired, 0) != 0;
}

#ifndef HKV_UPSERT_TILE
#define HKV_UPSERT_TILE 4
#endif
#ifndef HKV_UPSERT_MIN_BLOCKS
#define HKV_UPSERT_MIN_BLOCKS 5
#endif
// accum_or_assign: 5 blocks (48 registers) measured faster than 6 (40, more
// spills) and 4 (64)
#ifndef HKV_ACCUM_MIN_BLOCKS
#define HKV_ACCUM_MIN_BLOCKS 5
#endif
// accum grid: many short blocks (64 per SM) measured faster than one
// resident wave (278 -> 257 us per 1 Mi keys)
#ifndef HKV_ACCUM_BLOCKS_PER_SM
#define HKV_ACCUM_BLOCKS_PER_SM 64
#endif
// insert_and_evict keeps more state across its rounds (the victim and its
// output): at 64 registers (4 blocks of 256 per SM) it spills nothing and
// ran 4 % faster than at 48 with spills
#ifndef HKV_EVICT_MIN_BLOCKS
#define HKV_EVICT_MIN_BLOCKS 4
#endif
constexpr uint32_t kUpsertTile = HKV_UPSERT_TILE;

// Outputs of key i once its result is final: the per-key status, no
// address for find_or_insert* keys that got no slot, and insert_and_evict's
// report of a refused input (reference insert_and_evict_kernel.h:553-557,
// :675-683: the input with its desired score).
template <int Mode, int VW, uint32_t W>
__device__ __forceinline__ void upsert_finish(const TableView& t, const TileW<W>& tile,
                                              const UpsertArgs& a, uint64_t i,
                                              uint64_t key, uint64_t desired, int res,
                                              const RowHead<VW, W>& head) {
  if (a.status != nullptr && tile.lane == 0)
    a.status[i * (a.status_stride ? a.status_stride : 1)] = res;
  if constexpr (Mode == kModeFindOrInsertPtr) {
    // refused, reserved or timed-out keys get no address
    if (tile.lane == 0 && res != kDuplicate && res != kOccupiedEmpty &&
        res != kOccupiedReclaimed && res != kEvict) {
      a.value_ptrs[i] = nullptr;
      if (a.founds != nullptr) a.founds[i] = false;
      if (a.locked_key_ptrs != nullptr) a.locked_key_ptrs[i] = nullptr;
    }
  }
  if constexpr (Mode == kModeInsertAndEvict) {
    if (res == kRefused && a.report_refused) {
      const uint32_t vb = t.value_bytes;
      unsigned long long o = 0;
      if (tile.lane == 0) {
        o = warp_claim(a.ev_counter);
        if (!HKV_BOUND(t, o < a.n, 4)) o = 0;
        a.ev_keys[o] = key;
        if (a.ev_scores) a.ev_scores[o] = desired;
      }
      o = tile.shfl(o, 0);
      head.store(a.ev_values + o * vb, a.values_in + key_row(a, i) * vb, vb / VW, tile.lane);
    }
  }
}

// Keys a warp's probe rounds found absent from a full bucket wait here (per
// warp, in shared memory) until the warp has a whole round of them.
#ifndef HKV_UPSERT_SPLIT
#define HKV_UPSERT_SPLIT 1
#endif
constexpr uint32_t kDeferCap = 16;

// The upsert loop: keys [0, n) of `a`, warp `warp` of `nwarps` taking
// keys warp * KPW, then every nwarps * KPW.
//
// A warp works on KPW keys at a time in warp-uniform rounds (the lock
// discipline above), so a round lasts as long as its slowest key. At a high
// load factor half of the keys are absent from full buckets and take the
// eviction path (a 1 KiB score scan, the victim's exchange and re-check),
// the others a short hit or empty-slot path. With HKV_UPSERT_SPLIT the
// warp's probe rounds take new keys and finish every key that needs no
// eviction; a key absent from a full bucket is deferred to the warp's queue,
// and once KPW keys wait there an evict round runs them together, so the
// short and the long paths no longer share rounds.
template <int Mode, int S, int VW, bool kLocks>
__device__ __forceinline__ void upsert_body(const TableView& t, const UpsertArgs& a,
                                            uint64_t clk, uint64_t warp,
                                            uint64_t nwarps) {
  constexpr uint32_t W = kUpsertTile;
  constexpr uint32_t KPW = 32 / W;  // keys per warp
  const TileW<W> tile;
  const uint32_t wl = threadIdx.x & 31;
  const uint64_t n = a.dn != nullptr ? *a.dn : a.n;
  const uint32_t vb = t.value_bytes;
  const uint32_t nv = vb / VW;
  // find_or_insert with values_in set (the table's own calls, with the
  // caller's rows in both; the sharded owner, with the input rows in a
  // peer's memory) reads an input row only for a key it inserts, and writes
  // values_io only for a key it finds
  const uint8_t* in_rows = Mode == kModeFindOrInsert
                               ? (a.values_in != nullptr ? nullptr : a.values_io)
                               : a.values_in;
  // keys are read one iteration ahead, the head of the input row before the
  // probe, so neither waits behind the bucket's round trips
  const uint64_t stride = nwarps * KPW;
  uint64_t next = warp * KPW + wl / W < n ? a.keys[warp * KPW + wl / W] : 0;
  if constexpr (HKV_UPSERT_SPLIT && Mode == kModeInsertAndEvict) {
  static_assert(KPW <= kDeferCap / 2, "the queue takes one probe round on top of KPW - 1 keys");
  __shared__ uint64_t s_defer[8][kDeferCap];  // blockDim.x == 256: 8 warps
  uint64_t* dq = s_defer[threadIdx.x >> 5];
  uint32_t qhead = 0, qcnt = 0;  // warp-uniform
  uint64_t base = warp * KPW;
  while (true) {
    const bool evict = qcnt >= KPW || (base >= n && qcnt > 0);
    if (!evict && base >= n) break;
    uint64_t i = 0, key = 0;
    bool have;
    if (evict) {
      const uint32_t take = min(qcnt, KPW);
      have = wl / W < take;
      if (have) {
        i = dq[(qhead + wl / W) % kDeferCap];
        key = a.keys[i];
      }
      qhead = (qhead + take) % kDeferCap;
      qcnt -= take;
    } else {
      i = base + wl / W;
      have = i < n;
      if (have) {
        key = next;
        if (i + stride < n) next = a.keys[i + stride];
      }
      base += stride;
    }
    uint64_t desired = 0, t0 = 0;
    int res = kIllegal;
    bool todo = false;
    RowHead<VW, W> head;
    Locate l;
    l.bkt = 0;
    l.pos = 0;
    l.d4 = 0;
    if (have && !is_reserved(key)) {
      if (Mode != kModeFindOrInsertPtr && in_rows != nullptr)
        head.load(in_rows + key_row(a, i) * vb, nv, tile.lane);
      desired = desired_when_missed<S>(a.scores, i, a.epoch, clk);
      l = locate(t, key);
      todo = true;
    }
    const int phase = evict ? kPhaseEvict : kPhaseProbe;
    for (int round = 0;; round++) {
      bool again = false;
      if (todo) {
        res = upsert_round<Mode, S, VW, W, kLocks>(t, tile, a, i, key, desired, l, head,
                                                   phase);
        if (res == kRetry) {
          if (retry_expired(t, tile, t0, 101)) {
            res = kTimedOut;
            todo = false;
          } else {
            again = true;
          }
        } else {
          todo = false;
        }
      }
      if (!__any_sync(0xFFFFFFFFu, again)) break;
      backoff(round);
    }
    const bool deferred = have && res == kDeferred;
    const uint32_t dm = __ballot_sync(0xFFFFFFFFu, deferred && tile.lane == 0);
    if (deferred && tile.lane == 0)
      dq[(qhead + qcnt + __popc(dm & ((1u << wl) - 1))) % kDeferCap] = i;
    qcnt += __popc(dm);
    __syncwarp();  // the queue entries are read by other lanes of the warp
    if (have && !deferred) upsert_finish<Mode, VW, W>(t, tile, a, i, key, desired, res, head);
  }
  } else {
  for (uint64_t base = warp * KPW; base < n; base += stride) {
    const uint64_t i = base + wl / W;
    uint64_t key = 0, desired = 0, t0 = 0;
    int res = kIllegal;
    bool todo = false;
    RowHead<VW, W> head;
    Locate l;
    l.bkt = 0;
    l.pos = 0;
    l.d4 = 0;
    if (i < n) {
      key = next;
      if (i + stride < n) next = a.keys[i + stride];
      if (!is_reserved(key)) {
        if (Mode != kModeFindOrInsertPtr && in_rows != nullptr)
          head.load(in_rows + key_row(a, i) * vb, nv, tile.lane);
        desired = desired_when_missed<S>(a.scores, i, a.epoch, clk);
        l = locate(t, key);
        todo = true;
      }
    }
    // warp-uniform rounds; see the lock discipline above
    for (int round = 0;; round++) {
      bool again = false;
      if (todo) {
        res = upsert_round<Mode, S, VW, W, kLocks>(t, tile, a, i, key, desired, l, head);
        if (res == kRetry) {
          if (retry_expired(t, tile, t0, 101)) {
            res = kTimedOut;
            todo = false;
          } else {
            again = true;
          }
        } else {
          todo = false;
        }
      }
      if (!__any_sync(0xFFFFFFFFu, again)) break;
      backoff(round);
    }
    if (i < n) upsert_finish<Mode, VW, W>(t, tile, a, i, key, desired, res, head);
  }
  }
}

// kLocks: launched while the caller may hold keys locked (lock_keys,
// find_or_insert* with locked_key_ptrs); evictions then pass them by.
template <int Mode, int S, int VW, bool kLocks = false>
__global__ void __launch_bounds__(256, Mode == kModeInsertAndEvict ? HKV_EVICT_MIN_BLOCKS
                                                                   : HKV_UPSERT_MIN_BLOCKS)
    upsert_kernel(TableView t, UpsertArgs a) {
  __shared__ uint64_t s_clock;
  if (threadIdx.x == 0) s_clock = global_timer_ns();
  __syncthreads();
  upsert_body<Mode, S, VW, kLocks>(t, a, s_clock,
                           (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) / 32,
                           (uint64_t)gridDim.x * (blockDim.x / 32));
}

// How a lookup of existing keys walks a bucket in the reference:
//  kWalk      groups of 4 digests from the start group, first digest hit
//             holding the key (lock_keys_kernel.h:78-124);
//  kWalkStop  the same with find_without_lock's stop rule: an EMPTY_KEY slot
//             with an empty digest reached before the key hides it
//             (find_utils.h:31-86; assign_scores);
//  kWindow    find_and_lock's 32-slot windows from pos (find_utils.h:94-147;
//             accum_or_assign): the first slot holding the key in linear
//             order, unless an earlier window holds an EMPTY_KEY slot, which
//             find_and_lock would claim first.
enum LocateRule : int { kWalk = 0, kWalkStop = 1, kWindow = 2 };

// A tile of W lanes (kBucket / W digests per lane) finds the slot holding
// `key` with plain loads, the first in the rule's order when a layout holds
// two copies. Returns the slot, -1 if absent (or hidden by the stop rule),
// -2 if a locked digest-hit slot may hold the key (the caller retries), and
// for kWindow -3 when an EMPTY_KEY slot comes first (the caller takes
// find_and_lock's full path). EMPTY_KEY slots are found through their empty
// digests, which every slot this library empties carries.
template <int Rule, uint32_t W>
__device__ __forceinline__ int tile_locate_existing(const TableView& t,
                                                      const TileW<W>& tile,
                                                      const Locate& l, uint64_t key) {
  constexpr uint32_t kD = TileW<W>::kDigests;
  constexpr uint32_t kDV = kD / 16;
  using M = typename std::conditional<(kD > 32), uint64_t, uint32_t>::type;
  const uint64_t* bk = t.keys + l.bkt * kBucket;
  const uint4* dl = reinterpret_cast<const uint4*>(t.digests + l.bkt * kBucket) + tile.lane * kDV;
  // a full bucket holds no EMPTY_KEY slot: no empty slot can come first
  const bool full =
      Rule != kWalk && (__ldcg(t.sizes + l.bkt) & kSizeMask) >= int32_t{kBucket};
  const uint32_t lo = tile.lane * kD;
  M hits = 0, empt = 0;
#pragma unroll
  for (uint32_t j = 0; j < kDV; j++) {
    const uint4 dv = __ldcg(dl + j);
    hits |= static_cast<M>(bytes_eq16(dv, l.d4)) << (16 * j);
    if (Rule != kWalk)
      empt |= static_cast<M>(bytes_eq16(dv, kEmptyDigest * 0x01010101u)) << (16 * j);
  }
  uint32_t best = 0xFFFFFFFFu;
  bool busy = false;
  for (M h = hits; h; h &= h - 1) {
    const uint32_t q = lo + low_bit(h);
    const uint64_t k = ld_relaxed_u64(bk + q);
    if (k == key) {
      const uint32_t r = Rule == kWindow ? linear_rank(q, l.pos) : hit_rank(q, l.pos);
      best = min(best, (r << 8) | q);
    }
    busy |= (k == kLockedKey);
  }
#pragma unroll
  for (int o = W / 2; o > 0; o >>= 1) best = min(best, tile.shfl_xor(best, o));
  if (best == 0xFFFFFFFFu) return tile.ballot(busy) ? -2 : -1;
  const uint32_t p = best & 0xFF;
  if constexpr (Rule != kWalk) {
    bool first = false;
    if (!full) {
      const uint32_t bound = Rule == kWindow ? linear_rank(p, l.pos) & ~31u : walk_bound(p, l.pos);
      for (M e = empt & linear_below<M, kD>(lo, l.pos, bound); e; e &= e - 1)
        if (ld_relaxed_u64(bk + lo + low_bit(e)) == kEmptyKey) first = true;
    }
    if (tile.ballot(first)) return Rule == kWindow ? -3 : -1;
  }
  return static_cast<int>(p);
}

// erase (remove_kernel.h:79-110) visits the groups from the start group and
// tombstones the first digest hit holding the key in each, visiting the
// start group twice (offsets 0 and B): normally the key's one slot, on
// layouts with two copies every copy it reaches. Each lane erases its own
// slots; returns false when no slot held the key but a digest-hit slot was
// locked (the caller retries).
template <uint32_t W>
__device__ __forceinline__ bool tile_erase(const TableView& t, const TileW<W>& tile,
                                           const Locate& l, uint64_t key) {
  constexpr uint32_t kD = TileW<W>::kDigests;
  constexpr uint32_t kDV = kD / 16;
  using M = typename std::conditional<(kD > 32), uint64_t, uint32_t>::type;
  constexpr M kNib1 = static_cast<M>(0xEEEEEEEEEEEEEEEEull);  // bits 1-3 of each group
  constexpr M kNib2 = static_cast<M>(0xCCCCCCCCCCCCCCCCull);  // bits 2-3 of each group
  uint64_t* bk = t.keys + l.bkt * kBucket;
  const uint4* dl = reinterpret_cast<const uint4*>(t.digests + l.bkt * kBucket) + tile.lane * kDV;
  const uint32_t lo = tile.lane * kD;
  M hits = 0;
#pragma unroll
  for (uint32_t j = 0; j < kDV; j++)
    hits |= static_cast<M>(bytes_eq16(__ldcg(dl + j), l.d4)) << (16 * j);
  M held = 0;
  bool busy = false;
  for (M h = hits; h; h &= h - 1) {
    const uint32_t j = low_bit(h);
    const uint64_t k = ld_relaxed_u64(bk + lo + j);
    if (k == key) held |= static_cast<M>(1) << j;
    busy |= (k == kLockedKey);
  }
  // first holder of each group of 4 (groups start at multiples of 4 slots)
  M upto = held;
  upto |= (upto << 1) & kNib1;
  upto |= (upto << 2) & kNib2;
  M erase = held & ~((upto << 1) & kNib1);
  const uint32_t g0 = l.pos & ~3u;
  if (g0 >= lo && g0 < lo + kD) {
    // the second visit of the start group takes its next holder
    const M rest = held & ~erase & (static_cast<M>(0xF) << (g0 - lo));
    erase |= rest & (~rest + 1);
  }
  // The key word turns into the tombstone in one CAS; score, digest and size
  // follow with plain writes, as the reference's erase writes them
  // (remove_kernel.h:96-101, no lock): no other operation of this launch
  // touches the slot, and the next launch sees every write.
  for (M e = erase; e; e &= e - 1) {
    const uint64_t s = l.bkt * kBucket + lo + low_bit(e);
    if (cas_u64(t.keys + s, key, kReclaimKey) == key) {
      t.scores[s] = 0;
      t.digests[s] = kReclaimDigest;
      atomicSub(t.sizes + l.bkt, 1);
    }
  }
  return tile.ballot(held != 0) || !tile.ballot(busy);
}

// ============================================================================
// accum_or_assign (reference accum_or_assign_kernel.h:55-155 with
// find_and_lock, find_utils.h:94-228). A present key is found through its
// digest line by an 8-lane tile and locked with one CAS; any other key takes
// the whole warp: 32-slot windows from pos, waiting on LOCKED slots
// (bounded), so duplicate keys in one batch serialise on the key word.
// ============================================================================
struct AccumArgs {
  const uint64_t* keys;
  const uint8_t* values;
  const bool* accum_or_assigns;
  const uint64_t* scores;
  uint64_t n;
  uint64_t epoch;
  uint8_t* status;
  uint32_t vec16;  // rows and inputs allow 16-byte vectors (float rows only)
};

template <class VT>
struct AccumOps;
template <>
struct AccumOps<float> {
  static __device__ __forceinline__ float add(float a, float b) { return a + b; }
};
template <>
struct AccumOps<__half> {
  static __device__ __forceinline__ __half add(__half a, __half b) {
    return __float2half_rn(__half2float(a) + __half2float(b));
  }
};
template <>
struct AccumOps<__nv_bfloat16> {
  static __device__ __forceinline__ __nv_bfloat16 add(__nv_bfloat16 a,
                                                      __nv_bfloat16 b) {
    return __float2bfloat16_rn(__bfloat162float(a) + __bfloat162float(b));
  }
};

// Returns Occupy; on success the warp owns `slot` and `evk` holds the key it
// displaced (EMPTY_KEY / RECLAIM_KEY / victim).
__device__ __forceinline__ int warp_find_and_lock(const TableView& t,
                                                  const Locate& l, uint64_t key,
                                                  uint64_t desired,
                                                  uint32_t& slot,
                                                  uint64_t& evk) {
  const uint32_t lane = threadIdx.x & 31;
  uint64_t* bk = t.keys + l.bkt * kBucket;
  const uint64_t* bs = t.scores + l.bkt * kBucket;
  const uint64_t t0 = global_timer_ns();
  auto expired = [&]() { return global_timer_ns() - t0 > kSpinLimitNs; };
restart:
  if (expired()) return kTimedOut;
  for (uint32_t w = 0; w < kBucket; w += 32) {
    const uint32_t q = (l.pos + w + lane) & (kBucket - 1);
    while (true) {
      const uint64_t k = ld_relaxed_u64(bk + q);
      const uint32_t hit = __ballot_sync(0xFFFFFFFFu, k == key);
      if (hit) {
        const int src = __ffs(hit) - 1;
        uint64_t old = 0;
        if (static_cast<int>(lane) == src)
          old = cas_acquire_u64(bk + q, key, kLockedKey);
        old = __shfl_sync(0xFFFFFFFFu, old, src);
        if (old == key) {
          slot = __shfl_sync(0xFFFFFFFFu, q, src);
          evk = key;
          return kDuplicate;
        }
        if (expired()) return kTimedOut;
        __nanosleep(64);
        continue;
      }
      if (__ballot_sync(0xFFFFFFFFu, k == kLockedKey)) {
        if (expired()) return kTimedOut;
        __nanosleep(64);
        continue;
      }
      uint32_t em = __ballot_sync(0xFFFFFFFFu, k == kEmptyKey);
      while (em) {
        const int src = __ffs(em) - 1;
        uint64_t old = 0;
        if (static_cast<int>(lane) == src)
          old = cas_acquire_u64(bk + q, kEmptyKey, kLockedKey);
        old = __shfl_sync(0xFFFFFFFFu, old, src);
        if (old == kEmptyKey) {
          slot = __shfl_sync(0xFFFFFFFFu, q, src);
          evk = kEmptyKey;
          return kOccupiedEmpty;
        }
        if (old == key || old == kLockedKey) goto restart;
        em &= ~(1u << src);
      }
      break;
    }
  }
  // eviction: each lane the first strictly-smallest score over its slots
  uint64_t lm = kMaxScore, lk = kEmptyKey;
  uint32_t lp = 0;
  for (uint32_t w = 0; w < kBucket; w += 32) {
    const uint32_t q = (l.pos + w + lane) & (kBucket - 1);
    const uint64_t sc = ld_relaxed_u64(bs + q);
    if (sc < lm) {
      uint64_t k;
      bool gave_up = false;
      while ((k = ld_relaxed_u64(bk + q)) == kLockedKey) {
        if (expired()) {
          gave_up = true;
          break;
        }
        __nanosleep(64);
      }
      if (!gave_up && k != kEmptyKey && k != kUserLockedKey) {
        lm = sc;
        lp = q;
        lk = k;
      }
    }
  }
  uint64_t gm = lm;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) gm = min(gm, __shfl_xor_sync(0xFFFFFFFFu, gm, o));
  if (desired < gm) return kRefused;
  const uint32_t vote = __ballot_sync(0xFFFFFFFFu, lm <= gm);
  if (vote) {
    const int src = __ffs(vote) - 1;
    int ok = 0;
    if (static_cast<int>(lane) == src) {
      if (cas_acquire_u64(bk + lp, lk, kLockedKey) == lk) {
        if (ld_relaxed_u64(bs + lp) <= gm)
          ok = 1;
        else
          store_release_u64(bk + lp, lk);
      }
    }
    ok = __shfl_sync(0xFFFFFFFFu, ok, src);
    if (ok) {
      slot = __shfl_sync(0xFFFFFFFFu, lp, src);
      evk = __shfl_sync(0xFFFFFFFFu, lk, src);
      return evk == kReclaimKey ? kOccupiedReclaimed : kEvict;
    }
  }
  __nanosleep(128);
  goto restart;
}

// With `slot` locked (res as warp_find_and_lock returns it): undo when the
// operation does not apply (reference :114-128), else accumulate or assign
// the row, set size, digest and score, and release. `width` lanes of the
// calling group take part; sync() orders their row writes before the release.
template <int S, class VT, class Sync>
__device__ __forceinline__ int accum_apply(const TableView& t, const AccumArgs& a,
                                           uint64_t i, uint64_t key, bool is_accum,
                                           uint64_t desired, const Locate& l,
                                           uint32_t slot, uint64_t evk, int res,
                                           uint32_t lane, uint32_t width, Sync sync) {
  uint64_t* bk = t.keys + l.bkt * kBucket;
  const uint64_t s = l.bkt * kBucket + slot;
  if ((is_accum && res != kDuplicate) || (!is_accum && res == kDuplicate)) {
    if (lane == 0) store_release_u64(bk + slot, res == kDuplicate ? key : evk);
    return kIllegal;
  }
  const uint32_t vb = t.value_bytes;
  const uint32_t ne = vb / sizeof(VT);
  VT* dst = reinterpret_cast<VT*>(value_ptr(t, l.bkt, slot));
  const VT* src = reinterpret_cast<const VT*>(a.values + i * vb);
  if (std::is_same<VT, float>::value && a.vec16) {
    // four elements per access, each added as in the scalar loop
    float4* d4 = reinterpret_cast<float4*>(dst);
    const float4* s4 = reinterpret_cast<const float4*>(src);
    for (uint32_t e = lane; e < vb / 16; e += width) {
      float4 v = s4[e];
      if (is_accum) {
        const float4 o = d4[e];
        v.x = v.x + o.x;
        v.y = v.y + o.y;
        v.z = v.z + o.z;
        v.w = v.w + o.w;
      }
      d4[e] = v;
    }
  } else {
    for (uint32_t e = lane; e < ne; e += width)
      dst[e] = is_accum ? AccumOps<VT>::add(src[e], dst[e]) : src[e];
  }
  if (lane == 0) {
    if (res == kOccupiedEmpty || res == kOccupiedReclaimed) atomicAdd(t.sizes + l.bkt, 1);
    const bool ins = res != kDuplicate;
    uint64_t ns;
    const uint64_t old =
        (ins || (S != kLfu && S != kEpochLfu)) ? 0 : ld_relaxed_u64(t.scores + s);
    if (score_on_write<S>(old, a.scores, i, desired, ins, &ns)) {
      t.digests[s] = static_cast<uint8_t>(l.d4);
      t.scores[s] = ns;
    }
  }
  sync();
  if (lane == 0) store_release_u64(bk + slot, key);
  return res;
}

// Four keys per warp, one 8-lane tile each: a present, unlocked key is found
// through its digest line and locked with one CAS (the common case). The
// others (absent keys, keys whose slot another lane holds, keys being
// inserted) then go one at a time through the whole warp's window scan,
// which waits on locked slots, so repeats of a key serialise on its word.
constexpr uint32_t kAccumTile = 4;
template <int S, class VT>
__global__ void __launch_bounds__(256, HKV_ACCUM_MIN_BLOCKS)
    accum_kernel(TableView t, AccumArgs a) {
  constexpr uint32_t W = kAccumTile;
  constexpr uint32_t KPW = 32 / W;  // keys per warp
  __shared__ uint64_t s_clock;
  if (threadIdx.x == 0) s_clock = global_timer_ns();
  __syncthreads();
  const uint64_t clk = s_clock;
  const TileW<W> tile;
  const uint32_t wl = threadIdx.x & 31;
  const uint64_t nwarps = (uint64_t)gridDim.x * (blockDim.x / 32);
  const uint64_t warp = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) / 32;
  for (uint64_t base = warp * KPW; base < a.n; base += nwarps * KPW) {
    const uint64_t i = base + wl / W;
    const bool in = i < a.n;
    const uint64_t key = in ? a.keys[i] : 0;
    const bool valid = in && !is_reserved(key);
    int res = kIllegal;
    bool pending = false;
    uint64_t desired = 0;
    bool is_accum = false;
    Locate l;
    l.bkt = 0;
    l.pos = 0;
    l.d4 = 0;
    if (valid) {
      desired = desired_when_missed<S>(a.scores, i, a.epoch, clk);
      is_accum = a.accum_or_assigns[i];
      l = locate(t, key);
      const int p = tile_locate_existing<kWindow>(t, tile, l, key);
      bool got = false;
      if (p >= 0 && tile.lane == 0)
        got = cas_acquire_u64(t.keys + l.bkt * kBucket + p, key, kLockedKey) == key;
      if (tile.shfl(got, 0))
        res = accum_apply<S, VT>(t, a, i, key, is_accum, desired, l,
                                 static_cast<uint32_t>(p), key, kDuplicate, tile.lane, W,
                                 [&]() { tile.sync(); });
      else
        pending = true;
    }
    uint32_t todo = __ballot_sync(0xFFFFFFFFu, pending && tile.lane == 0);
    while (todo) {
      const int src = __ffs(todo) - 1;
      todo &= todo - 1;
      const uint64_t wi = __shfl_sync(0xFFFFFFFFu, i, src);
      const uint64_t wk = __shfl_sync(0xFFFFFFFFu, key, src);
      const uint64_t wd = __shfl_sync(0xFFFFFFFFu, desired, src);
      const bool wa = __shfl_sync(0xFFFFFFFFu, is_accum, src);
      Locate wlc;
      wlc.bkt = __shfl_sync(0xFFFFFFFFu, l.bkt, src);
      wlc.pos = __shfl_sync(0xFFFFFFFFu, l.pos, src);
      wlc.d4 = __shfl_sync(0xFFFFFFFFu, l.d4, src);
      uint32_t slot = 0;
      uint64_t evk = 0;
      int r = warp_find_and_lock(t, wlc, wk, wd, slot, evk);
      if (r == kTimedOut) {
        if (wl == 0) atomicOr(t.error, kErrSpinTimeout);
      } else if (r != kRefused) {
        r = accum_apply<S, VT>(t, a, wi, wk, wa, wd, wlc, slot, evk, r, wl, 32,
                               []() { __syncwarp(); });
      }
      if (wl / W == static_cast<uint32_t>(src) / W) res = r;
    }
    if (in && a.status != nullptr && tile.lane == 0) a.status[i] = res;
  }
}

// ============================================================================
// assign_scores (reference assign_scores_kernel_with_filter.h:38-141) and
// erase (reference remove_kernel.h:33-113)
// ============================================================================
// Score update of existing keys (reference assign_scores_kernel_with_filter.h
// :38-141, score rule update_without_missed) or erase (reference
// remove_kernel.h:33-113: RECLAIM tombstone, score 0, reclaim digest, size
// decrement), in the warp-uniform rounds of the upsert family. One key per
// kExistTile-lane tile; the next key is read one iteration ahead.
constexpr uint32_t kExistTile = 4;
template <int S, bool kErase>
__global__ void __launch_bounds__(256, 8)
    existing_key_kernel(TableView t, const uint64_t* __restrict__ keys,
                        const uint64_t* __restrict__ scores, uint64_t n,
                        uint64_t epoch) {
  constexpr uint32_t W = kExistTile;
  constexpr uint32_t KPW = 32 / W;  // keys per warp
  __shared__ uint64_t s_clock;
  if (threadIdx.x == 0) s_clock = global_timer_ns();
  __syncthreads();
  const uint64_t clk = s_clock;
  const TileW<W> tile;
  const uint32_t wl = threadIdx.x & 31;
  const uint64_t nwarps = (uint64_t)gridDim.x * (blockDim.x / 32);
  const uint64_t warp = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) / 32;
  const uint64_t stride = nwarps * KPW;
  uint64_t next = warp * KPW + wl / W < n ? keys[warp * KPW + wl / W] : 0;
  for (uint64_t base = warp * KPW; base < n; base += stride) {
    const uint64_t i = base + wl / W;
    uint64_t key = 0, t0 = 0;
    bool todo = false;
    Locate l;
    l.bkt = 0;
    l.pos = 0;
    l.d4 = 0;
    if (i < n) {
      key = next;
      if (i + stride < n) next = keys[i + stride];
      if (!is_reserved(key)) {
        l = locate(t, key);
        todo = true;
      }
    }
    for (int round = 0;; round++) {
      bool again = false;
      if constexpr (kErase) {
        if (todo) {
          if (tile_erase(t, tile, l, key))
            todo = false;
          else if (retry_expired(t, tile, t0, 202))
            todo = false;
          else
            again = true;
        }
      } else if (todo) {
        const int p = tile_locate_existing<kWalkStop>(t, tile, l, key);
        if (p >= 0) {
          // The score of the slot found, as the reference updates it
          // (assign_scores_kernel_with_filter.h:65-140, no lock): no other
          // operation of this launch moves the key. The Lfu rules add, so a
          // key repeated in the batch takes every addition: an atomic add,
          // or for EpochLfu's saturating low half a CAS loop.
          if (tile.lane == 0) {
            uint64_t* sp = t.scores + l.bkt * kBucket + p;
            uint64_t ns;
            if constexpr (S == kLfu) {
              if (scores != nullptr)
                atomicAdd(reinterpret_cast<unsigned long long*>(sp), scores[i]);
            } else if constexpr (S == kEpochLfu) {
              uint64_t old = ld_relaxed_u64(sp);
              while (score_without_missed<S>(old, scores, i, epoch, clk, &ns)) {
                const uint64_t prev = cas_u64(sp, old, ns);
                if (prev == old) break;
                old = prev;
              }
            } else if (score_without_missed<S>(0, scores, i, epoch, clk, &ns)) {
              *sp = ns;
            }
          }
          todo = false;
        } else if (p == -1) {
          todo = false;
        } else if (retry_expired(t, tile, t0, 201)) {
          todo = false;
        } else {
          again = true;
        }
      }
      if (!__any_sync(0xFFFFFFFFu, again)) break;
      backoff(round);
    }
  }
}

// lock_keys (reference lock_keys_kernel.h:17-140): each present key is
// found through its digests, locked, given its score by the hit rule
// (update_with_digest with new_insert = false) and left locked with the
// caller-lock word; its key-word address goes to locked_key_ptrs[i]. Absent
// keys get nullptr and false.
template <int S>
__global__ void __launch_bounds__(256, 8)
    lock_keys_kernel(TableView t, const uint64_t* __restrict__ keys,
                     uint64_t** __restrict__ locked_key_ptrs, bool* __restrict__ succeeded,
                     const uint64_t* __restrict__ scores, uint64_t n, uint64_t epoch) {
  constexpr uint32_t W = kExistTile;
  constexpr uint32_t KPW = 32 / W;  // keys per warp
  __shared__ uint64_t s_clock;
  if (threadIdx.x == 0) s_clock = global_timer_ns();
  __syncthreads();
  const uint64_t clk = s_clock;
  const TileW<W> tile;
  const uint32_t wl = threadIdx.x & 31;
  const uint64_t nwarps = (uint64_t)gridDim.x * (blockDim.x / 32);
  const uint64_t warp = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) / 32;
  for (uint64_t base = warp * KPW; base < n; base += nwarps * KPW) {
    const uint64_t i = base + wl / W;
    uint64_t key = 0, t0 = 0;
    bool todo = false, ok = false;
    uint64_t* addr = nullptr;
    Locate l;
    l.bkt = 0;
    l.pos = 0;
    l.d4 = 0;
    if (i < n) {
      key = keys[i];
      if (!is_reserved(key)) {
        l = locate(t, key);
        todo = true;
      }
    }
    for (int round = 0;; round++) {
      bool again = false;
      if (todo) {
        const int p = tile_locate_existing<kWalk>(t, tile, l, key);
        bool got = false;
        const uint64_t s = l.bkt * kBucket + (p < 0 ? 0 : p);
        if (p >= 0 && tile.lane == 0)
          got = cas_acquire_u64(t.keys + s, key, kLockedKey) == key;
        if (tile.shfl(got, 0)) {
          if (tile.lane == 0) {
            uint64_t ns;
            const uint64_t old =
                (S == kLfu || S == kEpochLfu) ? ld_relaxed_u64(t.scores + s) : 0;
            const uint64_t desired = desired_when_missed<S>(scores, i, epoch, clk);
            if (score_on_write<S>(old, scores, i, desired, false, &ns)) t.scores[s] = ns;
            atomicAdd(t.sizes + l.bkt, 1 << kLockShift);
            store_release_u64(t.keys + s, kUserLockedKey);
          }
          addr = t.keys + s;
          ok = true;
          todo = false;
        } else if (p == -1) {
          todo = false;
        } else if (retry_expired(t, tile, t0, 203)) {
          todo = false;
        } else {
          again = true;
        }
      }
      if (!__any_sync(0xFFFFFFFFu, again)) break;
      backoff(round);
    }
    if (i < n && tile.lane == 0) {
      locked_key_ptrs[i] = ok ? addr : nullptr;
      if (succeeded != nullptr) succeeded[i] = ok;
    }
  }
}

// unlock_keys (reference unlock_keys_kernel.h:17-60): a key word that still
// holds the caller-lock word gets its key back; any other pointer (null,
// outside this table's key array, or a word that is not locked) fails.
__global__ void __launch_bounds__(256)
    unlock_keys_kernel(TableView t, uint64_t n, uint64_t* const* __restrict__ locked_key_ptrs,
                       const uint64_t* __restrict__ keys, bool* __restrict__ succeeded) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    uint64_t* p = locked_key_ptrs[i];
    const uint64_t key = keys[i];
    bool ok = false;
    if (p != nullptr && p >= t.keys && p < t.keys + t.capacity && !is_reserved(key)) {
      const uint64_t slot = static_cast<uint64_t>(p - t.keys);
      ok = cas_u64(p, kUserLockedKey, kLockedKey) == kUserLockedKey;
      if (ok) {
        atomicSub(t.sizes + (slot >> kBucketShift), 1 << kLockShift);
        store_release_u64(p, key);
      }
    }
    if (succeeded != nullptr) succeeded[i] = ok;
  }
}

// clear (reference clear_kernel.h:29-60) is init_buckets_kernel without the
// score reset.

// ============================================================================
// export_batch (reference dump_kernel.h:37-123): slots [offset, offset+len).
// A block takes 256 consecutive slots: each warp ballot-compacts its 32, the
// block reserves its whole output range with one atomic (one per 256 slots
// on a single counter word), and the warp's lanes then copy the 16-byte
// vectors of its live rows. Output order is not deterministic (same as the
// reference).
// ============================================================================
template <int VW>
__global__ void __launch_bounds__(256)
    export_kernel(TableView t, uint64_t offset, uint64_t len,
                  unsigned long long* __restrict__ counter,
                  uint64_t* __restrict__ out_keys, uint8_t* __restrict__ out_values,
                  uint64_t* __restrict__ out_scores) {
  using V = typename VecOf<VW>::T;
  __shared__ uint32_t warp_cnt[8];
  __shared__ unsigned long long block_base;
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t wi = threadIdx.x >> 5;
  const uint32_t vb = t.value_bytes;
  const uint32_t nv = vb / VW;
  for (uint64_t c0 = uint64_t{blockIdx.x} * 256; c0 < len; c0 += uint64_t{gridDim.x} * 256) {
    const uint64_t r = c0 + threadIdx.x;
    const uint64_t s = offset + r;
    uint64_t k = kEmptyKey;
    if (r < len) k = t.keys[s];
    const bool live = !is_reserved(k);
    const uint32_t vote = __ballot_sync(0xFFFFFFFFu, live);
    if (lane == 0) warp_cnt[wi] = __popc(vote);
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t total = 0;
      for (uint32_t j = 0; j < 8; j++) total += warp_cnt[j];
      block_base = total ? atomicAdd(counter, static_cast<unsigned long long>(total)) : 0;
    }
    __syncthreads();
    unsigned long long base = block_base;
    for (uint32_t j = 0; j < wi; j++) base += warp_cnt[j];
    if (live) {
      const uint64_t o = base + __popc(vote & ((1u << lane) - 1u));
      out_keys[o] = k;
      if (out_scores != nullptr) out_scores[o] = t.scores[s];
    }
    if (out_values != nullptr) {
      const uint32_t nvec = __popc(vote) * nv;
      const uint64_t w0 = offset + c0 + wi * 32;  // slot of this warp's lane 0
      for (uint32_t x = lane; x < nvec; x += 32) {
        const uint32_t rank = x / nv;
        const uint32_t v = x - rank * nv;
        const uint64_t ss = w0 + __fns(vote, 0, static_cast<int>(rank) + 1);
        const V* sp = reinterpret_cast<const V*>(
            value_ptr(t, ss >> kBucketShift, static_cast<uint32_t>(ss & (kBucket - 1))));
        reinterpret_cast<V*>(out_values + (base + rank) * vb)[v] = sp[v];
      }
    }
    __syncthreads();  // warp_cnt and block_base are rewritten next chunk
  }
}

// ============================================================================
// Rehash after the bucket count doubles (reference rehash_kernel.h:30-207),
// in two passes.
//
// The reference scans an old bucket from slot 0, moves the first key whose
// new bucket differs (copy_key_to_new_bucket :30-67: first EMPTY slot of the
// new bucket from the key's start position, cyclically), back-shifts the
// entries behind the hole (defragmentation_for_rehash :77-135: the first
// entry before the next EMPTY_KEY that may move into the hole moves there,
// and the hole follows it) and restarts at slot 0, so every restart finds
// the lowest slot that holds a key to move.
//
// Pass 1, rehash_replay_kernel: one thread per old bucket replays exactly
// that on a packed copy of the bucket in shared memory (per slot: start
// position, EMPTY_KEY flag, must-move flag, original slot: 16 bits), its
// must-move flags also held as a 128-bit register mask (the next key to
// move is the lowest must-move bit; a back-shift stops at the next
// EMPTY_KEY slot). An entry may fill a hole d slots behind it only if it
// sits at least d slots past its start position, and moves only bring
// entries closer to theirs, so the search for a filler also stops at the
// bucket's largest displacement. The chain of shift steps is inherently
// sequential, so a bucket gets one thread and an SM replays 768 buckets at
// once. Thread c keeps slots q and q + 1 in the two halves of word (q / 2)
// of column c, so the 32 threads of a warp always touch 32 different banks.
// Output per old bucket: the original slot of the entry that ends in each
// slot of the old and of the new bucket (one byte each, 0xFF: empty; the
// new bucket's bytes written as keys move), and both buckets' sizes.
//
// Both passes read the old key and score arrays; pass 2 writes every slot of
// both buckets into the new (doubled) arrays, so the old metadata is neither
// copied nor the new buckets cleared first.
//
// Pass 2, rehash_apply_kernel: one warp per old bucket moves keys, scores,
// digests and value rows by those maps: rows bound for the new bucket
// straight from their old slots, rows that change slot inside the old
// bucket through the warp's scratch rows. The final layout is the
// reference's, slot for slot.
// ============================================================================
constexpr uint32_t kReplayBuckets = 256;  // buckets (threads) per replay block
// packed slot: start position (bits 0-6), EMPTY_KEY (7), bound for the new
// bucket (8), original slot (9-15)
constexpr uint32_t kEntEmpty = 0x80u;
constexpr uint32_t kEntMove = 0x100u;
constexpr uint32_t kEntSrcShift = 9;
// packed slots (2 bytes, [slot / 2][bucket][2]) and per bucket the
// must-move mask and the largest displacement: 70 KiB, three blocks per SM
constexpr size_t kReplaySmem = size_t{kBucket} * kReplayBuckets * 2 +
                               size_t{kReplayBuckets} * 3 * 8;

__device__ __forceinline__ uint32_t ent_index(uint32_t q, uint32_t c) {
  return ((q >> 1) * kReplayBuckets + c) * 2 + (q & 1);
}


__device__ __forceinline__ void bit_set(uint64_t& m0, uint64_t& m1, uint32_t x) {
  if (x < 64)
    m0 |= uint64_t{1} << x;
  else
    m1 |= uint64_t{1} << (x - 64);
}
__device__ __forceinline__ void bit_clear(uint64_t& m0, uint64_t& m1, uint32_t x) {
  if (x < 64)
    m0 &= ~(uint64_t{1} << x);
  else
    m1 &= ~(uint64_t{1} << (x - 64));
}

// First clear bit of the 128-bit mask (m0: slots 0-63, m1: 64-127) at or
// after `from`, cyclically; kBucket when every slot is set.
__device__ __forceinline__ uint32_t first_free_from(uint64_t m0, uint64_t m1, uint32_t from) {
  const uint64_t f0 = ~m0, f1 = ~m1;
  if (from < 64) {
    const uint64_t c = f0 & (~uint64_t{0} << from);
    if (c) return __ffsll(static_cast<long long>(c)) - 1;
    if (f1) return 64 + __ffsll(static_cast<long long>(f1)) - 1;
    if (f0) return __ffsll(static_cast<long long>(f0)) - 1;
    return kBucket;
  }
  const uint64_t c = f1 & (~uint64_t{0} << (from - 64));
  if (c) return 64 + __ffsll(static_cast<long long>(c)) - 1;
  if (f0) return __ffsll(static_cast<long long>(f0)) - 1;
  if (f1) return 64 + __ffsll(static_cast<long long>(f1)) - 1;
  return kBucket;
}

__global__ void __launch_bounds__(kReplayBuckets)
    rehash_replay_kernel(TableView t, uint64_t old_nb, const uint64_t* __restrict__ old_keys,
                         uint8_t* __restrict__ maps) {
  extern __shared__ uint64_t replay_smem[];
  // [3][kReplayBuckets]: must-move mask (2 words), largest displacement
  uint64_t* mask = replay_smem;
  uint16_t* E = reinterpret_cast<uint16_t*>(replay_smem + 3 * kReplayBuckets);
  constexpr uint32_t kWarps = kReplayBuckets / 32;
  const uint32_t lane = threadIdx.x & 31, wi = threadIdx.x >> 5;
  const uint32_t c = threadIdx.x;  // this thread's bucket column
  const uint64_t new_cap = t.capacity;  // power of two after doubling
  for (uint64_t b0 = uint64_t{blockIdx.x} * kReplayBuckets; b0 < old_nb;
       b0 += uint64_t{gridDim.x} * kReplayBuckets) {
    // pack: warp wi reads buckets wi, wi + kWarps, ... with coalesced loads
    for (uint32_t i0 = wi; i0 < kReplayBuckets; i0 += 4 * kWarps) {
      // four buckets' keys in flight per warp
      uint64_t kk[4][4];
#pragma unroll
      for (uint32_t u = 0; u < 4; u++)
#pragma unroll
        for (uint32_t j = 0; j < 4; j++) {
          const uint64_t bu = b0 + i0 + u * kWarps;
          kk[u][j] = bu < old_nb ? old_keys[bu * kBucket + lane + 32 * j] : kEmptyKey;
        }
#pragma unroll
      for (uint32_t u = 0; u < 4; u++) {
      const uint32_t i = i0 + u * kWarps;
      if (b0 + i >= old_nb) break;
      const uint64_t b = b0 + i;
      uint32_t mv[4], dmax = 0;
#pragma unroll
      for (uint32_t j = 0; j < 4; j++) {
        const uint32_t q = lane + 32 * j;
        const uint64_t k = kk[u][j];
        const uint64_t h = murmur3(k);
        uint32_t e = static_cast<uint32_t>(h & (kBucket - 1)) | (q << kEntSrcShift);
        if (k == kEmptyKey)
          e |= kEntEmpty;
        else if (k != kReclaimKey && ((h & (new_cap - 1)) >> kBucketShift) != b)
          e |= kEntMove;
        E[ent_index(q, i)] = static_cast<uint16_t>(e);
        if (!(e & kEntEmpty)) dmax = max(dmax, (q - static_cast<uint32_t>(h)) & (kBucket - 1));
        mv[j] = __ballot_sync(0xFFFFFFFFu, (e & kEntMove) != 0);
      }
      dmax = __reduce_max_sync(0xFFFFFFFFu, dmax);
      // the new bucket's map row starts empty; the replay fills what it moves
      reinterpret_cast<uint32_t*>(maps + b * 2 * kBucket + kBucket)[lane] = 0xFFFFFFFFu;
      if (lane == 0) {
        mask[2 * kReplayBuckets + i] = dmax;
        mask[0 * kReplayBuckets + i] = mv[0] | (uint64_t{mv[1]} << 32);
        mask[1 * kReplayBuckets + i] = mv[2] | (uint64_t{mv[3]} << 32);
      }
      }
    }
    __syncthreads();
    const uint64_t b = b0 + c;
    if (b < old_nb) {
      uint64_t mv0 = mask[0 * kReplayBuckets + c], mv1 = mask[1 * kReplayBuckets + c];
      // slot q of this column: col[(q / 2) * 2 kReplayBuckets + q % 2]
      uint16_t* col = E + 2 * c;
      // no entry can fill a hole farther behind it than this
      const uint32_t reach = static_cast<uint32_t>(mask[2 * kReplayBuckets + c]) + 1;
      uint8_t* nmap = maps + b * 2 * kBucket + kBucket;
      uint64_t nocc0 = 0, nocc1 = 0;
      int32_t moved = 0, removed = 0;
      while (mv0 | mv1) {
        const uint32_t q = mv0 ? __ffsll(static_cast<long long>(mv0)) - 1
                               : 64 + __ffsll(static_cast<long long>(mv1)) - 1;
        const uint32_t e = col[(q >> 1) * 2 * kReplayBuckets + (q & 1)];
        // the new start position: new capacity >= kBucket, so the key's low
        // hash bits are its start position in either bucket
        const uint32_t p = first_free_from(nocc0, nocc1, e & (kBucket - 1));
        if (p < kBucket) {
          nmap[p] = static_cast<uint8_t>(e >> kEntSrcShift);
          bit_set(nocc0, nocc1, p);
          moved++;
        }
        removed++;
        col[(q >> 1) * 2 * kReplayBuckets + (q & 1)] = kEntEmpty;
        bit_clear(mv0, mv1, q);
        // back-shift behind the hole. The reference lets the entry at cur
        // fill the hole at rm when its start position lies outside the
        // cyclic interval (rm, cur] (rehash_kernel.h:101-103): the same as
        // sitting at least `off` = cur - rm slots past its start position.
        uint32_t rm = q;
        for (uint32_t off = 1; off < reach;) {
          const uint32_t cur = (rm + off) & (kBucket - 1);
          const uint32_t ce = col[(cur >> 1) * 2 * kReplayBuckets + (cur & 1)];
          if (ce & kEntEmpty) break;
          if (((cur - ce) & (kBucket - 1)) >= off) {
            col[(rm >> 1) * 2 * kReplayBuckets + (rm & 1)] = static_cast<uint16_t>(ce);
            col[(cur >> 1) * 2 * kReplayBuckets + (cur & 1)] = kEntEmpty;
            if (ce & kEntMove) {
              bit_clear(mv0, mv1, cur);
              bit_set(mv0, mv1, rm);
            }
            rm = cur;
            off = 1;
          } else {
            off++;
          }
        }
      }
      t.sizes[b] -= removed;
      t.sizes[b + old_nb] = moved;
    }
    __syncthreads();
    // maps: bytes [0, kBucket) the original slot of each final old-bucket
    // slot (written here), [kBucket, 2 kBucket) of each new-bucket slot
    // (written by the replay); 0xFF: empty
    for (uint32_t i = wi; i < kReplayBuckets && b0 + i < old_nb; i += kWarps) {
      uint32_t ow = 0;
#pragma unroll
      for (uint32_t k = 0; k < 4; k++) {
        const uint32_t q = lane * 4 + k;
        const uint32_t e = E[ent_index(q, i)];
        const uint32_t os = (e & kEntEmpty) ? 0xFFu : (e >> kEntSrcShift) & 0x7Fu;
        ow |= os << (8 * k);
      }
      reinterpret_cast<uint32_t*>(maps + (b0 + i) * 2 * kBucket)[lane] = ow;
    }
    __syncthreads();
  }
}

struct RehashStage {
  uint64_t okeys[kBucket];    // the old bucket's keys and scores before the rehash
  uint64_t oscores[kBucket];
  uint8_t osrc[kBucket];      // original slot of the entry ending at q (old bucket)
  uint8_t nsrc[kBucket];      // original slot of the entry ending at q (new bucket)
  uint8_t lsrc[2][kBucket];   // rows to copy: [0] into the new bucket,
  uint8_t ldst[2][kBucket];   // [1] to another slot of the old bucket
};

// Copies the rows lsrc[k] -> ldst[k], k < cnt (slots of bucket sb / db, or
// the warp's scratch rows). Rows of nv <= 32 vectors: the lanes form 32 / nv
// groups of nv, each group one row, four rows' loads in flight; longer rows:
// the warp walks each row 32 vectors at a time.
template <int VW>
__device__ __forceinline__ void warp_copy_list(const TableView& t, uint64_t sb, uint64_t db,
                                               uint8_t* scratch, bool src_scratch,
                                               bool dst_scratch, const uint8_t* lsrc,
                                               const uint8_t* ldst, uint32_t cnt,
                                               uint32_t lane) {
  using V = typename VecOf<VW>::T;
  const uint32_t vb = t.value_bytes;
  const uint32_t nv = vb / VW;
  auto sptr = [&](uint32_t q) {
    return reinterpret_cast<const V*>(src_scratch ? scratch + uint64_t{q} * vb
                                                  : value_ptr(t, sb, q));
  };
  auto dptr = [&](uint32_t q) {
    return reinterpret_cast<V*>(dst_scratch ? scratch + uint64_t{q} * vb : value_ptr(t, db, q));
  };
  if (nv <= 32) {
    const uint32_t rpi = 32 / nv, lq = lane / nv, lv = lane - lq * nv;
    if (lq >= rpi) return;
    uint32_t k = lq;
    for (; k + 3 * rpi < cnt; k += 4 * rpi) {
      V x[4];
#pragma unroll
      for (uint32_t u = 0; u < 4; u++) x[u] = sptr(lsrc[k + u * rpi])[lv];
#pragma unroll
      for (uint32_t u = 0; u < 4; u++) dptr(ldst[k + u * rpi])[lv] = x[u];
    }
    for (; k < cnt; k += rpi) dptr(ldst[k])[lv] = sptr(lsrc[k])[lv];
  } else {
    for (uint32_t k = 0; k < cnt; k++) {
      const V* sp = sptr(lsrc[k]);
      V* dp = dptr(ldst[k]);
      for (uint32_t v = lane; v < nv; v += 32) dp[v] = sp[v];
    }
  }
}

template <int VW>
__global__ void __launch_bounds__(256)
    rehash_apply_kernel(TableView t, uint64_t old_nb, const uint64_t* __restrict__ old_keys,
                        const uint64_t* __restrict__ old_scores,
                        const uint8_t* __restrict__ maps, uint8_t* __restrict__ scratch) {
  __shared__ RehashStage stage[8];
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t wi = threadIdx.x >> 5;
  RehashStage& st = stage[wi];
  const uint64_t nwarps = (uint64_t)gridDim.x * (blockDim.x / 32);
  const uint64_t gw = blockIdx.x * (uint64_t)(blockDim.x / 32) + wi;
  uint8_t* rows = scratch + gw * kBucket * t.value_bytes;  // this warp's scratch rows
  constexpr uint32_t kNone = 0xFFu;
  const uint32_t lt = (1u << lane) - 1;
  for (uint64_t b = gw; b < old_nb; b += nwarps) {
    const uint64_t nbk = b + old_nb;
#pragma unroll
    for (uint32_t j = 0; j < 4; j++) {
      const uint32_t q = lane + 32 * j;
      st.okeys[q] = old_keys[b * kBucket + q];
      st.oscores[q] = old_scores[b * kBucket + q];
    }
    const uint32_t* mw = reinterpret_cast<const uint32_t*>(maps + b * 2 * kBucket);
    reinterpret_cast<uint32_t*>(st.osrc)[lane] = mw[lane];
    reinterpret_cast<uint32_t*>(st.nsrc)[lane] = mw[32 + lane];
    __syncwarp();
    // the rows that move: into the new bucket, and to another slot of the
    // old bucket (reclaimed slots carry no row)
    uint32_t c0 = 0, c1 = 0;
#pragma unroll
    for (uint32_t j = 0; j < 4; j++) {
      const uint32_t q = lane + 32 * j;
      const uint32_t n = st.nsrc[q], o = st.osrc[q];
      const bool p0 = n != kNone;
      const bool p1 = o != kNone && o != q && st.okeys[o] != kReclaimKey;
      const uint32_t m0 = __ballot_sync(0xFFFFFFFFu, p0);
      const uint32_t m1 = __ballot_sync(0xFFFFFFFFu, p1);
      if (p0) {
        const uint32_t at = c0 + __popc(m0 & lt);
        st.lsrc[0][at] = static_cast<uint8_t>(n);
        st.ldst[0][at] = static_cast<uint8_t>(q);
      }
      if (p1) {
        const uint32_t at = c1 + __popc(m1 & lt);
        st.lsrc[1][at] = static_cast<uint8_t>(o);
        st.ldst[1][at] = static_cast<uint8_t>(q);
      }
      c0 += __popc(m0);
      c1 += __popc(m1);
    }
    __syncwarp();
    // new bucket rows from the old slots, and the old bucket's moving rows
    // into scratch, before any old row is overwritten
    warp_copy_list<VW>(t, b, nbk, rows, false, false, st.lsrc[0], st.ldst[0], c0, lane);
    warp_copy_list<VW>(t, b, b, rows, false, true, st.lsrc[1], st.ldst[1], c1, lane);
    __syncwarp();
    warp_copy_list<VW>(t, b, b, rows, true, false, st.ldst[1], st.ldst[1], c1, lane);
#pragma unroll
    for (uint32_t j = 0; j < 4; j++) {
      const uint32_t q = lane + 32 * j;
      const uint32_t o = st.osrc[q], n = st.nsrc[q];
      const uint64_t ok = o == kNone ? kEmptyKey : st.okeys[o];
      const uint64_t nk = n == kNone ? kEmptyKey : st.okeys[n];
      t.keys[b * kBucket + q] = ok;
      t.scores[b * kBucket + q] = o == kNone ? 0 : st.oscores[o];
      t.digests[b * kBucket + q] =
          ok == kEmptyKey ? kEmptyDigest : digest_of_hash(murmur3(ok));
      t.keys[nbk * kBucket + q] = nk;
      t.scores[nbk * kBucket + q] = n == kNone ? 0 : st.oscores[n];
      t.digests[nbk * kBucket + q] =
          nk == kEmptyKey ? kEmptyDigest : digest_of_hash(murmur3(nk));
    }
    __syncwarp();
  }
}

}  // namespace hkvb
