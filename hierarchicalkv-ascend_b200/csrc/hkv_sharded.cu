// hkv_sharded.cu -- table sharded over the GPUs of one node (no reference
// counterpart: the reference drives a single device).
//
// Each rank owns one TableImpl; a key belongs to owner = (Murmur3(key) >> 40)
// % world (hash bits 40.. so that a shard's keys do not share the low hash
// bits that choose their bucket and start slot). A collective call takes
// every rank's batch, merges duplicate keys of insert-like batches
// (hkv_dedup.cuh; skipped for unique_key batches), moves each key to its
// owner, runs the local operation there (the same key from several ranks is
// applied in rank order) and brings results back. Two transports:
//   * peer memory (default when the shards never grow): CUDA IPC windows
//     over NVLink, data written locally and read remotely, device flags
//     between the steps, no host synchronisation (see the transport
//     section below);
//   * NCCL grouped send/recv: counts, then keys / scores / value rows, with
//     one host synchronisation per call to size the receive buffers.
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "hkv_table.cuh"

namespace hkvb {
namespace {

#define NCCL_TRY(expr)                                                   \
  do {                                                                   \
    ncclResult_t r_ = (expr);                                            \
    if (r_ != ncclSuccess)                                               \
      throw HkvError{HKV_ERR_CUDA, std::string(#expr) + ": " +           \
                                       ncclGetErrorString(r_)};          \
  } while (0)

constexpr int kMaxWorld = 64;

struct Offsets {
  uint64_t off[kMaxWorld];
};

__device__ __forceinline__ uint32_t owner_of(uint64_t key, uint32_t world) {
  return static_cast<uint32_t>((murmur3(key) >> 40) % world);
}

// Count representatives per destination and give each its rank within it.
__global__ void route_count_kernel(const uint64_t* __restrict__ ukeys,
                                   const uint32_t* __restrict__ dm, uint64_t n,
                                   uint32_t world, uint32_t* __restrict__ counts,
                                   uint32_t* __restrict__ dest,
                                   uint32_t* __restrict__ rank_in_dest) {
  __shared__ uint32_t local[kMaxWorld];
  __shared__ uint32_t base[kMaxWorld];
  const uint64_t m = dm != nullptr ? *dm : n;
  for (uint64_t b0 = blockIdx.x * (uint64_t)blockDim.x; b0 < m;
       b0 += (uint64_t)gridDim.x * blockDim.x) {
    for (uint32_t w = threadIdx.x; w < world; w += blockDim.x) local[w] = 0;
    __syncthreads();
    const uint64_t u = b0 + threadIdx.x;
    uint32_t d = 0, r = 0;
    if (u < m) {
      d = owner_of(ukeys[u], world);
      r = atomicAdd(&local[d], 1u);
    }
    __syncthreads();
    for (uint32_t w = threadIdx.x; w < world; w += blockDim.x)
      base[w] = local[w] ? atomicAdd(&counts[w], local[w]) : 0u;
    __syncthreads();
    if (u < m) {
      dest[u] = d;
      rank_in_dest[u] = base[d] + r;
    }
    __syncthreads();
  }
}

// Scatter representatives (key, score, value row) into the send buffers.
template <int VW>
__global__ void route_pack_kernel(const uint64_t* __restrict__ ukeys,
                                  const uint64_t* __restrict__ uscores,
                                  const uint8_t* __restrict__ rows,
                                  const uint32_t* __restrict__ row_of,
                                  const uint32_t* __restrict__ dm, uint64_t n,
                                  const uint32_t* __restrict__ dest,
                                  const uint32_t* __restrict__ rank_in_dest,
                                  Offsets soff, uint32_t vb,
                                  uint64_t* __restrict__ skeys,
                                  uint64_t* __restrict__ sscores,
                                  uint8_t* __restrict__ srows) {
  const Tile tile;
  const uint64_t m = dm != nullptr ? *dm : n;
  const uint64_t ntiles = (uint64_t)gridDim.x * (blockDim.x / kTile);
  for (uint64_t u = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) / kTile;
       u < m; u += ntiles) {
    const uint64_t p = soff.off[dest[u]] + rank_in_dest[u];
    if (tile.lane == 0) {
      skeys[p] = ukeys[u];
      if (sscores) sscores[p] = uscores[u];
    }
    if (srows)
      copy_row<VW>(srows + p * vb,
                   rows + static_cast<uint64_t>(row_of ? row_of[u] : u) * vb,
                   vb, tile.lane, kTile);
  }
}

// Bring results back to representatives, then to every occurrence.
// mode 0: find (rows only where found), 1: find_or_insert (rows where the
// owner found or inserted the key).
template <int VW>
__global__ void route_unpack_kernel(int mode, const uint32_t* __restrict__ uid_of,
                                    uint64_t n, const uint32_t* __restrict__ dest,
                                    const uint32_t* __restrict__ rank_in_dest,
                                    Offsets soff, uint32_t vb,
                                    const uint8_t* __restrict__ brows,
                                    const uint8_t* __restrict__ bflag,
                                    const uint64_t* __restrict__ bscores,
                                    uint8_t* __restrict__ values,
                                    bool* __restrict__ founds,
                                    uint64_t* __restrict__ scores) {
  const Tile tile;
  const uint64_t ntiles = (uint64_t)gridDim.x * (blockDim.x / kTile);
  for (uint64_t i = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) / kTile;
       i < n; i += ntiles) {
    const uint32_t u = uid_of != nullptr ? uid_of[i] : static_cast<uint32_t>(i);
    bool ok = false;
    uint64_t p = 0;
    if (u != 0xFFFFFFFFu) {
      p = soff.off[dest[u]] + rank_in_dest[u];
      const uint8_t f = bflag[p];
      ok = mode == 0 ? f != 0
                     : (f != kRefused && f != kIllegal && f != kTimedOut);
    }
    if (tile.lane == 0) {
      if (founds) founds[i] = ok;
      if (ok && scores && bscores) scores[i] = bscores[p];
    }
    if (ok && values)
      copy_row<VW>(values + i * vb, brows + p * vb, vb, tile.lane, kTile);
  }
}

#define SHARD_DISPATCH_VW(vw, ...) \
  do {                             \
    if ((vw) == 16) {              \
      constexpr int VW = 16;       \
      __VA_ARGS__;                 \
    } else if ((vw) == 4) {        \
      constexpr int VW = 4;        \
      __VA_ARGS__;                 \
    } else {                       \
      constexpr int VW = 1;        \
      __VA_ARGS__;                 \
    }                              \
  } while (0)

uint64_t ceil_div(uint64_t a, uint64_t b) { return (a + b - 1) / b; }

// ============================================================================
// Peer-memory transport. Every rank exposes one "window" of device memory to
// the others (CUDA IPC over NVLink). All bulk data is written locally and
// read by the peer that needs it: on these GPUs loads from a peer's memory
// run at about 740 GB/s while stores into it reach about 320 GB/s.
//   route   the requester sorts its keys (+ scores, + value rows) by owner
//           into its own send area, one region of max_batch entries per
//           owner, remembers where each key went, and stores
//           (epoch << 32 | count) into the owner's arrive[requester] flag;
//   serve   the owner waits for every arrive flag of this epoch, runs the
//           table kernel reading each requester's region over NVLink, and
//           writes the results into its own result area (one region per
//           requester), then stores epoch into every requester's done[owner];
//   finish  the requester waits for every done flag and reads its results
//           from the owners' result areas into the caller's buffers.
// A requester starts its next route only after its finish, which waited for
// every owner to finish serving (and so reading) this call, and an owner
// overwrites its result area only after every requester has arrived for the
// next call (and so finished reading this one): single buffers suffice. All
// waits are bounded (kSpinLimitNs): a rank that never arrives makes the
// others give up, flag kErrSpinTimeout and treat its region as empty.
// ============================================================================
// The result area holds, per requester region, value rows (vb bytes each,
// so a row keeps the alignment of the table's rows) and 16-byte tails: the
// score and the found flag for find, the Occupy status for find_or_insert.
struct WinLayout {
  uint64_t arrive, done;                       // kMaxWorld flags, 64 B apart
  uint64_t snd_keys, snd_scores, snd_rows;     // world regions of M (by owner)
  uint64_t res_rows, res_tail;                 // world regions of M (by requester)
  uint64_t bytes;
  uint64_t M;
  uint32_t vb;
};

struct PeerBases {
  uint8_t* base[kMaxWorld];
};

WinLayout make_layout(uint32_t world, uint64_t M, uint32_t vb) {
  auto up = [](uint64_t x) { return (x + 255) & ~uint64_t{255}; };
  WinLayout l{};
  uint64_t o = 0;
  l.arrive = o;
  o = up(o + kMaxWorld * 64);
  l.done = o;
  o = up(o + kMaxWorld * 64);
  const uint64_t R = uint64_t{world} * M;
  l.snd_keys = o;
  o = up(o + R * 8);
  l.snd_scores = o;
  o = up(o + R * 8);
  l.snd_rows = o;
  o = up(o + R * vb);
  l.res_rows = o;
  o = up(o + R * vb);
  l.res_tail = o;
  o = up(o + R * 16);
  l.bytes = o;
  l.M = M;
  l.vb = vb;
  return l;
}

__device__ __forceinline__ uint64_t* flag_at(uint8_t* base, uint64_t off,
                                             uint32_t i) {
  return reinterpret_cast<uint64_t*>(base + off + uint64_t{i} * 64);
}

// route: sort this rank's keys by owner into its own send area. `keys` are
// the batch keys (find, or distinct keys) or the merged representatives
// (count *dm); inv maps each send position back to its key.
template <int VW>
__global__ void __launch_bounds__(256)
    p2p_route_kernel(const uint64_t* __restrict__ keys,
                     const uint64_t* __restrict__ scores,
                     const uint8_t* __restrict__ rows,
                     const uint32_t* __restrict__ row_of,
                     const uint32_t* __restrict__ dm, uint64_t n,
                     uint32_t world, uint32_t self, PeerBases peers,
                     WinLayout lay, uint32_t* __restrict__ counters,
                     uint32_t* __restrict__ inv,
                     uint32_t* __restrict__ sent, uint64_t epoch,
                     int* __restrict__ err) {
  __shared__ uint32_t cnt[kMaxWorld];
  __shared__ uint32_t base[kMaxWorld];
  __shared__ uint64_t slot_of[256];
  __shared__ int last;
  const uint64_t m = dm != nullptr ? min(n, static_cast<uint64_t>(*dm)) : n;
  const uint32_t vb = lay.vb;
  uint8_t* win = peers.base[self];
  uint64_t* skeys = reinterpret_cast<uint64_t*>(win + lay.snd_keys);
  uint64_t* sscores = reinterpret_cast<uint64_t*>(win + lay.snd_scores);
  uint8_t* srows = win + lay.snd_rows;
  for (uint64_t b0 = uint64_t{blockIdx.x} * blockDim.x; b0 < m;
       b0 += uint64_t{gridDim.x} * blockDim.x) {
    for (uint32_t w = threadIdx.x; w < world; w += blockDim.x) cnt[w] = 0;
    __syncthreads();
    const uint64_t u = b0 + threadIdx.x;
    uint32_t d = 0, r = 0;
    uint64_t key = 0;
    if (u < m) {
      key = keys[u];
      d = owner_of(key, world);
      r = atomicAdd(&cnt[d], 1u);
    }
    __syncthreads();
    for (uint32_t w = threadIdx.x; w < world; w += blockDim.x)
      base[w] = cnt[w] ? atomicAdd(&counters[w], cnt[w]) : 0u;
    __syncthreads();
    uint64_t slot = ~uint64_t{0};
    if (u < m) {
      const uint64_t pos = uint64_t{base[d]} + r;
      if (pos < lay.M) {
        slot = uint64_t{d} * lay.M + pos;
        skeys[slot] = key;
        if (scores != nullptr) sscores[slot] = scores[u];
        inv[slot] = static_cast<uint32_t>(u);
      } else {
        atomicOr(err, kErrPeerOverflow);
      }
    }
    if (rows != nullptr) {
      slot_of[threadIdx.x] = slot;
      __syncthreads();
      // the block's rows, one 8-lane tile per row
      const Tile tile;
      for (uint32_t k = threadIdx.x / kTile; k < blockDim.x; k += blockDim.x / kTile) {
        const uint64_t uk = b0 + k;
        const uint64_t sk = slot_of[k];
        if (uk < m && sk != ~uint64_t{0})
          copy_row<VW>(srows + sk * vb,
                       rows + uint64_t{row_of != nullptr ? row_of[uk]
                                                         : static_cast<uint32_t>(uk)} * vb,
                       vb, tile.lane, kTile);
      }
    }
    __syncthreads();
  }
  // the last block to finish publishes the counts to the owners. Every
  // block's stores land in this GPU's L2 (the point peers read from) before
  // the block is counted; the flag store is a system-scope release, so an
  // owner that acquires it sees them.
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(&counters[world], 1u) == gridDim.x - 1;
  __syncthreads();
  if (last) {
    __threadfence();
    for (uint32_t w = threadIdx.x; w < world; w += blockDim.x) {
      const uint32_t c = min(atomicAdd(&counters[w], 0u), static_cast<uint32_t>(lay.M));
      sent[w] = c;
      st_release_sys_u64(flag_at(peers.base[w], lay.arrive, self), (epoch << 32) | c);
      counters[w] = 0;
    }
    if (threadIdx.x == 0) counters[world] = 0;
  }
}

// Waits (bounded) until flag_i holds epoch (in its high half when counted)
// for every i < world; writes the low halves to counts (0 for a flag that
// never came).
__device__ void wait_flags(uint8_t* base, uint64_t off, uint32_t world,
                           uint64_t epoch, bool counted, uint32_t* counts,
                           int* err, int site) {
  for (uint32_t w = threadIdx.x; w < world; w += blockDim.x) {
    const uint64_t* f = flag_at(base, off, w);
    const uint64_t t0 = global_timer_ns();
    uint64_t v = ld_acquire_sys_u64(f);
    bool ok = true;
    while ((counted ? (v >> 32) : v) != epoch) {
      if (global_timer_ns() - t0 > kSpinLimitNs) {
        ok = false;
        atomicOr(err, kErrSpinTimeout);
        atomicExch(err + 1, site);
        break;
      }
      __nanosleep(256);
      v = ld_acquire_sys_u64(f);
    }
    if (counts != nullptr) counts[w] = ok && counted ? static_cast<uint32_t>(v) : 0u;
  }
}

__global__ void p2p_wait_arrive_kernel(uint8_t* self_base, WinLayout lay,
                                       uint32_t world, uint64_t epoch,
                                       uint32_t* counts, int* err) {
  wait_flags(self_base, lay.arrive, world, epoch, true, counts, err, 301);
}

// serve: every result of this epoch is in place (written by the kernels
// before this one in stream order); tell each requester with a system-scope
// release
__global__ void p2p_signal_done_kernel(PeerBases peers, WinLayout lay,
                                       uint32_t world, uint32_t self,
                                       uint64_t epoch) {
  for (uint32_t w = threadIdx.x; w < world; w += blockDim.x)
    st_release_sys_u64(flag_at(peers.base[w], lay.done, self), epoch);
}

// finish of insert_or_assign: nothing comes back but the owners' done flags
__global__ void p2p_wait_done_kernel(uint8_t* self_base, WinLayout lay, uint32_t world,
                                     uint64_t epoch, int* err) {
  wait_flags(self_base, lay.done, world, epoch, false, nullptr, err, 302);
}

// finish: wait for every owner, then read the results in owner order. Block
// b reads owner b % world's result region for this rank front to back, so
// the tiles of a warp read consecutive rows and tails over NVLink; inv
// (written by route) maps each position back to its input (find, and
// find_or_insert of a batch without merged duplicates) or to its
// representative u (find_or_insert of a merged batch: the row goes to the
// representative's first occurrence row_of[u] and the status to ustatus[u],
// so each distinct key crosses NVLink once and its later occurrences copy it
// locally afterwards). A 4-lane tile per key issues the flag, score and row
// loads together, so a key costs one NVLink round trip. mode 0: find (rows,
// flags and scores of found keys); mode 1: find_or_insert, rows of the keys
// the owner found (an inserted key's row is the caller's own input row,
// already in place). sent[o] is the number of keys this rank routed to
// owner o.
template <int VW>
__global__ void __launch_bounds__(256)
    p2p_finish_ordered_kernel(int mode, PeerBases peers, WinLayout lay, uint32_t world,
                              uint32_t self, uint64_t epoch, int* err,
                              const uint32_t* __restrict__ sent,
                              const uint32_t* __restrict__ inv,
                              uint8_t* __restrict__ values, bool* __restrict__ founds,
                              uint64_t* __restrict__ scores,
                              const uint32_t* __restrict__ row_of,
                              uint8_t* __restrict__ ustatus) {
  wait_flags(peers.base[self], lay.done, world, epoch, false, nullptr, err, 302);
  __syncthreads();
  using V = typename VecOf<VW>::T;
  constexpr uint32_t W = 4;
  constexpr uint32_t kTilesPerBlock = 256 / W;
  constexpr uint32_t kHead = 4;  // row vectors per lane held in registers
  const TileW<W> tile;
  const uint32_t vb = lay.vb;
  const uint32_t nv = vb / VW;
  const uint32_t o = blockIdx.x % world;
  const uint64_t step = uint64_t{gridDim.x / world} * kTilesPerBlock;
  const uint64_t c = min(static_cast<uint64_t>(sent[o]), lay.M);
  const uint8_t* ob = peers.base[o];
  const uint64_t region = uint64_t{self} * lay.M;
  const uint32_t* invo = inv + uint64_t{o} * lay.M;
  for (uint64_t pos = uint64_t{blockIdx.x / world} * kTilesPerBlock + threadIdx.x / W;
       pos < c; pos += step) {
    const uint64_t slot = region + pos;
    const V* sp = reinterpret_cast<const V*>(ob + lay.res_rows + slot * vb);
    V head[kHead];
#pragma unroll
    for (uint32_t h = 0; h < kHead; h++)
      if (values != nullptr && tile.lane + h * W < nv) head[h] = __ldcg(sp + tile.lane + h * W);
    // tail: find -> score (8 bytes) | found flag; find_or_insert -> status
    uint4 tail = make_uint4(0, 0, 0, 0);
    if (tile.lane == 0)
      tail = __ldcg(reinterpret_cast<const uint4*>(ob + lay.res_tail) + slot);
    const uint32_t u = invo[pos];
    const uint64_t i = row_of != nullptr ? row_of[u] : u;
    const uint32_t f = tile.shfl(tail.z & 0xFFu, 0);
    const bool ok = mode == 0 ? f != 0 : (f != kRefused && f != kIllegal && f != kTimedOut);
    const uint64_t sc = (uint64_t{tail.y} << 32) | tail.x;
    if (tile.lane == 0) {
      if (founds != nullptr) founds[i] = ok;
      if (ok && scores != nullptr) scores[i] = sc;
      if (ustatus != nullptr) ustatus[u] = static_cast<uint8_t>(f);
    }
    if ((mode == 0 ? ok : f == kDuplicate) && values != nullptr) {
      V* dp = reinterpret_cast<V*>(values + i * vb);
#pragma unroll
      for (uint32_t h = 0; h < kHead; h++)
        if (tile.lane + h * W < nv) dp[tile.lane + h * W] = head[h];
      for (uint32_t v = tile.lane + kHead * W; v < nv; v += W) dp[v] = __ldcg(sp + v);
    }
  }
}

}  // namespace

class ShardedImpl {
 public:
  ShardedImpl(const hkv_options& o, int key_type, int value_type, int strategy,
              const uint8_t id[128], int rank, int world, uint64_t max_batch)
      : rank_(rank), world_(world) {
    HKV_REQUIRE(world >= 1 && world <= kMaxWorld, HKV_ERR_INVALID,
                "world_size must be in [1, 64]");
    HKV_REQUIRE(rank >= 0 && rank < world, HKV_ERR_INVALID, "bad rank");
    local_ = new TableImpl(o, key_type, value_type, strategy);
    CUDA_TRY(cudaSetDevice(local_->device()));
    ncclUniqueId uid;
    static_assert(sizeof(uid.internal) == 128, "NCCL unique id size");
    std::memcpy(uid.internal, id, 128);
    NCCL_TRY(ncclCommInitRank(&comm_, world, uid, rank));
    CUDA_TRY(cudaHostAlloc(&h_counts_, 2 * kMaxWorld * sizeof(uint32_t),
                           cudaHostAllocDefault));
    CUDA_TRY(cudaMalloc(&d_counts_, 2 * kMaxWorld * sizeof(uint32_t)));
    CUDA_TRY(cudaDeviceGetAttribute(&sm_count_, cudaDevAttrMultiProcessorCount,
                                    local_->device()));
    if (max_batch > 0 && world > 1 && local_->at_max_capacity())
      setup_p2p(max_batch);
  }
  ~ShardedImpl() {
    if (p2p_) {
      // every rank is here: no peer writes into a window after this barrier
      cudaStream_t s = nullptr;
      ncclAllReduce(d_counts_, d_counts_ + kMaxWorld, 1, ncclUint32, ncclSum,
                    comm_, s);
      cudaStreamSynchronize(s);
      for (int p = 0; p < world_; p++)
        if (p != rank_ && peers_.base[p]) cudaIpcCloseMemHandle(peers_.base[p]);
      cudaFree(win_);
      cudaFree(d_route_counters_);
      cudaFree(d_inv_);
      cudaFree(d_sent_);
    }
    if (comm_) ncclCommDestroy(comm_);
    delete local_;
    cudaFree(d_counts_);
    cudaFreeHost(h_counts_);
  }
  bool peer_transport() const { return p2p_; }
  TableImpl* local() { return local_; }

  // kind: 0 find, 1 find_or_insert, 2 insert_or_assign
  void run(int kind, size_t n, const uint64_t* keys, uint8_t* values,
           bool* founds, uint64_t* scores, cudaStream_t s, bool unique) {
    if (p2p_) return run_p2p(kind, n, keys, values, founds, scores, s, unique);
    const uint32_t vb = local_->value_bytes();
    const int st = local_->strategy();
    Workspace ws(s, local_->pool());
    const uint64_t nn = std::max<uint64_t>(n, 1);
    // Which buffers travel is fixed by the call kind and the strategy, so
    // every rank posts matching sends and receives.
    const bool send_rows = kind != 0;
    const bool send_scores =
        kind != 0 && (st == kLfu || st == kEpochLfu || st == kCustomized);
    // 1. merge duplicates (scores are inputs for insert-like calls only)
    const uint64_t* in_scores = kind == 0 ? nullptr : scores;
    DedupResult d;
    if (kind == 0 || unique) {
      // lookups are read-only, and a batch of distinct keys needs no merge:
      // every key travels as it is
      d.ukeys = const_cast<uint64_t*>(keys);
      d.rep_first = d.rep_last = d.uid_of = nullptr;
      d.uscores = const_cast<uint64_t*>(in_scores);
      d.dm = nullptr;
    } else if (n > 0) {
      d = dedup_batch(n, keys, in_scores, st, ws, s, sm_count_,
                      local_->error_word(), kind != 1);
    } else {
      d.ukeys = ws.get<uint64_t>(1);
      d.rep_first = d.rep_last = d.uid_of = ws.get<uint32_t>(1);
      d.uscores = nullptr;
      d.dm = ws.get<uint32_t>(1);
      CUDA_TRY(cudaMemsetAsync(d.dm, 0, sizeof(uint32_t), s));
    }
    if (send_scores && d.uscores == nullptr) {
      d.uscores = ws.get<uint64_t>(nn);
      CUDA_TRY(cudaMemsetAsync(d.uscores, 0, nn * 8, s));
    }
    // 2. route
    uint32_t* dest = ws.get<uint32_t>(nn);
    uint32_t* rid = ws.get<uint32_t>(nn);
    uint32_t* scnt = d_counts_;
    uint32_t* rcnt = d_counts_ + kMaxWorld;
    CUDA_TRY(cudaMemsetAsync(d_counts_, 0, 2 * kMaxWorld * sizeof(uint32_t), s));
    const int g = static_cast<int>(std::min<uint64_t>(ceil_div(nn, 256),
                                                      sm_count_ * 16ull));
    route_count_kernel<<<g, 256, 0, counted(s)>>>(d.ukeys, d.dm, n, world_, scnt, dest,
                                         rid);
    CUDA_TRY(cudaGetLastError());
    // 3a. exchange counts
    NCCL_TRY(ncclGroupStart());
    for (int p = 0; p < world_; p++) {
      NCCL_TRY(ncclSend(scnt + p, 1, ncclUint32, p, comm_, s));
      NCCL_TRY(ncclRecv(rcnt + p, 1, ncclUint32, p, comm_, s));
    }
    NCCL_TRY(ncclGroupEnd());
    CUDA_TRY(cudaMemcpyAsync(h_counts_, d_counts_, 2 * kMaxWorld * sizeof(uint32_t),
                             cudaMemcpyDeviceToHost, s));
    CUDA_TRY(cudaStreamSynchronize(s));
    Offsets so, ro;
    uint64_t sn = 0, rn = 0;
    for (int p = 0; p < world_; p++) {
      so.off[p] = sn;
      ro.off[p] = rn;
      sn += h_counts_[p];
      rn += h_counts_[kMaxWorld + p];
    }
    uint64_t* skeys = ws.get<uint64_t>(std::max<uint64_t>(sn, 1));
    uint64_t* sscores = send_scores ? ws.get<uint64_t>(std::max<uint64_t>(sn, 1)) : nullptr;
    uint8_t* srows = ws.get<uint8_t>(std::max<uint64_t>(sn, 1) * vb);
    uint64_t* rkeys = ws.get<uint64_t>(std::max<uint64_t>(rn, 1));
    uint64_t* rscores = ws.get<uint64_t>(std::max<uint64_t>(rn, 1));
    uint8_t* rrows = ws.get<uint8_t>(std::max<uint64_t>(rn, 1) * vb);
    uint8_t* rflag = ws.get<uint8_t>(std::max<uint64_t>(rn, 1));
    const int gt = static_cast<int>(std::min<uint64_t>(ceil_div(nn * kTile, 256),
                                                       sm_count_ * 32ull));
    const uint32_t* row_of = kind == 1 ? d.rep_first : d.rep_last;
    const int vw = local_->value_width({values, srows, rrows});
    SHARD_DISPATCH_VW(vw, route_pack_kernel<VW><<<gt, 256, 0, counted(s)>>>(
                              d.ukeys, d.uscores, send_rows ? values : nullptr,
                              row_of, d.dm, n, dest, rid, so, vb, skeys,
                              sscores, send_rows ? srows : nullptr));
    CUDA_TRY(cudaGetLastError());
    // 3b. forward exchange
    NCCL_TRY(ncclGroupStart());
    for (int p = 0; p < world_; p++) {
      const size_t c = h_counts_[p], r = h_counts_[kMaxWorld + p];
      if (c) NCCL_TRY(ncclSend(skeys + so.off[p], c, ncclUint64, p, comm_, s));
      if (r) NCCL_TRY(ncclRecv(rkeys + ro.off[p], r, ncclUint64, p, comm_, s));
      if (send_scores) {
        if (c) NCCL_TRY(ncclSend(sscores + so.off[p], c, ncclUint64, p, comm_, s));
        if (r) NCCL_TRY(ncclRecv(rscores + ro.off[p], r, ncclUint64, p, comm_, s));
      }
      if (send_rows) {
        if (c) NCCL_TRY(ncclSend(srows + so.off[p] * vb, c * vb, ncclUint8, p, comm_, s));
        if (r) NCCL_TRY(ncclRecv(rrows + ro.off[p] * vb, r * vb, ncclUint8, p, comm_, s));
      }
    }
    NCCL_TRY(ncclGroupEnd());
    // 4. local operation on the owner
    const uint64_t* rs = send_scores ? rscores : nullptr;
    if (kind == 0) {
      local_->find(rn, rkeys, rrows, reinterpret_cast<bool*>(rflag), rscores, s);
    } else if (kind == 1) {
      local_->find_or_insert(rn, rkeys, rrows, rs, s, false, false, rflag);
    } else {
      local_->insert_or_assign(rn, rkeys, rrows, rs, s, false, false);
    }
    CUDA_TRY(cudaGetLastError());
    if (kind == 2) return;  // nothing comes back
    // 5. backward exchange (rows, flags, scores for find) into send layout
    uint8_t* brows = srows;
    uint8_t* bflag = ws.get<uint8_t>(std::max<uint64_t>(sn, 1));
    uint64_t* bscores = (kind == 0 && scores) ? ws.get<uint64_t>(std::max<uint64_t>(sn, 1)) : nullptr;
    NCCL_TRY(ncclGroupStart());
    for (int p = 0; p < world_; p++) {
      const size_t c = h_counts_[p], r = h_counts_[kMaxWorld + p];
      if (r) NCCL_TRY(ncclSend(rrows + ro.off[p] * vb, r * vb, ncclUint8, p, comm_, s));
      if (c) NCCL_TRY(ncclRecv(brows + so.off[p] * vb, c * vb, ncclUint8, p, comm_, s));
      if (r) NCCL_TRY(ncclSend(rflag + ro.off[p], r, ncclUint8, p, comm_, s));
      if (c) NCCL_TRY(ncclRecv(bflag + so.off[p], c, ncclUint8, p, comm_, s));
      if (bscores) {
        if (r) NCCL_TRY(ncclSend(rscores + ro.off[p], r, ncclUint64, p, comm_, s));
        if (c) NCCL_TRY(ncclRecv(bscores + so.off[p], c, ncclUint64, p, comm_, s));
      }
    }
    NCCL_TRY(ncclGroupEnd());
    if (n == 0) return;
    SHARD_DISPATCH_VW(vw, route_unpack_kernel<VW><<<gt, 256, 0, counted(s)>>>(
                              kind == 0 ? 0 : 1, d.uid_of, n, dest, rid, so, vb,
                              brows, bflag, bscores, values,
                              kind == 0 ? founds : nullptr,
                              kind == 0 ? scores : nullptr));
    CUDA_TRY(cudaGetLastError());
  }

  // Collective: window allocation, IPC handle exchange over NCCL, peer
  // mapping. Any failure on any rank leaves every rank on the NCCL path.
  void setup_p2p(uint64_t max_batch) {
    const uint32_t vb = local_->value_bytes();
    lay_ = make_layout(world_, max_batch, vb);
    cudaStream_t s = nullptr;
    struct Rec {
      cudaIpcMemHandle_t h;
      int ok;
    };
    Rec mine{};
    mine.ok = cudaMalloc(&win_, lay_.bytes) == cudaSuccess;
    if (!mine.ok) {
      cudaGetLastError();
      win_ = nullptr;
    }
    if (mine.ok)
      mine.ok = cudaMemset(win_, 0, lay_.snd_keys) == cudaSuccess &&
                cudaIpcGetMemHandle(&mine.h, win_) == cudaSuccess;
    cudaGetLastError();
    std::vector<Rec> all(world_);
    exchange_bytes(&mine, all.data(), sizeof(Rec), s);
    int ok = 1;
    for (const Rec& r : all) ok &= r.ok;
    std::memset(&peers_, 0, sizeof peers_);
    if (ok) {
      for (int p = 0; p < world_; p++) {
        if (p == rank_) {
          peers_.base[p] = win_;
          continue;
        }
        void* ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, all[p].h, cudaIpcMemLazyEnablePeerAccess) !=
            cudaSuccess) {
          cudaGetLastError();
          ok = 0;
          break;
        }
        peers_.base[p] = static_cast<uint8_t*>(ptr);
      }
    }
    Rec again{};
    again.ok = ok;
    exchange_bytes(&again, all.data(), sizeof(Rec), s);
    for (const Rec& r : all) ok &= r.ok;
    if (ok) {
      ok = cudaMalloc(&d_route_counters_, (kMaxWorld + 1) * sizeof(uint32_t)) ==
               cudaSuccess &&
           cudaMemset(d_route_counters_, 0, (kMaxWorld + 1) * sizeof(uint32_t)) ==
               cudaSuccess &&
           cudaMalloc(&d_inv_, world_ * max_batch * sizeof(uint32_t)) == cudaSuccess &&
           cudaMalloc(&d_sent_, kMaxWorld * sizeof(uint32_t)) == cudaSuccess;
      cudaGetLastError();
      again.ok = ok;
      exchange_bytes(&again, all.data(), sizeof(Rec), s);
      for (const Rec& r : all) ok &= r.ok;
    }
    if (!ok) {
      for (int p = 0; p < world_; p++)
        if (p != rank_ && peers_.base[p]) cudaIpcCloseMemHandle(peers_.base[p]);
      std::memset(&peers_, 0, sizeof peers_);
      cudaFree(win_);
      cudaFree(d_route_counters_);
      cudaFree(d_inv_);
      cudaFree(d_sent_);
      win_ = nullptr;
      d_route_counters_ = nullptr;
      d_inv_ = nullptr;
      d_sent_ = nullptr;
      return;
    }
    max_batch_ = max_batch;
    p2p_ = true;
  }

  // all-gather of `bytes` host bytes per rank over NCCL (setup only)
  void exchange_bytes(const void* mine, void* all, size_t bytes, cudaStream_t s) {
    uint8_t* d = nullptr;
    CUDA_TRY(cudaMalloc(&d, bytes * (world_ + 1)));
    CUDA_TRY(cudaMemcpy(d, mine, bytes, cudaMemcpyHostToDevice));
    NCCL_TRY(ncclAllGather(d, d + bytes, bytes, ncclUint8, comm_, s));
    CUDA_TRY(cudaStreamSynchronize(s));
    CUDA_TRY(cudaMemcpy(all, d + bytes, bytes * world_, cudaMemcpyDeviceToHost));
    CUDA_TRY(cudaFree(d));
  }

  // kind: 0 find, 1 find_or_insert, 2 insert_or_assign (peer transport)
  void run_p2p(int kind, size_t n, const uint64_t* keys, uint8_t* values,
               bool* founds, uint64_t* scores, cudaStream_t s, bool unique) {
    HKV_REQUIRE(n <= max_batch_, HKV_ERR_INVALID,
                "sharded batch larger than the table's max_batch");
    const int st = local_->strategy();
    if (kind != 0) local_->check_strategy(scores, false);
    const bool send_scores =
        kind != 0 && (st == kLfu || st == kEpochLfu || st == kCustomized);
    const uint64_t M = max_batch_;
    const uint32_t vb = lay_.vb;
    const uint32_t me = static_cast<uint32_t>(rank_);
    int* err = local_->error_word();
    epoch_++;
    Workspace ws(s, local_->pool());
    // 1. route (insert-like calls merge duplicates first)
    const uint64_t* rkeys = keys;
    const uint64_t* rscores = nullptr;
    const uint32_t* row_of = nullptr;
    const uint32_t* dm = nullptr;
    const uint32_t* uid_of = nullptr;
    if (kind != 0 && unique) {
      rscores = send_scores ? scores : nullptr;
    } else if (kind != 0 && n > 0) {
      const DedupResult d = dedup_batch(n, keys, send_scores ? scores : nullptr,
                                        st, ws, s, sm_count_, err, kind != 1);
      rkeys = d.ukeys;
      rscores = d.uscores;
      row_of = kind == 1 ? d.rep_first : d.rep_last;
      dm = d.dm;
      uid_of = d.uid_of;
    }
    const int vw = kind == 0 ? 16
                             : local_->value_width({values, win_ + lay_.snd_rows});
    // a full wave (8 blocks of 256 per SM): the row copies are latency-bound
    const int gr = static_cast<int>(std::max<uint64_t>(
        1, std::min<uint64_t>(ceil_div(std::max<uint64_t>(n, 1), 256),
                              sm_count_ * 8ull)));
    SHARD_DISPATCH_VW(vw, p2p_route_kernel<VW><<<gr, 256, 0, counted(s)>>>(
                              rkeys, rscores, kind == 0 ? nullptr : values, row_of,
                              dm, n, world_, me, peers_, lay_, d_route_counters_,
                              d_inv_, d_sent_, epoch_, err));
    CUDA_TRY(cudaGetLastError());
    // 2. serve what the requesters sorted for this rank
    uint32_t* counts = d_counts_;  // kMaxWorld entries, device
    p2p_wait_arrive_kernel<<<1, kMaxWorld, 0, counted(s)>>>(win_, lay_, world_,
                                                             epoch_, counts, err);
    CUDA_TRY(cudaGetLastError());
    const uint64_t mine = uint64_t{me} * M;  // this owner's region in a send area
    if (kind == 0) {
      FindSegments seg;
      seg.row_stride = vb;
      seg.flag_stride = seg.score_stride = 16;
      for (int src = 0; src < world_; src++) {
        const uint64_t o = uint64_t{static_cast<uint32_t>(src)} * M;
        uint8_t* tail0 = win_ + lay_.res_tail + o * 16;
        seg.keys[src] = reinterpret_cast<const uint64_t*>(peers_.base[src] + lay_.snd_keys) + mine;
        seg.values[src] = win_ + lay_.res_rows + o * vb;
        seg.scores[src] = tail0;
        seg.founds[src] = tail0 + 8;
      }
      local_->find_segments(seg, static_cast<uint32_t>(world_), counts, M, s);
    } else {
      // one launch per requester, in rank order: a key sent by several
      // requesters is applied once per requester, in rank order (concurrent
      // inserts of one new key could both claim an empty slot)
      for (int src = 0; src < world_; src++) {
        const uint64_t o = uint64_t{static_cast<uint32_t>(src)} * M;
        uint8_t* pb = peers_.base[src];
        const uint64_t* k = reinterpret_cast<const uint64_t*>(pb + lay_.snd_keys) + mine;
        const uint64_t* sc =
            send_scores ? reinterpret_cast<const uint64_t*>(pb + lay_.snd_scores) + mine
                        : nullptr;
        // find_or_insert reads a requester's input row only for a key it
        // inserts, and leaves only found rows in the result area
        if (kind == 1)
          local_->upsert_counted(kModeFindOrInsert, M, counts + src, k,
                                 pb + lay_.snd_rows + mine * vb,
                                 win_ + lay_.res_rows + o * vb, sc,
                                 win_ + lay_.res_tail + o * 16 + 8, 16, s);
        else
          local_->upsert_counted(kModeInsertOrAssign, M, counts + src, k,
                                 pb + lay_.snd_rows + mine * vb, nullptr, sc, nullptr,
                                 1, s);
      }
    }
    p2p_signal_done_kernel<<<1, kMaxWorld, 0, counted(s)>>>(peers_, lay_, world_,
                                                             me, epoch_);
    CUDA_TRY(cudaGetLastError());
    // 3. finish: wait for every owner, then read the results
    const int vwf = (kind == 2 || values == nullptr)
                        ? 16
                        : local_->value_width({values, win_ + lay_.res_rows});
    if (kind == 0 || kind == 1) {
      // a multiple of world blocks: block b reads owner b % world's results
      const uint64_t per_owner = std::max<uint64_t>(
          1, std::min<uint64_t>(ceil_div(std::max<uint64_t>(n, 1) * 4, 256),
                                sm_count_ * 16ull / world_));
      const int gf = static_cast<int>(per_owner * world_);
      // a merged find_or_insert batch: representatives first, then their
      // later occurrences from the local copies (kIllegal until an owner's
      // status arrives: an overflowed representative is skipped)
      uint8_t* ustatus = nullptr;
      if (uid_of != nullptr) {
        ustatus = ws.get<uint8_t>(std::max<size_t>(n, 1));
        CUDA_TRY(cudaMemsetAsync(ustatus, kIllegal, n, s));
      }
      SHARD_DISPATCH_VW(vwf, p2p_finish_ordered_kernel<VW><<<gf, 256, 0, counted(s)>>>(
                                 kind, peers_, lay_, world_, me, epoch_, err, d_sent_,
                                 d_inv_, values, kind == 0 ? founds : nullptr,
                                 kind == 0 ? scores : nullptr, row_of, ustatus));
      if (uid_of != nullptr) {
        CUDA_TRY(cudaGetLastError());
        local_->scatter_found_rows(values, uid_of, row_of, ustatus, n, s);
      }
    } else {
      p2p_wait_done_kernel<<<1, kMaxWorld, 0, counted(s)>>>(win_, lay_, world_, epoch_, err);
    }
    CUDA_TRY(cudaGetLastError());
  }

  size_t size(cudaStream_t s) {
    const size_t local = local_->size(s);
    unsigned long long* d = nullptr;
    CUDA_TRY(cudaMallocFromPoolAsync(reinterpret_cast<void**>(&d), 8, local_->pool(), s));
    CUDA_TRY(cudaMemcpyAsync(d, &local, 8, cudaMemcpyHostToDevice, s));
    NCCL_TRY(ncclAllReduce(d, d, 1, ncclUint64, ncclSum, comm_, s));
    unsigned long long h = 0;
    CUDA_TRY(cudaMemcpyAsync(&h, d, 8, cudaMemcpyDeviceToHost, s));
    CUDA_TRY(cudaFreeAsync(d, s));
    CUDA_TRY(cudaStreamSynchronize(s));
    return h;
  }

 private:
  int rank_, world_;
  int sm_count_ = 148;
  TableImpl* local_ = nullptr;
  ncclComm_t comm_ = nullptr;
  uint32_t* d_counts_ = nullptr;
  uint32_t* h_counts_ = nullptr;
  // peer-memory transport
  bool p2p_ = false;
  uint64_t max_batch_ = 0;
  uint64_t epoch_ = 0;
  WinLayout lay_{};
  uint8_t* win_ = nullptr;
  PeerBases peers_{};
  uint32_t* d_route_counters_ = nullptr;
  uint32_t* d_inv_ = nullptr;    // [world][max_batch] input of each routed position
  uint32_t* d_sent_ = nullptr;   // [kMaxWorld] keys routed to each owner
};

void set_last_error(const std::string& m);

}  // namespace hkvb

struct hkv_sharded {
  hkvb::ShardedImpl* impl;
  hkv_table local;
};

using hkvb::HkvError;

#define HKV_API_BEGIN try {
#define HKV_API_END                     \
  return HKV_OK;                        \
  }                                     \
  catch (const HkvError& e) {           \
    hkvb::set_last_error(e.msg);        \
    return e.code;                      \
  }                                     \
  catch (const std::exception& e) {     \
    hkvb::set_last_error(e.what());     \
    return HKV_ERR_RUNTIME;             \
  }

#define HKV_SHARDED(x)                                                   \
  HKV_REQUIRE((x) != nullptr && (x)->impl != nullptr, HKV_ERR_INVALID,   \
              "null sharded table");                                     \
  hkvb::ShardedImpl* S = (x)->impl

extern "C" {

int hkv_nccl_unique_id(uint8_t out[128]) {
  HKV_API_BEGIN
  ncclUniqueId id;
  NCCL_TRY(ncclGetUniqueId(&id));
  std::memcpy(out, id.internal, 128);
  HKV_API_END
}

int hkv_sharded_create(const hkv_options* local_options, int key_type,
                       int value_type, int evict_strategy,
                       const uint8_t nccl_id[128], int rank, int world_size,
                       size_t max_batch, hkv_sharded** out) {
  HKV_API_BEGIN
  HKV_REQUIRE(local_options && nccl_id && out, HKV_ERR_INVALID, "null argument");
  *out = nullptr;
  auto* s = new hkv_sharded;
  try {
    s->impl = new hkvb::ShardedImpl(*local_options, key_type, value_type,
                                    evict_strategy, nccl_id, rank, world_size,
                                    max_batch);
  } catch (...) {
    delete s;
    throw;
  }
  s->local.impl = s->impl->local();
  *out = s;
  HKV_API_END
}

int hkv_sharded_destroy(hkv_sharded* s) {
  HKV_API_BEGIN
  if (s) {
    delete s->impl;
    delete s;
  }
  HKV_API_END
}

hkv_table* hkv_sharded_local(hkv_sharded* s) { return s ? &s->local : nullptr; }

int hkv_sharded_transport(hkv_sharded* s, int* out) {
  HKV_API_BEGIN
  HKV_SHARDED(s);
  HKV_REQUIRE(out != nullptr, HKV_ERR_INVALID, "null argument");
  *out = S->peer_transport() ? HKV_TRANSPORT_PEER : HKV_TRANSPORT_NCCL;
  HKV_API_END
}

int hkv_sharded_find_or_insert(hkv_sharded* s, size_t n, const void* keys,
                               void* values, const uint64_t* scores,
                               void* stream, bool unique_key) {
  HKV_API_BEGIN
  HKV_SHARDED(s);
  S->run(1, n, static_cast<const uint64_t*>(keys), static_cast<uint8_t*>(values),
         nullptr, const_cast<uint64_t*>(scores), static_cast<cudaStream_t>(stream),
         unique_key);
  HKV_API_END
}

int hkv_sharded_find(hkv_sharded* s, size_t n, const void* keys, void* values,
                     bool* founds, uint64_t* scores, void* stream) {
  HKV_API_BEGIN
  HKV_SHARDED(s);
  S->run(0, n, static_cast<const uint64_t*>(keys), static_cast<uint8_t*>(values),
         founds, scores, static_cast<cudaStream_t>(stream), false);
  HKV_API_END
}

int hkv_sharded_insert_or_assign(hkv_sharded* s, size_t n, const void* keys,
                                 const void* values, const uint64_t* scores,
                                 void* stream, bool unique_key) {
  HKV_API_BEGIN
  HKV_SHARDED(s);
  S->run(2, n, static_cast<const uint64_t*>(keys),
         const_cast<uint8_t*>(static_cast<const uint8_t*>(values)), nullptr,
         const_cast<uint64_t*>(scores), static_cast<cudaStream_t>(stream),
         unique_key);
  HKV_API_END
}

int hkv_sharded_size(hkv_sharded* s, void* stream, size_t* out) {
  HKV_API_BEGIN
  HKV_SHARDED(s);
  *out = S->size(static_cast<cudaStream_t>(stream));
  HKV_API_END
}

}  // extern "C"
