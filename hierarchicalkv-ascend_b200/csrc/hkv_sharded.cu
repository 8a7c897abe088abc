// hkv_sharded.cu -- table sharded over the GPUs of one node (no reference
// counterpart: the reference drives a single device).
//
// Each rank owns one TableImpl. A collective call takes every rank's batch:
//   1. merge duplicate keys of the local batch (hkv_dedup.cuh),
//   2. route each distinct key to owner = (Murmur3(key) >> 40) % world,
//   3. exchange per-peer counts, then keys / scores / value rows with NCCL
//      grouped send/recv (an all-to-all over NVLink/NVSwitch),
//   4. run the local operation on the owner (duplicates across sources are
//      merged again there),
//   5. return value rows (and found flags / scores) the same way and scatter
//      them to every occurrence in the caller's batch.
// The owner uses hash bits 40.. so that a shard's keys do not share the low
// hash bits that choose their bucket and start slot.
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

}  // namespace

class ShardedImpl {
 public:
  ShardedImpl(const hkv_options& o, int key_type, int value_type, int strategy,
              const uint8_t id[128], int rank, int world)
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
  }
  ~ShardedImpl() {
    if (comm_) ncclCommDestroy(comm_);
    delete local_;
    cudaFree(d_counts_);
    cudaFreeHost(h_counts_);
  }
  TableImpl* local() { return local_; }

  // kind: 0 find, 1 find_or_insert, 2 insert_or_assign
  void run(int kind, size_t n, const uint64_t* keys, uint8_t* values,
           bool* founds, uint64_t* scores, cudaStream_t s) {
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
    if (kind == 0) {
      // lookups are read-only: every occurrence travels as it is
      d.ukeys = const_cast<uint64_t*>(keys);
      d.rep_first = d.rep_last = d.uid_of = nullptr;
      d.uscores = nullptr;
      d.dm = nullptr;
    } else if (n > 0) {
      d = dedup_batch(n, keys, in_scores, st, ws, s, sm_count_,
                      local_->error_word());
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
                       hkv_sharded** out) {
  HKV_API_BEGIN
  HKV_REQUIRE(local_options && nccl_id && out, HKV_ERR_INVALID, "null argument");
  *out = nullptr;
  auto* s = new hkv_sharded;
  try {
    s->impl = new hkvb::ShardedImpl(*local_options, key_type, value_type,
                                    evict_strategy, nccl_id, rank, world_size);
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

int hkv_sharded_find_or_insert(hkv_sharded* s, size_t n, const void* keys,
                               void* values, const uint64_t* scores,
                               void* stream) {
  HKV_API_BEGIN
  HKV_SHARDED(s);
  S->run(1, n, static_cast<const uint64_t*>(keys), static_cast<uint8_t*>(values),
         nullptr, const_cast<uint64_t*>(scores), static_cast<cudaStream_t>(stream));
  HKV_API_END
}

int hkv_sharded_find(hkv_sharded* s, size_t n, const void* keys, void* values,
                     bool* founds, uint64_t* scores, void* stream) {
  HKV_API_BEGIN
  HKV_SHARDED(s);
  S->run(0, n, static_cast<const uint64_t*>(keys), static_cast<uint8_t*>(values),
         founds, scores, static_cast<cudaStream_t>(stream));
  HKV_API_END
}

int hkv_sharded_insert_or_assign(hkv_sharded* s, size_t n, const void* keys,
                                 const void* values, const uint64_t* scores,
                                 void* stream) {
  HKV_API_BEGIN
  HKV_SHARDED(s);
  S->run(2, n, static_cast<const uint64_t*>(keys),
         const_cast<uint8_t*>(static_cast<const uint8_t*>(values)), nullptr,
         const_cast<uint64_t*>(scores), static_cast<cudaStream_t>(stream));
  HKV_API_END
}

int hkv_sharded_size(hkv_sharded* s, void* stream, size_t* out) {
  HKV_API_BEGIN
  HKV_SHARDED(s);
  *out = S->size(static_cast<cudaStream_t>(stream));
  HKV_API_END
}

}  // extern "C"
