// Peer-memory exchange of the key-sharded store (one process per GPU).
//
// Rank r owns the keys the partitioner maps to r. Every rank keeps one
// exchange arena in its HBM with the same layout; all ranks map all arenas
// through CUDA IPC (plain peer mappings over NVLink, no multicast), so a
// kernel on rank s stores directly into rank d's arena. Per call:
//
//   forward : route the batch's keys by owner (stable histogram + scan, local);
//             publish the per-owner counts into every owner's count matrix;
//             scatter (key, batch position) straight into each owner's key
//             inbox, at the owner-side offset sum_{s' < s} count[s'][d];
//             the owner runs insert-on-miss / gather over its inbox (senders
//             in rank order) and stores every row straight into the
//             requester's row buffer at the requester's batch position;
//   backward: the same route for the gradient keys; (key, gradient row) are
//             scattered into each owner's gradient inbox; the owner appends
//             its inbox to its pending gradients (senders in rank order, so a
//             key's rows arrive in the order of the concatenated batch).
//
// Each phase ends with a flag per (kind, sender) in the receiver's arena,
// written with the sender's epoch for that kind by a one-block sync kernel
// that runs after the phase's data kernel completed; the same kernel then
// waits until every sender's flag reaches its own epoch. Waits are bounded in
// time: past the exchange's timeout the kernel records it and returns.
//
// One buffer per kind suffices when every rank makes the same sequence of
// calls:
//  - forward inbox / count matrix of owner p are last read by p's owner
//    kernels of call k, which precede p's ROWS flag of call k; a sender only
//    writes them for call k+1 after it saw every owner's ROWS flag of call k;
//  - a requester's row buffer is read before its KEYS flag of call k+1, which
//    every owner waits for before writing rows of call k+1;
//  - gradient inbox of owner p is read by p's accumulate of call k, which
//    precedes p's GCOUNTS flag of call k+1; senders wait for it before
//    scattering call k+1. The gradient count matrix is read only inside the
//    scatter kernel (the received total is staged there), which precedes p's
//    GRADS flag of call k, which senders wait for before publishing call k+1;
//  - a gradient batch routed like the last forward (no keys sent) lands in
//    the gradient inbox at the forward's slots and is accumulated with the
//    forward's key inbox: a sender scatters it only after its forward saw
//    owner p's ROWS flag, which p raises after its previous accumulate, and
//    p's key inbox is rewritten only after p's next COUNTS flag, which p
//    raises after this accumulate. The forward's total is staged by the
//    owner kernel.
#pragma once

#include "se_partition.cuh"

namespace se_gpu {

constexpr uint32_t kExMaxRanks = 64;

enum ExKind : int { kExCounts = 0, kExKeys = 1, kExRows = 2, kExGCounts = 3, kExGrads = 4, kExKinds = 5 };
constexpr uint64_t kSpinLimit = 1ull << 28;  // hard cap on polls (>= 128 ns each) behind the timeout

struct ExView {
  uint8_t *const *peer;  // [W] arena base of every rank (own included), device array
  uint32_t W, me;
  uint32_t M;            // keys per rank per call: rows of a row buffer; an inbox holds W * M
  uint32_t row_bytes, grad_bytes;
  uint64_t timeout_ns;
  // byte offsets inside every arena
  uint64_t o_flags, o_epochs, o_counts, o_gcounts, o_inkeys, o_inpos, o_inrow, o_gkeys, o_ingrads, o_rows, o_words,
      o_prefix;

  __device__ __forceinline__ uint32_t *flags(uint32_t r) const { return reinterpret_cast<uint32_t *>(peer[r] + o_flags); }
  __device__ __forceinline__ uint32_t *epochs() const { return reinterpret_cast<uint32_t *>(peer[me] + o_epochs); }
  __device__ __forceinline__ uint32_t *counts(uint32_t r, int kind) const {
    return reinterpret_cast<uint32_t *>(peer[r] + (kind == kExGCounts ? o_gcounts : o_counts));
  }
  __device__ __forceinline__ unsigned long long *inkeys(uint32_t r) const {
    return reinterpret_cast<unsigned long long *>(peer[r] + o_inkeys);
  }
  __device__ __forceinline__ uint32_t *inpos(uint32_t r) const { return reinterpret_cast<uint32_t *>(peer[r] + o_inpos); }
  // own [W * M]: row of each key inbox entry after the forward (kNoRow: none)
  __device__ __forceinline__ uint32_t *inrow() const { return reinterpret_cast<uint32_t *>(peer[me] + o_inrow); }
  __device__ __forceinline__ unsigned long long *gkeys(uint32_t r) const {
    return reinterpret_cast<unsigned long long *>(peer[r] + o_gkeys);
  }
  __device__ __forceinline__ uint8_t *ingrads(uint32_t r) const { return peer[r] + o_ingrads; }
  __device__ __forceinline__ uint8_t *rows(uint32_t r) const { return peer[r] + o_rows; }
  // own words: [kExTotal] received gradient rows (accumulate count),
  // [kExTotalStaged] its value before the GRADS wait, [kExStatus] timeout bits
  __device__ __forceinline__ uint32_t *words() const { return reinterpret_cast<uint32_t *>(peer[me] + o_words); }
  // own [W + 1]: first key inbox slot of every sender of the last forward, then the total
  __device__ __forceinline__ uint32_t *prefix() const { return reinterpret_cast<uint32_t *>(peer[me] + o_prefix); }
};

// kExFwdTotal: keys received by the last forward (the row count of a
// gradient batch routed like that forward's keys).
enum ExWord : int { kExTotal = 0, kExTotalStaged = 1, kExStatus = 2, kExFwdTotal = 3, kExWords = 4 };
// Status bit (above the per-kind timeout bits) for a slot or position outside
// the buffers, i.e. ranks created with different sizes; the access is skipped.
constexpr uint32_t kExBadIndex = 1u << 8;

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Thread 0 of a block: waits until every sender's flag of `kind` reached this
// rank's epoch of that kind. Gives up after x.timeout_ns (or kSpinLimit polls)
// and records bit 1 << kind in the status word; returns early when a wait of
// this rank already gave up (any bit set), so a failed exchange drains fast.
__device__ __forceinline__ bool ex_wait(const ExView &x, int kind) {
  const uint32_t e = x.epochs()[kind];
  const uint32_t *f = x.flags(x.me) + size_t(kind) * x.W;
  volatile uint32_t *status = x.words() + kExStatus;
  uint64_t polls = 0, start = 0;
  for (uint32_t s = 0; s < x.W; ++s) {
    while (ld_acquire_sys(f + s) < e) {
      ++polls;
      if ((polls & 63u) == 0) {
        if (*status) return false;
        const uint64_t now = globaltimer_ns();
        if (start == 0) start = now;
        if (now - start > x.timeout_ns || polls > kSpinLimit) {
          atomicOr(x.words() + kExStatus, 1u << kind);
          return false;
        }
      }
      __nanosleep(128);
    }
  }
  return true;
}

// True once a wait of this rank gave up: the data kernels then do nothing
// (every block alike), so a failed exchange stops moving data.
__device__ __forceinline__ bool ex_failed(const ExView &x) {
  return *reinterpret_cast<volatile uint32_t *>(x.words() + kExStatus) != 0u;
}

// All threads of one block: bumps this rank's epoch of `kind`, optionally
// stores this rank's per-owner counts into row `me` of every rank's count
// matrix, then raises flag (kind, me) on every rank with a system-scope
// release store.
__device__ void ex_raise(const ExView &x, int kind, const uint32_t *counts_local) {
  __shared__ uint32_t e;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t *ep = x.epochs() + kind;
    e = *ep + 1u;
    *ep = e;
  }
  __syncthreads();
  for (uint32_t p = threadIdx.x; p < x.W; p += blockDim.x) {
    if (counts_local) {
      uint32_t *cm = x.counts(p, kind) + size_t(x.me) * x.W;
      for (uint32_t d = 0; d < x.W; ++d) cm[d] = counts_local[d];
    }
    st_release_sys(x.flags(p) + size_t(kind) * x.W + x.me, e);
  }
  __syncthreads();
}

// One small block between a phase's data kernel and the kernels that read
// what the peers stored: raises this rank's flags of `kind` (the data kernel
// before it on the stream has completed, with all its stores, peer stores
// included, when pdl_wait returns), then waits until every sender's flag of
// `kind` reached this rank's epoch. A separate kernel per phase instead of a
// last-block tail in the data kernel (a GPU-scope fence and a counter atomic
// in every block, then the system-scope release: ~3 us per phase) and
// instead of a wait in every block of the next kernel.
// After KEYS it also lays out the key inbox once for the owner kernels (each
// sender's first slot and the total, bounded by the inbox); after GRADS it
// sets the row count of the accumulate that follows from `total_word` (0
// when the wait gave up).
__global__ void k_ex_sync(ExView x, int kind, int total_word) {
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  if (ex_failed(x)) {  // a failed exchange raises nothing more
    if (threadIdx.x == 0 && kind == kExGrads) x.words()[kExTotal] = 0u;
    return;
  }
  ex_raise(x, kind, nullptr);
  if (threadIdx.x != 0) return;
  const bool ok = ex_wait(x, kind);
  if (kind == kExGrads) {
    uint32_t *w = x.words();
    w[kExTotal] = ok ? w[total_word] : 0u;
    return;
  }
  if (!ok || kind != kExKeys) return;
  uint32_t *prefix = x.prefix();
  uint32_t run = 0;
  for (uint32_t s = 0; s < x.W; ++s) {
    prefix[s] = run;
    run += __ldcg(x.counts(x.me, kExCounts) + size_t(s) * x.W + x.me);
  }
  if (run > x.W * x.M) {
    atomicOr(x.words() + kExStatus, kExBadIndex);
    run = x.W * x.M;
  }
  prefix[x.W] = run;
  x.words()[kExFwdTotal] = run;
}

// Route counts of this rank's keys: per-tile histograms by owner. Launched
// with max(tiles, 1) blocks of kExTile keys.
// count_dev: when not null, the batch holds min(*count_dev, count) keys (the
// sender's distinct keys, counted on the device).
// With a deduplicated batch (pos_slot not null) the same grid also writes
// inverse[i], the distinct-key index of each of the npos batch positions
// (set_idx of the position's set slot), which the dedupe kernel's claims
// completed before this launch.
template <class K>
__global__ void __launch_bounds__(kRouteThreads)
k_ex_count(PartSpec s, ExView x, const K *__restrict__ keys, size_t count, uint32_t *__restrict__ tile_counts,
           const uint32_t *count_dev, const uint32_t *__restrict__ pos_slot, const uint32_t *set_idx,
           uint32_t *__restrict__ inverse, size_t npos) {
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  extern __shared__ uint32_t hist[];  // [W]
  if (ex_failed(x)) return;
  if (count_dev) count = min(count, size_t(*count_dev));
  for (uint32_t p = threadIdx.x; p < s.n; p += blockDim.x) hist[p] = 0;
  __syncthreads();
  const size_t i = size_t(blockIdx.x) * kRouteThreads + threadIdx.x;
  if (i < count) atomicAdd(&hist[partition_of<K>(s, keys[i])], 1u);
  if (pos_slot)
    for (size_t j = i; j < npos; j += size_t(gridDim.x) * kRouteThreads) {
      const uint32_t slot = pos_slot[j];
      inverse[j] = slot == kNoRow ? 0u : __ldcg(set_idx + slot);
    }
  __syncthreads();
  for (uint32_t p = threadIdx.x; p < s.n; p += blockDim.x) tile_counts[size_t(blockIdx.x) * s.n + p] = hist[p];
}

// One block: the partition-major exclusive offsets of every tile and the
// per-owner counts, which it stores into every owner's count matrix and
// publishes as `kind` (COUNTS or GCOUNTS); then waits for every sender's.
__global__ void __launch_bounds__(kRouteThreads)
k_ex_sync_counts(ExView x, int kind, uint32_t tiles, const uint32_t *__restrict__ tile_counts,
                 uint32_t *__restrict__ tile_offsets, uint32_t *__restrict__ counts) {
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  using Scan = cub::BlockScan<uint32_t, kRouteThreads>;
  __shared__ typename Scan::TempStorage tmp;
  __shared__ uint32_t carry;
  const uint32_t n = x.W;
  if (ex_failed(x)) return;  // a failed exchange raises nothing more
  uint32_t running = 0;  // partition base, valid in thread 0
  for (uint32_t p = 0; p < n; ++p) {
    if (threadIdx.x == 0) carry = running;
    __syncthreads();
    for (uint32_t t0 = 0; t0 < tiles; t0 += kRouteThreads) {
      const uint32_t t = t0 + threadIdx.x;
      const uint32_t c = t < tiles ? tile_counts[size_t(t) * n + p] : 0u;
      uint32_t excl, total;
      Scan(tmp).ExclusiveSum(c, excl, total);
      const uint32_t base = carry;
      if (t < tiles) tile_offsets[size_t(t) * n + p] = base + excl;
      __syncthreads();
      if (threadIdx.x == 0) carry = base + total;
      __syncthreads();
    }
    if (threadIdx.x == 0) {
      counts[p] = carry - running;
      running = carry;
    }
    __syncthreads();
  }
  ex_raise(x, kind, counts);
  if (threadIdx.x == 0) ex_wait(x, kind);
}

// Keys per route tile of the exchange: one per thread of a 256-thread block,
// so a 65,536-key batch spreads over 256 blocks.
constexpr int kExTile = kRouteThreads;

// Route scatter into the owners' inboxes (forward: keys and batch positions;
// backward: keys and gradient rows, copied block-wide in units U after the
// slots are known). Stable: a key's slot on owner d is
// sum_{s < me} counts[s][d] + (keys of earlier tiles for d) + (keys of
// earlier warps of this tile for d) + (earlier lanes of its warp for d).
// The keys are loaded and ranked within their warp before the wait for the
// peers' counts.
// Forward also records each key's (owner, slot) in key_pid / key_slot, so a
// gradient batch for the same keys can follow the same route (k_ex_scatter_rows).
template <class K, bool kGrads, class U>
__global__ void __launch_bounds__(kRouteThreads)
k_ex_scatter(PartSpec s, ExView x, const K *__restrict__ keys, size_t count, const uint32_t *__restrict__ tile_offsets,
             const uint32_t *__restrict__ counts_local, const uint8_t *__restrict__ grads,
             uint32_t *__restrict__ key_pid, uint32_t *__restrict__ key_slot, const uint32_t *count_dev) {
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  if (count_dev) count = min(count, size_t(*count_dev));
  extern __shared__ uint32_t sm[];
  uint32_t *warp_base = sm;                   // [kRouteWarps][W]
  uint32_t *remote = sm + kRouteWarps * s.n;  // [W] slot base on each owner minus the local prefix
  __shared__ uint32_t row_pid[kExTile], row_slot[kExTile];
  const int kind = kGrads ? kExGCounts : kExCounts;
  if (ex_failed(x)) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  const size_t tile_base = size_t(blockIdx.x) * kExTile;
  const size_t i = tile_base + threadIdx.x;
  const bool valid = i < count;
  K key{};
  uint32_t pid = 0xffffffffu;
  if (valid) {
    key = keys[i];
    pid = partition_of<K>(s, key);
  }
  const unsigned peers = __match_any_sync(0xffffffffu, pid);
  for (uint32_t j = threadIdx.x; j < kRouteWarps * s.n; j += blockDim.x) warp_base[j] = 0;
  __syncthreads();
  if (valid && (peers & lt) == 0) warp_base[size_t(warp) * s.n + pid] = __popc(peers);
  const uint32_t *cm = x.counts(x.me, kind);
  if (kGrads && blockIdx.x == 0 && threadIdx.x == 0) {
    uint32_t total = 0;
    for (uint32_t q = 0; q < x.W; ++q) total += __ldcg(cm + size_t(q) * x.W + x.me);
    x.words()[kExTotalStaged] = total;
  }
  for (uint32_t d = threadIdx.x; d < s.n; d += blockDim.x) {
    uint32_t base = 0, local_prefix = 0;
    for (uint32_t q = 0; q < x.me; ++q) base += __ldcg(cm + size_t(q) * x.W + d);
    for (uint32_t q = 0; q < d; ++q) local_prefix += counts_local[q];
    remote[d] = base - local_prefix;  // modular: added to the routed offset below
  }
  __syncthreads();
  for (uint32_t p = threadIdx.x; p < s.n; p += blockDim.x) {
    uint32_t run = tile_offsets[size_t(blockIdx.x) * s.n + p];
    for (int w = 0; w < kRouteWarps; ++w) {
      const uint32_t c = warp_base[size_t(w) * s.n + p];
      warp_base[size_t(w) * s.n + p] = run;
      run += c;
    }
  }
  __syncthreads();
  const uint32_t inbox = x.W * x.M;
  if (valid) {
    uint32_t slot = warp_base[size_t(warp) * s.n + pid] + __popc(peers & lt) + remote[pid];
    if (slot >= inbox) {
      atomicOr(x.words() + kExStatus, kExBadIndex);
      slot = inbox;  // marks the row as skipped below
    }
    if (slot == inbox) {
      if constexpr (kGrads) row_slot[threadIdx.x] = inbox;
      else key_slot[i] = inbox;
    } else if constexpr (kGrads) {
      x.gkeys(pid)[slot] = key_u64(key);
      row_pid[threadIdx.x] = pid;
      row_slot[threadIdx.x] = slot;
    } else {
      x.inkeys(pid)[slot] = key_u64(key);
      x.inpos(pid)[slot] = uint32_t(i);
      key_pid[i] = pid;
      key_slot[i] = slot;
    }
  }
  if constexpr (kGrads) {
    __syncthreads();
    const uint32_t units = x.grad_bytes / uint32_t(sizeof(U));
    const uint32_t rows = uint32_t(min(size_t(kExTile), count - min(count, tile_base)));
    const U *src = reinterpret_cast<const U *>(grads + tile_base * x.grad_bytes);
#pragma unroll 4
    for (uint32_t u = threadIdx.x; u < rows * units; u += blockDim.x) {
      const uint32_t r = u / units, c = u - r * units;
      if (row_slot[r] >= inbox) continue;
      U *dst = reinterpret_cast<U *>(x.ingrads(row_pid[r]) + size_t(row_slot[r]) * x.grad_bytes);
      dst[c] = src[u];
    }
  }
}

// Owner of the keys: after the keys of every sender arrived, finds (and with
// kInsert inserts) each key and stores its row into the requester's row
// buffer at the requester's batch position. Keys claimed by another group of
// the same launch go to the deferred list. Absent keys of a plain lookup get
// a zero row.
// Insert mode: the launch's last block (a GPU-scope fence and a counter in
// every block) then serves the deferred keys, whose claimants have all
// published their rows by then, and resets the counters for the next launch.
template <int LANES, int VEC>
__device__ __forceinline__ void ex_owner_deferred(const Layout &L, const uint8_t *slabs, const ExView &x,
                                                  uint32_t *def_count, const uint32_t *def_idx,
                                                  const unsigned long long *def_word, uint32_t *status);

template <int LANES, int VEC, bool kInsert>
__global__ void __launch_bounds__(256)
k_ex_owner(Dir d, Layout L, uint8_t *__restrict__ slabs, RowAlloc ra, InitSpec init,
           ExView x, uint32_t *def_count, uint32_t *def_idx, unsigned long long *def_word, uint32_t *status,
           uint32_t *done) {
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  __shared__ bool s_failed, s_last;
  if (threadIdx.x == 0) s_failed = ex_failed(x);
  __syncthreads();
  if (s_failed) return;  // whole block (the counters stay as they are: the exchange must be recreated)
  const uint32_t *prefix = x.prefix();  // written by the KEYS wait
  const uint32_t total = __ldcg(prefix + x.W);
  const size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t groups = size_t(gridDim.x) * blockDim.x / LANES;
  const uint32_t lane = uint32_t(t % LANES);
  const unsigned mask = group_mask<LANES>();
  const unsigned long long *inkeys = x.inkeys(x.me);
  const uint32_t *inpos = x.inpos(x.me);
  for (size_t i = t / LANES; i < total; i += groups) {
    const uint64_t key = __ldcg(inkeys + i);
    uint32_t pos = __ldcg(inpos + i);
    uint32_t src = 0;
    while (src + 1 < x.W && __ldcg(prefix + src + 1) <= i) ++src;
    if (pos >= x.M) {
      atomicOr(x.words() + kExStatus, kExBadIndex);
      pos = 0;  // inside the buffer; the row there is reported invalid by the status
    }
    void *out_row = x.rows(src) + size_t(pos) * x.row_bytes;
    int kind = kFound;
    uint32_t row = kNoRow;
    uint32_t *word = nullptr;
    if constexpr (kInsert) {
      if (lane == 0) {
        const InsertResult r = dir_find_or_insert(d, key);
        kind = r.kind;
        word = r.row_word;
        // found: published, claimed and not yet published (3), or erased and revived here
        if (kind == kFound) kind = resolve_found(word, &row, r.seen);
        else if (kind == kFull) raise_status(status, kStatusTableFull);
      }
      // lanes of this warp still in the loop: keys i - t / LANES + [0, total)
      const size_t live = (size_t(total) - (i - t / LANES)) * LANES;
      const uint32_t taken = take_rows_warp(ra, live_lanes(t, live), lane == 0 && kind == kInserted);
      if (lane == 0 && kind == kInserted) {
        row = taken;
        if (row >= ra.capacity) {
          raise_status(status, kStatusTableFull);
          kind = kFull;
        }
      }
      kind = __shfl_sync(mask, kind, 0, LANES);
      row = __shfl_sync(mask, row, 0, LANES);
    } else {
      row = dir_find<false>(d, key);
      if (row == kNoRow) kind = kFull;
    }
    // the row for a gradient batch routed like this forward (deferred keys: below)
    if (lane == 0 && kind != 3) x.inrow()[i] = (kind == kFound || kind == kInserted) ? row : kNoRow;
    if (kind == kFound) {  // L1 may serve the row (see copy_units)
      const uint8_t *slab = slabs + size_t(row) * L.stride;
      copy_row<VEC, 4, true>(out_row, slab, L.pdt, L.dim, lane * VEC, LANES * VEC);
    } else if (kind == kInserted) {
      uint8_t *slab = slabs + size_t(row) * L.stride;
      init_slab<LANES, VEC>(L, slab, init, key, lane, out_row);
      __threadfence();
      __syncwarp(mask);
      if (lane == 0) atomicExch(word, row);
    } else if (kind == 3) {
      if (lane == 0) {
        const uint32_t j = atomicAdd(def_count, 1u);
        def_idx[j] = uint32_t(i);
        def_word[j] = reinterpret_cast<unsigned long long>(word);
      }
    } else {
      for (uint32_t e = lane * VEC; e < L.dim; e += LANES * VEC) zero_elems<VEC>(out_row, L.pdt, e);
    }
  }
  if constexpr (kInsert) {
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      s_last = atomicAdd(done, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      ex_owner_deferred<LANES, VEC>(L, slabs, x, def_count, def_idx, def_word, status);
      __syncthreads();
      if (threadIdx.x == 0) {
        *def_count = 0u;
        *done = 0u;
      }
    }
  }
}

// Deferred keys of k_ex_owner (one block): their claimant has published the
// row by now.
template <int LANES, int VEC>
__device__ __forceinline__ void ex_owner_deferred(const Layout &L, const uint8_t *slabs, const ExView &x,
                                                  uint32_t *def_count, const uint32_t *def_idx,
                                                  const unsigned long long *def_word, uint32_t *status) {
  const size_t t = threadIdx.x;
  const size_t groups = blockDim.x / LANES;
  const uint32_t lane = uint32_t(t % LANES);
  const uint32_t count = __ldcg(def_count);
  for (size_t j = t / LANES; j < count; j += groups) {
    const uint32_t i = __ldcg(def_idx + j);
    uint32_t src = 0;
    while (src + 1 < x.W && __ldcg(x.prefix() + src + 1) <= i) ++src;
    uint32_t pos = __ldcg(x.inpos(x.me) + i);
    if (pos >= x.M) pos = 0;  // reported by k_ex_owner
    void *out_row = x.rows(src) + size_t(pos) * x.row_bytes;
    const uint32_t row = __ldcg(reinterpret_cast<const uint32_t *>(__ldcg(def_word + j)));
    if (lane == 0) x.inrow()[i] = row;
    if (row == kNoRow) {
      if (lane == 0) raise_status(status, kStatusTableFull);
      for (uint32_t e = lane * VEC; e < L.dim; e += LANES * VEC) zero_elems<VEC>(out_row, L.pdt, e);
      continue;
    }
    const uint8_t *slab = slabs + size_t(row) * L.stride;
    copy_row<VEC>(out_row, slab, L.pdt, L.dim, lane * VEC, LANES * VEC);
  }
}

// Requester: waits for the rows of every owner, then copies this rank's row
// buffer (batch order) to `out` in units U.
template <class U>
__global__ void __launch_bounds__(256)
k_ex_rows_out(ExView x, U *__restrict__ out, size_t units) {
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  if (ex_failed(x)) return;
  const U *src = reinterpret_cast<const U *>(x.rows(x.me));
  const size_t stride = size_t(gridDim.x) * blockDim.x;
  constexpr int kIlp = 4;  // loads in flight per thread
  for (size_t u0 = size_t(blockIdx.x) * blockDim.x + threadIdx.x; u0 < units; u0 += stride * kIlp) {
    U v[kIlp];
#pragma unroll
    for (int k = 0; k < kIlp; ++k)
      if (u0 + k * stride < units) v[k] = __ldcg(src + u0 + k * stride);
#pragma unroll
    for (int k = 0; k < kIlp; ++k)
      if (u0 + k * stride < units) out[u0 + k * stride] = v[k];
  }
}

// Gradient rows for the keys of the last forward, in that forward's route:
// row i goes to slot key_slot[i] of owner key_pid[i]'s gradient inbox, so it
// lines up with the key the owner holds in its key inbox. No wait: the slots
// were fixed by the forward.
template <class U>
__global__ void __launch_bounds__(256)
k_ex_scatter_rows(ExView x, const uint32_t *__restrict__ key_pid, const uint32_t *__restrict__ key_slot, size_t n,
                  const U *__restrict__ grads, uint32_t units, uint32_t team) {
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  __shared__ uint8_t *inbox_of[kExMaxRanks];
  if (ex_failed(x)) return;
  for (uint32_t p = threadIdx.x; p < x.W; p += blockDim.x) inbox_of[p] = x.ingrads(p);
  __syncthreads();
  // A team of `team` lanes (a power of two <= 32) copies one row; a warp
  // moves 32 / team rows per step and each team keeps kIlp rows in flight.
  constexpr int kIlp = 4;
  const uint32_t lane = threadIdx.x & 31u, sub = lane & (team - 1u), per = 32u / team;
  const size_t warp = (size_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const size_t step = ((size_t(gridDim.x) * blockDim.x) >> 5) * per;
  const uint32_t inbox = x.W * x.M;
  for (size_t r0 = warp * per + lane / team; r0 < n; r0 += step * kIlp) {
    const U *src[kIlp];
    U *dst[kIlp];
#pragma unroll
    for (int k = 0; k < kIlp; ++k) {
      const size_t r = r0 + k * step;
      const uint32_t slot = r < n ? key_slot[r] : inbox;
      // slot == inbox: past the batch, or skipped (and reported) by the forward
      dst[k] = slot < inbox ? reinterpret_cast<U *>(inbox_of[key_pid[r]] + size_t(slot) * x.grad_bytes) : nullptr;
      src[k] = grads + r * units;
    }
    for (uint32_t c = sub; c < units; c += team) {
      U v[kIlp];
#pragma unroll
      for (int k = 0; k < kIlp; ++k)
        if (dst[k]) v[k] = src[k][c];
#pragma unroll
      for (int k = 0; k < kIlp; ++k)
        if (dst[k]) dst[k][c] = v[k];
    }
  }
}

// ---------------------------------------------------------------------------
// Sender-side dedupe. A Zipf batch repeats its hot keys thousands of times;
// routing each distinct key once per sender keeps the owners' work and the
// NVLink traffic at the distinct keys, and the forward expands the rows
// locally. The gradient batch routed like such a forward is summed per
// distinct key on the sender first (pre-reduction: the order of the adds
// changes, so results match the plain route within fp32 reassociation).
// ---------------------------------------------------------------------------

// The counters of a deduplicated forward alternate between two sets by the
// forward's parity: forward c counts its distinct keys in count[c % 2],
// which the gradient batch routed like it still reads, and forward c's last
// kernel resets the other set (forward c - 1's, dead by then) for c + 1.
struct DedupeWs {
  unsigned long long *set_keys;  // [D] hash set of the batch's keys, kEmptyKey when free
  uint32_t *set_idx;             // [D + 1] distinct-key index of each set slot; [D]: the all-ones key
  uint32_t *pos_slot;            // [M] set slot of each batch position
  uint32_t *uslot;               // [M] set slot of each distinct key
  uint32_t *inverse;             // [M] distinct-key index of each batch position
  uint32_t *count;               // this forward's distinct keys
  uint32_t *spec;                // this forward's claim flag of the all-ones key
  uint32_t *other_count, *other_spec;  // the previous forward's, reset by this one
  uint32_t *done;                // blocks of k_ex_rows_out_dedupe that finished
  uint32_t mask;                 // D - 1
};

// Distinct keys of the batch, claim order: ukeys[idx] is the idx-th claimed
// key (same dtype as the batch), pos_slot[i] the set slot of position i.
// Each block first folds its 256 positions' keys in a shared-memory set, so
// only one thread per (block, distinct key) goes to the global set: a Zipf
// batch's hottest key costs one global CAS per block instead of one per
// position. Bounded probing; the global set holds at least twice the batch.
constexpr uint32_t kDedupeBlock = 256;
template <class K>
__global__ void __launch_bounds__(kDedupeBlock)
k_ex_dedupe(ExView x, const K *__restrict__ keys, size_t n, DedupeWs w, K *__restrict__ ukeys) {
  constexpr uint32_t H = 2 * kDedupeBlock;         // block set slots; H itself: the all-ones key
  __shared__ unsigned long long s_key[H];
  __shared__ uint32_t s_gslot[H + 1];              // global set slot of each block slot
  __shared__ bool s_failed;
  pdl_wait();
  pdl_trigger();
  const uint32_t tid = threadIdx.x;
  for (uint32_t h = tid; h < H; h += blockDim.x) s_key[h] = kEmptyKey;
  if (tid == 0) s_failed = ex_failed(x);
  __syncthreads();
  if (s_failed) return;  // whole block
  const size_t i = size_t(blockIdx.x) * blockDim.x + tid;
  const uint32_t D = w.mask + 1u;
  K k{};
  uint64_t key = kEmptyKey;
  uint32_t hl = kNoRow;  // block slot of this position's key
  bool leader = false;   // first position of the key in this block
  if (i < n) {
    k = keys[i];
    key = key_u64(k);
    if (key == kEmptyKey) {
      hl = H;
    } else {
      uint32_t h = uint32_t(splitmix64(key) >> 32) & (H - 1u);
      for (uint32_t probe = 0; probe < H; ++probe) {  // at most half full: ends at the key or a free slot
        const unsigned long long old = atomicCAS(&s_key[h], kEmptyKey, key);
        if (old == kEmptyKey || old == key) {
          leader = old == kEmptyKey;
          hl = h;
          break;
        }
        h = (h + 1u) & (H - 1u);
      }
    }
  }
  // the all-ones key's block leader: its first position in the block
  const unsigned spec_mask = __ballot_sync(0xffffffffu, hl == H);
  __shared__ uint32_t s_spec_first;
  if (tid == 0) s_spec_first = kNoRow;
  __syncthreads();
  if (spec_mask && (tid & 31u) == uint32_t(__ffs(spec_mask) - 1)) atomicMin(&s_spec_first, tid);
  __syncthreads();
  if (hl == H) leader = tid == s_spec_first;
  // leaders find or claim the key's global slot
  bool claimed = false;
  if (leader) {
    uint32_t slot = kNoRow;
    if (hl == H) {
      slot = D;
      claimed = atomicCAS(w.spec, 0u, 1u) == 0u;
    } else {
      uint32_t h = uint32_t(__umul64hi(splitmix64(key), uint64_t(D)));
      for (uint32_t probe = 0; probe < D; ++probe) {
        const unsigned long long old = atomicCAS(w.set_keys + h, kEmptyKey, key);
        if (old == kEmptyKey || old == key) {
          claimed = old == kEmptyKey;
          slot = h;
          break;
        }
        h = (h + 1u) & w.mask;
      }
    }
    s_gslot[hl] = slot;
  }
  // one counter atomic per warp for its claims
  const uint32_t lane = tid & 31u;
  const unsigned claims = __ballot_sync(0xffffffffu, claimed);
  if (claims) {
    uint32_t base = 0;
    if (lane == uint32_t(__ffs(claims) - 1)) base = atomicAdd(w.count, uint32_t(__popc(claims)));
    base = __shfl_sync(0xffffffffu, base, __ffs(claims) - 1);
    if (claimed) {
      const uint32_t idx = base + __popc(claims & ((1u << lane) - 1u));
      const uint32_t slot = s_gslot[hl];
      w.set_idx[slot] = idx;
      w.uslot[idx] = slot;
      ukeys[idx] = k;
    }
  }
  __syncthreads();
  if (i < n) w.pos_slot[i] = hl == kNoRow ? kNoRow : s_gslot[hl];
}

// Requester of a deduplicated forward: waits for the rows of every owner
// (stream order), then out[i] = row buffer[inverse[i]] in units U (a team of
// `team` lanes per position, kIlp positions in flight); also empties the
// dedupe set for the next forward, and its last block resets the previous
// forward's counters.
template <class U>
__global__ void __launch_bounds__(256)
k_ex_rows_out_dedupe(ExView x, U *__restrict__ out, size_t n, uint32_t units, DedupeWs w, uint32_t team) {
  pdl_wait();
  pdl_trigger();
  __shared__ bool s_failed;
  if (threadIdx.x == 0) s_failed = ex_failed(x);
  __syncthreads();
  const U *src = reinterpret_cast<const U *>(x.rows(x.me));
  const size_t tid = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t stride = size_t(gridDim.x) * blockDim.x;
  if (!s_failed) {
    constexpr int kIlp = 4;
    const uint32_t lane = threadIdx.x & 31u, sub = lane & (team - 1u), per = 32u / team;
    const size_t step = (stride >> 5) * per;
    for (size_t i0 = (tid >> 5) * per + lane / team; i0 < n; i0 += step * kIlp) {
      const U *s[kIlp];
      U *d[kIlp];
#pragma unroll
      for (int k = 0; k < kIlp; ++k) {
        const size_t i = i0 + k * step;
        const uint32_t idx = i < n ? __ldcg(w.inverse + i) : 0u;
        s[k] = i < n ? src + size_t(min(idx, x.M - 1u)) * units : nullptr;
        d[k] = i < n ? out + i * units : nullptr;
      }
      for (uint32_t c = sub; c < units; c += team) {
        U v[kIlp];
#pragma unroll
        for (int k = 0; k < kIlp; ++k)
          if (s[k]) v[k] = __ldcg(s[k] + c);
#pragma unroll
        for (int k = 0; k < kIlp; ++k)
          if (d[k]) d[k][c] = v[k];
      }
    }
  }
  const uint32_t nd = min(__ldcg(w.count), x.M);
  for (size_t j = tid; j < nd; j += stride) {
    const uint32_t slot = __ldcg(w.uslot + j);
    if (slot <= w.mask) w.set_keys[slot] = kEmptyKey;
  }
  __shared__ bool s_last;
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(w.done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    *w.other_count = 0u;
    *w.other_spec = 0u;
    *w.done = 0u;
  }
}

// Pre-reduced gradient rows of a deduplicated forward's keys: distinct key
// u's fp32 sum (pre[u], `dim` floats) goes to slot key_slot[u] of owner
// key_pid[u]'s gradient inbox, in the gradient dtype; the sum is zeroed for
// the next call. kVec (fp32 gradients, dim % 4 == 0): a team of `team`
// lanes moves one row in 16-byte units and keeps kIlp rows in flight;
// otherwise one warp per row, one value per lane.
template <bool kVec>
__global__ void __launch_bounds__(256)
k_ex_scatter_prerows(ExView x, const uint32_t *__restrict__ key_pid, const uint32_t *__restrict__ key_slot,
                     const uint32_t *count_dev, size_t n_max, float *__restrict__ pre, uint32_t dim, int gdt,
                     uint32_t team) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint8_t *inbox_of[kExMaxRanks];
  __shared__ bool s_failed;
  if (threadIdx.x == 0) s_failed = ex_failed(x);
  for (uint32_t p = threadIdx.x; p < x.W; p += blockDim.x) inbox_of[p] = x.ingrads(p);
  __syncthreads();
  if (s_failed) return;
  const size_t nd = min(size_t(__ldcg(count_dev)), n_max);
  const uint32_t inbox = x.W * x.M;
  const uint32_t lane = threadIdx.x & 31u;
  const size_t warp = (size_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const size_t warps = (size_t(gridDim.x) * blockDim.x) >> 5;
  if constexpr (kVec) {
    constexpr int kIlp = 4;
    const uint32_t sub = lane & (team - 1u), per = 32u / team, units = dim / 4u;
    const size_t step = warps * per;
    for (size_t u0 = warp * per + lane / team; u0 < nd; u0 += step * kIlp) {
      float4 *src[kIlp];
      float4 *dst[kIlp];
#pragma unroll
      for (int k = 0; k < kIlp; ++k) {
        const size_t u = u0 + k * step;
        const uint32_t slot = u < nd ? __ldcg(key_slot + u) : inbox;
        src[k] = u < nd ? reinterpret_cast<float4 *>(pre + u * dim) : nullptr;
        dst[k] = slot < inbox ? reinterpret_cast<float4 *>(inbox_of[__ldcg(key_pid + u)] + size_t(slot) * x.grad_bytes)
                              : nullptr;
      }
      for (uint32_t c = sub; c < units; c += team) {
        float4 v[kIlp];
#pragma unroll
        for (int k = 0; k < kIlp; ++k)
          if (src[k]) v[k] = __ldcg(src[k] + c);
#pragma unroll
        for (int k = 0; k < kIlp; ++k) {
          if (!src[k]) continue;
          src[k][c] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (dst[k]) dst[k][c] = v[k];
        }
      }
    }
  } else {
    for (size_t u = warp; u < nd; u += warps) {
      const uint32_t slot = __ldcg(key_slot + u);
      float *src = pre + u * dim;
      uint8_t *dst = slot < inbox ? inbox_of[__ldcg(key_pid + u)] + size_t(slot) * x.grad_bytes : nullptr;
      for (uint32_t e = lane; e < dim; e += 32) {
        const float v = __ldcg(src + e);
        src[e] = 0.0f;
        if (dst == nullptr) continue;
        if (gdt == SE_FLOAT32) reinterpret_cast<float *>(dst)[e] = v;
        else reinterpret_cast<uint16_t *>(dst)[e] = uint16_t(f_to_bits(gdt, v));
      }
    }
  }
}

}  // namespace se_gpu
