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
// written after a system-scope fence with the sender's epoch for that kind;
// a receiver waits until every sender's flag reaches its own epoch. Waits are
// bounded in time: past the exchange's timeout the kernel records it and returns.
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
//    GRADS flag of call k, which senders wait for before publishing call k+1.
#pragma once

#include "se_partition.cuh"

namespace se_gpu {

constexpr uint32_t kExMaxRanks = 64;

enum ExKind : int { kExCounts = 0, kExKeys = 1, kExRows = 2, kExGCounts = 3, kExGrads = 4, kExKinds = 5 };
constexpr uint64_t kSpinLimit = 1ull << 28;  // hard cap on polls (>= 128 ns each) behind the timeout

struct ExView {
  uint8_t *const *peer;  // [W] arena base of every rank (own included), device array
  uint32_t W, me;
  uint32_t row_bytes, grad_bytes;
  uint64_t timeout_ns;
  // byte offsets inside every arena
  uint64_t o_flags, o_epochs, o_counts, o_gcounts, o_inkeys, o_inpos, o_gkeys, o_ingrads, o_rows, o_words;

  __device__ __forceinline__ uint32_t *flags(uint32_t r) const { return reinterpret_cast<uint32_t *>(peer[r] + o_flags); }
  __device__ __forceinline__ uint32_t *epochs() const { return reinterpret_cast<uint32_t *>(peer[me] + o_epochs); }
  __device__ __forceinline__ uint32_t *counts(uint32_t r, int kind) const {
    return reinterpret_cast<uint32_t *>(peer[r] + (kind == kExGCounts ? o_gcounts : o_counts));
  }
  __device__ __forceinline__ unsigned long long *inkeys(uint32_t r) const {
    return reinterpret_cast<unsigned long long *>(peer[r] + o_inkeys);
  }
  __device__ __forceinline__ uint32_t *inpos(uint32_t r) const { return reinterpret_cast<uint32_t *>(peer[r] + o_inpos); }
  __device__ __forceinline__ unsigned long long *gkeys(uint32_t r) const {
    return reinterpret_cast<unsigned long long *>(peer[r] + o_gkeys);
  }
  __device__ __forceinline__ uint8_t *ingrads(uint32_t r) const { return peer[r] + o_ingrads; }
  __device__ __forceinline__ uint8_t *rows(uint32_t r) const { return peer[r] + o_rows; }
  // own words: [kExTotal] received gradient rows (accumulate count),
  // [kExTotalStaged] its value before the GRADS wait, [kExStatus] timeout bits
  __device__ __forceinline__ uint32_t *words() const { return reinterpret_cast<uint32_t *>(peer[me] + o_words); }
};

enum ExWord : int { kExTotal = 0, kExTotalStaged = 1, kExStatus = 2, kExWords = 4 };

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

// One block: bumps this rank's epoch of `kind`, optionally stores this rank's
// per-owner counts into row `me` of every rank's count matrix, then raises
// flag (kind, me) on every rank after a system-scope fence.
__global__ void k_ex_publish(ExView x, int kind, const uint32_t *counts_local) {
  __shared__ uint32_t e;
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
    __threadfence_system();
    st_release_sys(x.flags(p) + size_t(kind) * x.W + x.me, e);
  }
}

// Route scatter into the owners' inboxes (forward: keys and batch positions;
// backward: keys and gradient rows copied in units U). Same two-pass stable
// ranking as k_route_scatter; the slot on owner d is sum_{s < me} counts[s][d]
// plus the key's rank among this rank's keys for d.
template <class K, bool kGrads, class U>
__global__ void __launch_bounds__(kRouteThreads)
k_ex_scatter(PartSpec s, ExView x, const K *__restrict__ keys, size_t count, const uint32_t *__restrict__ tile_offsets,
             const uint32_t *__restrict__ counts_local, const uint8_t *__restrict__ grads) {
  extern __shared__ uint32_t sm[];
  uint32_t *warp_base = sm;                   // [kRouteWarps][W]
  uint32_t *remote = sm + kRouteWarps * s.n;  // [W] slot base on each owner minus the local prefix
  __shared__ bool ok;
  const int kind = kGrads ? kExGCounts : kExCounts;
  if (threadIdx.x == 0) ok = ex_wait(x, kind);
  __syncthreads();
  if (!ok) return;
  const uint32_t *cm = x.counts(x.me, kind);
  if (kGrads && blockIdx.x == 0 && threadIdx.x == 0) {
    uint32_t total = 0;
    for (uint32_t q = 0; q < x.W; ++q) total += __ldcg(cm + size_t(q) * x.W + x.me);
    x.words()[kExTotalStaged] = total;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  for (uint32_t j = threadIdx.x; j < kRouteWarps * s.n; j += blockDim.x) warp_base[j] = 0;
  for (uint32_t d = threadIdx.x; d < s.n; d += blockDim.x) {
    uint32_t base = 0, local_prefix = 0;
    for (uint32_t q = 0; q < x.me; ++q) base += __ldcg(cm + size_t(q) * x.W + d);
    for (uint32_t q = 0; q < d; ++q) local_prefix += counts_local[q];
    remote[d] = base - local_prefix;  // modular: added to the routed index below
  }
  __syncthreads();
  const size_t wbase = size_t(blockIdx.x) * kRouteTile + size_t(warp) * kRouteWarpKeys;
  uint32_t *mine = warp_base + size_t(warp) * s.n;
  for (int r = 0; r < kRouteWarpKeys; r += 32) {
    const size_t i = wbase + r + lane;
    const bool valid = i < count;
    const uint32_t pid = valid ? partition_of<K>(s, keys[i]) : 0xffffffffu;
    const unsigned peers = __match_any_sync(0xffffffffu, pid);
    if (valid && (peers & lt) == 0) mine[pid] += __popc(peers);
    __syncwarp();
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
  for (int r = 0; r < kRouteWarpKeys; r += 32) {
    const size_t i = wbase + r + lane;
    const bool valid = i < count;
    K key{};
    uint32_t pid = 0xffffffffu;
    if (valid) {
      key = keys[i];
      pid = partition_of<K>(s, key);
    }
    const unsigned peers = __match_any_sync(0xffffffffu, pid);
    uint32_t slot = 0;
    if (valid) slot = mine[pid] + __popc(peers & lt) + remote[pid];
    __syncwarp();
    if (valid) {
      if (kGrads) {
        x.gkeys(pid)[slot] = key_u64(key);
      } else {
        x.inkeys(pid)[slot] = key_u64(key);
        x.inpos(pid)[slot] = uint32_t(i);
      }
      if ((peers & lt) == 0) mine[pid] += __popc(peers);
    }
    __syncwarp();
    if constexpr (kGrads) {
      // the warp copies its (up to) 32 gradient rows one after another
      const uint32_t units = x.grad_bytes / uint32_t(sizeof(U));
      const unsigned any = __ballot_sync(0xffffffffu, valid);
      for (int k = 0; k < 32; ++k) {
        if (!((any >> k) & 1u)) continue;
        const uint32_t kp = __shfl_sync(0xffffffffu, pid, k);
        const uint32_t ks = __shfl_sync(0xffffffffu, slot, k);
        const size_t ki = wbase + r + k;
        const U *src = reinterpret_cast<const U *>(grads + ki * x.grad_bytes);
        U *dst = reinterpret_cast<U *>(x.ingrads(kp) + size_t(ks) * x.grad_bytes);
        for (uint32_t u = lane; u < units; u += 32) dst[u] = src[u];
      }
    }
  }
  __threadfence_system();
}

// Owner of the keys: after the keys of every sender arrived, finds (and with
// kInsert inserts) each key and stores its row into the requester's row
// buffer at the requester's batch position. Keys claimed by another group of
// the same launch go to the deferred list. Absent keys of a plain lookup get
// a zero row.
template <int LANES, int VEC, bool kInsert>
__global__ void __launch_bounds__(256)
k_ex_owner(Dir d, Layout L, uint8_t *__restrict__ slabs, uint32_t *next_row, uint64_t capacity, InitSpec init,
           ExView x, uint32_t *def_count, uint32_t *def_idx, unsigned long long *def_word, uint32_t *status) {
  __shared__ uint32_t prefix[kExMaxRanks + 1];
  __shared__ bool ok;
  if (threadIdx.x == 0) ok = ex_wait(x, kExKeys);
  __syncthreads();
  if (!ok) return;
  if (threadIdx.x == 0) {
    uint32_t run = 0;
    for (uint32_t s = 0; s < x.W; ++s) {
      prefix[s] = run;
      run += __ldcg(x.counts(x.me, kExCounts) + size_t(s) * x.W + x.me);
    }
    prefix[x.W] = run;
  }
  __syncthreads();
  const uint32_t total = prefix[x.W];
  const size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t groups = size_t(gridDim.x) * blockDim.x / LANES;
  const uint32_t lane = uint32_t(t % LANES);
  const unsigned mask = group_mask<LANES>();
  const unsigned long long *inkeys = x.inkeys(x.me);
  const uint32_t *inpos = x.inpos(x.me);
  for (size_t i = t / LANES; i < total; i += groups) {
    const uint64_t key = __ldcg(inkeys + i);
    const uint32_t pos = __ldcg(inpos + i);
    uint32_t src = 0;
    while (src + 1 < x.W && prefix[src + 1] <= i) ++src;
    void *out_row = x.rows(src) + size_t(pos) * x.row_bytes;
    int kind = kFound;
    uint32_t row = kNoRow;
    uint32_t *word = nullptr;
    if constexpr (kInsert) {
      if (lane == 0) {
        const InsertResult r = dir_find_or_insert(d, key);
        kind = r.kind;
        word = r.row_word;
        if (kind == kInserted) {
          row = atomicAdd(next_row, 1u);
          if (row >= capacity) {
            raise_status(status, kStatusTableFull);
            kind = kFull;
          }
        } else if (kind == kFound) {
          row = __ldcg(word);
          if (row == kNoRow) kind = 3;  // claimed, not yet published
        } else {
          raise_status(status, kStatusTableFull);
        }
      }
      kind = __shfl_sync(mask, kind, 0, LANES);
      row = __shfl_sync(mask, row, 0, LANES);
    } else {
      row = dir_find<false>(d, key);
      if (row == kNoRow) kind = kFull;
    }
    if (kind == kFound) {
      const uint8_t *slab = slabs + size_t(row) * L.stride;
      for (uint32_t e = lane * VEC; e < L.dim; e += LANES * VEC) copy_elems<VEC>(out_row, slab, L.pdt, e);
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
  __threadfence_system();
}

// Deferred keys of k_ex_owner: their claimant has published the row by now.
template <int LANES, int VEC>
__global__ void __launch_bounds__(256)
k_ex_owner_deferred(Layout L, const uint8_t *__restrict__ slabs, ExView x, const uint32_t *def_count,
                    const uint32_t *def_idx, const unsigned long long *def_word, uint32_t *status) {
  const size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t groups = size_t(gridDim.x) * blockDim.x / LANES;
  const uint32_t lane = uint32_t(t % LANES);
  const uint32_t count = *def_count;
  for (size_t j = t / LANES; j < count; j += groups) {
    const uint32_t i = def_idx[j];
    uint32_t run = 0, src = 0;
    for (uint32_t s = 0; s < x.W; ++s) {
      const uint32_t c = __ldcg(x.counts(x.me, kExCounts) + size_t(s) * x.W + x.me);
      if (i >= run && i < run + c) src = s;
      run += c;
    }
    const uint32_t pos = __ldcg(x.inpos(x.me) + i);
    void *out_row = x.rows(src) + size_t(pos) * x.row_bytes;
    const uint32_t row = __ldcg(reinterpret_cast<const uint32_t *>(def_word[j]));
    if (row == kNoRow) {
      if (lane == 0) raise_status(status, kStatusTableFull);
      for (uint32_t e = lane * VEC; e < L.dim; e += LANES * VEC) zero_elems<VEC>(out_row, L.pdt, e);
      continue;
    }
    const uint8_t *slab = slabs + size_t(row) * L.stride;
    for (uint32_t e = lane * VEC; e < L.dim; e += LANES * VEC) copy_elems<VEC>(out_row, slab, L.pdt, e);
  }
  __threadfence_system();
}

// Requester: waits for the rows of every owner, then copies this rank's row
// buffer (batch order) to `out` in units U.
template <class U>
__global__ void __launch_bounds__(256)
k_ex_rows_out(ExView x, U *__restrict__ out, size_t units) {
  __shared__ bool ok;
  if (threadIdx.x == 0) ok = ex_wait(x, kExRows);
  __syncthreads();
  if (!ok) return;
  const U *src = reinterpret_cast<const U *>(x.rows(x.me));
  for (size_t u = size_t(blockIdx.x) * blockDim.x + threadIdx.x; u < units; u += size_t(gridDim.x) * blockDim.x)
    out[u] = __ldcg(src + u);
}

// Owner, backward: waits for every sender's gradients and sets the number of
// received rows (the device count of the accumulate that follows; 0 when the
// wait gave up).
__global__ void k_ex_grads_total(ExView x) {
  if (threadIdx.x != 0) return;
  uint32_t *w = x.words();
  w[kExTotal] = ex_wait(x, kExGrads) ? w[kExTotalStaged] : 0u;
}

}  // namespace se_gpu
