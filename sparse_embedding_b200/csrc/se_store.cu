// B200 store: kernels for the forward gather, insert-on-miss, gradient
// accumulation and the fused segment-reduce + optimizer step, and the host
// object behind the C ABI in include/se_gpu.h.
//
// Per-key work is done by a group of LANES threads (4..32, a power of two):
// every lane of the group probes the same 64-byte bucket (one line, broadcast
// within the group), then the lanes split the row in 16-byte (VEC = 4
// elements) or element-wide chunks.

#include <cub/block/block_reduce.cuh>
#include <cub/block/block_scan.cuh>
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "se_common.cuh"
#include "se_host.hpp"
#include "se_store_kernels.cuh"
#include "se_accum.cuh"

namespace se_gpu {

// ===========================================================================
// Kernels
// ===========================================================================

template <class V> __device__ __forceinline__ V zero_unit();
template <> __device__ __forceinline__ uint4 zero_unit<uint4>() { return make_uint4(0, 0, 0, 0); }
template <> __device__ __forceinline__ uint2 zero_unit<uint2>() { return make_uint2(0, 0); }
template <> __device__ __forceinline__ uint32_t zero_unit<uint32_t>() { return 0u; }
template <> __device__ __forceinline__ uint16_t zero_unit<uint16_t>() { return 0; }

// forward_lookup (hogwild_embedding_store.hpp:4406-4534): probe, copy the
// param section of the row (simd_copy, memory_ops.hpp:31-35), zero on miss
// (4501-4503). Row copied in units V (16, 4 or 2 bytes).
template <int LANES, class V>
__global__ void __launch_bounds__(256)
k_lookup(Dir d, const uint8_t *__restrict__ slabs, uint32_t stride, uint32_t row_units,
         const void *__restrict__ keys, int kdt, size_t n, V *__restrict__ out) {
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  const size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t i = t / LANES;
  const uint32_t lane = uint32_t(t % LANES);
  if (i >= n) return;
  const uint32_t row = dir_find<false>(d, load_key(keys, kdt, i));
  V *dst = out + i * row_units;
  if (row != kNoRow) {
    const V *src = reinterpret_cast<const V *>(slabs + size_t(row) * stride);
    constexpr int kIlp = LANES == 2 ? 8 : 4;  // loads in flight per lane
    for (uint32_t u = lane; u < row_units; u += LANES * kIlp) {
      V v[kIlp];
#pragma unroll
      for (int k = 0; k < kIlp; ++k)
        if (u + k * LANES < row_units) v[k] = src[u + k * LANES];
#pragma unroll
      for (int k = 0; k < kIlp; ++k)
        if (u + k * LANES < row_units) dst[u + k * LANES] = v[k];
    }
  } else {
    for (uint32_t u = lane; u < row_units; u += LANES) dst[u] = zero_unit<V>();
  }
}

// forward_lookup of wide rows through the TMA (rows of 512..1,024 bytes, a
// multiple of 16, 16-byte aligned slabs and output). Each warp takes 32
// consecutive batch positions per round: every lane resolves one key, the
// rows found are brought into the warp's shared-memory buffer with one bulk
// copy each (cp.async.bulk, completion counted in bytes on the warp's
// mbarrier), rows of absent keys are zero-filled there, and the warp's 32
// rows - consecutive in the output - leave with one bulk store. The next
// round's keys are resolved while this round's copies are in flight, so the
// buffer holds rows in flight for most of the kernel. The waits are bounded:
// a copy that never lands raises kStatusCopyTimeout.
constexpr uint32_t kBulkWarps = 4;  // warps per block; shared memory = 4 x 32 rows
constexpr uint32_t kBulkMinRow = 512, kBulkMaxRow = 1024;

__device__ __forceinline__ uint32_t bulk_probe(const Dir &d, const void *keys, int kdt, size_t i0, size_t n,
                                               uint32_t lane) {
  return i0 + lane < n ? dir_find<false>(d, load_key(keys, kdt, i0 + lane)) : kNoRow;
}

__global__ void __launch_bounds__(kBulkWarps * 32)
k_lookup_bulk(Dir d, const uint8_t *__restrict__ slabs, uint32_t stride, uint32_t row_bytes,
              const void *__restrict__ keys, int kdt, size_t n, uint8_t *__restrict__ out, uint32_t *status) {
  extern __shared__ __align__(128) uint8_t s_buf[];  // [kBulkWarps][32][row_bytes]
  __shared__ __align__(8) uint64_t s_bar[kBulkWarps];
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  uint8_t *buf = s_buf + size_t(warp) * 32u * row_bytes;
  uint8_t *slot = buf + size_t(lane) * row_bytes;
  uint64_t *bar = &s_bar[warp];
  if (lane == 0) mbar_init(bar, 1);
  __syncwarp();
  uint32_t parity = 0;
  const size_t step = size_t(gridDim.x) * kBulkWarps * 32u;
  size_t i0 = (size_t(blockIdx.x) * kBulkWarps + warp) * 32u;
  uint32_t row = bulk_probe(d, keys, kdt, i0, n, lane);
  for (; i0 < n; i0 += step) {
    const uint32_t cnt = uint32_t(min(size_t(32), n - i0));
    const unsigned found = __ballot_sync(0xffffffffu, row != kNoRow);
    // the bytes to come are announced before any copy can complete
    if (lane == 0) mbar_arrive_expect_tx(bar, uint32_t(__popc(found)) * row_bytes);
    __syncwarp();
    if (row != kNoRow) {
      bulk_copy_g2s(slot, slabs + size_t(row) * stride, row_bytes, bar);
    } else if (lane < cnt) {
      for (uint32_t u = 0; u < row_bytes / 16u; ++u) reinterpret_cast<uint4 *>(slot)[u] = make_uint4(0, 0, 0, 0);
      fence_proxy_async_smem();  // the zeros are seen by the bulk store
    }
    // the next round's keys while the copies are in flight
    row = i0 + step < n ? bulk_probe(d, keys, kdt, i0 + step, n, lane) : kNoRow;
    uint32_t polls = 0;
    bool landed = true;
    while (!mbar_try_wait(bar, parity)) {
      if (++polls > kCopySpinLimit) {
        landed = false;
        break;
      }
    }
    if (!__all_sync(0xffffffffu, landed)) {
      if (lane == 0) {
        raise_status(status, kStatusCopyTimeout);
        // the copies still in flight land before the block's shared memory is released
        for (uint32_t w = 0; w < kCopySpinLimit && !mbar_try_wait(bar, parity); ++w) __nanosleep(64);
      }
      __syncwarp();
      return;
    }
    parity ^= 1u;
    __syncwarp();
    if (lane == 0) {
      bulk_store_s2g(out + i0 * row_bytes, buf, cnt * row_bytes);
      bulk_wait_read();  // the buffer is free for the next round
    }
    __syncwarp();
  }
  if (lane == 0) {
    bulk_wait_all();
    mbar_inval(bar);
  }
}

template <int VEC>
__device__ __forceinline__ void zero_elems(void *dst, int dt, size_t e) {
  float z[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) z[j] = 0.0f;
  stv<VEC>(dst, dt, e, z);
}

// Copies elements e0, e0 + step, ... (< dim) of a row in VEC-element units,
// raw bits. ILP loads are in flight before their stores: a few lanes per key
// then keep a whole row's loads outstanding, and more keys fit in flight per SM.
// kCached: plain loads, which L1 may serve. A row found through the
// directory in an insert kernel was published before it was found, and no
// thread of the launch read its slab before its claimant initialised it (a
// fresh or recycled row belongs to no key until then), so no L1 line of it
// can be stale; hot keys' rows are then fetched from L2 once per SM instead
// of once per position. Otherwise loads go to L2 (ld.cg).
template <class U, int VEC, int ILP, bool kCached = false>
__device__ __forceinline__ void copy_units(void *dst, const void *src, uint32_t dim, uint32_t e0, uint32_t step) {
  const U *s = static_cast<const U *>(src);
  U *d = static_cast<U *>(dst);
  for (uint32_t e = e0; e < dim; e += step * ILP) {
    U v[ILP];
#pragma unroll
    for (int k = 0; k < ILP; ++k)
      if (e + k * step < dim) v[k] = kCached ? s[(e + k * step) / VEC] : __ldcg(s + (e + k * step) / VEC);
#pragma unroll
    for (int k = 0; k < ILP; ++k)
      if (e + k * step < dim) d[(e + k * step) / VEC] = v[k];
  }
}

template <int VEC, int ILP = 4, bool kCached = false>
__device__ __forceinline__ void copy_row(void *dst, const void *src, int dt, uint32_t dim, uint32_t e0,
                                         uint32_t step) {
  if (dt == SE_FLOAT32) {
    if constexpr (VEC == 4) copy_units<uint4, 4, ILP, kCached>(dst, src, dim, e0, step);
    else copy_units<unsigned int, 1, ILP, kCached>(dst, src, dim, e0, step);
  } else {
    if constexpr (VEC == 4) copy_units<uint2, 4, ILP, kCached>(dst, src, dim, e0, step);
    else copy_units<unsigned short, 1, ILP, kCached>(dst, src, dim, e0, step);
  }
}

// Initialises a freshly claimed slab: param from the initializer (also written
// to `out_row`), optimizer state from InitSpec, Adam step = 0.
template <int LANES, int VEC>
__device__ __forceinline__ void init_slab(const Layout &L, uint8_t *slab, const InitSpec &init,
                                          uint64_t key, uint32_t lane, void *out_row) {
  const uint32_t seed = uint32_t(key ^ (key >> 32));
  for (uint32_t e = lane * VEC; e < L.dim; e += LANES * VEC) {
    float v[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j)
      v[j] = init.kind == SE_INIT_UNIFORM ? uniform_value(seed, e + j, init.lo, init.diff) : 0.0f;
    stv<VEC>(slab, L.pdt, e, v);
    stv<VEC>(out_row, L.pdt, e, v);
    if (L.nstate >= 1) {
      float s[VEC];
#pragma unroll
      for (int j = 0; j < VEC; ++j) s[j] = init.state0;
      stv<VEC>(slab + L.state0, L.odt, e, s);
    }
    if (L.nstate >= 2) {
      float s[VEC];
#pragma unroll
      for (int j = 0; j < VEC; ++j) s[j] = 0.0f;
      stv<VEC>(slab + L.state1, L.odt, e, s);
    }
  }
  if (L.nstate >= 2 && lane == 0) *reinterpret_cast<uint32_t *>(slab + L.step) = 0u;
  if (L.score != 0u && lane == 0) *reinterpret_cast<unsigned long long *>(slab + L.score) = 0ull;  // a new row's score
}

// The last block of k_lookup_or_insert: copies the published rows of the
// positions whose key another group of the launch claimed (row bytes as
// 32-bit words, or 16-bit for odd half-precision rows; they are few), then
// resets the launch's counters. Out of line, so the main path keeps its
// register budget.
// Arguments by value (scalars): a reference to a kernel parameter would make
// every thread copy the parameter struct to its stack.
__device__ __noinline__ void finish_deferred(uint32_t stride, size_t row_bytes, const uint8_t *slabs, size_t n,
                                             void *out, uint32_t *def_count, const uint32_t *def_pos,
                                             const unsigned long long *def_word, uint32_t *status, uint32_t *done,
                                             uint32_t *fc_rows, uint32_t *fc_n, bool cache) {
  __threadfence();
  const uint32_t count = __ldcg(def_count);
  const bool words = row_bytes % 4 == 0;
  const uint32_t units = uint32_t(words ? row_bytes / 4 : row_bytes / 2);
  for (uint32_t j = threadIdx.x / 32; j < count; j += blockDim.x / 32) {
    const uint32_t lane = threadIdx.x & 31u;
    const size_t pos = __ldcg(def_pos + j);
    const uint32_t row = __ldcg(reinterpret_cast<const uint32_t *>(__ldcg(def_word + j)));
    uint8_t *dst = static_cast<uint8_t *>(out) + pos * row_bytes;
    if (cache && lane == 0) fc_rows[pos] = row;
    if (row == kNoRow && lane == 0) raise_status(status, kStatusTableFull);
    const uint8_t *src = slabs + size_t(row) * stride;
    for (uint32_t u = lane; u < units; u += 32) {
      if (words) reinterpret_cast<uint32_t *>(dst)[u] = row == kNoRow ? 0u : __ldcg(reinterpret_cast<const uint32_t *>(src) + u);
      else reinterpret_cast<uint16_t *>(dst)[u] = row == kNoRow ? uint16_t(0) : reinterpret_cast<const uint16_t *>(src)[u];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    *def_count = 0u;  // for the next launch
    *done = 0u;
    if (fc_n) *fc_n = cache ? uint32_t(n) : 0u;
  }
}

// lookup_or_insert (hogwild_embedding_store.hpp:4925-4980 ->
// SlotStore::find_or_insert_batch 3057-3353). One claimant per absent key
// initialises and publishes its row; other positions of the same key found
// the claim before the row was published, are listed, and are finished by
// the launch's last block once every claimant has published.
template <int LANES, int VEC>
__global__ void __launch_bounds__(256)
k_lookup_or_insert(Dir d, Layout L, uint8_t *__restrict__ slabs, RowAlloc ra, InitSpec init, const void *__restrict__ keys, int kdt,
                   size_t n, void *__restrict__ out, uint32_t *def_count, uint32_t *def_pos,
                   unsigned long long *def_word, uint32_t *status, uint32_t *done, FwdCache fc) {
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  const size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t i = t / LANES;
  const uint32_t lane = uint32_t(t % LANES);
  const unsigned mask = group_mask<LANES>();
  const size_t row_bytes = size_t(L.dim) * (L.pdt == SE_FLOAT32 ? 4 : 2);
  const bool cache = fc.keys != nullptr && n <= fc.cap;
  if (i < n) {
    const uint64_t key = load_key(keys, kdt, i);
    int kind = kFound;
    uint32_t row = kNoRow;
    uint32_t *word = nullptr;
    if (lane == 0) {
      const InsertResult r = dir_find_or_insert(d, key);
      kind = r.kind;
      word = r.row_word;
      // found: published, claimed in this launch (3), or erased and revived here
      if (kind == kFound) kind = resolve_found(word, &row, r.seen);
      else if (kind == kFull) raise_status(status, kStatusTableFull);
    }
    const uint32_t taken = take_rows_warp(ra, live_lanes(t, n * LANES), lane == 0 && kind == kInserted);
    if (lane == 0 && kind == kInserted) {
      row = taken;
      if (row >= ra.capacity) {
        raise_status(status, kStatusTableFull);
        kind = kFull;
      }
    }
    kind = __shfl_sync(mask, kind, 0, LANES);
    row = __shfl_sync(mask, row, 0, LANES);
    void *out_row = static_cast<uint8_t *>(out) + i * row_bytes;
    if (cache && lane == 0) {
      fc.keys[i] = key;
      fc.rows[i] = (kind == kFound || kind == kInserted) ? row : kNoRow;  // deferred: filled below
    }
    if (kind == kFound) {
      const uint8_t *slab = slabs + size_t(row) * L.stride;
      copy_row<VEC, LANES == 2 ? 8 : 4, true>(out_row, slab, L.pdt, L.dim, lane * VEC, LANES * VEC);
    } else if (kind == kInserted) {
      uint8_t *slab = slabs + size_t(row) * L.stride;
      init_slab<LANES, VEC>(L, slab, init, key, lane, out_row);
      __threadfence();  // every lane's slab writes are visible device-wide ...
      __syncwarp(mask);
      if (lane == 0) atomicExch(word, row);  // ... before the row is published
    } else if (kind == 3) {
      if (lane == 0) {
        const uint32_t j = atomicAdd(def_count, 1u);
        def_pos[j] = uint32_t(i);
        def_word[j] = reinterpret_cast<unsigned long long>(word);
      }
    } else {
      for (uint32_t e = lane * VEC; e < L.dim; e += LANES * VEC) zero_elems<VEC>(out_row, L.pdt, e);
    }
  }
  // The last block to finish serves the positions whose key another group
  // claimed: every claimant has published its row (fence, then the count).
  __shared__ bool s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(done, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last)
    finish_deferred(L.stride, row_bytes, slabs, n, out, def_count, def_pos, def_word, status, done, fc.rows, fc.n,
                    cache);
}

// Per-row counting of the pending entries for optimizer_step's grouping,
// done where the entries are appended: each row present gets a segment the
// first time one of its entries is counted; entries whose key is absent when
// appended are listed and probed again at step time (k_group_fix).
struct CountWs {
  uint32_t *row_cnt;    // [capacity] entries of a row in this window (zero between steps)
  uint32_t *row_seg;    // [capacity] segment of a row in this window
  uint32_t *seg_row;    // [pending capacity] row of each segment
  uint32_t *seg_ctr;    // segments registered in this window
  uint32_t *unres;      // [pending capacity] entries whose key was absent when appended
  uint32_t *unres_ctr;  // their count
};

// Whole warp, one entry per lane (valid lanes only): counts the entries'
// rows (one atomic per distinct row of the warp) and registers new segments
// (one atomic per warp).
__device__ __forceinline__ void count_entries(const CountWs &c, bool valid, uint32_t row, uint32_t entry) {
  const uint32_t lane = threadIdx.x & 31u;
  const unsigned lt = (1u << lane) - 1u;
  const bool absent = valid && row == kNoRow;
  const unsigned abs_mask = __ballot_sync(0xffffffffu, absent);
  if (abs_mask) {
    uint32_t base = 0;
    if (lane == __ffs(abs_mask) - 1) base = atomicAdd(c.unres_ctr, uint32_t(__popc(abs_mask)));
    base = __shfl_sync(0xffffffffu, base, __ffs(abs_mask) - 1);
    if (absent) c.unres[base + __popc(abs_mask & lt)] = entry;
  }
  const uint32_t key = valid && row != kNoRow ? row : kNoRow;
  const unsigned peers = __match_any_sync(0xffffffffu, key);
  bool fresh = false;
  if (key != kNoRow && (peers & lt) == 0) fresh = atomicAdd(&c.row_cnt[key], uint32_t(__popc(peers))) == 0u;
  const unsigned fresh_mask = __ballot_sync(0xffffffffu, fresh);
  if (fresh_mask) {
    uint32_t base = 0;
    if (lane == __ffs(fresh_mask) - 1) base = atomicAdd(c.seg_ctr, uint32_t(__popc(fresh_mask)));
    base = __shfl_sync(0xffffffffu, base, __ffs(fresh_mask) - 1);
    if (fresh) {
      const uint32_t sid = base + __popc(fresh_mask & lt);
      c.seg_row[sid] = key;
      c.row_seg[key] = sid;
    }
  }
}

// accumulate_gradients, append phase: GradientAccumulator::validate_input
// (gradient_accumulator.hpp:88-104) and the entry scaling of accumulate_hashed
// (106-128): scaled = g / gradient_scale must be finite and within both the
// gradient and the parameter dtype; the stored row is g (scale 1) or the
// scaled value rounded to the gradient dtype.
//
// With kBag the gradient row of entry i is row grad_row[i] of `grads` (the
// backward of a sum-pooled bag: every key of bag b gets the bag's gradient).
template <int VEC, bool kBag = false>
__global__ void __launch_bounds__(256)
k_accumulate(Dir d, const void *__restrict__ keys, int kdt, size_t n_max, const uint32_t *n_dev,
             const void *__restrict__ grads, int gdt, uint32_t dim, float scale, float maxv,
             unsigned long long *__restrict__ pkeys_base, uint32_t *__restrict__ prows_base,
             void *__restrict__ pgrads_base, size_t pcap, uint32_t *pending, uint32_t *done, uint32_t *status,
             uint32_t *err, CountWs cw, int count_rows, const uint32_t *__restrict__ known_rows,
             const uint32_t *__restrict__ grad_row, FwdCache fc) {
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  const size_t stride = size_t(gridDim.x) * blockDim.x;
  const size_t tid = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  // Rows are appended at the committed pending count; the batch size is the
  // host's n_max or, for exchanged batches, a count in device memory.
  const uint32_t base = *pending;
  const size_t n = n_dev ? min(size_t(*n_dev), n_max) : n_max;
  if (size_t(base) + n > pcap) {
    // The buffers were sized from the host's count of pending rows; a device
    // count beyond it means calls of this store were not stream-ordered.
    // Every block takes this exit, so nothing is appended or committed.
    if (tid == 0) raise_status(err, kStatusPendingOverflow);
    return;
  }
  unsigned long long *pkeys = pkeys_base + base;
  uint32_t *prows = prows_base + base;
  // rows the last lookup_or_insert resolved for the same keys at the same positions
  const size_t cached = fc.n ? min(size_t(__ldcg(fc.n)), size_t(fc.cap)) : 0;
  void *pgrads = static_cast<uint8_t *>(pgrads_base) + size_t(base) * dim * (gdt == SE_FLOAT32 ? 4 : 2);
  // Keys and their rows (the directory probe overlaps the gradient copy; a
  // key absent now is probed again by optimizer_step). With count_rows the
  // rows are counted for the step's grouping here (warp-uniform loop).
  for (size_t i0 = tid - (tid & 31u); i0 < n; i0 += stride) {
    const size_t i = i0 + (tid & 31u);
    const bool valid = i < n;
    uint32_t row = kNoRow;
    if (valid) {
      const uint64_t key = load_key(keys, kdt, i);
      pkeys[i] = key;
      // rows an exchange's owner kernel already resolved for these keys, or
      // the last lookup_or_insert of the same keys; else a probe
      if (known_rows) {
        row = known_rows[i];
      } else {
        row = kNoRow;
        if (i < cached && __ldcg(fc.keys + i) == key) row = __ldcg(fc.rows + i);
        if (row == kNoRow) row = dir_find<false>(d, key);
      }
      prows[i] = row;
    }
    if (count_rows) count_entries(cw, valid, row, base + uint32_t(i));
  }
  const size_t chunks = n * dim / VEC;
  bool bad = false;
  constexpr int kIlp = 4;  // chunks loaded before any is stored: more bytes in flight per thread
  for (size_t c0 = tid; c0 < chunks; c0 += stride * kIlp) {
    float g[kIlp][VEC];
#pragma unroll
    for (int k = 0; k < kIlp; ++k) {
      if (c0 + k * stride >= chunks) continue;
      size_t e = (c0 + k * stride) * VEC;
      if constexpr (kBag) {
        const size_t i = e / dim;  // VEC divides dim: a chunk stays inside one entry
        e = size_t(grad_row[i]) * dim + (e - i * dim);
      }
      ldv<VEC>(grads, gdt, e, g[k]);
    }
#pragma unroll
    for (int k = 0; k < kIlp; ++k) {
      if (c0 + k * stride >= chunks) continue;
      if (scale == 1.0f) {  // g / 1 == g: no division (uniform branch)
#pragma unroll
        for (int j = 0; j < VEC; ++j) bad |= !(fabsf(g[k][j]) <= maxv);
      } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          g[k][j] = __fdiv_rn(g[k][j], scale);
          bad |= !(fabsf(g[k][j]) <= maxv);
        }
      }
      stv<VEC>(pgrads, gdt, (c0 + k * stride) * VEC, g[k]);
    }
  }
  if (bad) raise_status(status, kStatusBadGradient);
  // The last block to finish commits the rows (every block has read `base`;
  // the rows themselves are read by later kernels only, so no fence).
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *pending = base + uint32_t(n);
      *done = 0u;
    }
  }
}

struct OptSpec {
  int kind;
  float lr, b1, b2, eps, wd, omb1, omb2;
  uint32_t simd_cut;   // elements below use the reference's vector formulas
  const float *bc;     // Adam bias corrections: bc[2t], bc[2t+1]
  float factor;        // gradient_scale / normalization_steps
  int raw;             // gradient used as stored (GradT == ParamT, factor 1)
  const uint32_t *poison;  // nonzero: the window holds a batch that failed validation
  // dynamic learning rate (dynamic_lr_policy.hpp:32-124): the row's lr from its score
  int lr_kind;             // enum se_lr_policy; SE_LR_CONSTANT: lr for every row
  float lr_min_ratio;
  unsigned long long lr_max_score;
  const float *lr_lut;     // cosine multipliers [0, max_score], or the custom LUT
};

// Learning rate of a row with score `sc` (the reference's compute_lr, with
// its compiled fused multiply-add in the cosine policy).
__device__ __forceinline__ float row_lr(const OptSpec &o, unsigned long long sc) {
  const float base = o.lr;
  switch (o.lr_kind) {
  case SE_LR_SQRT_DECAY: return sc == 0ull ? base : __fdiv_rn(base, __fsqrt_rn(__ull2float_rn(sc)));
  case SE_LR_LOG_DECAY: return __fdiv_rn(base, log2f(__fadd_rn(2.0f, __ull2float_rn(sc))));
  case SE_LR_INVERSE_DECAY: return sc == 0ull ? base : __fdiv_rn(base, __ull2float_rn(sc));
  case SE_LR_COSINE_FREQUENCY: {
    const float min_lr = __fmul_rn(base, o.lr_min_ratio);
    if (sc >= o.lr_max_score) return min_lr;
    return __fmaf_rn(__fsub_rn(base, min_lr), o.lr_lut[sc], min_lr);
  }
  case SE_LR_CUSTOM_LUT: return __fmul_rn(base, o.lr_lut[sc >= o.lr_max_score ? o.lr_max_score : sc]);
  default: return base;
  }
}

// Applies the optimizer to VEC elements [e, e+VEC) of one row, given the
// reduced gradient in the gradient dtype's precision.
//   SGD:     simd_sgd_update (sgd_ops.hpp:30-78): g = fma(wd, p, g); p = fma(-lr, g, p).
//   Adam:    simd_adam_update (adam_ops.hpp:30-232), vector body below
//            simd_cut, compiled scalar tail above it.
//   Adagrad: no reference counterpart; acc = fma(g, g, acc),
//            p = fma(-lr, g / (sqrt(acc) + eps), p).
// Parameters and optimizer state of VEC elements of one row, loaded ahead of
// the gradient reduction so their latency overlaps it.
template <int VEC> struct RowState {
  float p[VEC], s0[VEC], s1[VEC];
};

template <int VEC>
__device__ __forceinline__ void load_state(const Layout &L, const uint8_t *slab, const OptSpec &o, uint32_t e,
                                           RowState<VEC> &r) {
  ldv<VEC>(slab, L.pdt, e, r.p);
  if (o.kind == SE_OPT_ADAGRAD || o.kind == SE_OPT_ADAM) ldv<VEC>(slab + L.state0, L.odt, e, r.s0);
  if (o.kind == SE_OPT_ADAM) ldv<VEC>(slab + L.state1, L.odt, e, r.s1);
}

// kDyn: the store has a dynamic learning-rate policy (the row's lr from its
// score); a separate instantiation keeps the constant-lr kernels unchanged.
template <int VEC, bool kDyn = false>
__device__ __forceinline__ void apply_loaded(const Layout &L, uint8_t *slab, const OptSpec &o, uint32_t t,
                                             uint32_t e, const float (&gsum)[VEC], RowState<VEC> &r) {
  float g[VEC];
  float (&p)[VEC] = r.p;
  float lr = o.lr;
  if constexpr (kDyn) lr = row_lr(o, *reinterpret_cast<const unsigned long long *>(slab + L.score));
  // GradientBatchView::assign (gradient_accumulator.hpp:38-53): g * scale / N -> ParamT.
#pragma unroll
  for (int j = 0; j < VEC; ++j) g[j] = o.raw ? gsum[j] : round_to(L.pdt, __fmul_rn(gsum[j], o.factor));
  if (o.kind == SE_OPT_SGD) {
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float gg = __fmaf_rn(o.wd, p[j], g[j]);
      p[j] = __fmaf_rn(-lr, gg, p[j]);
    }
  } else if (o.kind == SE_OPT_ADAGRAD) {
    float (&a)[VEC] = r.s0;
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      float gg = g[j];
      if (o.wd > 0.0f) gg = __fmaf_rn(o.wd, p[j], gg);
      a[j] = __fmaf_rn(gg, gg, a[j]);
      const float denom = __fadd_rn(__fsqrt_rn(a[j]), o.eps);
      p[j] = __fmaf_rn(-lr, __fdiv_rn(gg, denom), p[j]);
    }
    stv<VEC>(slab + L.state0, L.odt, e, a);
  } else if (o.kind == SE_OPT_ADAM) {
    const float (&m)[VEC] = r.s0;
    const float (&v)[VEC] = r.s1;
    float ms[VEC], vs[VEC];
    const float bc1 = o.bc[2 * t], bc2 = o.bc[2 * t + 1];
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      float gg = g[j];
      if (o.wd > 0.0f) gg = __fmaf_rn(o.wd, p[j], gg);
      const bool vec_body = e + j < o.simd_cut;
      const float mi = __fmaf_rn(o.b1, m[j], __fmul_rn(o.omb1, gg));
      const float addv = vec_body ? __fmul_rn(o.omb2, __fmul_rn(gg, gg))
                                  : __fmul_rn(__fmul_rn(o.omb2, gg), gg);
      const float vi = __fmaf_rn(o.b2, v[j], addv);
      ms[j] = mi;
      vs[j] = vi;
      const float m_hat = __fmul_rn(mi, bc1);
      const float v_hat = __fmul_rn(vi, bc2);
      const float denom = __fadd_rn(__fsqrt_rn(v_hat), o.eps);
      if (vec_body) p[j] = __fmaf_rn(-lr, __fdiv_rn(m_hat, denom), p[j]);
      else p[j] = __fsub_rn(p[j], __fdiv_rn(__fmul_rn(lr, m_hat), denom));
    }
    stv<VEC>(slab + L.state0, L.odt, e, ms);
    stv<VEC>(slab + L.state1, L.odt, e, vs);
  }
  stv<VEC>(slab, L.pdt, e, p);
}

template <int VEC, bool kDyn = false>
__device__ __forceinline__ void apply_chunk(const Layout &L, uint8_t *slab, const OptSpec &o,
                                            uint32_t t, uint32_t e, const float (&gsum)[VEC]) {
  RowState<VEC> r;
  load_state<VEC>(L, slab, o, e, r);
  apply_loaded<VEC, kDyn>(L, slab, o, t, e, gsum, r);
}

// Adds the gradient rows spos[k0..k1) (in order) into acc, rounding to the
// gradient dtype after each add like TransientArena's simd_accumulate
// (memory_ops.hpp:37-70). Loads run eight rows ahead of the adds.
template <int VEC, int AHEAD = 8>
__device__ __forceinline__ void sum_rows(const void *pgrads, int gdt, uint32_t dim, const uint32_t *spos,
                                         uint32_t k0, uint32_t k1, uint32_t e, float (&acc)[VEC]) {
  uint32_t k = k0;
  for (; k + AHEAD <= k1; k += AHEAD) {
    float g[AHEAD][VEC];
#pragma unroll
    for (int u = 0; u < AHEAD; ++u) ldv<VEC>(pgrads, gdt, size_t(spos[k + u]) * dim + e, g[u]);
#pragma unroll
    for (int u = 0; u < AHEAD; ++u)
#pragma unroll
      for (int j = 0; j < VEC; ++j) acc[j] = round_to(gdt, __fadd_rn(acc[j], g[u][j]));
  }
  for (; k < k1; ++k) {
    float g0[VEC];
    ldv<VEC>(pgrads, gdt, size_t(spos[k]) * dim + e, g0);
#pragma unroll
    for (int j = 0; j < VEC; ++j) acc[j] = round_to(gdt, __fadd_rn(acc[j], g0[j]));
  }
}

// ---------------------------------------------------------------------------
// optimizer_step: grouping of the pending gradient rows by key without a
// sort. Per-row counters in HBM (zero between steps) give each key present
// this step a segment; rows are placed into their segment by atomics, and
// each segment's positions are put back in arrival order before it is
// reduced, so every key is summed in the reference's order (per key, arrival
// order, from +0.0) regardless of placement order.
// ---------------------------------------------------------------------------

struct GroupWs {
  uint32_t *rows;      // [P] row of each pending entry, kNoRow when its key is absent
  uint32_t *row_cnt;   // [capacity] entries of a row this step (all zero between steps)
  uint32_t *row_seg;   // [capacity] segment of a row this step
  uint32_t *seg_row;   // [P] row of each segment
  uint32_t *seg_cnt;   // [P] entries of each segment
  uint32_t *seg_off;   // [P] first slot of each segment in pos
  uint32_t *seg_fill;  // [P] placement counters (all zero between steps)
  uint32_t *pos;       // [P] entry positions grouped by segment
  uint4 *items;        // work items of k_group_hot: (segment, part, parts, first item)
  float *partials;     // [items][dim] partial sums of multi-part segments
  uint32_t *ctr;       // [0] segments, [1] slots allocated, [2] work items, [3] long segments
  uint32_t *long_list;  // [P] segments of short_max+1 .. long_max rows (listed by k_group_alloc)
  uint32_t short_max, long_max;  // row bounds of the apply kernel's short and long segments
  uint32_t cap;        // P: entries the [P] buffers hold (the host's pending count)
  uint32_t sorted;     // 1: pos was filled by a stable sort (each segment's slice in arrival order)
  uint32_t *status;    // table status word (kStatusPendingOverflow)
  // cleared by the last block of k_group_hot, the step's last kernel, for
  // the next window: ctr[0..3], the unresolved count, the pending count
  uint32_t *done, *unres_ctr, *pending;
};

// Pending entries of this step: the device count, bounded by the buffers.
__device__ __forceinline__ uint32_t step_count(const uint32_t *count_p, const GroupWs &w) {
  const uint32_t c = *count_p;
  return c <= w.cap ? c : w.cap;
}

// Phase 1 (the counting itself ran when the entries were appended): entries
// whose key was absent then are probed again; still absent, their gradients
// are dropped and counted (hogwild_embedding_store.hpp:1942-1952), else they
// are counted now.
__global__ void __launch_bounds__(256)
k_group_fix(Dir d, const unsigned long long *__restrict__ pkeys, const uint32_t *count_p, GroupWs w, CountWs c,
            unsigned long long *dropped) {
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  if (blockIdx.x == 0 && threadIdx.x == 0 && *count_p > w.cap) raise_status(w.status, kStatusPendingOverflow);
  const uint32_t nunres = min(*c.unres_ctr, w.cap);
  const uint32_t count = step_count(count_p, w);
  for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < nunres; j += gridDim.x * blockDim.x) {
    const uint32_t i = c.unres[j];
    if (i >= count) continue;
    const uint32_t row = dir_find<false>(d, pkeys[i]);
    if (row == kNoRow) {
      atomicAdd(dropped, 1ull);
      continue;
    }
    w.rows[i] = row;
    if (atomicAdd(&c.row_cnt[row], 1u) == 0u) {
      const uint32_t sid = atomicAdd(c.seg_ctr, 1u);
      c.seg_row[sid] = row;
      c.row_seg[row] = sid;
    }
  }
}

// Counting of host-input batches, which are only kept once their validation
// passed: entries [*base_p, *base_p + n) of the pending rows.
__global__ void __launch_bounds__(256)
k_count_range(const uint32_t *__restrict__ prows, const uint32_t *base_p, uint32_t n, uint32_t pcap, CountWs c) {
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  const uint32_t base = *base_p;
  if (uint64_t(base) + n > pcap) return;  // refused by k_accumulate (reported there)
  const uint32_t stride = gridDim.x * blockDim.x;
  const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
  for (uint32_t i0 = tid - (tid & 31u); i0 < n; i0 += stride) {
    const uint32_t i = i0 + (tid & 31u);
    const bool valid = i < n;
    count_entries(c, valid, valid ? prows[base + i] : kNoRow, base + i);
  }
}

constexpr int kBlockThreads = 1024;
constexpr uint32_t kSerialMax = 64;          // rows summed serially (bit-exact order)
constexpr uint32_t kPartEntries = 512;       // target rows per k_group_hot work item
constexpr uint32_t kHotWindowBits = 1u << 17;  // positions per bitmap window
constexpr uint32_t kRoundEntries = 2048;     // rows compacted per round

// Phase 2: a contiguous slot range per segment (block-aggregated allocation).
__global__ void __launch_bounds__(256) k_group_alloc(GroupWs w, const uint32_t *count_p) {
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  using Scan = cub::BlockScan<uint32_t, 256>;
  __shared__ typename Scan::TempStorage tmp;
  __shared__ uint32_t s_base;
  const uint32_t nseg = w.ctr[0];
  const uint32_t sid = blockIdx.x * blockDim.x + threadIdx.x;
  if (blockIdx.x * blockDim.x >= nseg) return;  // whole block past the end
  const uint32_t cnt = sid < nseg ? w.row_cnt[w.seg_row[sid]] : 0u;
  uint32_t excl, total;
  Scan(tmp).ExclusiveSum(cnt, excl, total);
  if (threadIdx.x == 0) s_base = atomicAdd(&w.ctr[1], total);
  __syncthreads();
  if (sid < nseg) {
    w.seg_off[sid] = s_base + excl;
    w.seg_cnt[sid] = cnt;
    if (cnt > w.short_max && cnt <= w.long_max) w.long_list[atomicAdd(&w.ctr[3], 1u)] = sid;
    if (cnt > w.long_max) {
      // work items of k_group_hot: windows of the batch's positions
      // parts: ranks of a sorted slice, or windows of the batch's positions
      const uint32_t count = step_count(count_p, w);
      const uint32_t by_rows = (cnt + kPartEntries - 1) / kPartEntries;
      const uint32_t nparts = w.sorted ? by_rows : max(by_rows, (count + kHotWindowBits - 1) / kHotWindowBits);
      const uint32_t base = atomicAdd(&w.ctr[2], nparts);
      for (uint32_t q = 0; q < nparts; ++q) w.items[base + q] = make_uint4(sid, q, nparts, base);
    }
  }
}

// Phase 3: every entry takes a slot of its segment (warp-aggregated).
__global__ void __launch_bounds__(256) k_group_place(const uint32_t *count_p, GroupWs w) {
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  const uint32_t count = step_count(count_p, w);
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t row = i < count ? w.rows[i] : kNoRow;
  const uint32_t sid = row != kNoRow ? w.row_seg[row] : 0xffffffffu;
  const unsigned peers = __match_any_sync(0xffffffffu, sid);
  const uint32_t rank = __popc(peers & ((1u << lane) - 1u));
  uint32_t base = 0;
  if (sid != 0xffffffffu && rank == 0) base = atomicAdd(&w.seg_fill[sid], uint32_t(__popc(peers)));
  base = __shfl_sync(0xffffffffu, base, __ffs(peers) - 1);
  if (sid != 0xffffffffu) w.pos[w.seg_off[sid] + base + rank] = i;
}

// Phase 3 for large windows (more pending rows than one hot-key bitmap
// window): the key of each entry is its segment's first slot, so a stable
// radix sort of (key, position) lays every segment's positions out in
// arrival order. Entries without a row sort past every segment.
__global__ void __launch_bounds__(256)
k_group_sortkeys(const uint32_t *count_p, GroupWs w, uint32_t *__restrict__ keys, uint32_t *__restrict__ vals,
                 uint32_t last_key) {
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  const uint32_t count = step_count(count_p, w);
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= w.cap) return;
  const uint32_t row = i < count ? w.rows[i] : kNoRow;
  keys[i] = row != kNoRow ? w.seg_off[w.row_seg[row]] : last_key;
  vals[i] = i;
}

__device__ __forceinline__ uint32_t next_step(const Layout &L, uint8_t *slab) {
  uint32_t *sp = reinterpret_cast<uint32_t *>(slab + L.step);
  const uint32_t t = *sp + 1u;
  *sp = t;
  return t;
}


// Sums a segment of at most kApplySlots * LANES rows in the reference's
// order and applies the optimizer, by one group of LANES lanes: the group
// ranks the positions (arrival order) into `ord` (shared memory), and loads
// the row's parameters and state before the sum so both latencies overlap.
constexpr int kApplySlots = 4;

template <int LANES, int VEC, int SLOTS, int AHEAD, bool kDyn>
__device__ __forceinline__ void group_segment(const Layout &L, uint8_t *slabs, const OptSpec &o, int gdt,
                                              const void *pgrads, const GroupWs &w, uint32_t s, uint32_t cnt,
                                              uint32_t off, uint32_t row, uint32_t lane, unsigned mask,
                                              uint32_t *ord) {
  uint8_t *slab = slabs + size_t(row) * L.stride;
  const uint32_t e0 = lane * VEC;
  RowState<VEC> rs;
  if (e0 < L.dim) load_state<VEC>(L, slab, o, e0, rs);
  const uint32_t nslots = (cnt + LANES - 1) / LANES;
  uint32_t p[SLOTS], rank[SLOTS];
#pragma unroll
  for (int j = 0; j < SLOTS; ++j) {
    const uint32_t idx = lane + uint32_t(j) * LANES;
    p[j] = idx < cnt ? w.pos[off + idx] : 0xffffffffu;
    rank[j] = 0;
  }
#pragma unroll
  for (int jj = 0; jj < SLOTS; ++jj) {
    if (uint32_t(jj) < nslots) {
      for (int q = 0; q < LANES; ++q) {
        const uint32_t v = __shfl_sync(mask, p[jj], q, LANES);
#pragma unroll
        for (int j = 0; j < SLOTS; ++j) rank[j] += v < p[j] ? 1u : 0u;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < SLOTS; ++j)
    if (lane + uint32_t(j) * LANES < cnt) ord[rank[j]] = p[j];
  __syncwarp(mask);
  uint32_t step = 0;
  if (o.kind == SE_OPT_ADAM) {
    if (lane == 0) step = next_step(L, slab);
    step = __shfl_sync(mask, step, 0, LANES);
  }
  for (uint32_t e = e0; e < L.dim; e += LANES * VEC) {
    float acc[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) acc[j] = 0.0f;
    sum_rows<VEC, AHEAD>(pgrads, gdt, L.dim, ord, 0, cnt, e, acc);
    if (e == e0) apply_loaded<VEC, kDyn>(L, slab, o, step, e, acc, rs);
    else apply_chunk<VEC, kDyn>(L, slab, o, step, e, acc);
  }
  __syncwarp(mask);
}

// Phase 4: one group per segment of at most kApplySlots * LANES rows (the
// bulk of the keys), summed serially in arrival order; larger segments
// become the block work items of k_group_hot. (Tried and slower: the long
// segments in a concurrent kernel of their own, and half the lanes per
// segment.)
template <int LANES, int VEC, bool kDyn>
__global__ void __launch_bounds__(256, 3)
k_group_apply(Layout L, uint8_t *__restrict__ slabs, OptSpec o, int gdt, const void *__restrict__ pgrads,
              GroupWs w, const uint32_t *count_p) {
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  constexpr int GPB = 256 / LANES;
  __shared__ uint32_t s_ord[GPB][kApplySlots * LANES];
  const size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t groups = size_t(gridDim.x) * blockDim.x / LANES;
  const uint32_t lane = uint32_t(t % LANES);
  const uint32_t gib = threadIdx.x / LANES;
  const unsigned mask = group_mask<LANES>();
  const uint32_t nseg = w.ctr[0];
  const bool poisoned = *o.poison != 0u;
  // The long segments (serial chains of up to long_max rows) get groups of
  // their own, so no group runs a long chain after its share of short ones.
  const uint32_t nlong = w.ctr[3];
  const size_t long_groups = min(size_t(nlong), groups / 4);
  const size_t g = t / LANES;
  if (g < long_groups) {
    for (size_t j = g; j < nlong; j += long_groups) {
      const uint32_t s = w.long_list[j];
      const uint32_t cnt = w.seg_cnt[s], off = w.seg_off[s], row = w.seg_row[s];
      if (!poisoned)
        group_segment<LANES, VEC, kApplySlots, 4, kDyn>(L, slabs, o, gdt, pgrads, w, s, cnt, off, row, lane, mask,
                                                  s_ord[gib]);
      if (lane == 0) {
        w.row_cnt[row] = 0u;
        w.seg_fill[s] = 0u;
      }
    }
  }
  // Every other group: the short segments.
  const size_t short_groups = groups - long_groups;
  for (size_t s = g - long_groups; g >= long_groups && s < nseg; s += short_groups) {
    const uint32_t cnt = w.seg_cnt[s], off = w.seg_off[s], row = w.seg_row[s];
    if (cnt > w.short_max) continue;  // a long segment or one of k_group_hot's
    if (cnt > 0 && !poisoned)
      group_segment<LANES, VEC, 1, 4, kDyn>(L, slabs, o, gdt, pgrads, w, uint32_t(s), cnt, off, row, lane, mask,
                                      s_ord[gib]);
    if (lane == 0) {
      w.row_cnt[row] = 0u;
      w.seg_fill[s] = 0u;
    }
  }
  // k_group_hot (launched first, running beside this kernel) has completed
  // once pdl_wait returns; then the last block clears the window's counters
  // (every block of both kernels has read them).
  pdl_wait();
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(w.done, 1u) == gridDim.x - 1) {
    w.ctr[0] = w.ctr[1] = w.ctr[2] = w.ctr[3] = 0u;
    *w.unres_ctr = 0u;
    *w.pending = 0u;
    *w.done = 0u;
  }
}

// Phase 5: segments of more than kApplySlots * LANES rows. Each segment is cut into parts
// by windows of batch positions; one 1024-thread block per part finds the
// segment's rows inside its window in arrival order (bitmap over the
// window), reduces them, and either applies the optimizer (one part) or
// leaves a partial sum for the last part to finish, which adds the partial
// sums in window order. A single-part segment of at most kSerialMax rows is
// summed serially (the reference's order); larger ones in runs of
// 1024/LANES groups whose sums are added by a fixed pairwise tree. Everything
// is fixed by the shapes, so results are deterministic.
template <int LANES, int VEC, bool kDyn>
__global__ void __launch_bounds__(kBlockThreads)
k_group_hot(Layout L, uint8_t *__restrict__ slabs, OptSpec o, int gdt, const void *__restrict__ pgrads,
            GroupWs w, const uint32_t *count_p) {
  pdl_wait();
  pdl_trigger();  // k_group_apply runs beside this kernel (disjoint segments)
  const uint32_t count = step_count(count_p, w);
  using Scan = cub::BlockScan<uint32_t, kBlockThreads>;
  constexpr int NG = kBlockThreads / LANES;
  constexpr uint32_t WPT = kHotWindowBits / 32 / kBlockThreads;  // bitmap words per thread
  __shared__ uint32_t bitmap[kHotWindowBits / 32];
  __shared__ typename Scan::TempStorage scan_tmp;
  __shared__ uint32_t s_pos[kRoundEntries];
  __shared__ float part[kBlockThreads / 32][LANES][VEC];  // one run sum per warp
  __shared__ uint32_t s_last, s_step;
  const uint32_t lane = threadIdx.x % LANES;
  const uint32_t grp = threadIdx.x / LANES;
  const uint32_t nitems = w.ctr[2];
  const bool poisoned = *o.poison != 0u;
  for (uint32_t x = blockIdx.x; x < nitems; x += gridDim.x) {
    const uint4 it = w.items[x];
    const uint32_t s = it.x, q = it.y, nparts = it.z, first = it.w;
    const uint32_t cnt = w.seg_cnt[s], off = w.seg_off[s], row = w.seg_row[s];
    uint32_t win = (count + nparts - 1) / nparts;
    win = (win + 31u) & ~31u;
    const uint32_t w0 = min(q * win, count), w1 = min(w0 + win, count);
    const uint32_t nwords = (w1 - w0 + 31u) / 32u;
    // Sorted: the part is ranks [lo, lo + total) of the segment's slice.
    const uint32_t per = (cnt + nparts - 1) / nparts;
    const uint32_t lo = min(q * per, cnt);
    uint32_t excl = 0, total = 0;
    if (w.sorted) {
      total = min(lo + per, cnt) - lo;
    } else {
      // The segment's rows inside [w0, w1), as a bitmap over the window.
      for (uint32_t j = 0; j < WPT; ++j) bitmap[threadIdx.x * WPT + j] = 0u;
      __syncthreads();
      for (uint32_t k = threadIdx.x; k < cnt; k += kBlockThreads) {
        const uint32_t p = w.pos[off + k];
        if (p >= w0 && p < w1) atomicOr(&bitmap[(p - w0) >> 5], 1u << ((p - w0) & 31u));
      }
      __syncthreads();
      uint32_t bits = 0;
      for (uint32_t j = 0; j < WPT; ++j) {
        const uint32_t wi = threadIdx.x * WPT + j;
        bits += wi < nwords ? __popc(bitmap[wi]) : 0u;
      }
      Scan(scan_tmp).ExclusiveSum(bits, excl, total);
    }
    // Compacts the part's rows of rank [r0, r0 + kRoundEntries) into s_pos.
    auto compact = [&](uint32_t r0) {
      if (w.sorted) {
        const uint32_t m = min(total - r0, kRoundEntries);
        for (uint32_t k = threadIdx.x; k < m; k += kBlockThreads) s_pos[k] = w.pos[off + lo + r0 + k];
        return;
      }
      uint32_t rank = excl;
      for (uint32_t j = 0; j < WPT; ++j) {
        const uint32_t wi = threadIdx.x * WPT + j;
        uint32_t word = wi < nwords ? bitmap[wi] : 0u;
        while (word) {
          const uint32_t b = __ffs(word) - 1;
          word &= word - 1;
          if (rank >= r0 && rank - r0 < kRoundEntries) s_pos[rank - r0] = w0 + wi * 32u + b;
          ++rank;
        }
      }
    };
    const bool one_round = total <= kRoundEntries;
    const bool serial = nparts == 1 && cnt <= kSerialMax;
    uint8_t *slab = slabs + size_t(row) * L.stride;
    if (one_round) compact(0);
    if (threadIdx.x == 0) s_step = (nparts == 1 && !poisoned && o.kind == SE_OPT_ADAM) ? next_step(L, slab) : 0u;
    __syncthreads();
    for (uint32_t base = 0; base < L.dim; base += LANES * VEC) {
      const uint32_t e = base + lane * VEC;
      float acc[VEC];  // running sum of the window (group 0)
#pragma unroll
      for (int j = 0; j < VEC; ++j) acc[j] = 0.0f;
      for (uint32_t r0 = 0; r0 < total; r0 += kRoundEntries) {
        if (!one_round) {
          __syncthreads();
          compact(r0);
          __syncthreads();
        }
        const uint32_t n = min(total - r0, kRoundEntries);
        if (serial) {
          if (grp == 0 && e < L.dim) sum_rows<VEC, 4>(pgrads, gdt, L.dim, s_pos, 0, n, e, acc);
        } else {
          const uint32_t per = (n + NG - 1) / NG;
          const uint32_t k0 = min(grp * per, n), k1 = min(k0 + per, n);
          float a[VEC];
#pragma unroll
          for (int j = 0; j < VEC; ++j) a[j] = 0.0f;
          if (e < L.dim) sum_rows<VEC, 4>(pgrads, gdt, L.dim, s_pos, k0, k1, e, a);
          // Fixed reduction order over the runs: a butterfly across the
          // groups of a warp (shuffles), then the warps' sums added in warp
          // order by group 0 - two block barriers instead of one per level.
#pragma unroll
          for (int off = LANES; off < 32; off <<= 1)
#pragma unroll
            for (int j = 0; j < VEC; ++j) a[j] = round_to(gdt, __fadd_rn(a[j], __shfl_xor_sync(0xffffffffu, a[j], off)));
          const uint32_t warp = threadIdx.x >> 5;
          if ((threadIdx.x & 31u) < uint32_t(LANES))
#pragma unroll
            for (int j = 0; j < VEC; ++j) part[warp][lane][j] = a[j];
          __syncthreads();
          if (grp == 0)
            for (uint32_t wi = 0; wi < kBlockThreads / 32; ++wi)
#pragma unroll
              for (int j = 0; j < VEC; ++j) acc[j] = round_to(gdt, __fadd_rn(acc[j], part[wi][lane][j]));
          __syncthreads();
        }
      }
      if (grp == 0 && e < L.dim) {
        if (nparts == 1) {
          if (!poisoned) apply_chunk<VEC, kDyn>(L, slab, o, s_step, e, acc);
        } else {
          float *dst = w.partials + size_t(first + q) * L.dim;
#pragma unroll
          for (int j = 0; j < VEC; ++j) dst[e + j] = acc[j];
        }
      }
    }
    if (nparts > 1) {
      // The last part to finish adds the parts' sums in window order.
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) {
        // atomic placement left the counter at cnt, sorted placement at 0
        const uint32_t old = atomicAdd(&w.seg_fill[s], 1u);
        s_last = old == (w.sorted ? 0u : cnt) + nparts - 1 ? 1u : 0u;
        s_step = (s_last && !poisoned && o.kind == SE_OPT_ADAM) ? next_step(L, slab) : 0u;
      }
      __syncthreads();
      if (s_last && grp == 0 && !poisoned) {
        __threadfence();
        for (uint32_t e = lane * VEC; e < L.dim; e += LANES * VEC) {
          float tot[VEC];
#pragma unroll
          for (int j = 0; j < VEC; ++j) tot[j] = 0.0f;
          for (uint32_t g = 0; g < nparts; ++g) {
            const float *src = w.partials + size_t(first + g) * L.dim + e;
#pragma unroll
            for (int j = 0; j < VEC; ++j) tot[j] = round_to(gdt, __fadd_rn(tot[j], __ldcg(src + j)));
          }
          apply_chunk<VEC, kDyn>(L, slab, o, s_step, e, tot);
        }
      }
    }
    if (threadIdx.x == 0 && (nparts == 1 || s_last)) {
      w.row_cnt[row] = 0u;
      w.seg_fill[s] = 0u;
    }
    __syncthreads();
  }
}

// optimizer_step in atomic mode (the sums of se_accum.cuh): one group of
// LANES lanes per claimed slot. The slot's key is resolved in the directory
// now, as SlotStore::update_batch re-resolves keys at step time
// (hogwild_embedding_store.hpp:2735-2901); an absent key drops its rows and
// counts them (1942-1952). The sum is scaled to ParamT and applied like the
// ordered mode's reduced gradient (apply_chunk). Every slot is then freed
// for the next window: sum zeroed, count and key cleared; the last block
// resets the claim counters.
// OPT: the optimizer kind, fixed at compile time so the registers of the
// loads in flight are those of one optimizer's state.
template <int LANES, int VEC, bool kDyn, int OPT>
__global__ void __launch_bounds__(256, 3)  // 3 blocks per SM: ~29K slots of 4 lanes in one wave
k_acc_apply(AccTab a, Dir d, Layout L, uint8_t *__restrict__ slabs, OptSpec o_in, int apply,
            unsigned long long *dropped) {
  OptSpec o = o_in;
  o.kind = OPT;
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  const uint32_t G = a.mask + 1u;
  const size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t groups = size_t(gridDim.x) * blockDim.x / LANES;
  const uint32_t lane = uint32_t(t % LANES);
  const unsigned mask = group_mask<LANES>();
  // the group's first list entry is loaded with the entry count (one round
  // trip; the list holds G + 1 entries, so the load stays inside it), each
  // next one at the end of the iteration before it
  size_t g = t / LANES;
  uint4 ent = g <= size_t(G) ? __ldcg(a.list + g) : make_uint4(kNoRow, kNoRow, 0u, kNoRow);
  const uint32_t nslots = min(__ldcg(a.ctr), G + 1u);
  const bool run = apply && *o.poison == 0u;
  const uint32_t epoch = __ldcg(a.epoch);
  while (g < nslots) {
    const uint32_t slot = ent.x;
    if (slot != kNoRow) {  // else a hole left by a key another block claimed
      float *acc = a.vals + size_t(ent.w) * L.dim;  // the slot's dense sum row
      // the row the accumulate listed (from lookup_or_insert) while no erase
      // happened since; else the key is resolved in the directory now
      uint32_t row = ent.z == epoch ? ent.y : kNoRow;
      if (lane == 0 && apply && row == kNoRow) row = dir_find<false>(d, uint64_t(__ldcg(&a.slots[slot].x)));
      row = __shfl_sync(mask, row, 0, LANES);
      if (apply && row == kNoRow) {
        if (lane == 0) atomicAdd(dropped, (unsigned long long)__ldcg(a.cnt + slot));
      } else if (run) {
        uint8_t *slab = slabs + size_t(row) * L.stride;
        uint32_t step = 0;
        if (o.kind == SE_OPT_ADAM) {
          if (lane == 0) step = next_step(L, slab);
          step = __shfl_sync(mask, step, 0, LANES);
        }
        // kChunks chunks per lane and pass: every load of the pass (sum,
        // parameters, state) is in flight before the first update
        constexpr int kChunks = 4;
        for (uint32_t e0 = lane * VEC; e0 < L.dim; e0 += LANES * VEC * kChunks) {
          float gs[kChunks][VEC];
          RowState<VEC> rs[kChunks];
  #pragma unroll
          for (int k = 0; k < kChunks; ++k) {
            const uint32_t e = e0 + uint32_t(k) * LANES * VEC;
            if (e >= L.dim) continue;
            if constexpr (VEC == 4) {
              const float4 v = __ldcg(reinterpret_cast<const float4 *>(acc + e));
              gs[k][0] = v.x; gs[k][1] = v.y; gs[k][2] = v.z; gs[k][3] = v.w;
            } else {
              gs[k][0] = __ldcg(acc + e);
            }
            load_state<VEC>(L, slab, o, e, rs[k]);
          }
          // the sum is fp32; the ordered mode's is rounded to the gradient
          // dtype after every add
  #pragma unroll
          for (int k = 0; k < kChunks; ++k) {
            const uint32_t e = e0 + uint32_t(k) * LANES * VEC;
            if (e < L.dim) apply_loaded<VEC, kDyn>(L, slab, o, step, e, gs[k], rs[k]);
          }
        }
      }
      for (uint32_t e = lane * VEC; e < L.dim; e += LANES * VEC) {
        if constexpr (VEC == 4) *reinterpret_cast<float4 *>(acc + e) = make_float4(0.f, 0.f, 0.f, 0.f);
        else acc[e] = 0.0f;
      }
      if (lane == 0) {
        a.cnt[slot] = 0u;
        a.slots[slot] = make_ulonglong2(kEmptyKey, kAccFree);
      }
    }
    g += groups;
    if (g < nslots) ent = __ldcg(a.list + g);
  }
  // every block has read the claim counter: the last one resets the counters
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(a.ctr + 2, 1u) == gridDim.x - 1) {
    a.ctr[0] = 0u;
    a.ctr[2] = 0u;
    a.ctr[3] = 0u;
  }
}

// Rebuild into a larger directory.
__global__ void k_rehash(const Bucket *__restrict__ old_b, uint64_t old_n, Dir nd, uint32_t *status) {
  const uint64_t slot = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (slot >= old_n * kBucketSlots) return;
  const Bucket &b = old_b[slot / kBucketSlots];
  const int s = int(slot % kBucketSlots);
  const uint64_t key = b.keys[s];
  if (key == kEmptyKey || b.rows[s] == kDeadRow) return;  // erased keys are dropped here
  if (!dir_insert_unique(nd, key, b.rows[s])) raise_status(status, kStatusTableFull);
}

// ---------------------------------------------------------------------------
// Mutation API: contains, assign, erase (hogwild_embedding_store.hpp:4838-5106)
// ---------------------------------------------------------------------------

// contains (hogwild_embedding_store.hpp:4983-5009): a key is present when any
// table holds it; one launch per table, the first one overwrites `out`.
__global__ void __launch_bounds__(256)
k_contains(Dir d, const void *__restrict__ keys, int kdt, size_t n, uint8_t *__restrict__ out, int first) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const bool found = dir_find<false>(d, load_key(keys, kdt, i)) != kNoRow;
  out[i] = uint8_t(found || (!first && out[i] != 0));
}

// Optimizer state of a row that is created with given parameters.
template <int LANES, int VEC>
__device__ __forceinline__ void init_state(const Layout &L, uint8_t *slab, const InitSpec &init, uint32_t lane) {
  for (uint32_t e = lane * VEC; e < L.dim; e += LANES * VEC) {
    if (L.nstate >= 1) {
      float s[VEC];
#pragma unroll
      for (int j = 0; j < VEC; ++j) s[j] = init.state0;
      stv<VEC>(slab + L.state0, L.odt, e, s);
    }
    if (L.nstate >= 2) {
      float s[VEC];
#pragma unroll
      for (int j = 0; j < VEC; ++j) s[j] = 0.0f;
      stv<VEC>(slab + L.state1, L.odt, e, s);
    }
  }
  if (L.nstate >= 2 && lane == 0) *reinterpret_cast<uint32_t *>(slab + L.step) = 0u;
  if (L.score != 0u && lane == 0) *reinterpret_cast<unsigned long long *>(slab + L.score) = 0ull;
}

// validate_unique_mutation_batch (hogwild_embedding_store.hpp:5278-5305) on
// the device: the batch's keys go into a scratch open-addressing set of at
// least twice as many slots (all-ones = empty); a key that finds itself
// there already marks the batch. words[0] counts the all-ones key itself,
// words[1] is the mark.
__global__ void __launch_bounds__(256)
k_assign_dups(const void *__restrict__ keys, int kdt, size_t n, unsigned long long *__restrict__ set,
              uint64_t nslots, uint32_t *words) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint64_t key = load_key(keys, kdt, i);
  if (key == kEmptyKey) {
    if (atomicAdd(words, 1u) > 0u) words[1] = 1u;
    return;
  }
  const uint64_t mask = nslots - 1;
  uint64_t pos = splitmix64(key) & mask;
  for (uint64_t probe = 0; probe < nslots; ++probe) {
    const unsigned long long old = atomicCAS(&set[pos], kEmptyKey, key);
    if (old == kEmptyKey) return;
    if (old == key) {
      words[1] = 1u;
      return;
    }
    pos = (pos + 1) & mask;
  }
}

// assign (hogwild_embedding_store.hpp:4838-4923): a present key's parameters
// are overwritten and its optimizer state kept; an absent (or erased) key is
// inserted with the given parameters and fresh optimizer state. A batch that
// k_assign_dups marked (a key repeated) changes nothing.
template <int LANES, int VEC>
__global__ void __launch_bounds__(256)
k_assign(Dir d, Layout L, uint8_t *__restrict__ slabs, RowAlloc ra, InitSpec init, const void *__restrict__ keys,
         int kdt, size_t n, const void *__restrict__ values, const uint32_t *dup_mark, uint32_t *status) {
  const size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t i = t / LANES;
  const uint32_t lane = uint32_t(t % LANES);
  if (i >= n || *dup_mark != 0u) return;
  const unsigned mask = group_mask<LANES>();
  int kind = kFound;
  uint32_t row = kNoRow;
  uint32_t *word = nullptr;
  if (lane == 0) {
    const InsertResult r = dir_find_or_insert(d, load_key(keys, kdt, i));
    kind = r.kind;
    word = r.row_word;
    // unpublished (3) only after an insert that found the arena full
    if (kind == kFound) kind = resolve_found(word, &row);
    if (kind != kFound && kind != kInserted) kind = kFull;
  }
  const uint32_t taken = take_rows_warp(ra, live_lanes(t, n * LANES), lane == 0 && kind == kInserted);
  if (lane == 0) {
    if (kind == kInserted) row = taken;
    if (kind == kFull || row >= ra.capacity) {
      raise_status(status, kStatusTableFull);
      kind = kFull;
    }
  }
  kind = __shfl_sync(mask, kind, 0, LANES);
  row = __shfl_sync(mask, row, 0, LANES);
  if (kind == kFull) return;
  uint8_t *slab = slabs + size_t(row) * L.stride;
  const void *src = static_cast<const uint8_t *>(values) + i * size_t(L.dim) * (L.pdt == SE_FLOAT32 ? 4 : 2);
  copy_row<VEC>(slab, src, L.pdt, L.dim, lane * VEC, LANES * VEC);
  if (kind == kInserted) {
    init_state<LANES, VEC>(L, slab, init, lane);
    __threadfence();  // the slab is written device-wide ...
    __syncwarp(mask);
    if (lane == 0) atomicExch(word, row);  // ... before its row is published
  }
}

// Rows popped past the bottom of the free stack leave it below zero.
// Before an erase: clamps the free-stack top and bumps the table's erase
// epoch (rows listed by the atomic accumulate before it are probed again).
__global__ void k_free_clamp(int *free_top, uint32_t *erase_epoch) {
  if (*free_top < 0) *free_top = 0;
  ++*erase_epoch;
}

// erase / erase_dimension (hogwild_embedding_store.hpp:5011-5106): the key's
// slot becomes a tombstone (the all-ones key's side slot returns to "never
// inserted") and its row goes on the free stack, to be taken by a later
// insert. Absent keys and repeats are no-ops.
__global__ void __launch_bounds__(256)
k_erase(Dir d, const void *__restrict__ keys, int kdt, size_t n, int *free_top, uint32_t *free_rows,
        uint64_t capacity) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint64_t key = load_key(keys, kdt, i);
  uint32_t *word = dir_slot(d, key);
  if (word == nullptr) return;
  const bool side = key == kEmptyKey;
  const uint32_t old = atomicExch(word, side ? kNoRow : kDeadRow);
  if (side) atomicExch(d.special, 0u);
  if (old < kDeadRow && old < capacity) {
    const int j = atomicAdd(free_top, 1);
    if (uint64_t(j) < capacity) free_rows[j] = old;
  }
}

// After an erase, pending gradients are counted again from their keys'
// current rows: optimizer_step resolves keys when it runs
// (hogwild_embedding_store.hpp:2745-2750), so gradients of an erased key are
// dropped at the step, or applied to its new row if the key is inserted again
// before it. First the old counts are cleared ...
__global__ void __launch_bounds__(256)
k_requeue_clear(const uint32_t *__restrict__ prows, const uint32_t *count_p, uint32_t cap, uint64_t rows_cap,
                CountWs c) {
  const uint32_t count = min(*count_p, cap);
  const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
  if (tid == 0) {
    *c.seg_ctr = 0u;
    *c.unres_ctr = 0u;
  }
  for (uint32_t i = tid; i < count; i += gridDim.x * blockDim.x) {
    const uint32_t r = prows[i];
    if (r < rows_cap) c.row_cnt[r] = 0u;
  }
}

// ... then every entry is probed and counted again (keys absent now are
// listed for the step's probe, k_group_fix).
__global__ void __launch_bounds__(256)
k_requeue_count(Dir d, const unsigned long long *__restrict__ pkeys, uint32_t *__restrict__ prows,
                const uint32_t *count_p, uint32_t cap, CountWs c) {
  const uint32_t count = min(*count_p, cap);
  const uint32_t stride = gridDim.x * blockDim.x;
  const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
  for (uint32_t i0 = tid - (tid & 31u); i0 < count; i0 += stride) {
    const uint32_t i = i0 + (tid & 31u);
    const bool valid = i < count;
    const uint32_t row = valid ? dir_find<true>(d, pkeys[i]) : kNoRow;
    if (valid) prows[i] = row;
    count_entries(c, valid, row, i);
  }
}

// ---------------------------------------------------------------------------
// Scores (ScorePolicyRuntime::on_access, eviction/score_policy.hpp:40-100, as
// forward_lookup applies it to every key it finds, hogwild_embedding_store.hpp:4479-4490)
// ---------------------------------------------------------------------------

// LFU: one more access for every position whose key is present.
__global__ void __launch_bounds__(256)
k_touch_lfu(Dir d, Layout L, uint8_t *__restrict__ slabs, const void *__restrict__ keys, int kdt, size_t n) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t row = dir_find<false>(d, load_key(keys, kdt, i));
  if (row != kNoRow) atomicAdd(reinterpret_cast<unsigned long long *>(slabs + size_t(row) * L.stride + L.score), 1ull);
}

// LRU, first pass: rows and hit flags of the batch's positions.
__global__ void __launch_bounds__(256)
k_touch_find(Dir d, const void *__restrict__ keys, int kdt, size_t n, uint32_t *__restrict__ rows,
             uint32_t *__restrict__ hits) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t row = dir_find<false>(d, load_key(keys, kdt, i));
  rows[i] = row;
  hits[i] = row != kNoRow ? 1u : 0u;
}

// LRU, second pass: the h-th hit of the batch (in position order) takes the
// clock's value + h, and the row keeps the latest stamp; the clock advances
// by the batch's hits, as one access at a time would advance it.
__global__ void __launch_bounds__(256)
k_touch_lru(Layout L, uint8_t *__restrict__ slabs, const uint32_t *__restrict__ rows, const uint32_t *__restrict__ hits,
            const uint32_t *__restrict__ rank, size_t n, unsigned long long *clock) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const unsigned long long now = *clock;
  if (hits[i])
    atomicMax(reinterpret_cast<unsigned long long *>(slabs + size_t(rows[i]) * L.stride + L.score), now + rank[i]);
  // the advanced clock goes to clock[1] (other blocks may still read
  // clock[0]); the host moves it into clock[0] after the launch
  if (i == n - 1) clock[1] = now + rank[i] + hits[i];
}

// assign_scores: the first table holding a key takes its score (`done` marks
// keys already placed by an earlier table).
__global__ void __launch_bounds__(256)
k_assign_scores(Dir d, Layout L, uint8_t *__restrict__ slabs, const void *__restrict__ keys, int kdt, size_t n,
                const unsigned long long *__restrict__ scores, uint8_t *__restrict__ done) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n || done[i]) return;
  const uint32_t row = dir_find<false>(d, load_key(keys, kdt, i));
  if (row == kNoRow) return;
  *reinterpret_cast<unsigned long long *>(slabs + size_t(row) * L.stride + L.score) = scores[i];
  done[i] = 1;
}

__global__ void __launch_bounds__(256)
k_read_scores(Dir d, Layout L, const uint8_t *__restrict__ slabs, const void *__restrict__ keys, int kdt, size_t n,
              unsigned long long *__restrict__ out, uint8_t *__restrict__ done) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n || done[i]) return;
  const uint32_t row = dir_find<false>(d, load_key(keys, kdt, i));
  if (row == kNoRow) return;
  out[i] = *reinterpret_cast<const unsigned long long *>(slabs + size_t(row) * L.stride + L.score);
  done[i] = 1;
}

// ---------------------------------------------------------------------------
// Checkpoint interop: export of a table's present keys with their rows and
// optimizer state (export_batch / export_opt_state_batch,
// hogwild_embedding_store.hpp:6112-6300), assign_opt_states (6278-6351)
// ---------------------------------------------------------------------------

// 1 for each directory slot holding a present key (slot index nslots: the
// all-ones key's side slot).
__global__ void __launch_bounds__(256)
k_export_flag(Dir d, uint64_t nslots, uint32_t *__restrict__ flags) {
  const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i > nslots) return;
  uint32_t row;
  if (i == nslots) {
    row = d.special[1];
  } else {
    const Bucket &b = d.buckets[i / kBucketSlots];
    row = b.keys[i % kBucketSlots] == kEmptyKey ? kNoRow : b.rows[i % kBucketSlots];
  }
  flags[i] = row < kDeadRow ? 1u : 0u;
}

__global__ void __launch_bounds__(256)
k_export_list(Dir d, uint64_t nslots, const uint32_t *__restrict__ flags, const uint32_t *__restrict__ at,
              unsigned long long *__restrict__ keys, uint32_t *__restrict__ rows) {
  const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i > nslots || !flags[i]) return;
  const uint32_t j = at[i];
  if (i == nslots) {
    keys[j] = kEmptyKey;
    rows[j] = d.special[1];
  } else {
    const Bucket &b = d.buckets[i / kBucketSlots];
    keys[j] = b.keys[i % kBucketSlots];
    rows[j] = b.rows[i % kBucketSlots];
  }
}

// Entries [offset, offset + count) of a snapshot: key (narrowed to the key
// dtype), parameter row, optimizer state rows (state0 then state1), step.
template <int LANES>
__global__ void __launch_bounds__(256)
k_export_gather(Layout L, const uint8_t *__restrict__ slabs, const unsigned long long *__restrict__ keys,
                const uint32_t *__restrict__ rows, uint64_t offset, uint64_t count, int kdt, void *keys_out,
                uint8_t *__restrict__ values_out, uint8_t *__restrict__ states_out, uint32_t *__restrict__ steps_out) {
  const uint64_t t = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint64_t j = t / LANES;
  const uint32_t lane = uint32_t(t % LANES);
  if (j >= count) return;
  const uint64_t key = keys[offset + j];
  const uint8_t *slab = slabs + size_t(rows[offset + j]) * L.stride;
  const uint32_t pb = L.pdt == SE_FLOAT32 ? 4 : 2, ob = L.odt == SE_FLOAT32 ? 4 : 2;
  if (lane == 0 && keys_out) {
    if (kdt <= SE_KEY_UINT32) static_cast<uint32_t *>(keys_out)[j] = uint32_t(key);
    else static_cast<unsigned long long *>(keys_out)[j] = key;
  }
  if (values_out)
    for (uint32_t b = lane; b < L.dim * pb; b += LANES) values_out[j * L.dim * pb + b] = slab[b];
  if (states_out && L.nstate > 0) {
    const uint32_t sb = L.dim * ob;
    for (uint32_t b = lane; b < sb; b += LANES) {
      states_out[j * L.nstate * sb + b] = slab[L.state0 + b];
      if (L.nstate >= 2) states_out[j * L.nstate * sb + sb + b] = slab[L.state1 + b];
    }
  }
  if (lane == 0 && steps_out) steps_out[j] = L.nstate >= 2 ? *reinterpret_cast<const uint32_t *>(slab + L.step) : 0u;
}

// assign_opt_states: first every key must be present (mark[0] counts the
// absent ones); the write pass runs only when none is.
__global__ void __launch_bounds__(256)
k_opt_find(Dir d, const void *__restrict__ keys, int kdt, size_t n, uint32_t *__restrict__ rows, uint32_t *mark) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t row = dir_find<false>(d, load_key(keys, kdt, i));
  rows[i] = row;
  if (row == kNoRow) atomicAdd(mark, 1u);
}

template <int LANES>
__global__ void __launch_bounds__(256)
k_opt_assign(Layout L, uint8_t *__restrict__ slabs, const uint32_t *__restrict__ rows, size_t n,
             const uint8_t *__restrict__ states, const uint32_t *__restrict__ steps, const uint32_t *mark) {
  const size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t i = t / LANES;
  const uint32_t lane = uint32_t(t % LANES);
  if (i >= n || *mark != 0u) return;
  uint8_t *slab = slabs + size_t(rows[i]) * L.stride;
  const uint32_t sb = L.dim * (L.odt == SE_FLOAT32 ? 4 : 2);
  for (uint32_t b = lane; b < sb; b += LANES) {
    slab[L.state0 + b] = states[i * L.nstate * sb + b];
    if (L.nstate >= 2) slab[L.state1 + b] = states[i * L.nstate * sb + sb + b];
  }
  if (lane == 0 && steps && L.nstate >= 2) *reinterpret_cast<uint32_t *>(slab + L.step) = steps[i];
}

// ---------------------------------------------------------------------------
// Embedding bag: sum-pooled gather of multi-hot bags and its backward
// ---------------------------------------------------------------------------

// Rows of a bag batch's keys, inserting absent ones with lookup_or_insert's
// claim and initialisation (hogwild_embedding_store.hpp:4925-4980), written
// as row numbers for the pooling kernel; keys claimed by another group of
// the same launch are finished by k_bag_deferred.
template <int LANES, int VEC>
__global__ void __launch_bounds__(256)
k_bag_insert(Dir d, Layout L, uint8_t *__restrict__ slabs, RowAlloc ra, InitSpec init, const void *__restrict__ keys,
             int kdt, size_t n, uint32_t *__restrict__ rows_out, uint32_t *def_count, uint32_t *def_pos,
             unsigned long long *def_word, uint32_t *status) {
  const size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t i = t / LANES;
  const uint32_t lane = uint32_t(t % LANES);
  if (i >= n) return;
  const unsigned mask = group_mask<LANES>();
  const uint64_t key = load_key(keys, kdt, i);
  int kind = kFound;
  uint32_t row = kNoRow;
  uint32_t *word = nullptr;
  if (lane == 0) {
    const InsertResult r = dir_find_or_insert(d, key);
    kind = r.kind;
    word = r.row_word;
    if (kind == kFound) kind = resolve_found(word, &row, r.seen);
    else if (kind == kFull) raise_status(status, kStatusTableFull);
  }
  const uint32_t taken = take_rows_warp(ra, live_lanes(t, n * LANES), lane == 0 && kind == kInserted);
  if (lane == 0 && kind == kInserted) {
    row = taken;
    if (row >= ra.capacity) {
      raise_status(status, kStatusTableFull);
      kind = kFull;
    }
  }
  kind = __shfl_sync(mask, kind, 0, LANES);
  row = __shfl_sync(mask, row, 0, LANES);
  if (kind == kInserted) {
    uint8_t *slab = slabs + size_t(row) * L.stride;
    init_slab<LANES, VEC>(L, slab, init, key, lane, slab);  // no copy out: the parameters go to the slab only
    __threadfence();
    __syncwarp(mask);
    if (lane == 0) atomicExch(word, row);
  }
  if (lane == 0) {
    if (kind == 3) {
      const uint32_t j = atomicAdd(def_count, 1u);
      def_pos[j] = uint32_t(i);
      def_word[j] = reinterpret_cast<unsigned long long>(word);
    } else {
      rows_out[i] = (kind == kFound || kind == kInserted) ? row : kNoRow;
    }
  }
}

__global__ void __launch_bounds__(256)
k_bag_deferred(const uint32_t *def_count, const uint32_t *def_pos, const unsigned long long *def_word,
               uint32_t *__restrict__ rows_out, uint32_t *status) {
  const uint32_t count = *def_count;
  for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < count; j += gridDim.x * blockDim.x) {
    const uint32_t row = __ldcg(reinterpret_cast<const uint32_t *>(def_word[j]));
    if (row == kNoRow) raise_status(status, kStatusTableFull);
    rows_out[def_pos[j]] = row;
  }
}

__global__ void __launch_bounds__(256)
k_bag_find(Dir d, const void *__restrict__ keys, int kdt, size_t n, uint32_t *__restrict__ rows_out) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) rows_out[i] = dir_find<false>(d, load_key(keys, kdt, i));
}

// Bag of every key position: bag b covers [offsets[b], offsets[b+1]) clamped
// to [0, n] (positions outside every bag keep bag 0, so any offsets index in
// bounds). One warp per bag.
__global__ void __launch_bounds__(256)
k_bag_of(const int64_t *__restrict__ offsets, size_t nbags, size_t n, uint32_t *__restrict__ bag_of) {
  const size_t warps = size_t(gridDim.x) * blockDim.x / 32;
  const uint32_t lane = threadIdx.x & 31u;
  for (size_t b = (size_t(blockIdx.x) * blockDim.x + threadIdx.x) / 32; b < nbags; b += warps) {
    const int64_t lo = min(max(offsets[b], int64_t(0)), int64_t(n));
    const int64_t hi = min(max(offsets[b + 1], lo), int64_t(n));
    for (int64_t j = lo + lane; j < hi; j += 32) bag_of[j] = uint32_t(b);
  }
}

// out[b] = sum of the parameter rows of keys [offsets[b], offsets[b+1]) in
// key order: fp32 adds from +0.0 (an absent key adds a zero row), rounded
// once to the value dtype. Offsets are clamped to [0, n]. A group of LANES
// lanes per bag; each lane keeps four rows' loads in flight.
template <int LANES, int VEC>
__global__ void __launch_bounds__(256)
k_bag_pool(Layout L, const uint8_t *__restrict__ slabs, const uint32_t *__restrict__ rows, size_t n,
           const int64_t *__restrict__ offsets, size_t nbags, void *__restrict__ out) {
  const size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t groups = size_t(gridDim.x) * blockDim.x / LANES;
  const uint32_t lane = uint32_t(t % LANES);
  const size_t pb = L.pdt == SE_FLOAT32 ? 4 : 2;
  for (size_t b = t / LANES; b < nbags; b += groups) {
    const int64_t lo = min(max(offsets[b], int64_t(0)), int64_t(n));
    const int64_t hi = min(max(offsets[b + 1], lo), int64_t(n));
    void *orow = static_cast<uint8_t *>(out) + b * size_t(L.dim) * pb;
    for (uint32_t e = lane * VEC; e < L.dim; e += LANES * VEC) {
      float acc[VEC];
#pragma unroll
      for (int x = 0; x < VEC; ++x) acc[x] = 0.0f;
      int64_t j = lo;
      for (; j + 4 <= hi; j += 4) {
        float v[4][VEC];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t r = __ldg(rows + j + q);
          if (r != kNoRow) {
            ldv<VEC>(slabs + size_t(r) * L.stride, L.pdt, e, v[q]);
          } else {
#pragma unroll
            for (int x = 0; x < VEC; ++x) v[q][x] = 0.0f;
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int x = 0; x < VEC; ++x) acc[x] = __fadd_rn(acc[x], v[q][x]);
      }
      for (; j < hi; ++j) {
        const uint32_t r = __ldg(rows + j);
        float v[VEC];
        if (r != kNoRow) {
          ldv<VEC>(slabs + size_t(r) * L.stride, L.pdt, e, v);
        } else {
#pragma unroll
          for (int x = 0; x < VEC; ++x) v[x] = 0.0f;
        }
#pragma unroll
        for (int x = 0; x < VEC; ++x) acc[x] = __fadd_rn(acc[x], v[x]);
      }
      stv<VEC>(orow, L.pdt, e, acc);
    }
  }
}

// Reads the rows of a few keys (state inspection for tests).
__global__ void k_find_rows(Dir d, const unsigned long long *keys, uint32_t n, uint32_t *rows) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) rows[i] = dir_find<true>(d, keys[i]);
}

}  // namespace se_gpu

#include "se_exchange.cuh"

namespace se_gpu {

// ===========================================================================
// Host side
// ===========================================================================

namespace {

thread_local std::string t_last_error;
std::atomic<uint64_t> g_launches{0};

constexpr uint64_t kDefaultCapacity = 1u << 16;
constexpr double kMaxLoadPerBucket = 3.5;  // 70 % of 5 slots

uint64_t next_pow2(uint64_t x) {
  uint64_t p = 1;
  while (p < x) p <<= 1;
  return p;
}

// Lanes per key of the gathers: as few as keep each lane's share of the row
// at <= 8 units, so a warp probes 8 keys at once and each lane keeps its
// loads of the row in flight together.
// Threads per block of a one-thread-per-work-item kernel of up to 256-thread
// blocks: fewer (a multiple of 32, at least 64) when the work fills about
// one wave, so that every SM holds the same number of blocks (4 on each of
// the 148 SMs) instead of 3 on some and 4 on others.
unsigned balanced_block(size_t threads) {
  const size_t per = (threads + 148 * 4 - 1) / (148 * 4);
  const size_t bt = (per + 31) / 32 * 32;
  return unsigned(std::min<size_t>(256, std::max<size_t>(64, bt)));
}

// The TMA path of forward_lookup: rows of 512..1,024 bytes in 16-byte units,
// slabs and output 16-byte aligned.
bool bulk_lookup_fits(size_t row_bytes, uint32_t stride, const void *out, const void *slabs) {
  return row_bytes >= kBulkMinRow && row_bytes <= kBulkMaxRow && row_bytes % 16 == 0 && stride % 16 == 0 &&
         uintptr_t(out) % 16 == 0 && uintptr_t(slabs) % 16 == 0;
}

uint32_t gather_lanes(uint64_t units) {
  uint32_t l = 4;
  while (l < 32 && uint64_t(l) * 8 < units) l <<= 1;
  return l;
}

// Lanes per key of the forward kernels (k_lookup, k_lookup_or_insert): two
// lanes per key while each lane's share stays <= 8 units, so a 65,536-key
// batch of 256-byte rows is 131,072 threads - one wave of resident blocks -
// and every lane keeps its 8 loads of the row in flight together.
uint32_t forward_lanes(uint64_t units) {
  uint32_t l = 2;
  while (l < 32 && uint64_t(l) * 8 < units) l <<= 1;
  return l;
}

uint32_t pick_lanes(uint64_t units) {
  uint32_t l = 4;
  while (l < 32 && l < units) l <<= 1;
  return l;
}

float host_dtype_max(int dt) {
  if (dt == SE_FLOAT16) return 65504.0f;
  if (dt == SE_FLOAT32) return 3.40282347e38f;
  return 3.38953139e38f;
}

template <class T> T *dalloc(size_t count) {
  void *p = nullptr;
  if (count == 0) count = 1;
  cuda_check(cudaMalloc(&p, count * sizeof(T)), "cudaMalloc");
  return static_cast<T *>(p);
}

void dfree(void *p) {
  if (p) cudaFree(p);
}

// Device buffer that only grows; contents are not preserved.
template <class T> struct Scratch {
  T *ptr = nullptr;
  size_t cap = 0;
  T *get(size_t n) {
    if (n > cap) {
      dfree(ptr);
      ptr = nullptr;
      cap = std::max(n, cap * 2);
      ptr = dalloc<T>(cap);
    }
    return ptr;
  }
  ~Scratch() { dfree(ptr); }
};

// Counters of a table, one device block.
enum Ctr : int {
  kCtrNextRow = 0,
  kCtrSpecialClaim = 1,
  kCtrSpecialRow = 2,
  kCtrDeferred = 3,
  kCtrGroup = 4,       // words 4-7: GroupWs counters ([0] segments of the window), cleared after each step
  kCtrStatus = 12,      // insert / directory errors
  kCtrGradStatus = 13,  // gradient validation of the current accumulate call
  kCtrDropped = 8,      // u64 at words 8-9
  kCtrPoison = 10,      // sticky: a device-input gradient batch failed validation
  kCtrPending = 11,     // pending gradient rows committed on the device
  kCtrAccDone = 14,     // blocks of the running k_accumulate that have finished
  kCtrPendingBackup = 15,
  kCtrUnres = 16,      // pending entries whose key was absent when appended (cleared after each step)
  kCtrStepDone = 17,   // blocks of the running k_group_hot that have finished
  kCtrFreeTop = 18,    // int: rows of erased keys on the free stack (may read below zero; see take_row)
  kCtrFwdDone = 19,    // blocks of the running k_lookup_or_insert that have finished
  kCtrFwdN = 20,       // keys cached by the last lookup_or_insert (FwdCache::n)
  kCtrFwdDeferred = 21,  // k_lookup_or_insert's deferred positions (zero between launches)
  kCtrEraseEpoch = 22,   // erases so far (rows listed by the atomic accumulate carry it)
  kCtrOwnerDone = 23,    // blocks of the running k_ex_owner (insert) that have finished
  kCtrOwnerDeferred = 24,  // k_ex_owner's deferred keys (zero between launches)
  kCtrWords = 32,
};

struct Table {
  int64_t dim = 0;
  Layout L{};
  int vec = 1;
  uint32_t lanes = 4;
  // directory
  Bucket *buckets = nullptr;
  uint64_t nbuckets = 0;
  // arena
  uint8_t *slabs = nullptr;
  uint64_t capacity = 0;
  uint64_t rows_bound = 0;  // upper bound of rows in use
  bool bound_stale = false;  // graph-captured inserts may have added rows since
  uint32_t *ctr = nullptr;
  // pending gradients
  unsigned long long *pkeys = nullptr;
  uint32_t *prows = nullptr;  // row of each pending key at accumulate time
  uint8_t *pgrads = nullptr;
  // counted with the pending entries (pcap entries each): row of each
  // segment, entries whose key was absent when appended
  uint32_t *seg_row = nullptr, *unres = nullptr;
  uint64_t pcap = 0, pcount = 0;
  // per-row grouping counters of optimizer_step (capacity entries each)
  uint32_t *row_cnt = nullptr, *row_seg = nullptr;
  // rows of erased keys, reused by inserts (capacity entries)
  uint32_t *free_rows = nullptr;
  uint64_t tombs = 0;  // upper bound of erased keys' tombstones in the directory
  bool erased = false;  // inserts look at the free stack only once a key was erased
  // step and insert work buffers
  Scratch<uint32_t> g_seg_cnt, g_seg_off, g_seg_fill, g_pos, g_long, def_pos;
  Scratch<uint32_t> g_sort_kin, g_sort_kout, g_sort_vin;  // sorted placement of large windows
  Scratch<uint8_t> g_sort_tmp;
  // checkpoint export snapshot: present keys and their rows, directory order
  Scratch<unsigned long long> exp_keys;
  Scratch<uint32_t> exp_rows;
  uint64_t exp_count = 0;
  bool exp_taken = false;
  Scratch<uint4> g_items;
  Scratch<float> g_partials;
  Scratch<unsigned long long> def_word;
  uint64_t seg_fill_zeroed = 0;  // entries of g_seg_fill known to be zero
  // keys and rows of the last lookup_or_insert, for the accumulate that follows (ordered mode)
  Scratch<unsigned long long> fwd_keys;
  Scratch<uint32_t> fwd_rows;
  // atomic accumulation mode (se_accum.cuh): per-key fp32 sums of the window
  bool atomic = false;
  uint32_t acc_tile = 0, acc_hbits = 0;  // rows per block of k_acc_atomic, its hash-set bits
  uint64_t acc_slots = 0;                // G (0: not allocated yet)
  uint64_t acc_vcap = 0;                 // dense sum rows
  ulonglong2 *acc_keys = nullptr;        // slots: (key, dense row)
  float *acc_vals = nullptr;
  uint32_t *acc_cnt = nullptr, *acc_ctr = nullptr;
  uint4 *acc_list = nullptr;
  AccTab acc_tab() const {
    return AccTab{acc_keys, acc_vals, acc_cnt, acc_list, acc_ctr, ctr + kCtrEraseEpoch, uint32_t(acc_slots - 1),
                  uint32_t(dim), uint32_t(acc_vcap)};
  }

  Dir dir() const { return Dir{buckets, nbuckets, ctr + kCtrSpecialClaim}; }
  // the keys and rows the last lookup_or_insert cached, for reading
  FwdCache fwd_cache() const {
    return FwdCache{fwd_keys.ptr, fwd_rows.ptr, fwd_keys.ptr ? ctr + kCtrFwdN : nullptr,
                    uint32_t(std::min<size_t>(std::min(fwd_keys.cap, fwd_rows.cap), 0xffffffffu))};
  }
  RowAlloc alloc() const {
    return RowAlloc{ctr + kCtrNextRow, erased ? reinterpret_cast<int *>(ctr + kCtrFreeTop) : nullptr, free_rows,
                    capacity};
  }
  ~Table() {
    dfree(buckets);
    dfree(slabs);
    dfree(ctr);
    dfree(pkeys);
    dfree(prows);
    dfree(pgrads);
    dfree(row_cnt);
    dfree(row_seg);
    dfree(free_rows);
    dfree(seg_row);
    dfree(unres);
    dfree(acc_keys);
    dfree(acc_vals);
    dfree(acc_cnt);
    dfree(acc_list);
    dfree(acc_ctr);
  }
  CountWs count_ws() const {
    return CountWs{row_cnt, row_seg, seg_row, ctr + kCtrGroup, unres, ctr + kCtrUnres};
  }
};

struct ProfRec {
  std::string name;
  cudaEvent_t a, b;
};

}  // namespace

struct StoreImpl {
  se_store_config cfg{};
  // forward_lookup of 512..1,024-byte rows through the TMA bulk kernel
  // (SE_GPU_WIDE_GATHER=bulk when the store is created); the default is the
  // vector-load gather, which measured faster on B200 at 512-byte rows
  // (82 % against 70 % of the HBM copy peak)
  bool bulk_gather = [] {
    const char *v = std::getenv("SE_GPU_WIDE_GATHER");
    return v != nullptr && std::string(v) == "bulk";
  }();
  std::vector<int64_t> dims;
  int device = 0;
  cudaStream_t own = nullptr;
  std::mutex mu;
  std::vector<std::unique_ptr<Table>> tables;
  float *bc = nullptr;  // Adam bias corrections, 2 floats per step
  uint64_t bc_steps = 0;
  uint64_t steps_taken = 0;
  uint32_t *status_host = nullptr;  // pinned
  uint64_t *u64_host = nullptr;     // pinned
  Scratch<uint8_t> stage_keys, stage_vals;
  Scratch<unsigned long long> dup_set;  // assign's repeated-key check
  Scratch<uint32_t> dup_words;
  Scratch<uint8_t> stage_offs;             // embedding-bag offsets staged from the host
  // scores and dynamic learning rates
  float *lr_lut = nullptr;                 // cosine multipliers or the custom LUT, on the device
  uint64_t lr_max = 0;                     // cosine max_score / custom LUT's last index
  unsigned long long *lru_clock = nullptr; // [0] the LRU access clock, [1] its next value
  Scratch<uint8_t> score_done;
  Scratch<uint32_t> bag_rows, bag_of_buf;  // rows of a bag batch's keys; bag of each key
  bool profiling = false;
  std::vector<ProfRec> prof;
  std::vector<cudaEvent_t> event_pool;

  ~StoreImpl() {
    if (own) cudaStreamSynchronize(own);
    tables.clear();
    dfree(bc);
    dfree(lr_lut);
    dfree(lru_clock);
    if (status_host) cudaFreeHost(status_host);
    if (u64_host) cudaFreeHost(u64_host);
    for (auto &r : prof) {
      cudaEventDestroy(r.a);
      cudaEventDestroy(r.b);
    }
    for (auto e : event_pool) cudaEventDestroy(e);
    if (own) cudaStreamDestroy(own);
  }

  // NULL is the legacy default stream, as everywhere in CUDA.
  static cudaStream_t pick(void *s) { return static_cast<cudaStream_t>(s); }

  Table &table(int64_t dim) {
    for (auto &t : tables)
      if (t->dim == dim) return *t;
    throw Error(SE_ERR_RUNTIME, "invalid dim access: no physical table for dim " + std::to_string(dim));
  }

  // ---- profiling ------------------------------------------------------------
  cudaEvent_t take_event() {
    if (event_pool.empty()) {
      cudaEvent_t e;
      cuda_check(cudaEventCreate(&e), "cudaEventCreate");
      return e;
    }
    cudaEvent_t e = event_pool.back();
    event_pool.pop_back();
    return e;
  }
  struct Prof {
    StoreImpl *s;
    cudaStream_t st;
    ProfRec rec{};
    // Inside stream capture the records become external event nodes, which
    // are recorded (and can be timed) every time the graph is launched.
    static void record(cudaEvent_t e, cudaStream_t st) {
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      cudaStreamIsCapturing(st, &cs);
      if (cs == cudaStreamCaptureStatusActive) cudaEventRecordWithFlags(e, st, cudaEventRecordExternal);
      else cudaEventRecord(e, st);
    }
    Prof(StoreImpl *store, const char *name, cudaStream_t stream) : s(store), st(stream) {
      if (!s->profiling) return;
      rec.name = name;
      rec.a = s->take_event();
      rec.b = s->take_event();
      record(rec.a, st);
    }
    ~Prof() {
      if (!s->profiling) return;
      record(rec.b, st);
      s->prof.push_back(rec);
    }
  };

  // ---- table construction and growth ---------------------------------------
  void init_table(Table &t, int64_t dim, uint64_t cap) {
    const int pdt = cfg.value_dtype, odt = cfg.optimizer_dtype;
    const uint32_t pb = uint32_t(dim) * uint32_t(value_bytes(pdt));
    const uint32_t ob = uint32_t(dim) * uint32_t(value_bytes(odt));
    auto up16 = [](uint32_t x) { return (x + 15u) & ~15u; };
    uint32_t nstate = 0;
    if (cfg.enable_optimizer && cfg.optimizer_kind == SE_OPT_ADAGRAD) nstate = 1;
    if (cfg.enable_optimizer && cfg.optimizer_kind == SE_OPT_ADAM) nstate = 2;
    t.dim = dim;
    t.L.dim = uint32_t(dim);
    t.L.pdt = pdt;
    t.L.odt = odt;
    t.L.nstate = nstate;
    t.L.state0 = up16(pb);
    t.L.state1 = t.L.state0 + (nstate >= 1 ? up16(ob) : 0u);
    t.L.step = t.L.state1 + (nstate >= 2 ? up16(ob) : 0u);
    t.L.stride = t.L.step + (nstate >= 2 ? 16u : 0u);
    t.L.score = 0u;
    if (cfg.score_policy != SE_SCORE_NONE) {  // a u64 score after the optimizer state
      t.L.score = t.L.stride;
      t.L.stride += 16u;
    }
    t.vec = dim % 4 == 0 ? 4 : 1;
    t.lanes = pick_lanes(uint64_t(dim) / uint64_t(t.vec));
    // atomic mode: k_acc_atomic keeps a tile's sums in 32 KB of shared memory
    t.atomic = cfg.accumulation == SE_ACCUM_ATOMIC && dim <= int64_t(kAccMaxDim);
    if (t.atomic) {
      uint32_t tile = 1;
      while (tile < kAccMaxTile && uint64_t(tile) * 2 * uint64_t(dim) * 4 <= kAccSmemBytes) tile <<= 1;
      t.acc_tile = tile;
      t.acc_hbits = 1;
      while ((1u << t.acc_hbits) < 2 * tile) ++t.acc_hbits;
    }
    t.ctr = dalloc<uint32_t>(kCtrWords);
    cuda_check(cudaMemset(t.ctr, 0, kCtrWords * 4), "memset counters");
    cuda_check(cudaMemset(t.ctr + kCtrSpecialRow, 0xff, 4), "memset special");
    t.capacity = std::max<uint64_t>(cap, 64);
    t.slabs = dalloc<uint8_t>(size_t(t.capacity) * t.L.stride);
    alloc_row_arrays(t, t.capacity);
    t.nbuckets = next_pow2(uint64_t(double(t.capacity) / kMaxLoadPerBucket) + 1);
    t.buckets = dalloc<Bucket>(t.nbuckets);
    cuda_check(cudaMemset(t.buckets, 0xff, t.nbuckets * sizeof(Bucket)), "memset directory");
  }

  // Per-row grouping counters, zero between steps.
  // Rows counted since the last step keep their counts and segments when
  // the arena grows (the first `keep` rows are copied).
  void alloc_row_arrays(Table &t, uint64_t cap, uint64_t keep = 0, cudaStream_t st = nullptr) {
    uint32_t *nc = dalloc<uint32_t>(cap), *ns = dalloc<uint32_t>(cap), *nf = dalloc<uint32_t>(cap);
    cuda_check(cudaMemsetAsync(nc, 0, cap * 4, st), "memset row counters");
    if (keep) {
      cuda_check(cudaMemcpyAsync(nc, t.row_cnt, keep * 4, cudaMemcpyDeviceToDevice, st), "grow row counters");
      cuda_check(cudaMemcpyAsync(ns, t.row_seg, keep * 4, cudaMemcpyDeviceToDevice, st), "grow row counters");
      cuda_check(cudaMemcpyAsync(nf, t.free_rows, keep * 4, cudaMemcpyDeviceToDevice, st), "grow free rows");
    }
    cuda_check(cudaStreamSynchronize(st), "sync");
    dfree(t.row_cnt);
    dfree(t.row_seg);
    dfree(t.free_rows);
    t.row_cnt = nc;
    t.row_seg = ns;
    t.free_rows = nf;
  }

  uint64_t read_rows_used(Table &t, cudaStream_t st) {
    cuda_check(cudaMemcpyAsync(status_host, t.ctr + kCtrNextRow, 4, cudaMemcpyDeviceToHost, st), "read rows");
    cuda_check(cudaStreamSynchronize(st), "sync");
    const uint64_t used = status_host[0];
    check_status(t, st);
    return used;
  }

  // Keys present: rows taken from the arena minus the rows of erased keys
  // waiting on the free stack.
  uint64_t read_live_keys(Table &t, cudaStream_t st) {
    const uint64_t used = read_rows_used(t, st);
    cuda_check(cudaMemcpyAsync(status_host, t.ctr + kCtrFreeTop, 4, cudaMemcpyDeviceToHost, st), "read rows");
    cuda_check(cudaStreamSynchronize(st), "sync");
    const int32_t free_top = int32_t(status_host[0]);
    return used - uint64_t(free_top > 0 ? free_top : 0);
  }

  static bool capturing(cudaStream_t st) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    return cs == cudaStreamCaptureStatusActive;
  }

  // Guarantees room for `extra` more rows in the arena and the directory.
  // Under stream capture nothing can grow: the call only checks the room
  // reserved beforehand. Replays of the captured graph do not come through
  // here, so the rows they insert are bounded by the arena alone (the insert
  // kernels report a full arena), and the next call outside capture re-reads
  // the rows in use.
  void ensure_rows(Table &t, uint64_t extra, cudaStream_t st) {
    if (capturing(st)) {
      t.bound_stale = true;
      const uint64_t need = t.rows_bound + extra;
      if (need > t.capacity || need + t.tombs > uint64_t(double(t.nbuckets) * kMaxLoadPerBucket))
        throw Error(SE_ERR_TABLE_FULL, "insert captured in a CUDA graph needs " + std::to_string(extra) +
                                           " reserved rows; reserve capacity before capturing");
      return;
    }
    if (t.bound_stale) {
      t.rows_bound = read_rows_used(t, st);
      t.bound_stale = false;
    }
    uint64_t need = t.rows_bound + extra;
    const auto dir_limit = [&](uint64_t nb) { return uint64_t(double(nb) * kMaxLoadPerBucket); };
    // The bound carries each call's whole batch (the new rows are known only
    // on the device), so it drifts above the rows in use. When it leaves no
    // room for one more call of this size after this one, the rows in use
    // are read again (a sync): a call captured next in a CUDA graph, which
    // can neither read them nor grow the arena, then finds its room whenever
    // the rows in use leave it. The arena grows only when this call needs it.
    // Directory slots in use: at most the rows ever taken plus the erased
    // keys' tombstones (a rehash drops those).
    if (need + extra > t.capacity || need + extra + t.tombs > dir_limit(t.nbuckets)) {
      t.rows_bound = read_rows_used(t, st);
      need = t.rows_bound + extra;
      if (need > 0xfffffff0ull) throw Error(SE_ERR_TABLE_FULL, "table exceeds 2^32 rows");
      if (need > t.capacity) {
        const uint64_t ncap = std::max<uint64_t>(need, t.capacity * 2);
        uint8_t *ns = dalloc<uint8_t>(size_t(ncap) * t.L.stride);
        cuda_check(cudaMemcpyAsync(ns, t.slabs, size_t(t.rows_bound) * t.L.stride,
                                   cudaMemcpyDeviceToDevice, st), "grow arena");
        cuda_check(cudaStreamSynchronize(st), "sync");
        dfree(t.slabs);
        t.slabs = ns;
        const uint64_t old_cap = t.capacity;
        t.capacity = ncap;
        alloc_row_arrays(t, ncap, old_cap, st);
      }
      if (need + t.tombs > dir_limit(t.nbuckets)) {
        uint64_t nb = t.nbuckets;
        while (dir_limit(nb) < std::max(need, t.capacity)) nb *= 2;
        Bucket *nbk = dalloc<Bucket>(nb);
        cuda_check(cudaMemsetAsync(nbk, 0xff, nb * sizeof(Bucket), st), "memset directory");
        Dir nd{nbk, nb, t.ctr + kCtrSpecialClaim};
        const uint64_t slots = t.nbuckets * kBucketSlots;
        k_rehash<<<grid_for(slots, 256, 0x7fffffffu), 256, 0, st>>>(t.buckets, t.nbuckets, nd,
                                                                   t.ctr + kCtrStatus);
        launched("k_rehash");
        cuda_check(cudaStreamSynchronize(st), "sync");
        dfree(t.buckets);
        t.buckets = nbk;
        t.nbuckets = nb;
        t.tombs = 0;
      }
    }
    t.rows_bound = need;
  }

  void ensure_pending(Table &t, uint64_t extra, cudaStream_t st) {
    const uint64_t need = t.pcount + extra;
    if (need <= t.pcap) return;
    if (need > 0xffffffffull) throw Error(SE_ERR_RUNTIME, "more than 2^32 pending gradient rows");
    const uint64_t ncap = std::max<uint64_t>(need, std::max<uint64_t>(t.pcap * 2, 1024));
    const size_t gb = size_t(t.dim) * value_bytes(cfg.gradient_dtype);
    auto *nk = dalloc<unsigned long long>(ncap);
    auto *nr = dalloc<uint32_t>(ncap);
    auto *ng = dalloc<uint8_t>(size_t(ncap) * gb);
    auto *nsr = dalloc<uint32_t>(ncap);
    auto *nu = dalloc<uint32_t>(ncap);
    if (t.pcount) {
      cuda_check(cudaMemcpyAsync(nk, t.pkeys, t.pcount * 8, cudaMemcpyDeviceToDevice, st), "grow pending");
      cuda_check(cudaMemcpyAsync(nr, t.prows, t.pcount * 4, cudaMemcpyDeviceToDevice, st), "grow pending");
      cuda_check(cudaMemcpyAsync(ng, t.pgrads, size_t(t.pcount) * gb, cudaMemcpyDeviceToDevice, st),
                 "grow pending");
      cuda_check(cudaMemcpyAsync(nsr, t.seg_row, t.pcount * 4, cudaMemcpyDeviceToDevice, st), "grow pending");
      cuda_check(cudaMemcpyAsync(nu, t.unres, t.pcount * 4, cudaMemcpyDeviceToDevice, st), "grow pending");
    }
    cuda_check(cudaStreamSynchronize(st), "sync");
    dfree(t.pkeys);
    dfree(t.prows);
    dfree(t.pgrads);
    dfree(t.seg_row);
    dfree(t.unres);
    t.pkeys = nk;
    t.prows = nr;
    t.pgrads = ng;
    t.seg_row = nsr;
    t.unres = nu;
    t.pcap = ncap;
  }

  // Atomic mode: room in the sum table for `extra` more gradient rows of the
  // window (at most half the slots in use). A larger table takes the claimed
  // slots over (k_acc_move); under stream capture nothing can grow.
  void ensure_acc(Table &t, uint64_t extra, cudaStream_t st) {
    const uint64_t need = 2 * (t.pcount + extra);
    if (need <= t.acc_slots) return;
    if (capturing(st))
      throw Error(SE_ERR_RUNTIME, "gradient window captured in a CUDA graph outgrows its sum table; run one "
                                  "step of the same size before capturing");
    if (need > (1ull << 31)) throw Error(SE_ERR_RUNTIME, "more than 2^30 gradient rows in one window");
    const uint64_t G = next_pow2(std::max<uint64_t>(need, 1024));
    const uint64_t V = G / 2;  // dense sum rows: one per gradient row of the window at most
    auto *nk = dalloc<ulonglong2>(G + 1);
    auto *nv = dalloc<float>(size_t(V) * size_t(t.dim));
    auto *nc = dalloc<uint32_t>(G + 1);
    auto *nl = dalloc<uint4>(G + 1);
    auto *nctr = dalloc<uint32_t>(4);
    cuda_check(cudaMemsetAsync(nk, 0xff, (G + 1) * sizeof(ulonglong2), st), "memset sums");  // all free
    cuda_check(cudaMemsetAsync(nv, 0, size_t(V) * size_t(t.dim) * 4, st), "memset sums");
    cuda_check(cudaMemsetAsync(nc, 0, (G + 1) * 4, st), "memset sums");
    cuda_check(cudaMemsetAsync(nctr, 0, 16, st), "memset sums");
    const AccTab to{nk, nv, nc, nl, nctr, t.ctr + kCtrEraseEpoch, uint32_t(G - 1), uint32_t(t.dim), uint32_t(V)};
    if (t.acc_slots) {
      // the claimed slots move; their dense sums are copied as they are
      cuda_check(cudaMemcpyAsync(nv, t.acc_vals, size_t(t.acc_vcap) * size_t(t.dim) * 4, cudaMemcpyDeviceToDevice,
                                 st), "grow sums");
      k_acc_move<<<grid_for(t.acc_slots + 1, 256, 148 * 8), 256, 0, st>>>(t.acc_tab(), to, t.ctr + kCtrStatus);
      launched("k_acc_move");
    }
    cuda_check(cudaStreamSynchronize(st), "sync");
    dfree(t.acc_keys);
    dfree(t.acc_vals);
    dfree(t.acc_cnt);
    dfree(t.acc_list);
    dfree(t.acc_ctr);
    t.acc_keys = nk;
    t.acc_vals = nv;
    t.acc_cnt = nc;
    t.acc_list = nl;
    t.acc_ctr = nctr;
    t.acc_slots = G;
    t.acc_vcap = V;
  }

  void ensure_bc(uint64_t steps) {
    if (steps < bc_steps) return;
    uint64_t n = std::max<uint64_t>(4096, bc_steps * 2);
    while (n <= steps) n *= 2;
    std::vector<float> h(2 * n);
    h[0] = 1.0f;
    h[1] = 1.0f;
    // AdamOptimizer bias-correction table (adam_optimizer.hpp:55-61, and the
    // same formula past the table, 144-148): std::pow(float, float) is powf.
    for (uint64_t s = 1; s < n; ++s) {
      const float sf = float(s);
      h[2 * s] = 1.0f / (1.0f - std::pow(cfg.beta1, sf));
      h[2 * s + 1] = 1.0f / (1.0f - std::pow(cfg.beta2, sf));
    }
    float *nb = dalloc<float>(2 * n);
    cuda_check(cudaMemcpy(nb, h.data(), h.size() * 4, cudaMemcpyHostToDevice), "upload bc");
    dfree(bc);
    bc = nb;
    bc_steps = n;
  }

  // ---- host/device staging ----------------------------------------------------
  const void *stage_in(Scratch<uint8_t> &buf, const void *p, size_t bytes, cudaStream_t st) {
    if (bytes == 0 || is_device_ptr(p)) return p;
    uint8_t *d = buf.get(bytes);
    cuda_check(cudaMemcpyAsync(d, p, bytes, cudaMemcpyHostToDevice, st), "stage H2D");
    return d;
  }

  // ---- operations ----------------------------------------------------------
  void lookup(const void *keys, size_t n, int64_t dim, void *out, void *sp, bool insert) {
    std::lock_guard<std::mutex> lock(mu);
    DeviceGuard dg(device);
    if (dim <= 0) throw std::invalid_argument("dim must be > 0");
    Table &t = table(dim);
    if (n == 0) return;
    if (n > 0x7fffffffull) throw std::invalid_argument("batch exceeds 2^31 keys");
    cudaStream_t st = pick(sp);
    const size_t vb = value_bytes(cfg.value_dtype);
    const size_t out_bytes = n * size_t(dim) * vb;
    const void *dkeys = stage_in(stage_keys, keys, n * key_bytes(cfg.key_dtype), st);
    const bool host_out = !is_device_ptr(out);
    void *dout = host_out ? stage_vals.get(out_bytes) : out;
    if (!insert && bulk_gather && bulk_lookup_fits(size_t(dim) * vb, t.L.stride, dout, t.slabs)) {
      const size_t row_bytes = size_t(dim) * vb;
      const size_t smem = size_t(kBulkWarps) * 32u * row_bytes;
      // 32 positions per warp and round, warps striding over the batch; one
      // wave of resident blocks at most
      const uint32_t per_sm = uint32_t(std::max<size_t>(1, (227u * 1024u) / (smem + 1024u)));
      const size_t rounds = (n + 31) / 32;
      const unsigned grid = unsigned(std::min<size_t>((rounds + kBulkWarps - 1) / kBulkWarps, size_t(148) * per_sm));
      allow_dynamic_smem(k_lookup_bulk, smem);
      Prof pr(this, "k_lookup_bulk", st);
      pdl(k_lookup_bulk, grid, kBulkWarps * 32, smem, st, t.dir(), t.slabs, t.L.stride, uint32_t(row_bytes), dkeys,
          cfg.key_dtype, n, static_cast<uint8_t *>(dout), t.ctr + kCtrStatus);
      launched("k_lookup_bulk");
      if (cfg.score_policy == SE_SCORE_LFU || cfg.score_policy == SE_SCORE_LRU) touch_scores(t, dkeys, n, st);
    } else if (!insert) {
      const size_t row_bytes = size_t(dim) * vb;
      const uintptr_t al = uintptr_t(dout) | uintptr_t(row_bytes);
      const Dir d = t.dir();
      auto go = [&](auto lanes_tag, auto vtag) {
        constexpr int LN = decltype(lanes_tag)::value;
        using V = decltype(vtag);
        const uint32_t units = uint32_t(row_bytes / sizeof(V));
        Prof pr(this, "k_lookup", st);
        pdl(k_lookup<LN, V>, grid_for(n * LN, 256, 0x7fffffffu), 256, 0, st,
            d, t.slabs, t.L.stride, units, dkeys, cfg.key_dtype, n, static_cast<V *>(dout));
        launched("k_lookup");
      };
      auto by_lanes = [&](auto vtag) {
        using V = decltype(vtag);
        const uint32_t ln = forward_lanes(row_bytes / sizeof(V));
        switch (ln) {
        case 2: go(std::integral_constant<int, 2>{}, vtag); break;
        case 4: go(std::integral_constant<int, 4>{}, vtag); break;
        case 8: go(std::integral_constant<int, 8>{}, vtag); break;
        case 16: go(std::integral_constant<int, 16>{}, vtag); break;
        default: go(std::integral_constant<int, 32>{}, vtag); break;
        }
      };
      if (al % 16 == 0) by_lanes(uint4{});
      else if (al % 4 == 0) by_lanes(uint32_t{});
      else by_lanes(uint16_t{});
      if (cfg.score_policy == SE_SCORE_LFU || cfg.score_policy == SE_SCORE_LRU) touch_scores(t, dkeys, n, st);
    } else {
      ensure_rows(t, n, st);
      const bool under_capture = capturing(st);
      uint32_t *dpos = under_capture ? t.def_pos.ptr : t.def_pos.get(n);
      unsigned long long *dword = under_capture ? t.def_word.ptr : t.def_word.get(n);
      if (under_capture && (t.def_pos.cap < n || t.def_word.cap < n))
        throw Error(SE_ERR_RUNTIME, "lookup_or_insert captured in a CUDA graph needs a batch of the same size "
                                    "run once before capturing");
      // keys and rows stay cached for the accumulate of the same keys
      FwdCache fc{nullptr, nullptr, t.ctr + kCtrFwdN, 0};
      if (!under_capture || (t.fwd_keys.cap >= n && t.fwd_rows.cap >= n)) {
        fc.keys = t.fwd_keys.get(n);
        fc.rows = t.fwd_rows.get(n);
        fc.cap = uint32_t(std::min<size_t>(std::min(t.fwd_keys.cap, t.fwd_rows.cap), 0xffffffffu));
      }
      InitSpec init{cfg.init_kind, cfg.init_min, cfg.init_max - cfg.init_min,
                    cfg.optimizer_kind == SE_OPT_ADAGRAD ? cfg.initial_accumulator : 0.0f};
      const bool vec4 = t.vec == 4 && (uintptr_t(dout) % 16 == 0);
      auto go = [&](auto lanes_tag, auto vec_tag) {
        constexpr int LN = decltype(lanes_tag)::value;
        constexpr int VC = decltype(vec_tag)::value;
        Prof pr(this, "k_lookup_or_insert", st);
        const unsigned bt = balanced_block(n * LN);
        pdl(k_lookup_or_insert<LN, VC>, grid_for(n * LN, bt, 0x7fffffffu), bt, 0, st,
            t.dir(), t.L, t.slabs, t.alloc(), init, dkeys, cfg.key_dtype, n,
            dout, t.ctr + kCtrFwdDeferred, dpos, dword, t.ctr + kCtrStatus, t.ctr + kCtrFwdDone, fc);
        launched("k_lookup_or_insert");
      };
      auto by_lanes = [&](auto vec_tag) {
        const uint32_t ln = forward_lanes(vec4 ? uint64_t(dim) / 4 : uint64_t(dim));
        switch (ln) {
        case 2: go(std::integral_constant<int, 2>{}, vec_tag); break;
        case 4: go(std::integral_constant<int, 4>{}, vec_tag); break;
        case 8: go(std::integral_constant<int, 8>{}, vec_tag); break;
        case 16: go(std::integral_constant<int, 16>{}, vec_tag); break;
        default: go(std::integral_constant<int, 32>{}, vec_tag); break;
        }
      };
      if (vec4) by_lanes(std::integral_constant<int, 4>{});
      else by_lanes(std::integral_constant<int, 1>{});
    }
    if (host_out) {
      cuda_check(cudaMemcpyAsync(out, dout, out_bytes, cudaMemcpyDeviceToHost, st), "copy out");
      cuda_check(cudaStreamSynchronize(st), "sync");
      if (insert) check_status(t, st);
    }
  }

  // Reads and clears the table's insert status word and raises on
  // kernel-reported errors. Calls with device outputs do not wait for their
  // kernels; their errors surface at the next synchronising call.
  void check_status(Table &t, cudaStream_t st) {
    cuda_check(cudaMemcpyAsync(status_host, t.ctr + kCtrStatus, 4, cudaMemcpyDeviceToHost, st), "status");
    cuda_check(cudaMemcpyAsync(status_host + 1, t.ctr + kCtrPoison, 4, cudaMemcpyDeviceToHost, st), "status");
    cuda_check(cudaMemsetAsync(t.ctr + kCtrStatus, 0, 4, st), "status clear");
    cuda_check(cudaStreamSynchronize(st), "sync");
    const uint32_t s = status_host[0];
    if (s & kStatusTableFull) throw Error(SE_ERR_TABLE_FULL, "embedding table is full");
    if (s & kStatusBadRow) throw Error(SE_ERR_RUNTIME, "row index outside the arena");
    if (s & kStatusPendingOverflow)
      throw Error(SE_ERR_RUNTIME, "pending gradient rows on the device exceed the host's count: calls on this "
                                  "store were not ordered on one stream (rows past the buffers were dropped)");
    if (status_host[1] && t.pcount == 0) {
      // the poisoned window has been stepped (and discarded): report it once
      cuda_check(cudaMemsetAsync(t.ctr + kCtrPoison, 0, 4, st), "status clear");
      cuda_check(cudaStreamSynchronize(st), "sync");
      throw std::overflow_error(
          "gradient scale storage exceeds configured dtype (a device gradient batch failed validation; "
          "its accumulation window was discarded)");
    }
  }

  // ---- mutation API ----------------------------------------------------------
  // contains (hogwild_embedding_store.hpp:4983-5009).
  void contains(const void *keys, size_t n, uint8_t *out, void *sp) {
    std::lock_guard<std::mutex> lock(mu);
    DeviceGuard dg(device);
    if (n == 0) return;
    if (n > 0x7fffffffull) throw std::invalid_argument("batch exceeds 2^31 keys");
    cudaStream_t st = pick(sp);
    const void *dkeys = stage_in(stage_keys, keys, n * key_bytes(cfg.key_dtype), st);
    const bool host_out = !is_device_ptr(out);
    uint8_t *dout = host_out ? stage_vals.get(n) : out;
    if (tables.empty()) cuda_check(cudaMemsetAsync(dout, 0, n, st), "memset");
    int first = 1;
    for (auto &t : tables) {
      Prof pr(this, "k_contains", st);
      k_contains<<<grid_for(n, 256, 0x7fffffffu), 256, 0, st>>>(t->dir(), dkeys, cfg.key_dtype, n, dout, first);
      launched("k_contains");
      first = 0;
    }
    if (host_out) {
      cuda_check(cudaMemcpyAsync(out, dout, n, cudaMemcpyDeviceToHost, st), "copy out");
      cuda_check(cudaStreamSynchronize(st), "sync");
    }
  }

  // assign (hogwild_embedding_store.hpp:4838-4923) with the batch check of
  // validate_unique_mutation_batch (5278-5305).
  void assign(const void *keys, size_t n, int64_t dim, const void *values, void *sp) {
    std::lock_guard<std::mutex> lock(mu);
    DeviceGuard dg(device);
    if (dim <= 0) throw std::invalid_argument("dim must be > 0");
    Table &t = table(dim);
    if (n == 0) return;
    if (n > 0x7fffffffull) throw std::invalid_argument("batch exceeds 2^31 keys");
    cudaStream_t st = pick(sp);
    ensure_rows(t, n, st);
    const size_t vb = value_bytes(cfg.value_dtype);
    const void *dkeys = stage_in(stage_keys, keys, n * key_bytes(cfg.key_dtype), st);
    const void *dvals = stage_in(stage_vals, values, n * size_t(dim) * vb, st);
    // repeated keys: checked on the device before anything is written
    const uint64_t nslots = next_pow2(2 * uint64_t(n));
    unsigned long long *set = dup_set.get(nslots);
    uint32_t *words = dup_words.get(2);
    cuda_check(cudaMemsetAsync(set, 0xff, nslots * 8, st), "memset");
    cuda_check(cudaMemsetAsync(words, 0, 8, st), "memset");
    k_assign_dups<<<grid_for(n, 256, 0x7fffffffu), 256, 0, st>>>(dkeys, cfg.key_dtype, n, set, nslots, words);
    launched("k_assign_dups");
    InitSpec init{cfg.init_kind, cfg.init_min, cfg.init_max - cfg.init_min,
                  cfg.optimizer_kind == SE_OPT_ADAGRAD ? cfg.initial_accumulator : 0.0f};
    const bool vec4 = t.vec == 4 && (uintptr_t(dvals) % 16 == 0);
    auto go = [&](auto lanes_tag, auto vec_tag) {
      constexpr int LN = decltype(lanes_tag)::value;
      constexpr int VC = decltype(vec_tag)::value;
      Prof pr(this, "k_assign", st);
      k_assign<LN, VC><<<grid_for(n * LN, 256, 0x7fffffffu), 256, 0, st>>>(
          t.dir(), t.L, t.slabs, t.alloc(), init, dkeys, cfg.key_dtype, n, dvals, words + 1, t.ctr + kCtrStatus);
      launched("k_assign");
    };
    auto by_lanes = [&](auto vec_tag) {
      const uint32_t ln = gather_lanes(vec4 ? uint64_t(dim) / 4 : uint64_t(dim));
      switch (ln) {
      case 4: go(std::integral_constant<int, 4>{}, vec_tag); break;
      case 8: go(std::integral_constant<int, 8>{}, vec_tag); break;
      case 16: go(std::integral_constant<int, 16>{}, vec_tag); break;
      default: go(std::integral_constant<int, 32>{}, vec_tag); break;
      }
    };
    if (vec4) by_lanes(std::integral_constant<int, 4>{});
    else by_lanes(std::integral_constant<int, 1>{});
    // the reference raises before it mutates anything: read the mark now
    cuda_check(cudaMemcpyAsync(status_host, words + 1, 4, cudaMemcpyDeviceToHost, st), "read mark");
    cuda_check(cudaStreamSynchronize(st), "sync");
    if (status_host[0] != 0u) throw std::invalid_argument("mutation batch contains duplicate dimension and key");
    if (!is_device_ptr(keys) || !is_device_ptr(values)) check_status(t, st);
  }

  // erase (hogwild_embedding_store.hpp:5011-5062): every table; or
  // erase_dimension (5064-5106): the table of `dim`.
  void erase(const void *keys, size_t n, int64_t dim, void *sp) {
    std::lock_guard<std::mutex> lock(mu);
    DeviceGuard dg(device);
    Table *only = nullptr;
    if (dim != 0) {
      for (auto &t : tables)
        if (t->dim == dim) only = t.get();
      if (only == nullptr) throw std::invalid_argument("erase dimension is not configured");
    }
    if (n == 0) return;
    if (n > 0x7fffffffull) throw std::invalid_argument("batch exceeds 2^31 keys");
    cudaStream_t st = pick(sp);
    const void *dkeys = stage_in(stage_keys, keys, n * key_bytes(cfg.key_dtype), st);
    for (auto &tp : tables) {
      Table &t = *tp;
      if (only != nullptr && only != &t) continue;
      int *free_top = reinterpret_cast<int *>(t.ctr + kCtrFreeTop);
      k_free_clamp<<<1, 1, 0, st>>>(free_top, t.ctr + kCtrEraseEpoch);
      launched("k_free_clamp");
      {
        Prof pr(this, "k_erase", st);
        k_erase<<<grid_for(n, 256, 0x7fffffffu), 256, 0, st>>>(t.dir(), dkeys, cfg.key_dtype, n, free_top,
                                                               t.free_rows, t.capacity);
        launched("k_erase");
      }
      t.tombs += n;
      t.erased = true;
      // an erased key's row may be reused: rows cached by the last
      // lookup_or_insert are no longer trusted
      cuda_check(cudaMemsetAsync(t.ctr + kCtrFwdN, 0, 4, st), "cache clear");
      // ordered mode: pending rows are counted again (atomic mode resolves keys at the step)
      if (t.pcount > 0 && !t.atomic) {
        const unsigned grid = grid_for(t.pcount, 256, 148 * 8);
        k_requeue_clear<<<grid, 256, 0, st>>>(t.prows, t.ctr + kCtrPending, uint32_t(t.pcap), t.capacity,
                                              t.count_ws());
        launched("k_requeue_clear");
        k_requeue_count<<<grid, 256, 0, st>>>(t.dir(), t.pkeys, t.prows, t.ctr + kCtrPending, uint32_t(t.pcap),
                                              t.count_ws());
        launched("k_requeue_count");
      }
    }
    if (!is_device_ptr(keys)) cuda_check(cudaStreamSynchronize(st), "sync");
  }

  // ---- scores and dynamic learning rates -------------------------------------
  // Store construction (bindings/module.cpp:144-158; dynamic_lr_policy.hpp:32-124).
  void init_scores(se_store_config &c) {
    if (c.score_policy < SE_SCORE_NONE || c.score_policy > SE_SCORE_MANUAL)
      throw std::invalid_argument("unknown score policy");
    if (c.lr_policy < SE_LR_CONSTANT || c.lr_policy > SE_LR_CUSTOM_LUT)
      throw std::invalid_argument("unknown dynamic learning-rate policy");
    if (c.lr_policy != SE_LR_CONSTANT && c.score_policy == SE_SCORE_NONE)
      throw std::invalid_argument("dynamic learning-rate policy requires a score policy");
    std::vector<float> lut;
    if (c.lr_policy == SE_LR_COSINE_FREQUENCY) {
      // CosineFrequencyLrPolicy's table: (1 + cos(pi * i / max_score)) / 2
      if (!std::isfinite(c.lr_min_ratio) || c.lr_min_ratio < 0.0f || c.lr_min_ratio > 1.0f)
        throw std::invalid_argument("min_lr_ratio must be finite and in [0, 1]");
      if (c.lr_max_score == 0) throw std::invalid_argument("max_score must be greater than zero");
      if (c.lr_max_score > (uint64_t(1) << 28)) throw std::invalid_argument("max_score above 2^28 is not supported");
      lut.resize(size_t(c.lr_max_score) + 1);
      const float pi = static_cast<float>(3.14159265358979323846);
      for (uint64_t i = 0; i <= c.lr_max_score; ++i) {
        const float ratio = static_cast<float>(i) / static_cast<float>(c.lr_max_score);
        const float cos_val = std::cos(pi * ratio);
        lut[size_t(i)] = (1.0f + cos_val) / 2.0f;
      }
      lr_max = c.lr_max_score;
    } else if (c.lr_policy == SE_LR_CUSTOM_LUT) {
      if (c.lr_lut == nullptr || c.lr_lut_len == 0) throw std::invalid_argument("lut must not be empty");
      for (size_t i = 0; i < c.lr_lut_len; ++i)
        if (!std::isfinite(c.lr_lut[i]) || c.lr_lut[i] < 0.0f)
          throw std::invalid_argument("lut multipliers must be finite and non-negative");
      lut.assign(c.lr_lut, c.lr_lut + c.lr_lut_len);
      lr_max = c.lr_lut_len - 1;
    }
    c.lr_lut = nullptr;  // the caller's array is not kept
    c.lr_lut_len = lut.size();
    cfg.lr_lut = nullptr;
    cfg.lr_lut_len = lut.size();
    if (!lut.empty()) {
      lr_lut = dalloc<float>(lut.size());
      cuda_check(cudaMemcpy(lr_lut, lut.data(), lut.size() * 4, cudaMemcpyHostToDevice), "upload lut");
    }
    if (c.score_policy == SE_SCORE_LRU) {
      const unsigned long long start[2] = {1ull, 1ull};  // the reference's clock starts at 1
      lru_clock = dalloc<unsigned long long>(2);
      cuda_check(cudaMemcpy(lru_clock, start, 16, cudaMemcpyHostToDevice), "init clock");
    }
  }

  // on_access for every position of a lookup whose key is present.
  void touch_scores(Table &t, const void *dkeys, size_t n, cudaStream_t st) {
    if (cfg.score_policy == SE_SCORE_LFU) {
      k_touch_lfu<<<grid_for(n, 256, 0x7fffffffu), 256, 0, st>>>(t.dir(), t.L, t.slabs, dkeys, cfg.key_dtype, n);
      launched("k_touch_lfu");
    } else if (cfg.score_policy == SE_SCORE_LRU) {
      uint32_t *rows = bag_rows.get(n), *hits = exp_flags.get(n), *rank = exp_at.get(n);
      size_t tmp_bytes = 0;
      cuda_check(cub::DeviceScan::ExclusiveSum(nullptr, tmp_bytes, hits, rank, int(n), st), "scan size");
      uint8_t *tmp = exp_tmp.get(tmp_bytes);
      k_touch_find<<<grid_for(n, 256, 0x7fffffffu), 256, 0, st>>>(t.dir(), dkeys, cfg.key_dtype, n, rows, hits);
      launched("k_touch_find");
      cuda_check(cub::DeviceScan::ExclusiveSum(tmp, tmp_bytes, hits, rank, int(n), st), "scan");
      k_touch_lru<<<grid_for(n, 256, 0x7fffffffu), 256, 0, st>>>(t.L, t.slabs, rows, hits, rank, n, lru_clock);
      launched("k_touch_lru");
      cuda_check(cudaMemcpyAsync(lru_clock, lru_clock + 1, 8, cudaMemcpyDeviceToDevice, st), "clock");
    }
  }

  // assign_scores (hogwild_embedding_store.hpp:5202-5250), without row lengths.
  void assign_scores(const void *keys, size_t n, const uint64_t *scores, void *sp) {
    std::lock_guard<std::mutex> lock(mu);
    DeviceGuard dg(device);
    if (cfg.score_policy == SE_SCORE_NONE) throw Error(SE_ERR_RUNTIME, "assign_scores requires a score-enabled policy");
    if (n == 0) return;
    if (scores == nullptr) throw std::invalid_argument("assign_scores row counts differ");
    cudaStream_t st = pick(sp);
    const void *dkeys = stage_in(stage_keys, keys, n * key_bytes(cfg.key_dtype), st);
    const auto *dsc = static_cast<const unsigned long long *>(stage_in(stage_vals, scores, n * 8, st));
    uint8_t *done = score_done.get(n);
    cuda_check(cudaMemsetAsync(done, 0, n, st), "memset");
    for (auto &t : tables) {
      k_assign_scores<<<grid_for(n, 256, 0x7fffffffu), 256, 0, st>>>(t->dir(), t->L, t->slabs, dkeys, cfg.key_dtype,
                                                                      n, dsc, done);
      launched("k_assign_scores");
    }
    cuda_check(cudaStreamSynchronize(st), "sync");
  }

  void read_scores(const void *keys, size_t n, uint64_t *out, void *sp) {
    std::lock_guard<std::mutex> lock(mu);
    DeviceGuard dg(device);
    if (cfg.score_policy == SE_SCORE_NONE) throw Error(SE_ERR_RUNTIME, "the store keeps no scores (score policy none)");
    if (n == 0) return;
    cudaStream_t st = pick(sp);
    const void *dkeys = stage_in(stage_keys, keys, n * key_bytes(cfg.key_dtype), st);
    const bool host_out = !is_device_ptr(out);
    auto *dout = reinterpret_cast<unsigned long long *>(host_out ? stage_vals.get(n * 8) : static_cast<void *>(out));
    uint8_t *done = score_done.get(n);
    cuda_check(cudaMemsetAsync(done, 0, n, st), "memset");
    cuda_check(cudaMemsetAsync(dout, 0, n * 8, st), "memset");
    for (auto &t : tables) {
      k_read_scores<<<grid_for(n, 256, 0x7fffffffu), 256, 0, st>>>(t->dir(), t->L, t->slabs, dkeys, cfg.key_dtype, n,
                                                                    dout, done);
      launched("k_read_scores");
    }
    if (host_out) cuda_check(cudaMemcpyAsync(out, dout, n * 8, cudaMemcpyDeviceToHost, st), "copy out");
    cuda_check(cudaStreamSynchronize(st), "sync");
  }

  // ---- checkpoint interop ------------------------------------------------------
  Scratch<uint32_t> exp_flags, exp_at;
  Scratch<uint8_t> exp_tmp;

  // export_batch / export_opt_state_batch (hogwild_embedding_store.hpp:6112-6300):
  // lists the table's present keys; se_export_read copies slices of the list.
  uint64_t export_snapshot(int64_t dim, void *sp) {
    std::lock_guard<std::mutex> lock(mu);
    DeviceGuard dg(device);
    Table &t = table(dim);
    cudaStream_t st = pick(sp);
    const uint64_t nslots = t.nbuckets * kBucketSlots;
    if (nslots + 1 > 0x7fffffffull) throw Error(SE_ERR_NOT_IMPLEMENTED, "export of a directory above 2^31 slots");
    const int m = int(nslots + 1);
    uint32_t *flags = exp_flags.get(m), *at = exp_at.get(m);
    size_t tmp_bytes = 0;
    cuda_check(cub::DeviceScan::ExclusiveSum(nullptr, tmp_bytes, flags, at, m, st), "scan size");
    uint8_t *tmp = exp_tmp.get(tmp_bytes);
    k_export_flag<<<grid_for(uint64_t(m), 256, 0x7fffffffu), 256, 0, st>>>(t.dir(), nslots, flags);
    launched("k_export_flag");
    cuda_check(cub::DeviceScan::ExclusiveSum(tmp, tmp_bytes, flags, at, m, st), "scan");
    uint32_t last[2];
    cuda_check(cudaMemcpyAsync(&last[0], at + m - 1, 4, cudaMemcpyDeviceToHost, st), "read count");
    cuda_check(cudaMemcpyAsync(&last[1], flags + m - 1, 4, cudaMemcpyDeviceToHost, st), "read count");
    cuda_check(cudaStreamSynchronize(st), "sync");
    const uint64_t total = uint64_t(last[0]) + last[1];
    unsigned long long *keys = t.exp_keys.get(std::max<uint64_t>(total, 1));
    uint32_t *rows = t.exp_rows.get(std::max<uint64_t>(total, 1));
    k_export_list<<<grid_for(uint64_t(m), 256, 0x7fffffffu), 256, 0, st>>>(t.dir(), nslots, flags, at, keys, rows);
    launched("k_export_list");
    cuda_check(cudaStreamSynchronize(st), "sync");
    t.exp_count = total;
    t.exp_taken = true;
    return total;
  }

  void export_read(int64_t dim, uint64_t offset, uint64_t count, void *keys_out, void *values_out,
                   void *states_out, uint32_t *steps_out, void *sp) {
    std::lock_guard<std::mutex> lock(mu);
    DeviceGuard dg(device);
    Table &t = table(dim);
    if (!t.exp_taken) throw std::logic_error("se_export_read needs a snapshot (se_export_snapshot) of this table");
    if (offset > t.exp_count || count > t.exp_count - offset)
      throw std::invalid_argument("export slice is outside the snapshot");
    if (count == 0) return;
    cudaStream_t st = pick(sp);
    const size_t kb = key_bytes(cfg.key_dtype), vb = value_bytes(cfg.value_dtype) * size_t(dim);
    const size_t sb = value_bytes(cfg.optimizer_dtype) * size_t(dim) * t.L.nstate;
    // outputs in host memory go through one device buffer, copied back below
    struct Out { void *user; size_t bytes; size_t at; };
    Out outs[4] = {{keys_out, kb * count, 0}, {values_out, vb * count, 0}, {t.L.nstate ? states_out : nullptr,
                   sb * count, 0}, {steps_out, 4 * count, 0}};
    size_t staged = 0;
    for (auto &o : outs)
      if (o.user && !is_device_ptr(o.user)) {
        o.at = staged;
        staged += (o.bytes + 255) & ~size_t(255);
      }
    uint8_t *buf = staged ? stage_vals.get(staged) : nullptr;
    void *dev[4];
    for (int i = 0; i < 4; ++i)
      dev[i] = outs[i].user == nullptr ? nullptr : is_device_ptr(outs[i].user) ? outs[i].user : buf + outs[i].at;
    k_export_gather<32><<<grid_for(count * 32, 256, 0x7fffffffu), 256, 0, st>>>(
        t.L, t.slabs, t.exp_keys.ptr, t.exp_rows.ptr, offset, count, cfg.key_dtype, dev[0],
        static_cast<uint8_t *>(dev[1]), static_cast<uint8_t *>(dev[2]), static_cast<uint32_t *>(dev[3]));
    launched("k_export_gather");
    for (int i = 0; i < 4; ++i)
      if (outs[i].user && dev[i] != outs[i].user)
        cuda_check(cudaMemcpyAsync(outs[i].user, dev[i], outs[i].bytes, cudaMemcpyDeviceToHost, st), "copy out");
    if (staged) cuda_check(cudaStreamSynchronize(st), "sync");
  }

  // assign_opt_states (hogwild_embedding_store.hpp:6278-6351): all keys must be
  // present; nothing is written otherwise.
  void assign_opt_states(int64_t dim, const void *keys, size_t n, const void *states, size_t num_values,
                         const uint32_t *steps, void *sp) {
    std::lock_guard<std::mutex> lock(mu);
    DeviceGuard dg(device);
    if (dim <= 0) throw std::invalid_argument("assign_opt_states dimension has no physical table");
    Table *tp = nullptr;
    for (auto &x : tables)
      if (x->dim == dim) tp = x.get();
    if (tp == nullptr) throw std::invalid_argument("assign_opt_states dimension has no physical table");
    Table &t = *tp;
    if (!cfg.enable_optimizer || cfg.optimizer_kind == SE_OPT_NONE)
      throw std::invalid_argument("assign_opt_states dimension has no optimizer");
    const size_t opt_dim = size_t(dim) * t.L.nstate;
    if (opt_dim == 0 || num_values != n * opt_dim)
      throw std::invalid_argument("assign_opt_states payload size does not match dimension");
    if (n == 0) return;
    cudaStream_t st = pick(sp);
    const void *dkeys = stage_in(stage_keys, keys, n * key_bytes(cfg.key_dtype), st);
    const void *dstates = stage_in(stage_vals, states, num_values * value_bytes(cfg.optimizer_dtype), st);
    const uint32_t *dsteps = steps ? static_cast<const uint32_t *>(stage_in(stage_offs, steps, n * 4, st)) : nullptr;
    uint32_t *rows = bag_rows.get(n);
    uint32_t *mark = dup_words.get(2);
    cuda_check(cudaMemsetAsync(mark, 0, 4, st), "memset");
    k_opt_find<<<grid_for(n, 256, 0x7fffffffu), 256, 0, st>>>(t.dir(), dkeys, cfg.key_dtype, n, rows, mark);
    launched("k_opt_find");
    k_opt_assign<32><<<grid_for(n * 32, 256, 0x7fffffffu), 256, 0, st>>>(
        t.L, t.slabs, rows, n, static_cast<const uint8_t *>(dstates), dsteps, mark);
    launched("k_opt_assign");
    cuda_check(cudaMemcpyAsync(status_host, mark, 4, cudaMemcpyDeviceToHost, st), "read mark");
    cuda_check(cudaStreamSynchronize(st), "sync");
    if (status_host[0] != 0u) throw std::invalid_argument("assign_opt_states key is absent from dimension table");
  }

  // ---- embedding bag ------------------------------------------------------------
  // Offsets in host memory are checked (CSR: start at 0, non-decreasing, end
  // at n); device offsets are used as given, clamped by the kernels.
  static void check_offsets(const int64_t *offsets, size_t nbags, size_t n) {
    if (offsets == nullptr) throw std::invalid_argument("offsets is null");
    if (is_device_ptr(offsets)) return;
    if (offsets[0] != 0 || offsets[nbags] != int64_t(n))
      throw std::invalid_argument("offsets must start at 0 and end at the number of keys");
    for (size_t b = 0; b < nbags; ++b)
      if (offsets[b + 1] < offsets[b]) throw std::invalid_argument("offsets must be non-decreasing");
  }

  void embedding_bag(const void *keys, size_t n, const int64_t *offsets, size_t nbags, int64_t dim, void *out,
                     bool insert, void *sp) {
    std::lock_guard<std::mutex> lock(mu);
    DeviceGuard dg(device);
    if (dim <= 0) throw std::invalid_argument("dim must be > 0");
    Table &t = table(dim);
    if (nbags == 0) return;
    check_offsets(offsets, nbags, n);
    if (n > 0x7fffffffull) throw std::invalid_argument("batch exceeds 2^31 keys");
    cudaStream_t st = pick(sp);
    const size_t vb = value_bytes(cfg.value_dtype);
    const size_t out_bytes = nbags * size_t(dim) * vb;
    const void *dkeys = stage_in(stage_keys, keys, n * key_bytes(cfg.key_dtype), st);
    const auto *doffs = static_cast<const int64_t *>(stage_in(stage_offs, offsets, (nbags + 1) * 8, st));
    const bool host_out = !is_device_ptr(out);
    void *dout = host_out ? stage_vals.get(out_bytes) : out;
    uint32_t *rows = bag_rows.get(std::max<size_t>(n, 1));
    const bool vec4 = t.vec == 4;
    if (n > 0) {
      if (insert) {
        ensure_rows(t, n, st);
        cuda_check(cudaMemsetAsync(t.ctr + kCtrDeferred, 0, 4, st), "memset");
        uint32_t *dpos = t.def_pos.get(n);
        unsigned long long *dword = t.def_word.get(n);
        InitSpec init{cfg.init_kind, cfg.init_min, cfg.init_max - cfg.init_min,
                      cfg.optimizer_kind == SE_OPT_ADAGRAD ? cfg.initial_accumulator : 0.0f};
        auto go = [&](auto lanes_tag, auto vec_tag) {
          constexpr int LN = decltype(lanes_tag)::value;
          constexpr int VC = decltype(vec_tag)::value;
          Prof pr(this, "k_bag_insert", st);
          k_bag_insert<LN, VC><<<grid_for(n * LN, 256, 0x7fffffffu), 256, 0, st>>>(
              t.dir(), t.L, t.slabs, t.alloc(), init, dkeys, cfg.key_dtype, n, rows, t.ctr + kCtrDeferred, dpos,
              dword, t.ctr + kCtrStatus);
          launched("k_bag_insert");
        };
        // 4 lanes per key: only lane 0 probes, the others help initialise
        // new rows (measured: 32 lanes per key left SMs issue-bound)
        if (vec4) go(std::integral_constant<int, 4>{}, std::integral_constant<int, 4>{});
        else go(std::integral_constant<int, 4>{}, std::integral_constant<int, 1>{});
        k_bag_deferred<<<grid_for(n, 256, 148 * 4), 256, 0, st>>>(t.ctr + kCtrDeferred, dpos, dword, rows,
                                                                  t.ctr + kCtrStatus);
        launched("k_bag_deferred");
      } else {
        Prof pr(this, "k_bag_find", st);
        k_bag_find<<<grid_for(n, 256, 0x7fffffffu), 256, 0, st>>>(t.dir(), dkeys, cfg.key_dtype, n, rows);
        launched("k_bag_find");
      }
    }
    const bool pool4 = vec4 && uintptr_t(dout) % 16 == 0;
    auto pool = [&](auto lanes_tag, auto vec_tag) {
      constexpr int LN = decltype(lanes_tag)::value;
      constexpr int VC = decltype(vec_tag)::value;
      Prof pr(this, "k_bag_pool", st);
      k_bag_pool<LN, VC><<<grid_for(nbags * LN, 256, 148 * 64), 256, 0, st>>>(t.L, t.slabs, rows, n, doffs, nbags,
                                                                               dout);
      launched("k_bag_pool");
    };
    auto pool_lanes = [&](auto vec_tag) {
      switch (pick_lanes(pool4 ? uint64_t(dim) / 4 : uint64_t(dim))) {
      case 4: pool(std::integral_constant<int, 4>{}, vec_tag); break;
      case 8: pool(std::integral_constant<int, 8>{}, vec_tag); break;
      case 16: pool(std::integral_constant<int, 16>{}, vec_tag); break;
      default: pool(std::integral_constant<int, 32>{}, vec_tag); break;
      }
    };
    if (pool4) pool_lanes(std::integral_constant<int, 4>{});
    else pool_lanes(std::integral_constant<int, 1>{});
    if (host_out) {
      cuda_check(cudaMemcpyAsync(out, dout, out_bytes, cudaMemcpyDeviceToHost, st), "copy out");
      cuda_check(cudaStreamSynchronize(st), "sync");
      if (insert) check_status(t, st);
    } else if (!is_device_ptr(keys) || !is_device_ptr(offsets)) {
      cuda_check(cudaStreamSynchronize(st), "sync");  // the staging buffers are reused by the next call
    }
  }

  // Backward of the sum pooling: every key of bag b accumulates pooled_grads[b]
  // (accumulate_gradients of the expanded rows, without expanding them).
  void embedding_bag_backward(const void *keys, size_t n, const int64_t *offsets, size_t nbags, int64_t dim,
                              const void *pooled_grads, void *sp) {
    std::lock_guard<std::mutex> lock(mu);
    DeviceGuard dg(device);
    if (dim <= 0) throw std::invalid_argument("gradient row length must be positive");
    table(dim);
    if (nbags == 0 || n == 0) return;
    check_offsets(offsets, nbags, n);
    if (n > 0x7fffffffull) throw std::invalid_argument("batch exceeds 2^31 keys");
    cudaStream_t st = pick(sp);
    const auto *doffs = static_cast<const int64_t *>(stage_in(stage_offs, offsets, (nbags + 1) * 8, st));
    uint32_t *bag_of = bag_of_buf.get(n);
    cuda_check(cudaMemsetAsync(bag_of, 0, n * 4, st), "memset");
    k_bag_of<<<grid_for(nbags * 32, 256, 148 * 32), 256, 0, st>>>(doffs, nbags, n, bag_of);
    launched("k_bag_of");
    accumulate_locked(keys, n, nullptr, dim, pooled_grads, sp, -1, nullptr, bag_of, nbags);
  }

  void accumulate(const void *keys, size_t n, int64_t dim, const void *grads, void *sp) {
    std::lock_guard<std::mutex> lock(mu);
    accumulate_locked(keys, n, nullptr, dim, grads, sp);
  }

  // n_dev: optional device count (<= n) of the rows to take, for batches
  // whose size is only known on the device (exchanged batches); kdt: key
  // dtype of `keys` when it differs from the store's (exchanged keys are u64).
  // known_rows: the rows of `keys` when the caller resolved them already.
  // grad_row: device array, the row of `grads` (grad_rows rows) that entry i
  // takes (embedding-bag backward); null: row i.
  void accumulate_locked(const void *keys, size_t n, const uint32_t *n_dev, int64_t dim, const void *grads,
                         void *sp, int kdt = -1, const uint32_t *known_rows = nullptr,
                         const uint32_t *grad_row = nullptr, size_t grad_rows = 0) {
    DeviceGuard dg(device);
    if (dim <= 0) throw std::invalid_argument("gradient row length must be positive");
    Table &t = table(dim);
    if (n == 0) return;
    cudaStream_t st = pick(sp);
    if (t.atomic) {
      accumulate_atomic(t, keys, n, n_dev, grads, st, kdt, grad_row, grad_rows);
      return;
    }
    ensure_pending(t, n, st);
    const size_t gb = value_bytes(cfg.gradient_dtype);
    if (kdt < 0) kdt = cfg.key_dtype;
    const void *dkeys = stage_in(stage_keys, keys, n * key_bytes(kdt), st);
    const void *dgrads = stage_in(stage_vals, grads, (grad_row ? grad_rows : n) * size_t(dim) * gb, st);
    const float maxv = std::min(host_dtype_max(cfg.gradient_dtype), host_dtype_max(cfg.value_dtype));
    // dim % 4 == 0 keeps every appended row 16-byte (fp32) / 8-byte aligned.
    const bool vec4 = dim % 4 == 0 && uintptr_t(dgrads) % 16 == 0;
    // Host inputs: validate_input semantics of the reference - the call waits
    // for its check and raises before anything is accumulated. Device inputs:
    // the check runs on the device without stalling the stream; a failing
    // batch poisons the window (optimizer_step then applies nothing) and the
    // error is raised by the next synchronising call.
    const bool device_inputs = dkeys == keys && dgrads == grads;
    uint32_t *status_word = t.ctr + (device_inputs ? kCtrPoison : kCtrGradStatus);
    if (!device_inputs) {
      cuda_check(cudaMemsetAsync(status_word, 0, 4, st), "status clear");
      cuda_check(cudaMemcpyAsync(t.ctr + kCtrPendingBackup, t.ctr + kCtrPending, 4, cudaMemcpyDeviceToDevice, st),
                 "pending backup");
    }
    const CountWs cw = t.count_ws();
    {
      Prof pr(this, "k_accumulate", st);
      const size_t chunks = n * size_t(dim) / (vec4 ? 4 : 1);
      // 4 blocks per SM: enough 16-byte loads in flight to stream the rows,
      // and few blocks to count in for the commit
      const unsigned grid = grid_for(std::max(chunks, n), 256, 148 * 4);
      auto go = [&](auto kern) {
        pdl(kern, grid, 256, 0, st, t.dir(), dkeys, kdt, n, n_dev, dgrads, cfg.gradient_dtype, uint32_t(dim),
            cfg.gradient_scale, maxv, t.pkeys, t.prows, t.pgrads, size_t(t.pcap), t.ctr + kCtrPending,
            t.ctr + kCtrAccDone, status_word, t.ctr + kCtrStatus, cw, device_inputs ? 1 : 0, known_rows, grad_row,
            t.fwd_cache());
      };
      if (grad_row) {
        if (vec4) go(k_accumulate<4, true>);
        else go(k_accumulate<1, true>);
      } else {
        if (vec4) go(k_accumulate<4, false>);
        else go(k_accumulate<1, false>);
      }
      launched("k_accumulate");
    }
    if (!device_inputs) {
      // the rows just written are only kept when the whole batch passed
      cuda_check(cudaMemcpyAsync(status_host, status_word, 4, cudaMemcpyDeviceToHost, st), "status");
      cuda_check(cudaStreamSynchronize(st), "sync");
      if (status_host[0] & kStatusBadGradient) {
        cuda_check(cudaMemsetAsync(status_word, 0, 4, st), "status clear");
        cuda_check(cudaMemcpyAsync(t.ctr + kCtrPending, t.ctr + kCtrPendingBackup, 4, cudaMemcpyDeviceToDevice, st),
                   "pending rollback");
        cuda_check(cudaStreamSynchronize(st), "sync");
        throw std::overflow_error("gradient scale storage exceeds configured dtype");
      }
      // the batch is kept: count its rows for the step's grouping
      pdl(k_count_range, grid_for(n, 256, 148 * 4), 256, 0, st, t.prows, t.ctr + kCtrPendingBackup, uint32_t(n),
                                                               uint32_t(t.pcap), cw);
      launched("k_count_range");
    }
    t.pcount += n;  // upper bound of the rows pending on the device
  }

  // accumulate_gradients in atomic mode: the rows are added into the
  // window's per-key sums (k_acc_atomic). Host inputs are validated first and
  // the call raises before anything is added; device inputs are validated on
  // the device and a failing batch poisons the window (see accumulate_locked).
  void accumulate_atomic(Table &t, const void *keys, size_t n, const uint32_t *n_dev, const void *grads,
                         cudaStream_t st, int kdt, const uint32_t *grad_row, size_t grad_rows) {
    ensure_acc(t, n, st);
    const size_t gb = value_bytes(cfg.gradient_dtype);
    if (kdt < 0) kdt = cfg.key_dtype;
    const int64_t dim = t.dim;
    const void *dkeys = stage_in(stage_keys, keys, n * key_bytes(kdt), st);
    const size_t grad_elems = (grad_row ? grad_rows : n) * size_t(dim);
    const void *dgrads = stage_in(stage_vals, grads, grad_elems * gb, st);
    const float maxv = std::min(host_dtype_max(cfg.gradient_dtype), host_dtype_max(cfg.value_dtype));
    const bool vec4 = dim % 4 == 0 && uintptr_t(dgrads) % (cfg.gradient_dtype == SE_FLOAT32 ? 16 : 8) == 0;
    const bool device_inputs = dkeys == keys && dgrads == grads;
    uint32_t *status_word = t.ctr + (device_inputs ? kCtrPoison : kCtrGradStatus);
    if (!device_inputs) {
      cuda_check(cudaMemsetAsync(status_word, 0, 4, st), "status clear");
      {
        Prof pr(this, "k_acc_check", st);
        if (vec4) pdl(k_acc_check<4>, grid_for(grad_elems / 4, 256, 148 * 8), 256, 0, st, dgrads,
                      cfg.gradient_dtype, grad_elems, cfg.gradient_scale, maxv, status_word);
        else pdl(k_acc_check<1>, grid_for(grad_elems, 256, 148 * 8), 256, 0, st, dgrads, cfg.gradient_dtype,
                 grad_elems, cfg.gradient_scale, maxv, status_word);
        launched("k_acc_check");
      }
      cuda_check(cudaMemcpyAsync(status_host, status_word, 4, cudaMemcpyDeviceToHost, st), "status");
      cuda_check(cudaStreamSynchronize(st), "sync");
      if (status_host[0] & kStatusBadGradient) {
        cuda_check(cudaMemsetAsync(status_word, 0, 4, st), "status clear");
        cuda_check(cudaStreamSynchronize(st), "sync");
        throw std::overflow_error("gradient scale storage exceeds configured dtype");
      }
    }
    {
      Prof pr(this, "k_acc_atomic", st);
      // rows per block: the table's tile, or fewer so that a batch of about
      // one wave spreads evenly (4 resident blocks on each of the 148 SMs)
      const uint32_t tile = uint32_t(std::min<size_t>(t.acc_tile, std::max<size_t>(32, (n + 591) / 592)));
      const unsigned grid = grid_for(n, tile, 0x7fffffffu);
      const size_t smem = size_t(tile) * size_t(dim) * 4;  // the tile's rows (fp32 or 16-bit)
      auto go = [&](auto kern) {
        allow_dynamic_smem(kern, smem);
        pdl(kern, grid, kAccThreads, smem, st, t.acc_tab(), dkeys, kdt, n, n_dev, dgrads, cfg.gradient_dtype,
            cfg.gradient_scale, maxv, tile, t.acc_hbits, status_word, t.ctr + kCtrStatus, grad_row,
            t.fwd_cache());
      };
      if (grad_row) {
        if (vec4) go(k_acc_atomic<4, true>);
        else go(k_acc_atomic<1, true>);
      } else {
        if (vec4) go(k_acc_atomic<4, false>);
        else go(k_acc_atomic<1, false>);
      }
      launched("k_acc_atomic");
    }
    if (!device_inputs) cuda_check(cudaStreamSynchronize(st), "sync");  // staging buffers are reused
    t.pcount += n;  // upper bound of the window's distinct keys
  }

  // optimizer_step of an atomic-mode table (apply = 0: the window is only cleared).
  void step_atomic(Table &t, size_t nsteps, bool apply, cudaStream_t st) {
    OptSpec o = opt_spec(t, nsteps);
    // the sums are fp32: used as they are only for fp32 parameters and factor 1
    o.raw = cfg.value_dtype == SE_FLOAT32 && nsteps == 1 && cfg.gradient_scale == 1.0f;
    auto *dropped = reinterpret_cast<unsigned long long *>(t.ctr + kCtrDropped);
    const uint64_t slots = std::min<uint64_t>(t.pcount, t.acc_slots + 1);
    auto go = [&](auto lanes_tag, auto vec_tag) {
      constexpr int LN = decltype(lanes_tag)::value;
      constexpr int VC = decltype(vec_tag)::value;
      // one wave (3 blocks per SM); the groups stride over the slots, so no
      // block of a later wave starts only to find nothing to do
      const unsigned grid = grid_for(slots * LN, 256, 148 * 3);
      Prof pr(this, "k_acc_apply", st);
      auto launch = [&](auto kern) {
        pdl(kern, grid, 256, 0, st, t.acc_tab(), t.dir(), t.L, t.slabs, o, apply ? 1 : 0, dropped);
      };
      const bool dyn = cfg.lr_policy != SE_LR_CONSTANT;
      if (o.kind == SE_OPT_ADAM) {
        if (dyn) launch(k_acc_apply<LN, VC, true, SE_OPT_ADAM>);
        else launch(k_acc_apply<LN, VC, false, SE_OPT_ADAM>);
      } else if (o.kind == SE_OPT_ADAGRAD) {
        if (dyn) launch(k_acc_apply<LN, VC, true, SE_OPT_ADAGRAD>);
        else launch(k_acc_apply<LN, VC, false, SE_OPT_ADAGRAD>);
      } else {  // SGD, or no optimizer (the window is only cleared)
        if (dyn) launch(k_acc_apply<LN, VC, true, SE_OPT_SGD>);
        else launch(k_acc_apply<LN, VC, false, SE_OPT_SGD>);
      }
      launched("k_acc_apply");
    };
    auto by_lanes = [&](auto vec_tag) {
      // few lanes per slot, each with several chunks in flight: one wave of groups
      const uint32_t ln = gather_lanes(uint64_t(t.dim) / uint64_t(decltype(vec_tag)::value));
      switch (ln) {
      case 4: go(std::integral_constant<int, 4>{}, vec_tag); break;
      case 8: go(std::integral_constant<int, 8>{}, vec_tag); break;
      case 16: go(std::integral_constant<int, 16>{}, vec_tag); break;
      default: go(std::integral_constant<int, 32>{}, vec_tag); break;
      }
    };
    if (t.vec == 4) by_lanes(std::integral_constant<int, 4>{});
    else by_lanes(std::integral_constant<int, 1>{});
  }

  OptSpec opt_spec(const Table &t, size_t nsteps) const {
    OptSpec o{};
    o.kind = cfg.optimizer_kind;
    o.lr = cfg.lr;
    o.b1 = cfg.beta1;
    o.b2 = cfg.beta2;
    o.eps = cfg.eps;
    o.wd = cfg.weight_decay;
    o.omb1 = 1.0f - cfg.beta1;
    o.omb2 = 1.0f - cfg.beta2;
    const uint32_t wdt = uint32_t(cfg.simd_width > 0 ? cfg.simd_width : 1);
    o.simd_cut = (uint32_t(t.dim) / wdt) * wdt;
    o.bc = bc;
    o.factor = cfg.gradient_scale / float(nsteps);
    o.raw = cfg.gradient_dtype == cfg.value_dtype && nsteps == 1 && cfg.gradient_scale == 1.0f;
    o.poison = t.ctr + kCtrPoison;
    o.lr_kind = cfg.lr_policy;
    o.lr_min_ratio = cfg.lr_min_ratio;
    o.lr_max_score = lr_max;
    o.lr_lut = lr_lut;
    return o;
  }

  void optimizer_step(size_t nsteps, void *sp) {
    std::lock_guard<std::mutex> lock(mu);
    DeviceGuard dg(device);
    if (nsteps == 0) throw std::invalid_argument("normalization_steps must be positive");
    cudaStream_t st = pick(sp);
    const bool apply = cfg.enable_optimizer && cfg.optimizer_kind != SE_OPT_NONE;
    if (apply && cfg.optimizer_kind == SE_OPT_ADAM) ensure_bc(steps_taken + 2);
    steps_taken += 1;
    for (auto &tp : tables) {
      Table &t = *tp;
      if (t.pcount == 0) continue;
      if (t.atomic) {
        step_atomic(t, nsteps, apply, st);
      } else if (apply) {
        step_table(t, nsteps, st);  // its last kernel clears the window's counters
      } else {
        cuda_check(cudaMemsetAsync(t.ctr + kCtrGroup, 0, 16, st), "memset group counters");
        cuda_check(cudaMemsetAsync(t.ctr + kCtrUnres, 0, 4, st), "memset unresolved counter");
        cuda_check(cudaMemsetAsync(t.ctr + kCtrPending, 0, 4, st), "pending clear");
      }
      t.pcount = 0;
    }
  }

  void step_table(Table &t, size_t nsteps, cudaStream_t st) {
    const uint32_t P = uint32_t(t.pcount);
    GroupWs w{};
    w.rows = t.prows;
    w.row_cnt = t.row_cnt;
    w.row_seg = t.row_seg;
    w.seg_row = t.seg_row;  // filled as the entries were counted
    w.seg_cnt = t.g_seg_cnt.get(P);
    w.seg_off = t.g_seg_off.get(P);
    const size_t fill_cap_before = t.g_seg_fill.cap;
    w.seg_fill = t.g_seg_fill.get(P);
    if (t.g_seg_fill.cap != fill_cap_before || t.seg_fill_zeroed < P) {
      // placement counters are reset by the apply kernels after use; a new
      // or grown buffer starts from zero
      cuda_check(cudaMemsetAsync(w.seg_fill, 0, t.g_seg_fill.cap * 4, st), "memset seg_fill");
      t.seg_fill_zeroed = t.g_seg_fill.cap;
    }
    w.pos = t.g_pos.get(P);
    {
      const uint32_t lna = t.vec == 4 ? t.lanes : pick_lanes(uint64_t(t.dim));
      w.short_max = lna;                            // one slot per lane
      w.long_max = uint32_t(kApplySlots) * lna;     // larger: k_group_hot
      w.long_list = t.g_long.get(P);
    }
    // Upper bound on k_group_hot work items: segments of more than `lanes`
    // rows, each cut into max(ceil(rows / kPartEntries), ceil(P / window)) parts.
    // Sorted placement (more than one window of pending rows): no window
    // minimum, and only segments of more than long_max rows are items.
    const bool sorted = P > kHotWindowBits && P <= 0x7fffffffu;  // the sort takes an int count
    const uint64_t min_parts = (uint64_t(P) + kHotWindowBits - 1) / kHotWindowBits;
    const uint64_t max_items =
        sorted ? uint64_t(P) / kPartEntries + uint64_t(P) / (uint64_t(w.long_max) + 1) + 1
               : uint64_t(P) / kPartEntries + 1 + (uint64_t(P) / 5 + 1) * (min_parts + 1);
    w.items = reinterpret_cast<uint4 *>(t.g_items.get(max_items));
    w.partials = t.g_partials.get(max_items * uint64_t(t.dim));
    w.ctr = t.ctr + kCtrGroup;
    w.cap = P;
    // More pending rows than one hot-key window: segments are laid out by a
    // sort instead of windowed bitmaps (each bitmap pass costs P/32 words).
    w.sorted = sorted ? 1u : 0u;
    w.status = t.ctr + kCtrStatus;
    // ctr[0] (segments) was counted with the entries; ctr[1..3] are zero
    // (cleared with the window's other counters by the previous step)
    w.done = t.ctr + kCtrStepDone;
    w.unres_ctr = t.ctr + kCtrUnres;
    w.pending = t.ctr + kCtrPending;
    auto *dropped = reinterpret_cast<unsigned long long *>(t.ctr + kCtrDropped);
    const unsigned g = grid_for(P, 256);
    {
      Prof pr(this, "k_group_fix", st);
      pdl(k_group_fix, 148, 256, 0, st, t.dir(), t.pkeys, t.ctr + kCtrPending, w, t.count_ws(), dropped);
      launched("k_group_fix");
    }
    {
      Prof pr(this, "k_group_alloc", st);
      pdl(k_group_alloc, g, 256, 0, st, w, t.ctr + kCtrPending);
      launched("k_group_alloc");
    }
    if (w.sorted) {
      // stable sort of (segment's first slot, position): the key needs
      // bits for every slot below P plus one key past them
      int end_bit = 1;
      while ((uint64_t(1) << end_bit) <= uint64_t(P)) ++end_bit;
      uint32_t *kin = t.g_sort_kin.get(P), *kout = t.g_sort_kout.get(P), *vin = t.g_sort_vin.get(P);
      size_t tmp_bytes = 0;
      cuda_check(cub::DeviceRadixSort::SortPairs(nullptr, tmp_bytes, kin, kout, vin, w.pos, int(P), 0, end_bit, st),
                 "sort size");
      uint8_t *tmp = t.g_sort_tmp.get(tmp_bytes);
      {
        Prof pr(this, "k_group_sortkeys", st);
        pdl(k_group_sortkeys, g, 256, 0, st, t.ctr + kCtrPending, w, kin, vin, uint32_t((uint64_t(1) << end_bit) - 1));
        launched("k_group_sortkeys");
      }
      Prof pr(this, "k_group_place", st);
      cuda_check(cub::DeviceRadixSort::SortPairs(tmp, tmp_bytes, kin, kout, vin, w.pos, int(P), 0, end_bit, st),
                 "sort");
    } else {
      Prof pr(this, "k_group_place", st);
      pdl(k_group_place, g, 256, 0, st, t.ctr + kCtrPending, w);
      launched("k_group_place");
    }
    const OptSpec o = opt_spec(t, nsteps);
    const int gdt = cfg.gradient_dtype;
    auto go = [&](auto lanes_tag, auto vec_tag) {
      constexpr int LN = decltype(lanes_tag)::value;
      constexpr int VC = decltype(vec_tag)::value;
      // k_group_hot first (its blocks take whole SMs), k_group_apply beside it
      auto launch = [&](auto dyn_tag) {
        constexpr bool DY = decltype(dyn_tag)::value;
        {
          Prof pr(this, "k_group_hot", st);
          pdl(k_group_hot<LN, VC, DY>, 128, kBlockThreads, 0, st, t.L, t.slabs, o, gdt, t.pgrads, w,
              t.ctr + kCtrPending);
          launched("k_group_hot");
        }
        Prof pr(this, "k_group_apply", st);
        pdl(k_group_apply<LN, VC, DY>, grid_for(size_t(P) * LN, 256, 148 * 8), 256, 0, st,
            t.L, t.slabs, o, gdt, t.pgrads, w, t.ctr + kCtrPending);
        launched("k_group_apply");
      };
      if (cfg.lr_policy != SE_LR_CONSTANT) launch(std::true_type{});
      else launch(std::false_type{});
    };
    auto by_lanes = [&](auto vec_tag) {
      const uint32_t ln = decltype(vec_tag)::value == 4 ? t.lanes : pick_lanes(uint64_t(t.dim));
      switch (ln) {
      case 4: go(std::integral_constant<int, 4>{}, vec_tag); break;
      case 8: go(std::integral_constant<int, 8>{}, vec_tag); break;
      case 16: go(std::integral_constant<int, 16>{}, vec_tag); break;
      default: go(std::integral_constant<int, 32>{}, vec_tag); break;
      }
    };
    if (t.vec == 4) by_lanes(std::integral_constant<int, 4>{});
    else by_lanes(std::integral_constant<int, 1>{});
  }

  // clear (hogwild_embedding_store.hpp:5107-5154): every key of every table
  // is removed, the arenas are reset and the gradients of the current window
  // are discarded; capacity is kept. The store-wide LRU clock keeps running,
  // as the reference's score policy does.
  void clear(void *sp) {
    std::lock_guard<std::mutex> lock(mu);
    DeviceGuard dg(device);
    cudaStream_t st = pick(sp);
    for (auto &tp : tables) {
      Table &t = *tp;
      cuda_check(cudaMemsetAsync(t.buckets, 0xff, t.nbuckets * sizeof(Bucket), st), "clear directory");
      cuda_check(cudaMemsetAsync(t.ctr, 0, kCtrWords * 4, st), "clear counters");
      cuda_check(cudaMemsetAsync(t.ctr + kCtrSpecialRow, 0xff, 4, st), "clear special");
      cuda_check(cudaMemsetAsync(t.row_cnt, 0, t.capacity * 4, st), "clear row counters");
      if (t.acc_slots) {
        cuda_check(cudaMemsetAsync(t.acc_keys, 0xff, (t.acc_slots + 1) * sizeof(ulonglong2), st), "clear sums");
        cuda_check(cudaMemsetAsync(t.acc_vals, 0, size_t(t.acc_vcap) * size_t(t.dim) * 4, st), "clear sums");
        cuda_check(cudaMemsetAsync(t.acc_cnt, 0, (t.acc_slots + 1) * 4, st), "clear sums");
        cuda_check(cudaMemsetAsync(t.acc_ctr, 0, 16, st), "clear sums");
      }
      t.pcount = 0;
      t.rows_bound = 0;
      t.bound_stale = false;
      t.tombs = 0;
      t.erased = false;
      t.exp_count = 0;
      t.exp_taken = false;
    }
    cuda_check(cudaStreamSynchronize(st), "sync");
  }

  void read_state(int64_t dim, uint64_t key, void *param_out, void *state_out, uint32_t *step_out,
                  int32_t *found) {
    std::lock_guard<std::mutex> lock(mu);
    DeviceGuard dg(device);
    Table &t = table(dim);
    cudaStream_t st = own;
    cuda_check(cudaDeviceSynchronize(), "sync");
    auto *dk = dalloc<unsigned long long>(1);
    auto *dr = dalloc<uint32_t>(1);
    unsigned long long k = key;
    cuda_check(cudaMemcpy(dk, &k, 8, cudaMemcpyHostToDevice), "copy");
    k_find_rows<<<1, 32, 0, st>>>(t.dir(), dk, 1, dr);
    launched("k_find_rows");
    uint32_t row = kNoRow;
    cuda_check(cudaMemcpyAsync(&row, dr, 4, cudaMemcpyDeviceToHost, st), "copy");
    cuda_check(cudaStreamSynchronize(st), "sync");
    dfree(dk);
    dfree(dr);
    *found = row != kNoRow;
    if (row == kNoRow) return;
    std::vector<uint8_t> slab(t.L.stride);
    cuda_check(cudaMemcpy(slab.data(), t.slabs + size_t(row) * t.L.stride, t.L.stride,
                          cudaMemcpyDeviceToHost), "copy slab");
    const size_t pb = size_t(t.dim) * value_bytes(cfg.value_dtype);
    const size_t ob = size_t(t.dim) * value_bytes(cfg.optimizer_dtype);
    if (param_out) std::memcpy(param_out, slab.data(), pb);
    if (state_out && t.L.nstate >= 1) std::memcpy(state_out, slab.data() + t.L.state0, ob);
    if (state_out && t.L.nstate >= 2)
      std::memcpy(static_cast<uint8_t *>(state_out) + ob, slab.data() + t.L.state1, ob);
    if (step_out) {
      uint32_t s = 0;
      if (t.L.nstate >= 2) std::memcpy(&s, slab.data() + t.L.step, 4);
      *step_out = s;
    }
  }
};

// ---------------------------------------------------------------------------
// Peer-memory exchange (kernels in se_exchange.cuh)
// ---------------------------------------------------------------------------

constexpr size_t kIpcHandleBytes = sizeof(cudaIpcMemHandle_t);

struct ExchangeImpl {
  StoreImpl *store = nullptr;
  int device = 0;
  uint32_t W = 1, me = 0;
  uint64_t M = 0;  // keys per rank per call
  int64_t dim = 0;
  PartSpec spec{};
  uint8_t *arena = nullptr;
  size_t arena_bytes = 0;
  std::vector<uint8_t *> peers;    // arena of every rank in this process's address space
  std::vector<bool> opened;        // peers[r] came from cudaIpcOpenMemHandle
  uint8_t **d_peers = nullptr;     // device copy of `peers`
  ExView view{};
  bool connected = false;
  // route scratch of the forward and backward direction
  uint32_t *route[2] = {nullptr, nullptr};
  uint32_t tiles_cap = 0;
  uint32_t *status_host = nullptr;  // pinned
  // (owner, slot) of every key of the last forward (of every distinct key
  // when it was deduplicated), and its batch size
  uint32_t *key_pid = nullptr, *key_slot = nullptr;
  size_t last_fwd_n = 0;
  bool have_fwd = false;
  // sender-side dedupe (se_exchange_set_dedupe): workspace, distinct keys of
  // the batch (key dtype), fp32 per-key gradient sums of the routed backward
  bool dedupe = false, fwd_deduped = false;
  uint32_t parity = 0;
  unsigned long long *dd_set = nullptr;
  uint32_t *dd_idx = nullptr, *dd_pos_slot = nullptr, *dd_uslot = nullptr, *dd_inverse = nullptr, *dd_ctr = nullptr;
  uint8_t *dd_ukeys = nullptr;
  float *dd_pre = nullptr;
  uint64_t dd_slots = 0;

  ~ExchangeImpl() {
    DeviceGuard dg(device);
    cudaDeviceSynchronize();
    for (uint32_t r = 0; r < peers.size(); ++r)
      if (opened[r]) cudaIpcCloseMemHandle(peers[r]);
    dfree(d_peers);
    dfree(arena);
    dfree(route[0]);
    dfree(route[1]);
    dfree(key_pid);
    dfree(key_slot);
    dfree(dd_set);
    dfree(dd_idx);
    dfree(dd_pos_slot);
    dfree(dd_uslot);
    dfree(dd_inverse);
    dfree(dd_ctr);
    dfree(dd_ukeys);
    dfree(dd_pre);
    if (status_host) cudaFreeHost(status_host);
  }

  // Sender-side dedupe of forwards (and pre-reduction of the gradient batch
  // routed like them). Every rank of the exchange must make the same choice.
  void set_dedupe(bool enable) {
    DeviceGuard dg(device);
    std::lock_guard<std::mutex> lock(store->mu);
    if (enable && dd_set == nullptr) {
      dd_slots = next_pow2(std::max<uint64_t>(2 * M, 64));
      dd_set = dalloc<unsigned long long>(dd_slots);
      dd_idx = dalloc<uint32_t>(dd_slots + 1);
      dd_pos_slot = dalloc<uint32_t>(M);
      dd_uslot = dalloc<uint32_t>(M);
      dd_inverse = dalloc<uint32_t>(M);
      dd_ctr = dalloc<uint32_t>(8);
      dd_ukeys = dalloc<uint8_t>(M * 8);
      dd_pre = dalloc<float>(M * size_t(dim));
      cuda_check(cudaMemset(dd_set, 0xff, dd_slots * 8), "memset dedupe");
      cuda_check(cudaMemset(dd_ctr, 0, 32), "memset dedupe");
      cuda_check(cudaMemset(dd_pre, 0, M * size_t(dim) * 4), "memset dedupe");
      cuda_check(cudaDeviceSynchronize(), "sync");
    }
    dedupe = enable;
  }

  DedupeWs dedupe_ws() const {
    return DedupeWs{dd_set, dd_idx, dd_pos_slot, dd_uslot, dd_inverse, dd_ctr + parity, dd_ctr + 2 + parity,
                    dd_ctr + (parity ^ 1u), dd_ctr + 2 + (parity ^ 1u), dd_ctr + 4, uint32_t(dd_slots - 1)};
  }

  void create(StoreImpl *s, int kind, uint32_t world, uint32_t rank, uint64_t max_keys, int64_t row_dim,
              uint32_t timeout_ms) {
    if (world == 0 || world > kExMaxRanks) throw std::invalid_argument("world_size must be in [1, 64]");
    if (rank >= world) throw std::invalid_argument("rank must be < world_size");
    if (max_keys == 0 || max_keys > (1ull << 26)) throw std::invalid_argument("max_keys_per_rank must be in [1, 2^26]");
    if (uint64_t(world) * max_keys >= (1ull << 32))
      throw std::invalid_argument("world_size * max_keys_per_rank must be below 2^32");
    if (row_dim <= 0) throw std::invalid_argument("dim must be > 0");
    if (timeout_ms == 0) throw std::invalid_argument("timeout_ms must be > 0");
    store = s;
    device = s->device;
    s->table(row_dim);  // the dim must have a table
    W = world;
    me = rank;
    M = max_keys;
    dim = row_dim;
    spec = make_spec(kind, world);
    DeviceGuard dg(device);
    const uint64_t WM = uint64_t(W) * M;
    const uint32_t row_bytes = uint32_t(dim * int64_t(value_bytes(s->cfg.value_dtype)));
    const uint32_t grad_bytes = uint32_t(dim * int64_t(value_bytes(s->cfg.gradient_dtype)));
    auto up = [](uint64_t x) { return (x + 255u) & ~uint64_t(255u); };
    uint64_t o = 0;
    auto take = [&](uint64_t bytes) {
      const uint64_t at = o;
      o = up(o + bytes);
      return at;
    };
    view.W = W;
    view.me = me;
    view.M = uint32_t(M);
    view.row_bytes = row_bytes;
    view.grad_bytes = grad_bytes;
    view.timeout_ns = uint64_t(timeout_ms) * 1000000ull;
    view.o_flags = take(4ull * kExKinds * W);
    view.o_epochs = take(4ull * kExKinds);
    view.o_words = take(4ull * kExWords);
    view.o_prefix = take(4ull * (W + 1));
    view.o_counts = take(4ull * W * W);
    view.o_gcounts = take(4ull * W * W);
    view.o_inkeys = take(8 * WM);
    view.o_inpos = take(4 * WM);
    view.o_inrow = take(4 * WM);
    view.o_gkeys = take(8 * WM);
    view.o_ingrads = take(WM * grad_bytes);
    view.o_rows = take(M * row_bytes);
    arena_bytes = o;
    arena = dalloc<uint8_t>(arena_bytes);
    cuda_check(cudaMemset(arena, 0, arena_bytes), "memset exchange arena");
    tiles_cap = uint32_t((M + kExTile - 1) / kExTile);
    for (auto &r : route) r = dalloc<uint32_t>(2 * size_t(tiles_cap) * W + W);
    key_pid = dalloc<uint32_t>(M);
    key_slot = dalloc<uint32_t>(M);
    d_peers = dalloc<uint8_t *>(W);
    cuda_check(cudaMallocHost(&status_host, 16), "cudaMallocHost");
    peers.assign(W, nullptr);
    opened.assign(W, false);
    peers[me] = arena;
    cuda_check(cudaDeviceSynchronize(), "sync");
  }

  void handle(void *out, size_t bytes) const {
    if (bytes < kIpcHandleBytes) throw std::invalid_argument("handle buffer is smaller than a CUDA IPC handle");
    DeviceGuard dg(device);
    cudaIpcMemHandle_t h;
    cuda_check(cudaIpcGetMemHandle(&h, arena), "cudaIpcGetMemHandle");
    std::memcpy(out, &h, kIpcHandleBytes);
  }

  void finish_connect() {
    cuda_check(cudaMemcpy(d_peers, peers.data(), W * sizeof(uint8_t *), cudaMemcpyHostToDevice), "upload peers");
    {  // the owner kernel's counters start at zero (its last block resets them after every launch)
      std::lock_guard<std::mutex> lock(store->mu);
      Table &t = store->table(dim);
      cuda_check(cudaMemset(t.ctr + kCtrOwnerDeferred, 0, 4), "memset");
      cuda_check(cudaMemset(t.ctr + kCtrOwnerDone, 0, 4), "memset");
    }
    view.peer = d_peers;
    connected = true;
  }

  // handles: one CUDA IPC handle per rank, rank order (own entry ignored).
  void connect(const void *handles, size_t bytes) {
    if (connected) throw std::invalid_argument("exchange is already connected");
    if (bytes < kIpcHandleBytes * W) throw std::invalid_argument("need world_size IPC handles");
    DeviceGuard dg(device);
    for (uint32_t r = 0; r < W; ++r) {
      if (r == me) continue;
      cudaIpcMemHandle_t h;
      std::memcpy(&h, static_cast<const uint8_t *>(handles) + r * kIpcHandleBytes, kIpcHandleBytes);
      void *p = nullptr;
      cuda_check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
      peers[r] = static_cast<uint8_t *>(p);
      opened[r] = true;
    }
    finish_connect();
  }

  void require_connected() const {
    if (!connected) throw std::invalid_argument("exchange is not connected");
  }

  InitSpec init_spec() const {
    const se_store_config &c = store->cfg;
    return InitSpec{c.init_kind, c.init_min, c.init_max - c.init_min,
                    c.optimizer_kind == SE_OPT_ADAGRAD ? c.initial_accumulator : 0.0f};
  }

  // Route of this rank's keys (per-tile counts, offsets, per-owner counts),
  // published to every rank as `kind`; returns after every rank's counts
  // arrived (stream order).
  // count_dev: the batch's size on the device (at most n), or null.
  template <class K>
  const uint32_t *run_route(const K *keys, size_t n, int dir, int kind, cudaStream_t st,
                            const uint32_t *count_dev = nullptr, const DedupeWs *dws = nullptr) {
    const uint32_t tiles = std::max(uint32_t((n + kExTile - 1) / kExTile), 1u);
    uint32_t *tile_counts = route[dir], *tile_offsets = tile_counts + size_t(tiles_cap) * W;
    uint32_t *counts = tile_offsets + size_t(tiles_cap) * W;
    pdl(k_ex_count<K>, tiles, kRouteThreads, W * 4, st, spec, view, keys, n, tile_counts, count_dev,
        dws ? static_cast<const uint32_t *>(dws->pos_slot) : nullptr,
        dws ? static_cast<const uint32_t *>(dws->set_idx) : nullptr, dws ? dws->inverse : nullptr, n);
    launched("k_ex_count");
    pdl(k_ex_sync_counts, 1, kRouteThreads, 0, st, view, kind, tiles, tile_counts, tile_offsets, counts);
    launched("k_ex_sync_counts");
    return counts;
  }

  // Stream-ordered end of a phase: raises this rank's flags of `kind` and
  // waits for every rank's (total_word: see k_ex_sync).
  void sync(int kind, cudaStream_t st, int total_word = kExTotal) {
    pdl(k_ex_sync, 1, 32, 0, st, view, kind, total_word);
    launched("k_ex_sync");
  }

  void check_batch(const void *keys, size_t n, const void *rows, const char *rows_name) const {
    require_connected();
    if (n > M) throw std::invalid_argument("batch exceeds the exchange's max_keys_per_rank");
    if (n && (!is_device_ptr(keys) || !is_device_ptr(rows)))
      throw std::invalid_argument(std::string("exchange takes device keys and ") + rows_name);
  }

  void forward(const void *keys, size_t n, void *out, bool insert, cudaStream_t st) {
    check_batch(keys, n, out, "output rows");
    std::lock_guard<std::mutex> lock(store->mu);
    DeviceGuard dg(device);
    Table &t = store->table(dim);
    const uint32_t tiles = uint32_t((n + kExTile - 1) / kExTile);
    const bool dd = dedupe && n > 0;
    if (dd) parity ^= 1u;
    const DedupeWs dws = dedupe_ws();
    dispatch_key(store->cfg.key_dtype, [&](auto tag) {
      using K = decltype(tag);
      const K *k = static_cast<const K *>(keys);
      const uint32_t *count_dev = nullptr;
      if (dd) {  // route each distinct key of the batch once
        StoreImpl::Prof pr(store, "k_ex_dedupe", st);
        pdl(k_ex_dedupe<K>, grid_for(n, 256, 0x7fffffffu), 256, 0, st, view, k, n, dws,
            reinterpret_cast<K *>(dd_ukeys));
        launched("k_ex_dedupe");
        k = reinterpret_cast<const K *>(dd_ukeys);
        count_dev = dws.count;
      }
      // the route count of a deduplicated batch also writes its inverse
      const uint32_t *counts = run_route<K>(k, n, 0, kExCounts, st, count_dev, dd ? &dws : nullptr);
      StoreImpl::Prof pr(store, "k_ex_scatter_keys", st);
      pdl(k_ex_scatter<K, false, uint4>, std::max(tiles, 1u), kRouteThreads, (kRouteWarps + 1) * W * 4, st,
          spec, view, k, n, route[0] + size_t(tiles_cap) * W, counts, nullptr, key_pid, key_slot, count_dev);
      launched("k_ex_scatter");
    });
    fwd_deduped = dd;
    sync(kExKeys, st);
    // owner side: at most W * M keys arrive
    const uint64_t WM = uint64_t(W) * M;
    if (insert) store->ensure_rows(t, WM, st);
    uint32_t *def_idx = t.def_pos.get(WM);
    unsigned long long *def_word = t.def_word.get(WM);
    const InitSpec init = init_spec();
    auto go = [&](auto lanes_tag, auto vec_tag) {
      constexpr int LN = decltype(lanes_tag)::value;
      constexpr int VC = decltype(vec_tag)::value;
      const unsigned grid = grid_for(M * LN, 256, 148 * 16);
      StoreImpl::Prof pr(store, "k_ex_owner", st);
      if (insert) {
        pdl(k_ex_owner<LN, VC, true>, grid, 256, 0, st, t.dir(), t.L, t.slabs, t.alloc(),
                                                        init, view, t.ctr + kCtrOwnerDeferred, def_idx, def_word,
                                                        t.ctr + kCtrStatus, t.ctr + kCtrOwnerDone);
        launched("k_ex_owner");
      } else {
        pdl(k_ex_owner<LN, VC, false>, grid, 256, 0, st, t.dir(), t.L, t.slabs, t.alloc(),
                                                         init, view, nullptr, nullptr, nullptr,
                                                         t.ctr + kCtrStatus, nullptr);
        launched("k_ex_owner");
      }
    };
    auto by_lanes = [&](auto vec_tag) {
      const uint32_t ln = gather_lanes(t.vec == 4 ? uint64_t(dim) / 4 : uint64_t(dim));
      switch (ln) {
      case 4: go(std::integral_constant<int, 4>{}, vec_tag); break;
      case 8: go(std::integral_constant<int, 8>{}, vec_tag); break;
      case 16: go(std::integral_constant<int, 16>{}, vec_tag); break;
      default: go(std::integral_constant<int, 32>{}, vec_tag); break;
      }
    };
    if (t.vec == 4) by_lanes(std::integral_constant<int, 4>{});
    else by_lanes(std::integral_constant<int, 1>{});
    sync(kExRows, st);
    last_fwd_n = n;
    have_fwd = true;
    // requester side: this rank's rows, batch order
    const size_t bytes = n * size_t(view.row_bytes);
    const uintptr_t al = uintptr_t(out) | uintptr_t(bytes);
    auto copy_out = [&](auto utag) {
      using U = decltype(utag);
      const size_t units = bytes / sizeof(U);
      StoreImpl::Prof pr(store, "k_ex_rows_out", st);
      if (dd) {  // expand the distinct keys' rows to the batch's positions
        const uint32_t row_units = uint32_t(view.row_bytes / sizeof(U));
        uint32_t team = 1;
        while (team < 32 && team < row_units) team <<= 1;
        pdl(k_ex_rows_out_dedupe<U>, grid_for(n * team, 256, 148 * 8), 256, 0, st, view, static_cast<U *>(out), n,
            row_units, dws, team);
      } else {
        pdl(k_ex_rows_out<U>, grid_for(units, 256, 148 * 8), 256, 0, st, view, static_cast<U *>(out), units);
      }
      launched("k_ex_rows_out");
    };
    if (al % 16 == 0) copy_out(uint4{});
    else if (al % 4 == 0) copy_out(uint32_t{});
    else copy_out(uint16_t{});
  }

  void backward(const void *keys, size_t n, const void *grads, cudaStream_t st) {
    check_batch(keys, n, grads, "gradient rows");
    std::lock_guard<std::mutex> lock(store->mu);
    DeviceGuard dg(device);
    const uint32_t tiles = uint32_t((n + kExTile - 1) / kExTile);
    const uintptr_t al = uintptr_t(grads) | uintptr_t(view.grad_bytes);
    dispatch_key(store->cfg.key_dtype, [&](auto tag) {
      using K = decltype(tag);
      const K *k = static_cast<const K *>(keys);
      const uint32_t *counts = run_route<K>(k, n, 1, kExGCounts, st);
      auto scatter = [&](auto utag) {
        using U = decltype(utag);
        StoreImpl::Prof pr(store, "k_ex_scatter_grads", st);
        pdl(k_ex_scatter<K, true, U>, std::max(tiles, 1u), kRouteThreads, (kRouteWarps + 1) * W * 4, st,
            spec, view, k, n, route[1] + size_t(tiles_cap) * W, counts, static_cast<const uint8_t *>(grads), nullptr,
            nullptr, nullptr);
        launched("k_ex_scatter");
      };
      if (al % 16 == 0) scatter(uint4{});
      else if (al % 4 == 0) scatter(uint32_t{});
      else scatter(uint16_t{});
    });
    sync(kExGrads, st, kExTotalStaged);
    const auto *total = reinterpret_cast<const uint32_t *>(arena + view.o_words) + kExTotal;
    store->accumulate_locked(arena + view.o_gkeys, size_t(W) * M, total, dim, arena + view.o_ingrads, st,
                             SE_KEY_UINT64);
  }

  // Gradients for the keys of the last forward (lookup) of this exchange, in
  // that batch's order: rows follow the forward's route, and the owners
  // accumulate them with the keys already in their key inboxes.
  void backward_routed(const void *grads, size_t n, cudaStream_t st) {
    require_connected();
    if (!have_fwd) throw std::invalid_argument("no lookup on this exchange to route the gradients by");
    if (n != last_fwd_n) throw std::invalid_argument("gradient rows must match the keys of the last lookup");
    if (n && !is_device_ptr(grads)) throw std::invalid_argument("exchange takes device gradient rows");
    std::lock_guard<std::mutex> lock(store->mu);
    DeviceGuard dg(device);
    if (fwd_deduped) {
      prereduce_and_scatter(grads, n, st);
    } else {
      const uintptr_t al = uintptr_t(grads) | uintptr_t(view.grad_bytes);
      auto scatter = [&](auto utag) {
        using U = decltype(utag);
        const uint32_t units = view.grad_bytes / uint32_t(sizeof(U));
        uint32_t team = 1;
        while (team < 32 && team < units) team <<= 1;
        StoreImpl::Prof pr(store, "k_ex_scatter_rows", st);
        pdl(k_ex_scatter_rows<U>, grid_for(n * team, 256, 148 * 8), 256, 0, st,
            view, key_pid, key_slot, n, static_cast<const U *>(grads), units, team);
        launched("k_ex_scatter_rows");
      };
      if (al % 16 == 0) scatter(uint4{});
      else if (al % 4 == 0) scatter(uint32_t{});
      else scatter(uint16_t{});
    }
    sync(kExGrads, st, kExFwdTotal);
    const auto *total = reinterpret_cast<const uint32_t *>(arena + view.o_words) + kExTotal;
    store->accumulate_locked(arena + view.o_inkeys, size_t(W) * M, total, dim, arena + view.o_ingrads, st,
                             SE_KEY_UINT64, reinterpret_cast<const uint32_t *>(arena + view.o_inrow));
  }

  // Gradient batch of a deduplicated forward: the rows of each distinct key
  // are summed on this rank in fp32 (k_acc_atomic over dense rows indexed by
  // the forward's inverse), then each sum goes to the owner's inbox slot of
  // that key.
  void prereduce_and_scatter(const void *grads, size_t n, cudaStream_t st) {
    if (dim > int64_t(kAccMaxDim))
      throw std::invalid_argument("dedupe needs rows of at most 8,192 values");
    const DedupeWs dws = dedupe_ws();
    const int gdt = store->cfg.gradient_dtype;
    uint32_t tile = 1;
    while (tile < kAccMaxTile && uint64_t(tile) * 2 * uint64_t(dim) * 4 <= kAccSmemBytes) tile <<= 1;
    uint32_t hbits = 1;
    while ((1u << hbits) < 2 * tile) ++hbits;
    const AccTab dense{nullptr, dd_pre, nullptr, nullptr, nullptr, nullptr, 0u, uint32_t(dim), uint32_t(M)};
    const bool vec4 = dim % 4 == 0 && uintptr_t(grads) % (gdt == SE_FLOAT32 ? 16 : 8) == 0;
    {
      StoreImpl::Prof pr(store, "k_ex_prereduce", st);
      auto go = [&](auto kern) {
        allow_dynamic_smem(kern, size_t(tile) * size_t(dim) * 4);
        pdl(kern, grid_for(n, tile, 0x7fffffffu), kAccThreads, size_t(tile) * size_t(dim) * 4, st, dense,
            static_cast<const void *>(dws.inverse), int(SE_KEY_UINT32), n, static_cast<const uint32_t *>(nullptr),
            grads, gdt, 1.0f, INFINITY, tile, hbits, dd_ctr + 6, dd_ctr + 7, static_cast<const uint32_t *>(nullptr),
            FwdCache{nullptr, nullptr, nullptr, 0u});
      };
      if (vec4) go(k_acc_atomic<4, false, true>);
      else go(k_acc_atomic<1, false, true>);
      launched("k_acc_atomic");
    }
    StoreImpl::Prof pr(store, "k_ex_scatter_rows", st);
    if (gdt == SE_FLOAT32 && dim % 4 == 0) {  // 16-byte units: team lanes per row
      uint32_t team = 1;
      while (team < 32 && team < uint32_t(dim / 4)) team <<= 1;
      pdl(k_ex_scatter_prerows<true>, grid_for(n * team, 256, 148 * 8), 256, 0, st, view, key_pid, key_slot,
          dws.count, size_t(M), dd_pre, uint32_t(dim), gdt, team);
    } else {
      pdl(k_ex_scatter_prerows<false>, grid_for(n * 32, 256, 148 * 8), 256, 0, st, view, key_pid, key_slot,
          dws.count, size_t(M), dd_pre, uint32_t(dim), gdt, 32u);
    }
    launched("k_ex_scatter_prerows");
  }

  // Waits for the stream; raises a timed-out wait, then the owner's table errors.
  void check(cudaStream_t st) {
    require_connected();
    std::lock_guard<std::mutex> lock(store->mu);
    DeviceGuard dg(device);
    cuda_check(cudaMemcpyAsync(status_host, arena + view.o_words + 4 * kExStatus, 4, cudaMemcpyDeviceToHost, st),
               "exchange status");
    cuda_check(cudaStreamSynchronize(st), "sync");
    if (status_host[0] & kExBadIndex)
      throw Error(SE_ERR_RUNTIME, "exchange slot outside its buffers (ranks created with different sizes?); "
                                  "the exchange must be recreated");
    if (status_host[0]) {
      static const char *names[kExKinds] = {"counts", "keys", "rows", "gradient counts", "gradients"};
      std::string which;
      for (int k = 0; k < kExKinds; ++k)
        if (status_host[0] & (1u << k)) which += std::string(which.empty() ? "" : ", ") + names[k];
      throw Error(SE_ERR_RUNTIME, "exchange wait timed out (" + which +
                                      "): a peer rank did not take part; the exchange must be recreated");
    }
    store->check_status(store->table(dim), st);
  }
};

void set_last_error(const std::string &msg) { t_last_error = msg; }
void clear_last_error() { t_last_error.clear(); }
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

}  // namespace se_gpu

struct se_store {
  se_gpu::StoreImpl impl;
};

struct se_exchange {
  se_gpu::ExchangeImpl impl;
};

using namespace se_gpu;

namespace {

// Returns the common row length, or throws when lengths differ.
int64_t uniform_dim(const int64_t *row_lengths, size_t n, size_t num_row_lengths, bool gradient) {
  if (num_row_lengths != n)
    throw std::invalid_argument(gradient ? "gradient key and row-length counts must match"
                                         : "row_lengths count must match keys");
  if (n == 0) return 0;
  const int64_t d = row_lengths[0];
  for (size_t i = 0; i < n; ++i) {
    if (gradient && row_lengths[i] <= 0) throw std::invalid_argument("gradient row length must be positive");
    if (row_lengths[i] != d)
      throw Error(SE_ERR_NOT_IMPLEMENTED, "mixed row lengths in one call are not supported by the GPU store");
  }
  return d;
}

se_store *checked(se_store *s) {
  if (!s) throw std::invalid_argument("store handle is null");
  return s;
}

}  // namespace

extern "C" {

const char *se_last_error(void) { return se_gpu::t_last_error.c_str(); }
const char *se_version(void) { return "se_gpu sm_100a 0.1"; }
uint64_t se_kernel_launch_count(void) { return se_gpu::g_launches.load(); }

int se_store_create(const se_store_config *config, se_store **out_store) {
  return guarded([&] {
    if (!config || !out_store) throw std::invalid_argument("null config or output handle");
    const se_store_config &c = *config;
    if (c.num_dims == 0 || !c.dims) throw std::invalid_argument("dims must not be empty");
    for (size_t i = 0; i < c.num_dims; ++i)
      if (c.dims[i] <= 0) throw std::invalid_argument("dims must be positive");
    if (c.key_dtype < SE_KEY_INT32 || c.key_dtype > SE_KEY_UINT64)
      throw std::invalid_argument("unsupported key dtype code");
    for (int dt : {c.value_dtype, c.optimizer_dtype, c.gradient_dtype})
      if (dt < SE_FLOAT32 || dt > SE_BFLOAT16) throw std::invalid_argument("unsupported value dtype");
    if (!std::isfinite(c.gradient_scale) || c.gradient_scale <= 0.0f)
      throw std::invalid_argument("gradient_scale must be finite and greater than zero");
    if (c.accumulation != SE_ACCUM_ORDERED && c.accumulation != SE_ACCUM_ATOMIC)
      throw std::invalid_argument("accumulation must be 'ordered' or 'atomic'");
    auto s = std::make_unique<se_store>();
    StoreImpl &st = s->impl;
    st.cfg = c;
    st.device = c.device;
    DeviceGuard dg(c.device);
    cuda_check(cudaStreamCreateWithFlags(&st.own, cudaStreamNonBlocking), "cudaStreamCreate");
    cuda_check(cudaMallocHost(&st.status_host, 64), "cudaMallocHost");
    cuda_check(cudaMallocHost(&st.u64_host, 64), "cudaMallocHost");
    st.init_scores(st.cfg);  // validates the score and lr policies; uploads the LUT
    for (size_t i = 0; i < c.num_dims; ++i) {
      bool dup = false;
      for (auto &t : st.tables) dup |= t->dim == c.dims[i];
      if (dup) continue;
      st.dims.push_back(c.dims[i]);
      auto t = std::make_unique<Table>();
      st.init_table(*t, c.dims[i], c.initial_capacity ? c.initial_capacity : kDefaultCapacity);
      st.tables.push_back(std::move(t));
    }
    if (c.enable_optimizer && c.optimizer_kind == SE_OPT_ADAM) st.ensure_bc(1);
    cuda_check(cudaDeviceSynchronize(), "create sync");
    *out_store = s.release();
  });
}

int se_store_destroy(se_store *store) {
  return guarded([&] {
    if (!store) return;
    DeviceGuard dg(store->impl.device);
    delete store;
  });
}

int se_forward_lookup_dim(se_store *store, const void *keys, size_t n, int64_t dim, void *out,
                          void *stream) {
  return guarded([&] { checked(store)->impl.lookup(keys, n, dim, out, stream, false); });
}

int se_lookup_or_insert_dim(se_store *store, const void *keys, size_t n, int64_t dim, void *out,
                            void *stream) {
  return guarded([&] { checked(store)->impl.lookup(keys, n, dim, out, stream, true); });
}

int se_forward_lookup(se_store *store, const void *keys, size_t n, void *out, size_t num_out,
                      const int64_t *row_lengths, size_t num_row_lengths, void *stream) {
  return guarded([&] {
    const int64_t d = uniform_dim(row_lengths, n, num_row_lengths, false);
    if (n == 0) return;
    if (num_out != n * size_t(d)) throw std::invalid_argument("output size does not match row lengths");
    checked(store)->impl.lookup(keys, n, d, out, stream, false);
  });
}

int se_lookup_or_insert(se_store *store, const void *keys, size_t n, void *out, size_t num_out,
                        const int64_t *row_lengths, size_t num_row_lengths, void *stream) {
  return guarded([&] {
    const int64_t d = uniform_dim(row_lengths, n, num_row_lengths, false);
    if (n == 0) return;
    if (num_out != n * size_t(d)) throw std::invalid_argument("output size does not match row lengths");
    checked(store)->impl.lookup(keys, n, d, out, stream, true);
  });
}

int se_contains(se_store *store, const void *keys, size_t n, uint8_t *out, void *stream) {
  return guarded([&] { checked(store)->impl.contains(keys, n, out, stream); });
}

int se_assign_dim(se_store *store, const void *keys, size_t n, int64_t dim, const void *values, void *stream) {
  return guarded([&] { checked(store)->impl.assign(keys, n, dim, values, stream); });
}

int se_assign(se_store *store, const void *keys, size_t n, const void *values, size_t num_values,
              const int64_t *row_lengths, size_t num_row_lengths, void *stream) {
  return guarded([&] {
    const int64_t d = uniform_dim(row_lengths, n, num_row_lengths, false);
    if (n == 0) return;
    if (num_values != n * size_t(d)) throw std::invalid_argument("values size does not match row lengths");
    checked(store)->impl.assign(keys, n, d, values, stream);
  });
}

int se_assign_scores(se_store *store, const void *keys, size_t n, const uint64_t *scores, void *stream) {
  return guarded([&] { checked(store)->impl.assign_scores(keys, n, scores, stream); });
}

int se_read_scores(se_store *store, const void *keys, size_t n, uint64_t *scores_out, void *stream) {
  return guarded([&] { checked(store)->impl.read_scores(keys, n, scores_out, stream); });
}

int se_export_snapshot(se_store *store, int64_t dim, uint64_t *num_keys_out, void *stream) {
  return guarded([&] {
    if (num_keys_out == nullptr) throw std::invalid_argument("num_keys_out is null");
    *num_keys_out = checked(store)->impl.export_snapshot(dim, stream);
  });
}

int se_export_read(se_store *store, int64_t dim, uint64_t offset, uint64_t count, void *keys_out, void *values_out,
                   void *opt_states_out, uint32_t *steps_out, void *stream) {
  return guarded([&] {
    checked(store)->impl.export_read(dim, offset, count, keys_out, values_out, opt_states_out, steps_out, stream);
  });
}

int se_assign_opt_states(se_store *store, int64_t dim, const void *keys, size_t n, const void *opt_states,
                         size_t num_state_values, const uint32_t *steps, void *stream) {
  return guarded([&] {
    checked(store)->impl.assign_opt_states(dim, keys, n, opt_states, num_state_values, steps, stream);
  });
}

int se_embedding_bag(se_store *store, const void *keys, size_t n, const int64_t *offsets, size_t num_bags,
                     int64_t dim, void *out, int32_t insert, void *stream) {
  return guarded([&] { checked(store)->impl.embedding_bag(keys, n, offsets, num_bags, dim, out, insert != 0, stream); });
}

int se_embedding_bag_backward(se_store *store, const void *keys, size_t n, const int64_t *offsets,
                              size_t num_bags, int64_t dim, const void *pooled_grads, void *stream) {
  return guarded([&] {
    checked(store)->impl.embedding_bag_backward(keys, n, offsets, num_bags, dim, pooled_grads, stream);
  });
}

int se_erase(se_store *store, const void *keys, size_t n, void *stream) {
  return guarded([&] { checked(store)->impl.erase(keys, n, 0, stream); });
}

int se_erase_dimension(se_store *store, int64_t dim, const void *keys, size_t n, void *stream) {
  return guarded([&] {
    if (dim <= 0) throw std::invalid_argument(dim < 0 ? "erase dimension must be non-negative"
                                                      : "erase dimension is not configured");
    checked(store)->impl.erase(keys, n, dim, stream);
  });
}

int se_accumulate_gradients_dim(se_store *store, const void *keys, size_t n, int64_t dim,
                                const void *grads, void *stream) {
  return guarded([&] { checked(store)->impl.accumulate(keys, n, dim, grads, stream); });
}

int se_accumulate_gradients(se_store *store, const void *keys, size_t n, const void *grads,
                            size_t num_grad_scalars, const int64_t *row_lengths,
                            size_t num_row_lengths, void *stream) {
  return guarded([&] {
    const int64_t d = uniform_dim(row_lengths, n, num_row_lengths, true);
    if (n == 0) return;
    if (num_grad_scalars != n * size_t(d))
      throw std::invalid_argument("flat gradient scalar count does not match row lengths");
    checked(store)->impl.accumulate(keys, n, d, grads, stream);
  });
}

int se_optimizer_step(se_store *store, size_t normalization_steps, void *stream) {
  return guarded([&] { checked(store)->impl.optimizer_step(normalization_steps, stream); });
}

int se_store_size(se_store *store, uint64_t *out) {
  return guarded([&] {
    StoreImpl &s = checked(store)->impl;
    std::lock_guard<std::mutex> lock(s.mu);
    DeviceGuard dg(s.device);
    cuda_check(cudaDeviceSynchronize(), "sync");
    uint64_t total = 0;
    for (auto &t : s.tables) total += s.read_live_keys(*t, s.own);
    *out = total;
  });
}

int se_store_dim_size(se_store *store, int64_t dim, uint64_t *out) {
  return guarded([&] {
    StoreImpl &s = checked(store)->impl;
    std::lock_guard<std::mutex> lock(s.mu);
    DeviceGuard dg(s.device);
    cuda_check(cudaDeviceSynchronize(), "sync");
    *out = s.read_live_keys(s.table(dim), s.own);
  });
}

int se_store_reserve(se_store *store, size_t keys, int64_t dim) {
  return guarded([&] {
    StoreImpl &s = checked(store)->impl;
    std::lock_guard<std::mutex> lock(s.mu);
    DeviceGuard dg(s.device);
    if (dim <= 0) throw std::invalid_argument("dim must be > 0");
    Table &t = s.table(dim);
    cuda_check(cudaDeviceSynchronize(), "sync");
    const uint64_t used = s.read_rows_used(t, s.own);
    if (keys > used) {
      t.rows_bound = used;
      s.ensure_rows(t, keys - used, s.own);
      t.rows_bound = used;
    }
  });
}

int se_store_internal_shard_count(se_store *store, uint64_t *out) {
  return guarded([&] {
    const int32_t n = checked(store)->impl.cfg.internal_shards;
    *out = uint64_t(n > 0 ? n : 1);
  });
}

int se_store_entries_per_page(se_store *store, uint64_t *out) {
  return guarded([&] {
    checked(store);
    *out = 4096;  // reporting unit of the slab arena; the reference's default page geometry
  });
}

int se_store_dropped_gradients(se_store *store, uint64_t *out) {
  return guarded([&] {
    StoreImpl &s = checked(store)->impl;
    std::lock_guard<std::mutex> lock(s.mu);
    DeviceGuard dg(s.device);
    cuda_check(cudaDeviceSynchronize(), "sync");
    uint64_t total = 0;
    for (auto &t : s.tables) {
      cuda_check(cudaMemcpyAsync(s.u64_host, t->ctr + kCtrDropped, 8, cudaMemcpyDeviceToHost, s.own), "copy");
      cuda_check(cudaStreamSynchronize(s.own), "sync");
      total += s.u64_host[0];
    }
    *out = total;
  });
}

int se_store_read_state(se_store *store, int64_t dim, uint64_t key, void *param_out, void *state_out,
                        uint32_t *step_out, int32_t *found) {
  return guarded([&] { checked(store)->impl.read_state(dim, key, param_out, state_out, step_out, found); });
}

int se_store_clear(se_store *store, void *stream) {
  return guarded([&] { checked(store)->impl.clear(stream); });
}

int se_store_synchronize(se_store *store) {
  return guarded([&] {
    StoreImpl &s = checked(store)->impl;
    std::lock_guard<std::mutex> lock(s.mu);
    DeviceGuard dg(s.device);
    cuda_check(cudaDeviceSynchronize(), "sync");
    for (auto &t : s.tables) s.check_status(*t, s.own);
  });
}

int se_store_profile_enable(se_store *store, int32_t enable) {
  return guarded([&] {
    StoreImpl &s = checked(store)->impl;
    std::lock_guard<std::mutex> lock(s.mu);
    DeviceGuard dg(s.device);
    s.profiling = enable != 0;
    if (s.profiling && s.event_pool.size() < 4096) {
      while (s.event_pool.size() < 4096) {
        cudaEvent_t e;
        cuda_check(cudaEventCreate(&e), "cudaEventCreate");
        s.event_pool.push_back(e);
      }
    }
  });
}

int se_store_profile_read(se_store *store, const char *name, double *out_ms, uint64_t *out_launches) {
  return guarded([&] {
    StoreImpl &s = checked(store)->impl;
    std::lock_guard<std::mutex> lock(s.mu);
    DeviceGuard dg(s.device);
    cuda_check(cudaDeviceSynchronize(), "sync");
    double ms = 0;
    uint64_t count = 0;
    std::vector<ProfRec> keep;
    for (auto &r : s.prof) {
      if (name && r.name.find(name) == std::string::npos) {
        keep.push_back(r);
        continue;
      }
      float x = 0;
      cuda_check(cudaEventElapsedTime(&x, r.a, r.b), "elapsed");
      ms += x;
      ++count;
      s.event_pool.push_back(r.a);
      s.event_pool.push_back(r.b);
    }
    s.prof.swap(keep);
    *out_ms = ms;
    *out_launches = count;
  });
}


int se_exchange_create(se_store *store, int32_t partitioner_kind, uint32_t world_size, uint32_t rank,
                       uint64_t max_keys_per_rank, int64_t dim, uint32_t timeout_ms, se_exchange **out) {
  return guarded([&] {
    if (!out) throw std::invalid_argument("null output handle");
    auto ex = std::make_unique<se_exchange>();
    ex->impl.create(&checked(store)->impl, partitioner_kind, world_size, rank, max_keys_per_rank, dim, timeout_ms);
    *out = ex.release();
  });
}

int se_exchange_handle(se_exchange *ex, void *handle_out, size_t handle_bytes) {
  return guarded([&] {
    if (!ex || !handle_out) throw std::invalid_argument("null exchange or handle buffer");
    ex->impl.handle(handle_out, handle_bytes);
  });
}

int se_exchange_connect(se_exchange *ex, const void *handles, size_t handles_bytes) {
  return guarded([&] {
    if (!ex || !handles) throw std::invalid_argument("null exchange or handles");
    ex->impl.connect(handles, handles_bytes);
  });
}

int se_exchange_connect_local(se_exchange *const *exchanges, uint32_t count) {
  return guarded([&] {
    if (!exchanges || count == 0) throw std::invalid_argument("no exchanges given");
    for (uint32_t r = 0; r < count; ++r) {
      ExchangeImpl &e = exchanges[r]->impl;
      if (e.W != count || e.me != r) throw std::invalid_argument("exchanges[r] must be rank r of world_size == count");
      if (e.connected) throw std::invalid_argument("exchange is already connected");
    }
    for (uint32_t r = 0; r < count; ++r) {
      ExchangeImpl &e = exchanges[r]->impl;
      DeviceGuard dg(e.device);
      for (uint32_t q = 0; q < count; ++q) {
        const ExchangeImpl &o = exchanges[q]->impl;
        if (o.device != e.device) {
          const cudaError_t pe = cudaDeviceEnablePeerAccess(o.device, 0);
          if (pe == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
          else cuda_check(pe, "cudaDeviceEnablePeerAccess");
        }
        e.peers[q] = o.arena;
      }
      e.finish_connect();
    }
  });
}

int se_exchange_lookup(se_exchange *ex, const void *keys, size_t n, void *out, int32_t insert, void *stream) {
  return guarded([&] {
    if (!ex) throw std::invalid_argument("exchange handle is null");
    ex->impl.forward(keys, n, out, insert != 0, static_cast<cudaStream_t>(stream));
  });
}

int se_exchange_accumulate(se_exchange *ex, const void *keys, size_t n, const void *grads, void *stream) {
  return guarded([&] {
    if (!ex) throw std::invalid_argument("exchange handle is null");
    ex->impl.backward(keys, n, grads, static_cast<cudaStream_t>(stream));
  });
}

int se_exchange_accumulate_routed(se_exchange *ex, const void *grads, size_t n, void *stream) {
  return guarded([&] {
    if (!ex) throw std::invalid_argument("exchange handle is null");
    ex->impl.backward_routed(grads, n, static_cast<cudaStream_t>(stream));
  });
}

int se_exchange_set_dedupe(se_exchange *ex, int32_t enable) {
  return guarded([&] {
    if (!ex) throw std::invalid_argument("exchange handle is null");
    ex->impl.set_dedupe(enable != 0);
  });
}

int se_exchange_check(se_exchange *ex, void *stream) {
  return guarded([&] {
    if (!ex) throw std::invalid_argument("exchange handle is null");
    ex->impl.check(static_cast<cudaStream_t>(stream));
  });
}

int se_exchange_destroy(se_exchange *ex) {
  return guarded([&] { delete ex; });
}

}  // extern "C"
