// Atomic accumulation mode of the B200 store.
//
// The ordered mode appends every gradient row and reduces each key's rows in
// arrival order at optimizer_step (bit-exact with the reference's serial
// sum). This mode instead sums gradients as they arrive into a hash table
// keyed by key - the structure of TransientArena::accumulate_hashed
// (arena/transient_arena.hpp:119-145: one accumulator slot per key, found by
// hashing the key, each gradient row added into it) - with the additions
// made concurrent:
//
//   k_acc_atomic  one block per tile of the batch: the tile's distinct keys
//                 go into a shared-memory hash set, each gradient row is
//                 added into its key's shared-memory sum, then each distinct
//                 key finds (or claims) its slot of the table and adds the
//                 tile's sum with 16-byte vector reductions
//                 (red.global.add.v4.f32). Hot keys thus cost one reduction
//                 per tile, not one per row.
//   k_acc_apply   optimizer_step: one lane group per claimed slot resolves
//                 the key in the directory (absent keys drop their rows, as
//                 SlotStore::update_batch does,
//                 hogwild_embedding_store.hpp:1942-1952), applies the
//                 optimizer to the row with the slot's sum, and frees the
//                 slot (sum zeroed, key cleared) for the next window.
//
// Sums are fp32 whatever the gradient dtype; the order of a key's additions
// is not the arrival order, so updates equal the ordered mode's within the
// rounding of a reassociated fp32 sum (1e-5 relative for fp32 tables).
// Keys need not be present when their gradients arrive: they are resolved
// at optimizer_step, like the reference's transient arena keyed by key.
#pragma once

#include "se_store_kernels.cuh"

namespace se_gpu {

// Hash table of one store table's gradient sums for the current window.
// A slot holds (key, dense row) in one 16-byte word, claimed by one 128-bit
// CAS, so a block that finds the key learns its dense row in the same
// round trip. The sums live in `vals` by dense row: each block reserves one
// dense row per entry of its tile up front, and a claim takes the row
// reserved for that key; the rows in use stay in the front of `vals`, the
// same region every window (L2-resident from one step to the next).
struct AccTab {
  ulonglong2 *slots;         // [G + 1] (key, dense row); free: all ones; slot G holds the all-ones key
  float *vals;               // [vcap][dim] fp32 sums by dense row, zero when free
  uint32_t *cnt;             // [G + 1] gradient rows summed into each slot
  uint4 *list;               // [G + 1] (slot, cached row, erase epoch, dense row) of each claim; slot kNoRow: a hole
  uint32_t *ctr;             // [0] list entries, [2] finished apply blocks, [3] dense rows reserved
  const uint32_t *epoch;     // the table's erase epoch (bumped by every erase)
  uint32_t mask;             // G - 1; G is a power of two
  uint32_t dim;
  uint32_t vcap;             // dense rows `vals` holds
};

constexpr unsigned long long kAccFree = ~0ull;  // dense-row half of a free slot

// 128-bit compare-and-swap of a slot (sm_90+): returns the old word.
__device__ __forceinline__ ulonglong2 cas_slot(ulonglong2 *p, ulonglong2 expect, ulonglong2 desire) {
  ulonglong2 old;
  asm volatile("{\n .reg .b128 c, v, o;\n mov.b128 c, {%2, %3};\n mov.b128 v, {%4, %5};\n"
               " atom.global.cas.b128 o, [%6], c, v;\n mov.b128 {%0, %1}, o;\n}"
               : "=l"(old.x), "=l"(old.y)
               : "l"(expect.x), "l"(expect.y), "l"(desire.x), "l"(desire.y), "l"(p)
               : "memory");
  return old;
}

// Keys and rows the last lookup_or_insert resolved, by batch position (the
// accumulate of the same batch finds its rows here instead of probing the
// directory). *n is that batch's size; an erase clears it.
struct FwdCache {
  unsigned long long *keys;  // null: nothing is cached by this launch
  uint32_t *rows;
  uint32_t *n;               // null: the cache is not kept
  uint32_t cap;              // entries keys / rows hold
};

// Row of key `key` at batch position pos from the cache, or kNoRow.
// The count, the key and the row are loaded together (one round trip): every
// position below cap is inside the cache's arrays.
__device__ __forceinline__ uint32_t cached_row(const FwdCache &fc, size_t pos, uint64_t key) {
  if (fc.n == nullptr || fc.keys == nullptr || pos >= size_t(fc.cap)) return kNoRow;
  const uint32_t cached = __ldcg(fc.n);
  const unsigned long long k = __ldcg(fc.keys + pos);
  const uint32_t row = __ldcg(fc.rows + pos);
  return pos < size_t(cached) && k == key ? row : kNoRow;
}

constexpr uint32_t kAccThreads = 256;
constexpr uint32_t kAccMaxTile = 256;        // rows per block of k_acc_atomic
static_assert(kAccMaxTile <= kAccThreads, "k_acc_atomic gives each entry and each distinct key its own thread");
constexpr uint64_t kAccSmemBytes = 32768;    // shared-memory sums per block
constexpr uint32_t kAccMaxDim = 8192;        // longest row of an atomic-mode table (one row per tile)

// Slot of `key`, claiming a free one with dense row `rank` if the key has
// none (`claimed` tells the caller to list the slot); *vrow receives the
// key's dense row either way. Linear probing from the high bits of the
// SplitMix64 hash (hash-partitioned GPUs share the low bits); the all-ones
// key has slot G. kNoRow when every slot is taken (the host sizes the table
// at twice the window's rows).
__device__ __forceinline__ uint32_t acc_find_or_claim(const AccTab &a, uint64_t key, uint32_t rank, bool &claimed,
                                                      uint32_t &vrow) {
  claimed = false;
  const uint32_t G = a.mask + 1u;
  const ulonglong2 free_word = make_ulonglong2(kEmptyKey, kAccFree);
  const ulonglong2 mine = make_ulonglong2(key, rank);
  uint32_t s = key == kEmptyKey ? G : uint32_t(__umul64hi(splitmix64(key), uint64_t(G)));
  for (uint32_t probe = 0; probe < G; ++probe) {
    // one L2 round trip per slot: the CAS claims a free slot or reports the
    // key (and its dense row) already there
    const ulonglong2 old = cas_slot(a.slots + s, free_word, mine);
    if (old.x == kEmptyKey && old.y == kAccFree) {
      claimed = true;
      vrow = rank;
      return s;
    }
    if (old.x == key) {
      vrow = uint32_t(old.y);
      return s;
    }
    if (s == G) break;  // slot G holds only the all-ones key
    s = (s + 1u) & a.mask;
  }
  return kNoRow;
}

// Adds four floats at a 16-byte aligned address of global memory with one
// vector reduction (relaxed, device scope).
__device__ __forceinline__ void red_add_v4(float *p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// accumulate_gradients in atomic mode. Entries [blockIdx.x * tile, + tile)
// of the batch (n_max rows, or *n_dev when the batch size is known only on
// the device). Each gradient is validated and scaled on entry like
// GradientAccumulator::accumulate_hashed (gradient_accumulator.hpp:88-128):
// g / gradient_scale must be finite and within the gradient and parameter
// dtypes (failures raise kStatusBadGradient in *bad_word), and the value
// added is g (scale 1) or the scaled value rounded to the gradient dtype.
// With kBag, entry i takes gradient row grad_row[i] (embedding-bag backward).
//
// The tile's gradient rows are staged in shared memory (dynamic, tile x row
// bytes): one bulk copy through the TMA when the rows are contiguous and
// 16-byte aligned (one per row for bag rows), else plain loads. Meanwhile
// the keys are hashed; each distinct key gets a local index and a list of
// its entries (shared-memory linked list), and finds or claims its table
// slot. Then each (distinct key, 16-byte chunk) pair sums its entries'
// chunks from shared memory and adds the sum to the table with one vector
// reduction - no floating-point shared-memory atomics, conflict-free reads.
constexpr uint32_t kCopySpinLimit = 1u << 26;  // polls of the bulk-copy barrier before giving up

// Walks chunks c = c0, c0 + step, c0 + 2 step, ... of rows of `units`
// chunks as (row, chunk in row) without a division per step.
struct ChunkWalk {
  uint32_t j, u;           // row and chunk of the current c
  uint32_t dj, du, units;  // step = dj * units + du
  __device__ __forceinline__ ChunkWalk(uint32_t c0, uint32_t step, uint32_t units_)
      : j(c0 / units_), u(c0 % units_), dj(step / units_), du(step % units_), units(units_) {}
  __device__ __forceinline__ void next() {
    j += dj;
    u += du;
    if (u >= units) {
      u -= units;
      ++j;
    }
  }
};

template <int VEC, bool kBag, bool kDirect = false>
__global__ void __launch_bounds__(kAccThreads, 4)  // 4 blocks per SM: a 65,536-row batch in one wave
k_acc_atomic(AccTab a, const void *__restrict__ keys, int kdt, size_t n_max, const uint32_t *n_dev,
             const void *__restrict__ grads, int gdt, float scale, float maxv, uint32_t tile, uint32_t hbits,
             uint32_t *bad_word, uint32_t *status, const uint32_t *__restrict__ grad_row, FwdCache fc) {
  extern __shared__ __align__(16) uint8_t s_rows[];   // [tile][row bytes] the tile's gradient rows
  __shared__ unsigned long long s_hkey[2 * kAccMaxTile];  // hash set of the tile's keys
  __shared__ uint32_t s_hloc[2 * kAccMaxTile + 1];    // local index of each set slot; [H]: the all-ones key
  __shared__ int32_t s_next[kAccMaxTile];             // next entry of the same key, -1 at the end
  __shared__ int32_t s_head[kAccMaxTile];             // first entry of each local key
  __shared__ unsigned long long s_lkey[kAccMaxTile];  // key of each local index
  __shared__ uint32_t s_gslot[kAccMaxTile];           // table slot of each local index
  __shared__ uint32_t s_vrow[kAccMaxTile];            // dense sum row of each local index
  __shared__ uint32_t s_crank[kAccMaxTile];           // 1: this block claimed the local key's slot
  __shared__ uint32_t s_lrow[kAccMaxTile];            // row of each local key from the forward's cache, or kNoRow
  __shared__ uint32_t s_nloc, s_spec, s_claim_base, s_epoch, s_copy_ok, s_rank_base;
  __shared__ __align__(8) uint64_t s_bar;
  pdl_wait();
  pdl_trigger();  // the next kernel may launch; its pdl_wait still waits for this one
  const size_t n = n_dev ? min(size_t(*n_dev), n_max) : n_max;
  const size_t i0 = size_t(blockIdx.x) * tile;
  if (i0 >= n) return;  // whole block: past the end of a device-sized batch
  const uint32_t m = uint32_t(min(size_t(tile), n - i0));
  const uint32_t H = 1u << hbits;  // >= 2 * tile
  const uint32_t dim = a.dim;
  const uint32_t tid = threadIdx.x;
  const uint32_t gsize = gdt == SE_FLOAT32 ? 4u : 2u;
  const uint32_t row_bytes = dim * gsize;
  const uint32_t units = dim / VEC;
  const uint32_t lane = tid & 31u;
  // The entry of this thread (tile <= blockDim): its key and the row the
  // forward cached for it, loaded first so their latency overlaps the set-up.
  const bool has_entry = tid < m;
  uint64_t my_key = kEmptyKey;
  uint32_t my_row = kNoRow;
  if (has_entry) {
    my_key = load_key(keys, kdt, i0 + tid);
    if (!kDirect) my_row = cached_row(fc, i0 + tid, my_key);
  }
  // 0. stage the gradient rows
  const uint8_t *gsrc = static_cast<const uint8_t *>(grads);
  const bool tma = row_bytes % 16u == 0u && (reinterpret_cast<uintptr_t>(gsrc) & 15u) == 0u;
  if (tma) {
    if (tid == 0) {
      mbar_init(&s_bar, 1);
      mbar_arrive_expect_tx(&s_bar, m * row_bytes);
      if (!kBag) bulk_copy_g2s(s_rows, gsrc + i0 * row_bytes, m * row_bytes, &s_bar);
    }
    __syncthreads();  // the barrier is initialised before any copy names it
    if (kBag)
      for (uint32_t j = tid; j < m; j += blockDim.x)
        bulk_copy_g2s(s_rows + j * row_bytes, gsrc + size_t(grad_row[i0 + j]) * row_bytes, row_bytes, &s_bar);
  } else {
    for (uint32_t x = tid; x < m * (row_bytes / 2u); x += blockDim.x) {
      const uint32_t j = x / (row_bytes / 2u), h = x - j * (row_bytes / 2u);
      const size_t src = kBag ? size_t(grad_row[i0 + j]) : i0 + j;
      reinterpret_cast<uint16_t *>(s_rows)[x] = reinterpret_cast<const uint16_t *>(gsrc + src * row_bytes)[h];
    }
  }
  for (uint32_t h = tid; h < H; h += blockDim.x) s_hkey[h] = kEmptyKey;
  for (uint32_t q = tid; q < tile; q += blockDim.x) s_head[q] = -1;
  if (tid == 0) {
    s_nloc = 0u;
    s_spec = 0u;
    s_epoch = a.epoch ? __ldcg(a.epoch) : 0u;
    s_copy_ok = 1u;
    // dense sum rows for the tile's keys that this block may claim
    s_rank_base = kDirect ? 0u : atomicAdd(a.ctr + 3, m);
  }
  __syncthreads();
  // 1. the tile's distinct keys. The lanes of a warp holding the same key
  //    find each other (match); the lowest of them inserts the key into the
  //    block's hash set (the all-ones key, the set's empty marker, takes slot
  //    H), and the warp that inserts a key first gives it its local index.
  const unsigned entries = __ballot_sync(0xffffffffu, has_entry);
  const unsigned peers = __match_any_sync(0xffffffffu, my_key) & entries;
  const uint32_t leader = peers ? uint32_t(__ffs(peers) - 1) : lane;
  bool first = false;
  uint32_t h = H;
  if (has_entry && lane == leader) {
    if (my_key == kEmptyKey) {
      first = atomicCAS(&s_spec, 0u, 1u) == 0u;
    } else {
      h = uint32_t(splitmix64(my_key) >> 32) & (H - 1u);
      for (uint32_t probe = 0; probe < H; ++probe) {  // at most half full: ends at the key or a free slot
        const unsigned long long old = atomicCAS(&s_hkey[h], kEmptyKey, my_key);
        if (old == kEmptyKey || old == my_key) {
          first = old == kEmptyKey;
          break;
        }
        h = (h + 1u) & (H - 1u);
      }
    }
  }
  {  // local indices of the keys this warp inserted first (one counter atomic per warp)
    const unsigned ballot = __ballot_sync(0xffffffffu, first);
    uint32_t base = 0;
    if (ballot && lane == uint32_t(__ffs(ballot) - 1)) base = atomicAdd(&s_nloc, uint32_t(__popc(ballot)));
    base = __shfl_sync(0xffffffffu, base, ballot ? __ffs(ballot) - 1 : 0);
    if (first) {
      const uint32_t q = base + __popc(ballot & ((1u << lane) - 1u));
      s_hloc[h] = q;
      s_lkey[q] = my_key;
      s_lrow[q] = my_row;
    }
  }
  h = __shfl_sync(0xffffffffu, h, leader);
  __syncthreads();
  const uint32_t nloc = s_nloc;
  // 3. each warp's entries of a key join the key's list as one chain (lanes
  //    in order, linked by the group's leader with one exchange); each
  //    distinct key finds (or claims) its table slot (its L2 round trips
  //    overlap the lists and the copy)
  {
    const uint32_t q = has_entry ? s_hloc[h] : 0u;
    int32_t old = -1;
    if (has_entry && lane == leader) old = atomicExch(&s_head[q], int32_t(tid));
    old = __shfl_sync(0xffffffffu, old, leader);
    if (has_entry) {
      const unsigned above = peers & ~((2u << lane) - 1u);  // group lanes after this one
      s_next[tid] = above ? int32_t((tid & ~31u) + uint32_t(__ffs(above) - 1)) : old;
    }
  }
  {  // nloc <= tile <= blockDim: one local key per thread at most
    // optimizer_step's list positions for the tile's distinct keys, reserved
    // while the keys are claimed (one entry per local key: a key another
    // block claimed leaves a hole, which optimizer_step skips)
    uint32_t list_base = 0;
    if (!kDirect && tid == 0) list_base = atomicAdd(a.ctr, nloc);
    const uint32_t q = tid;
    const bool mine = q < nloc;
    bool claimed = false;
    uint32_t slot = kNoRow, vrow = kNoRow;
    if (mine) {
      const uint64_t key = s_lkey[q];
      if (kDirect) {
        slot = vrow = uint32_t(key);
      } else {
        const uint32_t rank = s_rank_base + q;
        if (rank < a.vcap) slot = acc_find_or_claim(a, key, rank, claimed, vrow);
        if (slot == kNoRow) raise_status(status, kStatusTableFull);
      }
      s_gslot[q] = slot;
      s_vrow[q] = vrow;
      s_crank[q] = claimed ? 1u : 0u;
    }
    if (!kDirect && tid == 0) s_claim_base = list_base;
  }
  __syncthreads();
  // the claimant lists the row lookup_or_insert cached for its key, so
  // optimizer_step need not probe the directory for it
  if (!kDirect)
    for (uint32_t q = tid; q < nloc; q += blockDim.x)
      a.list[s_claim_base + q] = s_crank[q] ? make_uint4(s_gslot[q], s_lrow[q], s_epoch, s_vrow[q])
                                            : make_uint4(kNoRow, kNoRow, 0u, kNoRow);
  if (tma) {  // every thread waits for the rows (bounded; the copy is local and completes)
    uint32_t polls = 0;
    while (!mbar_try_wait(&s_bar, 0u)) {
      if (++polls > kCopySpinLimit) {
        s_copy_ok = 0u;
        break;
      }
    }
  }
  __syncthreads();
  if (tma && tid == 0) {
    if (s_copy_ok) {
      mbar_inval(&s_bar);
    } else {
      raise_status(status, kStatusCopyTimeout);
      // wait (bounded) for the copy still in flight before the block's shared memory is released
      for (uint32_t w = 0; w < kCopySpinLimit && !mbar_try_wait(&s_bar, 0u); ++w) __nanosleep(64);
    }
  }
  if (!s_copy_ok) return;
  // 4. per (distinct key, chunk): the sum of its entries' chunks, validated
  //    and scaled on entry, added into the table
  bool bad = false;
  const uint32_t pairs = nloc * units;
  ChunkWalk w(tid, blockDim.x, units);
  for (uint32_t c = tid; c < pairs; c += blockDim.x, w.next()) {
    const uint32_t q = w.j, e = w.u * VEC;
    const uint32_t slot = s_gslot[q];
    float acc[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[v] = 0.0f;
    uint32_t count = 0;
    for (int32_t j = s_head[q]; j >= 0; j = s_next[j], ++count) {
      float g[VEC];
      ldv<VEC>(s_rows + size_t(j) * row_bytes, gdt, e, g);
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        if (scale == 1.0f) {  // g / 1 == g: no division (uniform branch)
          bad |= !(fabsf(g[v]) <= maxv);
        } else {
          const float sc = __fdiv_rn(g[v], scale);
          bad |= !(fabsf(sc) <= maxv);
          g[v] = round_to(gdt, sc);
        }
        acc[v] = __fadd_rn(acc[v], g[v]);
      }
    }
    if (slot == kNoRow) continue;
    float *dst = a.vals + size_t(s_vrow[q]) * dim + e;
    if constexpr (VEC == 4) red_add_v4(dst, acc[0], acc[1], acc[2], acc[3]);
    else atomicAdd(dst, acc[0]);
    if (!kDirect && w.u == 0u) atomicAdd(a.cnt + slot, count);
  }
  if (bad) raise_status(bad_word, kStatusBadGradient);
}

// Validation of a host batch before anything is added (the reference raises
// before accumulating, gradient_accumulator.hpp:88-104).
template <int VEC>
__global__ void __launch_bounds__(256)
k_acc_check(const void *__restrict__ grads, int gdt, size_t elems, float scale, float maxv, uint32_t *bad_word) {
  pdl_wait();
  pdl_trigger();
  bool bad = false;
  const size_t chunks = elems / VEC;
  for (size_t c = size_t(blockIdx.x) * blockDim.x + threadIdx.x; c < chunks; c += size_t(gridDim.x) * blockDim.x) {
    float g[VEC];
    ldv<VEC>(grads, gdt, c * VEC, g);
#pragma unroll
    for (int v = 0; v < VEC; ++v) bad |= !(fabsf(__fdiv_rn(g[v], scale)) <= maxv);
  }
  if (bad) raise_status(bad_word, kStatusBadGradient);
}

// Moves every claimed slot into a larger table (the window outgrew the old
// one between accumulate calls), keeping its dense row; the host copies the
// dense sums. One thread per listed slot.
__global__ void __launch_bounds__(256) k_acc_move(AccTab from, AccTab to, uint32_t *status) {
  const uint32_t G = from.mask + 1u;
  const uint32_t n = min(*from.ctr, G + 1u);
  if (blockIdx.x == 0 && threadIdx.x == 0) to.ctr[3] = from.ctr[3];  // dense rows stay where they are
  for (uint32_t g = blockIdx.x * blockDim.x + threadIdx.x; g < n; g += gridDim.x * blockDim.x) {
    const uint4 ent = from.list[g];
    const uint32_t slot = ent.x;
    if (slot == kNoRow) continue;  // a hole: the key was claimed by another block's entry
    const uint64_t key = from.slots[slot].x;
    bool claimed = false;
    uint32_t vrow = kNoRow;
    const uint32_t ns = acc_find_or_claim(to, key, ent.w, claimed, vrow);
    if (ns == kNoRow) {
      raise_status(status, kStatusTableFull);
      continue;
    }
    to.list[atomicAdd(to.ctr, 1u)] = make_uint4(ns, ent.y, ent.z, ent.w);
    to.cnt[ns] = from.cnt[slot];
  }
}

}  // namespace se_gpu
