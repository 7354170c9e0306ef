// Device code of the B200 store.
//
// HBM layout of one table (one per distinct dim):
//   directory  : 2^b buckets of 64 B = 5 keys (u64) + 5 row ids (u32) + pad,
//                open addressing with linear probing over buckets; replaces
//                FlatKeyDirectory + SegmentedLocatorTable
//                (core/flat_key_directory.hpp:42-85, core/segmented_locator_table.hpp:234-254).
//                The all-ones key is the empty marker; the one real key with
//                that value lives in a side slot (`special`).
//   slab arena : one contiguous slab per row, rows allocated by a bump
//                counter; slab = param[dim] | state0[dim] | state1[dim] | step,
//                each section 16-byte aligned (replaces EmbeddingArena and the
//                optimizer state arenas, hogwild_embedding_store.hpp:102-841,
//                optimizer/optimizer_state.hpp:37-156).
//   pending    : gradients accumulated since the last optimizer_step, in
//                arrival order (keys u64 + rows of the gradient dtype); the
//                step sorts them by row and reduces each key's rows in order
//                (replaces TransientArena, arena/transient_arena.hpp:119-269).
#pragma once

#include "se_common.cuh"

namespace se_gpu {

constexpr uint64_t kEmptyKey = ~0ull;
constexpr uint32_t kNoRow = 0xffffffffu;
// Row word of an erased key (a tombstone): the key keeps its slot, so probe
// sequences stay intact, and reads as absent; an insert of the same key
// revives the slot, a rehash drops it.
constexpr uint32_t kDeadRow = 0xfffffffeu;
constexpr int kBucketSlots = 5;

struct alignas(64) Bucket {
  unsigned long long keys[kBucketSlots];
  uint32_t rows[kBucketSlots];
  uint32_t pad;
};
static_assert(sizeof(Bucket) == 64, "bucket must be one 64-byte line");

struct Dir {
  Bucket *buckets;
  uint64_t nbuckets;  // power of two
  uint32_t *special;  // [0] claim flag of the all-ones key, [1] its row
};

// Slab layout of one row.
struct Layout {
  uint32_t dim;
  uint32_t stride;     // slab bytes, multiple of 16
  uint32_t state0;     // byte offsets
  uint32_t state1;
  uint32_t step;
  uint32_t nstate;     // 0, 1 (Adagrad) or 2 (Adam)
  int32_t pdt, odt;    // value / optimizer dtypes (SE_FLOAT32 / SE_FLOAT16 / SE_BFLOAT16)
  uint32_t score;      // offset of the row's u64 score; 0: the store keeps no scores
};

// Home bucket from the high bits of the SplitMix64 hash: the hash partitioner
// assigns GPUs by the low bits (partitioner.hpp:316-327), so a GPU's keys
// still spread over all of its buckets.
__device__ __forceinline__ uint64_t home_bucket(uint64_t h, uint64_t nbuckets) {
  return __umul64hi(h, nbuckets);
}

// Bucket loads: kLoadL2 bypasses L1 (ld.cg; words other SMs may be
// writing), kLoadReadOnly takes the read-only path (ld.global.nc; no writes
// during the launch), kLoadCached is a plain load that L1 may serve (stale
// views are allowed: every decision on an empty slot is checked by a CAS).
enum BucketLoad : int { kLoadL2 = 1, kLoadReadOnly = 0, kLoadCached = 2 };

template <int kMode>
__device__ __forceinline__ void load_bucket(const Bucket *b, uint64_t (&k)[kBucketSlots],
                                            uint32_t (&r)[kBucketSlots]) {
  const uint4 *p = reinterpret_cast<const uint4 *>(b);
  uint4 a0, a1, a2, a3;
  if constexpr (kMode == kLoadL2) {
    a0 = __ldcg(p); a1 = __ldcg(p + 1); a2 = __ldcg(p + 2); a3 = __ldcg(p + 3);
  } else if constexpr (kMode == kLoadCached) {
    a0 = p[0]; a1 = p[1]; a2 = p[2]; a3 = p[3];
  } else {
    a0 = __ldg(p); a1 = __ldg(p + 1); a2 = __ldg(p + 2); a3 = __ldg(p + 3);
  }
  k[0] = uint64_t(a0.x) | (uint64_t(a0.y) << 32);
  k[1] = uint64_t(a0.z) | (uint64_t(a0.w) << 32);
  k[2] = uint64_t(a1.x) | (uint64_t(a1.y) << 32);
  k[3] = uint64_t(a1.z) | (uint64_t(a1.w) << 32);
  k[4] = uint64_t(a2.x) | (uint64_t(a2.y) << 32);
  r[0] = a2.z; r[1] = a2.w; r[2] = a3.x; r[3] = a3.y; r[4] = a3.z;
}

// Row of `key`, or kNoRow when absent (or erased). Probing stops at the first
// bucket that holds the key or an empty slot; slots never return to empty
// (erasing leaves a tombstone), so the key cannot sit past an empty slot of
// its probe sequence. Bounded by the bucket count.
template <bool kCoherent>
__device__ __forceinline__ uint32_t dir_find(const Dir &d, uint64_t key) {
  if (key == kEmptyKey) return kCoherent ? __ldcg(d.special + 1) : __ldg(d.special + 1);
  const uint64_t mask = d.nbuckets - 1;
  uint64_t b = home_bucket(splitmix64(key), d.nbuckets);
  for (uint64_t probe = 0; probe < d.nbuckets; ++probe) {
    uint64_t k[kBucketSlots];
    uint32_t r[kBucketSlots];
    load_bucket<kCoherent ? kLoadL2 : kLoadReadOnly>(d.buckets + b, k, r);
    bool empty = false;
#pragma unroll
    for (int s = 0; s < kBucketSlots; ++s) {
      if (k[s] == key) return r[s] == kDeadRow ? kNoRow : r[s];
      empty |= k[s] == kEmptyKey;
    }
    if (empty) return kNoRow;
    b = (b + 1) & mask;
  }
  return kNoRow;
}

enum InsertKind : int { kFound = 0, kInserted = 1, kFull = 2 };

struct InsertResult {
  uint32_t *row_word;
  int kind;
  uint32_t seen;  // found: the row word as the probe read it (kNoRow for a claim)
};

// Find-or-claim by one thread. A claim CASes the key into the first empty
// slot of its probe sequence; the claimant then owns the row word. A key
// found with a tombstone row word is revived by the caller (revive_row).
__device__ __forceinline__ InsertResult dir_find_or_insert(const Dir &d, uint64_t key) {
  if (key == kEmptyKey) {
    const uint32_t old = atomicCAS(d.special, 0u, 1u);
    return {d.special + 1, old == 0u ? kInserted : kFound, kNoRow};
  }
  const uint64_t mask = d.nbuckets - 1;
  uint64_t b = home_bucket(splitmix64(key), d.nbuckets);
  for (uint64_t probe = 0; probe < d.nbuckets; ++probe) {
    Bucket *bk = d.buckets + b;
    uint64_t k[kBucketSlots];
    uint32_t r[kBucketSlots];
    load_bucket<kLoadCached>(bk, k, r);  // hot buckets from L1; claims are checked by the CAS
#pragma unroll
    for (int s = 0; s < kBucketSlots; ++s) {
      if (k[s] == key) return {&bk->rows[s], kFound, r[s]};
      if (k[s] == kEmptyKey) {
        const unsigned long long old = atomicCAS(&bk->keys[s], kEmptyKey, key);
        if (old == kEmptyKey) return {&bk->rows[s], kInserted, kNoRow};
        if (old == key) return {&bk->rows[s], kFound, kNoRow};
      }
    }
    b = (b + 1) & mask;
  }
  return {nullptr, kFull, kNoRow};
}

// A found key's row word: kInserted when it was a tombstone that this thread
// claimed back (its row is then taken like a new key's), 3 when the row is
// not published yet (claimed in this launch), else kFound with *row set.
// `seen` is the word as the probe read it: a published row there is final
// (rows change only by erase, which no insert kernel runs beside), so the
// word is read again only when the probe saw it unpublished or erased.
__device__ __forceinline__ int resolve_found(uint32_t *word, uint32_t *row, uint32_t seen = kNoRow) {
  if (seen < kDeadRow) {
    *row = seen;
    return kFound;
  }
  *row = __ldcg(word);
  if (*row == kDeadRow) return atomicCAS(word, kDeadRow, kNoRow) == kDeadRow ? kInserted : 3;
  return *row == kNoRow ? 3 : kFound;
}

// Row word of `key` (live, unpublished or a tombstone), or nullptr when the
// key never had a slot. Used by erase.
__device__ __forceinline__ uint32_t *dir_slot(const Dir &d, uint64_t key) {
  if (key == kEmptyKey) return d.special + 1;
  const uint64_t mask = d.nbuckets - 1;
  uint64_t b = home_bucket(splitmix64(key), d.nbuckets);
  for (uint64_t probe = 0; probe < d.nbuckets; ++probe) {
    uint64_t k[kBucketSlots];
    uint32_t r[kBucketSlots];
    load_bucket<kLoadL2>(d.buckets + b, k, r);
    bool empty = false;
#pragma unroll
    for (int s = 0; s < kBucketSlots; ++s) {
      if (k[s] == key) return &d.buckets[b].rows[s];
      empty |= k[s] == kEmptyKey;
    }
    if (empty) return nullptr;
    b = (b + 1) & mask;
  }
  return nullptr;
}

// Where claimants take their rows: the rows of erased keys first (a stack,
// `free_top` entries; pops may drive it below zero, which the next push
// clamps), else the bump counter. free_top is null for a table that never
// had a key erased.
struct RowAlloc {
  uint32_t *next_row;
  int *free_top;
  const uint32_t *free_rows;
  uint64_t capacity;
};

// Lanes of the calling warp whose global thread index t is below `active`
// (threads past the end of a launch's work have returned).
__device__ __forceinline__ unsigned live_lanes(size_t t, size_t active) {
  const size_t base = t & ~size_t(31);
  if (active >= base + 32) return 0xffffffffu;
  return active > base ? (1u << unsigned(active - base)) - 1u : 0u;
}

// Rows for the claimants of one warp (`claim` set) with one atomic per
// warp and source: every lane of `lanes` calls it; claimants get their row,
// others kNoRow. A row at or past the arena's capacity means it is full.
__device__ __forceinline__ uint32_t take_rows_warp(const RowAlloc &a, unsigned lanes, bool claim) {
  const unsigned claims = __ballot_sync(lanes, claim);
  if (claims == 0u) return kNoRow;
  const uint32_t lane = threadIdx.x & 31u;
  const int leader = __ffs(claims) - 1;
  const int cnt = __popc(claims);
  int top = 0;
  uint32_t bump = 0;
  if (int(lane) == leader) {
    if (a.free_top != nullptr && __ldcg(a.free_top) > 0) {
      top = atomicSub(a.free_top, cnt);
      if (uint64_t(max(top, 0)) > a.capacity) top = int(a.capacity);  // never more free rows than the arena holds
    }
    const int from_free = min(max(top, 0), cnt);
    if (from_free < cnt) bump = atomicAdd(a.next_row, uint32_t(cnt - from_free));
  }
  top = __shfl_sync(lanes, top, leader);
  bump = __shfl_sync(lanes, bump, leader);
  if (!claim) return kNoRow;
  const int from_free = min(max(top, 0), cnt);
  const int rank = __popc(claims & ((1u << lane) - 1u));
  if (rank < from_free) return __ldcg(a.free_rows + (top - 1 - rank));  // entries [top - from_free, top)
  return bump + uint32_t(rank - from_free);
}

// Plain insert used when rebuilding a larger directory (keys are distinct).
__device__ __forceinline__ bool dir_insert_unique(const Dir &d, uint64_t key, uint32_t row) {
  const uint64_t mask = d.nbuckets - 1;
  uint64_t b = home_bucket(splitmix64(key), d.nbuckets);
  for (uint64_t probe = 0; probe < d.nbuckets; ++probe) {
    Bucket *bk = d.buckets + b;
#pragma unroll
    for (int s = 0; s < kBucketSlots; ++s) {
      if (atomicCAS(&bk->keys[s], kEmptyKey, key) == kEmptyKey) {
        bk->rows[s] = row;
        return true;
      }
    }
    b = (b + 1) & mask;
  }
  return false;
}

// ---------------------------------------------------------------------------
// Keys and runtime-typed element access
// ---------------------------------------------------------------------------

// Key i of a key array of the given dtype, widened to u64 with sign extension.
__device__ __forceinline__ uint64_t load_key(const void *keys, int key_dtype, size_t i) {
  switch (key_dtype) {
  case SE_KEY_INT32: return key_u64(static_cast<const int32_t *>(keys)[i]);
  case SE_KEY_UINT32: return key_u64(static_cast<const uint32_t *>(keys)[i]);
  case SE_KEY_INT64: return key_u64(static_cast<const int64_t *>(keys)[i]);
  default: return static_cast<const uint64_t *>(keys)[i];
  }
}

__device__ __forceinline__ float bits_to_f(int dt, uint32_t bits16) {
  if (dt == SE_FLOAT16) return __half2float(__ushort_as_half(uint16_t(bits16)));
  return __uint_as_float(bits16 << 16);
}
__device__ __forceinline__ uint32_t f_to_bits(int dt, float f) {
  if (dt == SE_FLOAT16) return __half_as_ushort(__float2half_rn(f));
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// VEC consecutive elements starting at element index e of an array of dtype dt.
template <int VEC>
__device__ __forceinline__ void ldv(const void *base, int dt, size_t e, float (&f)[VEC]) {
  if constexpr (VEC == 4) {
    if (dt == SE_FLOAT32) {
      const float4 v = *reinterpret_cast<const float4 *>(static_cast<const float *>(base) + e);
      f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
    } else {
      const uint2 v = *reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(base) + e);
      f[0] = bits_to_f(dt, v.x & 0xffffu); f[1] = bits_to_f(dt, v.x >> 16);
      f[2] = bits_to_f(dt, v.y & 0xffffu); f[3] = bits_to_f(dt, v.y >> 16);
    }
  } else {
    if (dt == SE_FLOAT32) f[0] = static_cast<const float *>(base)[e];
    else f[0] = bits_to_f(dt, static_cast<const uint16_t *>(base)[e]);
  }
}

template <int VEC>
__device__ __forceinline__ void stv(void *base, int dt, size_t e, const float (&f)[VEC]) {
  if constexpr (VEC == 4) {
    if (dt == SE_FLOAT32) {
      *reinterpret_cast<float4 *>(static_cast<float *>(base) + e) = make_float4(f[0], f[1], f[2], f[3]);
    } else {
      uint2 v;
      v.x = f_to_bits(dt, f[0]) | (f_to_bits(dt, f[1]) << 16);
      v.y = f_to_bits(dt, f[2]) | (f_to_bits(dt, f[3]) << 16);
      *reinterpret_cast<uint2 *>(static_cast<uint16_t *>(base) + e) = v;
    }
  } else {
    if (dt == SE_FLOAT32) static_cast<float *>(base)[e] = f[0];
    else static_cast<uint16_t *>(base)[e] = uint16_t(f_to_bits(dt, f[0]));
  }
}

// Round a float to dtype dt and back (the value a store of dt would keep).
__device__ __forceinline__ float round_to(int dt, float f) {
  return dt == SE_FLOAT32 ? f : bits_to_f(dt, f_to_bits(dt, f));
}

// ---------------------------------------------------------------------------
// Row initialisation (UniformInitializer, initializer/uniform_initializer.hpp:36-53
// -> simd_uniform_init, simd/uniform_init_ops.hpp:32-134; ZerosInitializer)
// ---------------------------------------------------------------------------

struct InitSpec {
  int kind;         // SE_INIT_ZEROS / SE_INIT_UNIFORM
  float lo, diff;   // min, max - min
  float state0;     // initial value of optimizer state 0 (Adagrad accumulator)
};

// Element e of the uniform row of `key`: fmix32(seed + e) mapped to [1, 2),
// minus one, then fused (f - 1) * (max - min) + min. The reference's AVX-512
// body and its compiled scalar tail both fuse this step.
__device__ __forceinline__ float uniform_value(uint32_t seed, uint32_t e, float lo, float diff) {
  const uint32_t h = fmix32(seed + e);
  const float f = __uint_as_float((h >> 9) | 0x3f800000u) - 1.0f;
  return __fmaf_rn(f, diff, lo);
}

}  // namespace se_gpu
