// Device code of the partitioners and of the stable route (shared by the
// partition entry points and the peer-memory exchange of the store).
//
// The three registered partitioners (sparse_embedding/src/ops/partitioner.hpp:72-406)
// as bit-identical element-wise kernels, plus the stable route (histogram +
// scatter) and the row permutations used by the cross-GPU exchange. All are
// integer, HBM-bound kernels: per key they read K bytes and write 4
// (partition id) or 1 (filter mask) bytes; the route reads the keys twice
// (count, scatter) and writes K + 4 bytes per key.
#pragma once

#include <cub/block/block_scan.cuh>

#include <stdexcept>
#include <type_traits>

#include "se_common.cuh"

namespace se_gpu {
namespace {

// ---------------------------------------------------------------------------
// Per-key partition function
// ---------------------------------------------------------------------------

struct PartSpec {
  int kind;
  uint32_t n;
  bool pow2;
};

// ModuloPartitioner::partition_span (partitioner.hpp:92-132) with the signed
// floor modulo of modulo_partition (common/dtypes.hpp:97-111). A 64-bit
// signed remainder by n (1 <= n < 2^32) is exact, so no 128-bit arithmetic is
// needed on the device.
template <class K> __device__ __forceinline__ uint32_t modulo_of(K key, uint32_t n, bool pow2) {
  if (pow2) return uint32_t(uint64_t(int64_t(key)) & uint64_t(n - 1));
  if constexpr (sizeof(K) == 4 && std::is_signed<K>::value) {
    int64_t r = int64_t(key) % int64_t(n);
    return uint32_t(r < 0 ? r + int64_t(n) : r);
  } else if constexpr (std::is_signed<K>::value) {
    int64_t r = int64_t(key) % int64_t(n);
    return uint32_t(r < 0 ? r + int64_t(n) : r);
  } else {
    return uint32_t(uint64_t(key) % uint64_t(n));
  }
}

template <class K> __device__ __forceinline__ uint32_t partition_of(const PartSpec &s, K key) {
  if (s.kind == SE_PART_MODULO) return modulo_of<K>(key, s.n, s.pow2);
  if (s.kind == SE_PART_FAST_RANGE) {
    // fast_range_64 / fast_range_32 (partitioner.hpp:36-43, 191-204).
    if constexpr (sizeof(K) == 8) return uint32_t(__umul64hi(uint64_t(key), uint64_t(s.n)));
    else return uint32_t((uint64_t(uint32_t(key)) * s.n) >> 32);
  }
  // HashPartitioner (partitioner.hpp:282-340): splitmix64 for 8-byte keys,
  // murmur fmix32 for 4-byte keys; mask when n is a power of two, else fast range.
  if constexpr (sizeof(K) == 8) {
    const uint64_t h = splitmix64(uint64_t(key));
    return s.pow2 ? uint32_t(h & uint64_t(s.n - 1)) : uint32_t(__umul64hi(h, uint64_t(s.n)));
  } else {
    const uint32_t h = fmix32(uint32_t(key));
    return s.pow2 ? (h & (s.n - 1)) : uint32_t((uint64_t(h) * s.n) >> 32);
  }
}

// Host-side validation and key-type dispatch shared by the launchers.
PartSpec make_spec(int kind, uint32_t n) {
  if (n == 0) throw std::invalid_argument("num_shards must be > 0");
  if (kind < SE_PART_MODULO || kind > SE_PART_FAST_RANGE)
    throw std::invalid_argument("unknown partitioner kind");
  return PartSpec{kind, n, (n & (n - 1)) == 0};
}

void check_key_dtype(int key_dtype) {
  if (key_dtype < SE_KEY_INT32 || key_dtype > SE_KEY_UINT64)
    throw std::invalid_argument("unsupported key dtype code");
}

template <class F> void dispatch_key(int key_dtype, F &&f) {
  switch (key_dtype) {
  case SE_KEY_INT32: f(int32_t{}); break;
  case SE_KEY_UINT32: f(uint32_t{}); break;
  case SE_KEY_INT64: f(int64_t{}); break;
  default: f(uint64_t{}); break;
  }
}

template <class K>
__global__ void k_partition(PartSpec s, const K *__restrict__ keys, size_t count,
                            uint32_t *__restrict__ out) {
  const size_t stride = size_t(gridDim.x) * blockDim.x;
  for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride)
    out[i] = partition_of<K>(s, keys[i]);
}

template <class K>
__global__ void k_filter(PartSpec s, const K *__restrict__ keys, size_t count, uint32_t target,
                         uint8_t *__restrict__ mask) {
  const size_t stride = size_t(gridDim.x) * blockDim.x;
  for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride)
    mask[i] = partition_of<K>(s, keys[i]) == target ? 1 : 0;
}

// ---------------------------------------------------------------------------
// Stable route: counts per (tile, partition) -> partition-major exclusive
// offsets -> in-order scatter. A tile is 2048 keys; each of its 8 warps owns
// 256 consecutive keys and ranks them 32 at a time with __match_any_sync.
// ---------------------------------------------------------------------------

constexpr int kRouteThreads = 256;
constexpr int kRouteWarps = kRouteThreads / 32;
constexpr int kRouteWarpKeys = 256;
constexpr int kRouteTile = kRouteWarps * kRouteWarpKeys;
constexpr uint32_t kRouteMaxPartitions = 1024;

template <class K, int TILE = kRouteTile>
__global__ void k_route_count(PartSpec s, const K *__restrict__ keys, size_t count,
                              uint32_t *__restrict__ tile_counts) {
  extern __shared__ uint32_t hist[];
  for (uint32_t p = threadIdx.x; p < s.n; p += blockDim.x) hist[p] = 0;
  __syncthreads();
  const size_t base = size_t(blockIdx.x) * TILE;
  for (int j = threadIdx.x; j < TILE; j += blockDim.x) {
    const size_t i = base + j;
    if (i < count) atomicAdd(&hist[partition_of<K>(s, keys[i])], 1u);
  }
  __syncthreads();
  for (uint32_t p = threadIdx.x; p < s.n; p += blockDim.x)
    tile_counts[size_t(blockIdx.x) * s.n + p] = hist[p];
}

// One block: offsets[t][p] = sum_{q<p} total[q] + sum_{t'<t} c[t'][p].
__global__ void k_route_scan(const uint32_t *__restrict__ tile_counts, uint32_t tiles, uint32_t n,
                             uint32_t *__restrict__ tile_offsets, uint32_t *__restrict__ counts) {
  using Scan = cub::BlockScan<uint32_t, 1024>;
  __shared__ typename Scan::TempStorage tmp;
  __shared__ uint32_t carry;
  uint32_t running = 0;  // partition base, valid in thread 0
  for (uint32_t p = 0; p < n; ++p) {
    if (threadIdx.x == 0) carry = running;
    __syncthreads();
    for (uint32_t t0 = 0; t0 < tiles; t0 += 1024) {
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
}

template <class K>
__global__ void k_route_scatter(PartSpec s, const K *__restrict__ keys, size_t count,
                                const uint32_t *__restrict__ tile_offsets, K *__restrict__ send_keys,
                                uint32_t *__restrict__ send_pos) {
  extern __shared__ uint32_t warp_base[];  // [kRouteWarps][n]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  for (uint32_t j = threadIdx.x; j < kRouteWarps * s.n; j += blockDim.x) warp_base[j] = 0;
  __syncthreads();
  const size_t wbase = size_t(blockIdx.x) * kRouteTile + size_t(warp) * kRouteWarpKeys;
  uint32_t *mine = warp_base + size_t(warp) * s.n;
  // Pass A: per-warp counts per partition.
  for (int r = 0; r < kRouteWarpKeys; r += 32) {
    const size_t i = wbase + r + lane;
    const bool valid = i < count;
    const uint32_t pid = valid ? partition_of<K>(s, keys[i]) : 0xffffffffu;
    const unsigned peers = __match_any_sync(0xffffffffu, pid);
    if (valid && (peers & lt) == 0) mine[pid] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  // Exclusive prefix over warps, seeded with the tile's global offsets.
  for (uint32_t p = threadIdx.x; p < s.n; p += blockDim.x) {
    uint32_t run = tile_offsets[size_t(blockIdx.x) * s.n + p];
    for (int w = 0; w < kRouteWarps; ++w) {
      const uint32_t c = warp_base[size_t(w) * s.n + p];
      warp_base[size_t(w) * s.n + p] = run;
      run += c;
    }
  }
  __syncthreads();
  // Pass B: in-order placement.
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
    uint32_t dst = 0;
    if (valid) dst = mine[pid] + __popc(peers & lt);
    __syncwarp();
    if (valid) {
      send_keys[dst] = key;
      send_pos[dst] = uint32_t(i);
      if ((peers & lt) == 0) mine[pid] += __popc(peers);
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Row permutation (exchange un-permute / permute)
// ---------------------------------------------------------------------------

template <class V>
__global__ void k_permute_rows(const V *__restrict__ in, V *__restrict__ out,
                               const uint32_t *__restrict__ pos, size_t rows, size_t vecs_per_row,
                               int scatter) {
  const size_t total = rows * vecs_per_row;
  const size_t stride = size_t(gridDim.x) * blockDim.x;
  for (size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total; t += stride) {
    const size_t j = t / vecs_per_row, v = t - j * vecs_per_row;
    const size_t p = pos[j];
    if (scatter) out[j * vecs_per_row + v] = in[p * vecs_per_row + v];
    else out[p * vecs_per_row + v] = in[j * vecs_per_row + v];
  }
}

}  // namespace
}  // namespace se_gpu
