// Partition kernels: the three registered partitioners
// (sparse_embedding/src/ops/partitioner.hpp:72-406) as bit-identical
// element-wise kernels, plus the stable route (histogram + scatter) and the
// row permutations used by the cross-GPU exchange.
//
// All three are integer, HBM-bound kernels: per key they read K bytes and
// write 4 (partition id) or 1 (filter mask) bytes; the route kernels read the
// keys twice (count, scatter) and write K + 4 bytes per key.

#include <cub/block/block_scan.cuh>

#include <algorithm>
#include <map>
#include <tuple>
#include <mutex>
#include <string>

#include "se_common.cuh"
#include "se_host.hpp"

namespace se_gpu {

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

template <class K>
__global__ void k_route_count(PartSpec s, const K *__restrict__ keys, size_t count,
                              uint32_t *__restrict__ tile_counts) {
  extern __shared__ uint32_t hist[];
  for (uint32_t p = threadIdx.x; p < s.n; p += blockDim.x) hist[p] = 0;
  __syncthreads();
  const size_t base = size_t(blockIdx.x) * kRouteTile;
  for (int j = threadIdx.x; j < kRouteTile; j += blockDim.x) {
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

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

namespace {

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


// Scratch cached per (device, stream, use): calls on one stream are ordered,
// so they can share a buffer; a buffer only grows, and lives until the
// process exits. (Per-call stream-ordered allocation stalled multi-GPU steps.)
std::mutex g_route_mu;
std::map<std::tuple<int, cudaStream_t, int>, std::pair<void *, size_t>> g_route_bufs;

enum ScratchUse { kUseRoute = 0, kUseKeysIn = 1, kUseIdsOut = 2 };

// Host-memory partition/filter calls stage through shared buffers and wait for
// their result, so they run one at a time.
std::mutex g_host_call_mu;

void *stream_scratch(int device, cudaStream_t st, int use, size_t bytes) {
  std::lock_guard<std::mutex> lock(g_route_mu);
  auto &b = g_route_bufs[{device, st, use}];
  if (b.second < bytes) {
    if (b.first) {
      cuda_check(cudaStreamSynchronize(st), "route scratch sync");
      cuda_check(cudaFree(b.first), "cudaFree");
      b.first = nullptr;
    }
    const size_t cap = std::max<size_t>(bytes, std::max<size_t>(2 * b.second, 1 << 16));
    cuda_check(cudaMalloc(&b.first, cap), "cudaMalloc(stream scratch)");
    b.second = cap;
  }
  return b.first;
}

}  // namespace

}  // namespace se_gpu

using namespace se_gpu;

extern "C" int se_partition(int32_t kind, uint32_t num_partitions, int32_t key_dtype,
                            const void *keys, size_t num_keys, uint32_t *out, int32_t device,
                            void *stream_ptr) {
  return guarded([&] {
    const PartSpec s = make_spec(kind, num_partitions);
    check_key_dtype(key_dtype);
    if (num_keys == 0) return;
    DeviceGuard dg(device);
    cudaStream_t st = static_cast<cudaStream_t>(stream_ptr);
    const size_t kb = key_bytes(key_dtype) * num_keys, ob = 4 * num_keys;
    const bool dk = is_device_ptr(keys), dout = is_device_ptr(out);
    std::unique_lock<std::mutex> host_lock(g_host_call_mu, std::defer_lock);
    if (!dk || !dout) host_lock.lock();
    const void *dkeys = keys;
    if (!dk) {
      void *sk = stream_scratch(device, st, kUseKeysIn, kb);
      cuda_check(cudaMemcpyAsync(sk, keys, kb, cudaMemcpyHostToDevice, st), "copy keys");
      dkeys = sk;
    }
    uint32_t *dres = dout ? out : static_cast<uint32_t *>(stream_scratch(device, st, kUseIdsOut, ob));
    dispatch_key(key_dtype, [&](auto tag) {
      using K = decltype(tag);
      k_partition<K><<<grid_for(num_keys, 256, 148 * 16), 256, 0, st>>>(
          s, static_cast<const K *>(dkeys), num_keys, dres);
      launched("k_partition");
    });
    if (!dout) {
      cuda_check(cudaMemcpyAsync(out, dres, ob, cudaMemcpyDeviceToHost, st), "copy ids");
      cuda_check(cudaStreamSynchronize(st), "partition sync");
    }
  });
}

extern "C" int se_filter(int32_t kind, uint32_t num_partitions, int32_t key_dtype,
                         const void *keys, size_t num_keys, uint32_t target, uint8_t *mask,
                         int32_t device, void *stream_ptr) {
  return guarded([&] {
    const PartSpec s = make_spec(kind, num_partitions);
    check_key_dtype(key_dtype);
    if (num_keys == 0) return;
    DeviceGuard dg(device);
    cudaStream_t st = static_cast<cudaStream_t>(stream_ptr);
    const size_t kb = key_bytes(key_dtype) * num_keys;
    const bool dk = is_device_ptr(keys), dout = is_device_ptr(mask);
    std::unique_lock<std::mutex> host_lock(g_host_call_mu, std::defer_lock);
    if (!dk || !dout) host_lock.lock();
    const void *dkeys = keys;
    if (!dk) {
      void *sk = stream_scratch(device, st, kUseKeysIn, kb);
      cuda_check(cudaMemcpyAsync(sk, keys, kb, cudaMemcpyHostToDevice, st), "copy keys");
      dkeys = sk;
    }
    uint8_t *dres = dout ? mask : static_cast<uint8_t *>(stream_scratch(device, st, kUseIdsOut, num_keys));
    dispatch_key(key_dtype, [&](auto tag) {
      using K = decltype(tag);
      k_filter<K><<<grid_for(num_keys, 256, 148 * 16), 256, 0, st>>>(
          s, static_cast<const K *>(dkeys), num_keys, target, dres);
      launched("k_filter");
    });
    if (!dout) {
      cuda_check(cudaMemcpyAsync(mask, dres, num_keys, cudaMemcpyDeviceToHost, st), "copy mask");
      cuda_check(cudaStreamSynchronize(st), "filter sync");
    }
  });
}

extern "C" int se_partition_route(int32_t kind, uint32_t num_partitions, int32_t key_dtype,
                                  const void *keys, size_t num_keys, void *send_keys,
                                  uint32_t *send_positions, uint32_t *counts, int32_t device,
                                  void *stream_ptr) {
  return guarded([&] {
    const PartSpec s = make_spec(kind, num_partitions);
    check_key_dtype(key_dtype);
    if (num_partitions > kRouteMaxPartitions)
      throw std::invalid_argument("route supports at most 1024 partitions");
    if (num_keys > 0xffffffffull) throw std::invalid_argument("route supports < 2^32 keys");
    DeviceGuard dg(device);
    cudaStream_t st = static_cast<cudaStream_t>(stream_ptr);
    if (num_keys == 0) {
      cuda_check(cudaMemsetAsync(counts, 0, 4 * size_t(num_partitions), st), "memset counts");
      return;
    }
    if (!is_device_ptr(keys) || !is_device_ptr(send_keys) || !is_device_ptr(send_positions) ||
        !is_device_ptr(counts))
      throw std::invalid_argument("se_partition_route takes device pointers only");
    const uint32_t tiles = uint32_t((num_keys + kRouteTile - 1) / kRouteTile);
    const size_t words = size_t(tiles) * num_partitions;
    uint32_t *tile_counts = static_cast<uint32_t *>(stream_scratch(device, st, kUseRoute, 2 * words * 4));
    uint32_t *tile_offsets = tile_counts + words;
    dispatch_key(key_dtype, [&](auto tag) {
      using K = decltype(tag);
      const K *k = static_cast<const K *>(keys);
      k_route_count<K><<<tiles, kRouteThreads, num_partitions * 4, st>>>(s, k, num_keys, tile_counts);
      launched("k_route_count");
      k_route_scan<<<1, 1024, 0, st>>>(tile_counts, tiles, num_partitions, tile_offsets, counts);
      launched("k_route_scan");
      k_route_scatter<K><<<tiles, kRouteThreads, kRouteWarps * num_partitions * 4, st>>>(
          s, k, num_keys, tile_offsets, static_cast<K *>(send_keys), send_positions);
      launched("k_route_scatter");
    });
  });
}

extern "C" int se_permute_rows(const void *in_rows, void *out_rows, const uint32_t *positions,
                               size_t num_rows, size_t row_bytes, int32_t scatter, int32_t device,
                               void *stream_ptr) {
  return guarded([&] {
    if (num_rows == 0 || row_bytes == 0) return;
    DeviceGuard dg(device);
    cudaStream_t st = static_cast<cudaStream_t>(stream_ptr);
    if (!is_device_ptr(in_rows) || !is_device_ptr(out_rows) || !is_device_ptr(positions))
      throw std::invalid_argument("se_permute_rows takes device pointers only");
    const uintptr_t a = uintptr_t(in_rows) | uintptr_t(out_rows) | uintptr_t(row_bytes);
    auto run = [&](auto vtag) {
      using V = decltype(vtag);
      const size_t vpr = row_bytes / sizeof(V);
      k_permute_rows<V><<<grid_for(num_rows * vpr, 256, 148 * 32), 256, 0, st>>>(
          static_cast<const V *>(in_rows), static_cast<V *>(out_rows), positions, num_rows, vpr,
          scatter);
      launched("k_permute_rows");
    };
    if (a % 16 == 0) run(uint4{});
    else if (a % 4 == 0) run(uint32_t{});
    else run(uint8_t{});
  });
}

// ---------------------------------------------------------------------------
// se_partition_route_noalloc: the same three route kernels, with their scratch
// in a fixed device array instead of stream-ordered allocations, for callers
// that cannot allocate device memory during a step (a host framework that owns
// nearly all device memory through its own allocator, or a serving loop that
// must not fail or stall on an allocation mid-batch).
// ---------------------------------------------------------------------------

namespace se_gpu {
namespace {

// Per-tile partition counts followed by per-tile offsets; every word a call
// reads was written earlier in that call (k_route_count writes all counts of
// every tile, k_route_scan all offsets), so nothing needs clearing between
// calls. 2 x 65536 u32 = 512 KiB per device, kept until the process exits.
constexpr size_t kNoAllocWords = 65536;
static __device__ __align__(256) uint32_t g_route_scratch[2 * kNoAllocWords];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
uint32_t *g_scratch_ptr[kMaxDevices] = {};

// Device address of g_route_scratch on `device` (current), looked up once per
// device. In host code the symbol itself only names a host-side stand-in.
uint32_t *route_scratch(int device) {
  if (device < 0 || device >= kMaxDevices) throw std::invalid_argument("device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[device]) {
    void *p = nullptr;
    cuda_check(cudaGetSymbolAddress(&p, g_route_scratch), "cudaGetSymbolAddress(route scratch)");
    g_scratch_ptr[device] = static_cast<uint32_t *>(p);
  }
  return g_scratch_ptr[device];
}

}  // namespace
}  // namespace se_gpu

extern "C" int se_partition_route_noalloc(int32_t kind, uint32_t num_partitions, int32_t key_dtype,
                                          const void *keys, size_t num_keys, void *send_keys,
                                          uint32_t *send_positions, uint32_t *counts, int32_t device,
                                          void *stream_ptr) {
  return guarded([&] {
    const PartSpec s = make_spec(kind, num_partitions);
    check_key_dtype(key_dtype);
    if (num_partitions > kRouteMaxPartitions)
      throw std::invalid_argument("route supports at most 1024 partitions");
    const uint64_t tiles = (uint64_t(num_keys) + kRouteTile - 1) / kRouteTile;
    if (tiles * num_partitions > kNoAllocWords)
      throw std::invalid_argument("se_partition_route_noalloc: ceil(num_keys / 2048) * num_partitions = " +
                                  std::to_string(tiles * num_partitions) +
                                  " exceeds its fixed scratch of 65536 entries; use se_partition_route");
    DeviceGuard dg(device);
    uint32_t *scratch = route_scratch(device);
    cudaStream_t st = static_cast<cudaStream_t>(stream_ptr);
    if (num_keys == 0) {
      cuda_check(cudaMemsetAsync(counts, 0, 4 * size_t(num_partitions), st), "memset counts");
      return;
    }
    if (!is_device_ptr(keys) || !is_device_ptr(send_keys) || !is_device_ptr(send_positions) ||
        !is_device_ptr(counts))
      throw std::invalid_argument("se_partition_route_noalloc takes device pointers only");
    uint32_t *tile_counts = scratch;
    uint32_t *tile_offsets = scratch + kNoAllocWords;
    dispatch_key(key_dtype, [&](auto tag) {
      using K = decltype(tag);
      const K *k = static_cast<const K *>(keys);
      k_route_count<K><<<unsigned(tiles), kRouteThreads, num_partitions * 4, st>>>(s, k, num_keys, tile_counts);
      launched("k_route_count");
      k_route_scan<<<1, 1024, 0, st>>>(tile_counts, uint32_t(tiles), num_partitions, tile_offsets, counts);
      launched("k_route_scan");
      k_route_scatter<K><<<unsigned(tiles), kRouteThreads, kRouteWarps * num_partitions * 4, st>>>(
          s, k, num_keys, tile_offsets, static_cast<K *>(send_keys), send_positions);
      launched("k_route_scatter");
    });
  });
}
