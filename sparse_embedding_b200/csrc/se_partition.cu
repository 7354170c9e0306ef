// Partition entry points of the C ABI: partition / filter of host or device
// keys, the stable route used by the cross-GPU exchange, and row
// permutations. Device code: se_partition.cuh.

#include <algorithm>
#include <map>
#include <mutex>
#include <string>
#include <tuple>

#include "se_host.hpp"
#include "se_partition.cuh"

namespace se_gpu {

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

namespace {

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
