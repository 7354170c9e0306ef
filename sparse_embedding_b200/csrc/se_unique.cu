// Unique keys with inverse indices, first indices and counts: the GPU form
// of se::ops::unique_keys_inverse (sparse_embedding/src/ops/unique_ops.hpp:73-418)
// behind the Python async_unique (sparse_embedding/src/bindings/module.cpp:959-1072).
//
// The reference returns the distinct keys "unordered" (its sequential path
// in order of first appearance, its parallel path grouped by hash
// partition). This version always returns them in order of first
// appearance, so its results do not depend on sizes or threads:
//   1. every key goes into a scratch open-addressing set (2-4x the keys,
//      all-ones = empty, the all-ones key itself in a side slot); each slot
//      keeps the smallest position holding its key (atomicMin);
//   2. a position is a first appearance when its slot's minimum is itself;
//      an exclusive scan of those flags numbers the distinct keys;
//   3. each first appearance writes its key, its position and a zero count
//      under its number, and stores the number in its slot;
//   4. every position reads its slot's number (the inverse index) and adds
//      one to that key's count.

#include <cub/device/device_scan.cuh>

#include <algorithm>
#include <map>
#include <mutex>
#include <utility>

#include "se_host.hpp"
#include "se_partition.cuh"

namespace se_gpu {

namespace {

constexpr uint64_t kUniqueEmpty = ~0ull;
constexpr uint32_t kUniqueMaxKeys = 0x7fffffffu;  // validate_unique_input_size (unique_ops.hpp:42-47)

template <class K>
__global__ void __launch_bounds__(256)
k_unique_insert(const K *__restrict__ keys, uint32_t n, unsigned long long *__restrict__ set_keys,
                uint32_t *__restrict__ set_first, uint64_t nslots, uint32_t *__restrict__ slot_of) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint64_t key = key_u64(keys[i]);
  uint64_t slot = nslots;  // the side slot of the all-ones key
  if (key != kUniqueEmpty) {
    const uint64_t mask = nslots - 1;
    uint64_t pos = splitmix64(key) & mask;
    for (uint64_t probe = 0; probe < nslots; ++probe) {
      const unsigned long long old = atomicCAS(&set_keys[pos], kUniqueEmpty, key);
      if (old == kUniqueEmpty || old == key) {
        slot = pos;
        break;
      }
      pos = (pos + 1) & mask;
    }
  }
  atomicMin(&set_first[slot], i);
  slot_of[i] = uint32_t(slot);
}

__global__ void __launch_bounds__(256)
k_unique_flag(uint32_t n, const uint32_t *__restrict__ set_first, const uint32_t *__restrict__ slot_of,
              uint32_t *__restrict__ flags) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) flags[i] = __ldg(set_first + slot_of[i]) == i ? 1u : 0u;
}

template <class K>
__global__ void __launch_bounds__(256)
k_unique_emit(const K *__restrict__ keys, uint32_t n, const uint32_t *__restrict__ flags,
              const uint32_t *__restrict__ number, const uint32_t *__restrict__ slot_of,
              uint32_t *__restrict__ set_uid, K *__restrict__ unique_out, int32_t *__restrict__ first_out,
              int32_t *__restrict__ counts, uint32_t *__restrict__ num_unique) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t u = number[i];
  if (i == n - 1) *num_unique = u + flags[i];
  if (!flags[i]) return;
  set_uid[slot_of[i]] = u;
  unique_out[u] = keys[i];
  if (first_out) first_out[u] = int32_t(i);
  if (counts) counts[u] = 0;
}

__global__ void __launch_bounds__(256)
k_unique_inverse(uint32_t n, const uint32_t *__restrict__ slot_of, const uint32_t *__restrict__ set_uid,
                 int32_t *__restrict__ inverse, int32_t *__restrict__ counts) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t u = set_uid[slot_of[i]];
  if (inverse) inverse[i] = int32_t(u);
  if (counts) atomicAdd(counts + u, 1);
}

// Scratch cached per (device, stream): calls on one stream are ordered, so
// they share it; it only grows and lives until the process exits.
std::mutex g_unique_mu;
std::map<std::pair<int, cudaStream_t>, std::pair<void *, size_t>> g_unique_bufs;

uint8_t *unique_scratch(int device, cudaStream_t st, size_t bytes) {
  std::lock_guard<std::mutex> lock(g_unique_mu);
  auto &b = g_unique_bufs[{device, st}];
  if (b.second < bytes) {
    if (b.first) {
      cuda_check(cudaStreamSynchronize(st), "unique scratch sync");
      cuda_check(cudaFree(b.first), "cudaFree");
      b.first = nullptr;
    }
    const size_t cap = std::max<size_t>(bytes, std::max<size_t>(2 * b.second, 1 << 20));
    cuda_check(cudaMalloc(&b.first, cap), "cudaMalloc(unique scratch)");
    b.second = cap;
  }
  return static_cast<uint8_t *>(b.first);
}

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

}  // namespace se_gpu

using namespace se_gpu;

extern "C" int se_unique(int32_t key_dtype, const void *keys, size_t num_keys, void *unique_out,
                         int32_t *inverse_out, int32_t *first_out, int32_t *counts_out,
                         uint64_t *num_unique_out, int32_t device, void *stream_ptr) {
  return guarded([&] {
    check_key_dtype(key_dtype);
    if (num_unique_out == nullptr) throw std::invalid_argument("num_unique_out is null");
    if (num_keys > kUniqueMaxKeys)
      throw std::invalid_argument("Input size exceeds maximum supported 32-bit element count (2^31 - 1)");
    *num_unique_out = 0;
    if (num_keys == 0) return;
    if (unique_out == nullptr) throw std::invalid_argument("unique_keys_out is null");
    DeviceGuard dg(device);
    cudaStream_t st = static_cast<cudaStream_t>(stream_ptr);
    const uint32_t n = uint32_t(num_keys);
    const size_t kb = key_bytes(key_dtype);
    const uint64_t nslots = [&] {
      uint64_t p = 1;
      while (p < 2 * uint64_t(n)) p <<= 1;
      return p;
    }();
    size_t scan_bytes = 0;
    cuda_check(cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, static_cast<uint32_t *>(nullptr),
                                             static_cast<uint32_t *>(nullptr), int(n), st),
               "scan size");
    // scratch: set keys | set first | set uid | slot_of | flags | number | count | scan temp
    // | staged keys | staged outputs (host pointers only)
    const bool dk = is_device_ptr(keys);
    const bool du = is_device_ptr(unique_out);
    const bool di = inverse_out == nullptr || is_device_ptr(inverse_out);
    const bool df = first_out == nullptr || is_device_ptr(first_out);
    const bool dc = counts_out == nullptr || is_device_ptr(counts_out);
    size_t off = 0;
    auto take = [&](size_t bytes) {
      const size_t at = off;
      off += up256(bytes);
      return at;
    };
    const size_t o_sk = take(8 * (nslots + 1)), o_sf = take(4 * (nslots + 1)), o_su = take(4 * (nslots + 1));
    const size_t o_slot = take(4 * size_t(n)), o_flags = take(4 * size_t(n)), o_num = take(4 * size_t(n));
    const size_t o_cnt = take(4), o_scan = take(scan_bytes);
    const size_t o_keys = dk ? 0 : take(kb * n), o_uout = du ? 0 : take(kb * n);
    const size_t o_inv = di ? 0 : take(4 * size_t(n)), o_first = df ? 0 : take(4 * size_t(n));
    const size_t o_counts = dc ? 0 : take(4 * size_t(n));
    uint8_t *base = unique_scratch(device, st, off);
    auto *set_keys = reinterpret_cast<unsigned long long *>(base + o_sk);
    auto *set_first = reinterpret_cast<uint32_t *>(base + o_sf);
    auto *set_uid = reinterpret_cast<uint32_t *>(base + o_su);
    auto *slot_of = reinterpret_cast<uint32_t *>(base + o_slot);
    auto *flags = reinterpret_cast<uint32_t *>(base + o_flags);
    auto *number = reinterpret_cast<uint32_t *>(base + o_num);
    auto *count = reinterpret_cast<uint32_t *>(base + o_cnt);
    const void *dkeys = keys;
    if (!dk) {
      cuda_check(cudaMemcpyAsync(base + o_keys, keys, kb * n, cudaMemcpyHostToDevice, st), "copy keys");
      dkeys = base + o_keys;
    }
    void *duo = du ? unique_out : base + o_uout;
    int32_t *dinv = inverse_out == nullptr ? nullptr : di ? inverse_out : reinterpret_cast<int32_t *>(base + o_inv);
    int32_t *dfirst = first_out == nullptr ? nullptr : df ? first_out : reinterpret_cast<int32_t *>(base + o_first);
    // counts are also needed on the device when only their host copy is asked for
    int32_t *dcounts = counts_out == nullptr ? nullptr : dc ? counts_out : reinterpret_cast<int32_t *>(base + o_counts);
    cuda_check(cudaMemsetAsync(set_keys, 0xff, 8 * (nslots + 1), st), "memset");
    cuda_check(cudaMemsetAsync(set_first, 0xff, 4 * (nslots + 1), st), "memset");
    const unsigned grid = grid_for(n, 256, 0x7fffffffu);
    dispatch_key(key_dtype, [&](auto tag) {
      using K = decltype(tag);
      k_unique_insert<K><<<grid, 256, 0, st>>>(static_cast<const K *>(dkeys), n, set_keys, set_first, nslots,
                                               slot_of);
      launched("k_unique_insert");
      k_unique_flag<<<grid, 256, 0, st>>>(n, set_first, slot_of, flags);
      launched("k_unique_flag");
      cuda_check(cub::DeviceScan::ExclusiveSum(base + o_scan, scan_bytes, flags, number, int(n), st), "scan");
      k_unique_emit<K><<<grid, 256, 0, st>>>(static_cast<const K *>(dkeys), n, flags, number, slot_of, set_uid,
                                             static_cast<K *>(duo), dfirst, dcounts, count);
      launched("k_unique_emit");
      if (dinv || dcounts) {
        k_unique_inverse<<<grid, 256, 0, st>>>(n, slot_of, set_uid, dinv, dcounts);
        launched("k_unique_inverse");
      }
    });
    uint32_t u = 0;
    cuda_check(cudaMemcpyAsync(&u, count, 4, cudaMemcpyDeviceToHost, st), "read count");
    cuda_check(cudaStreamSynchronize(st), "unique sync");
    if (!du) cuda_check(cudaMemcpyAsync(unique_out, duo, kb * u, cudaMemcpyDeviceToHost, st), "copy out");
    if (!di) cuda_check(cudaMemcpyAsync(inverse_out, dinv, 4 * size_t(n), cudaMemcpyDeviceToHost, st), "copy out");
    if (!df) cuda_check(cudaMemcpyAsync(first_out, dfirst, 4 * size_t(u), cudaMemcpyDeviceToHost, st), "copy out");
    if (!dc) cuda_check(cudaMemcpyAsync(counts_out, dcounts, 4 * size_t(u), cudaMemcpyDeviceToHost, st), "copy out");
    if (!du || !di || !df || !dc) cuda_check(cudaStreamSynchronize(st), "unique sync");
    *num_unique_out = u;
  });
}
