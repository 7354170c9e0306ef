// Shared device definitions of the B200 store: scalar types, hashes,
// conversions and small helpers.
//
// Build with --fmad=false: products and sums are rounded separately unless a
// kernel asks for a fused multiply-add with __fmaf_rn, so each formula's fused
// steps are exactly the ones the reference's compiled CPU code performs.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace se_gpu {

// ---------------------------------------------------------------------------
// Value types. Each wraps a 16- or 32-bit storage type with float conversions
// (round to nearest even on the way down, like the reference's
// _mm512_cvtneps_pbh / _mm512_cvtps_ph stores, simd/intrinsics.hpp:37-60).
// ---------------------------------------------------------------------------

struct F32 {
  using T = float;
  static __device__ __forceinline__ float load(T x) { return x; }
  static __device__ __forceinline__ T store(float f) { return f; }
  static constexpr float kMax = 3.40282347e38f;
};
struct F16 {
  using T = __half;
  static __device__ __forceinline__ float load(T x) { return __half2float(x); }
  static __device__ __forceinline__ T store(float f) { return __float2half_rn(f); }
  static constexpr float kMax = 65504.0f;
};
struct BF16 {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float load(T x) { return __bfloat162float(x); }
  static __device__ __forceinline__ T store(float f) { return __float2bfloat16_rn(f); }
  static constexpr float kMax = 3.38953139e38f;
};

// ---------------------------------------------------------------------------
// Hashes
// ---------------------------------------------------------------------------

// SplitMix64 finalizer (hogwild_embedding_store.hpp:1272-1281; partitioner.hpp:226-234).
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z ^= z >> 30;
  z *= 0xbf58476d1ce4e5b9ull;
  z ^= z >> 27;
  z *= 0x94d049bb133111ebull;
  z ^= z >> 31;
  return z;
}

// Murmur3 fmix32 (partitioner.hpp:250-258; uniform_init_ops.hpp:119-124).
__host__ __device__ __forceinline__ uint32_t fmix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x85ebca6bu;
  x ^= x >> 13;
  x *= 0xc2b2ae35u;
  x ^= x >> 16;
  return x;
}

// Keys enter the store as uint64 with sign extension (hogwild_embedding_store.hpp:4449).
__device__ __forceinline__ uint64_t key_u64(int32_t k) { return uint64_t(int64_t(k)); }
__device__ __forceinline__ uint64_t key_u64(uint32_t k) { return uint64_t(k); }
__device__ __forceinline__ uint64_t key_u64(int64_t k) { return uint64_t(k); }
__device__ __forceinline__ uint64_t key_u64(uint64_t k) { return k; }

// ---------------------------------------------------------------------------
// Error reporting from kernels: bits OR-ed into a device status word that the
// host reads after the launch. No kernel traps or asserts.
// ---------------------------------------------------------------------------

enum StatusBits : uint32_t {
  kStatusTableFull = 1u,       // probe sequence or row arena exhausted
  kStatusBadGradient = 2u,     // gradient fails validate_input
  kStatusBadRow = 4u,          // row index outside the arena
  kStatusPendingOverflow = 8u, // device pending count beyond the host-sized buffers
  kStatusCopyTimeout = 16u,    // a bulk copy into shared memory did not complete in time
};

// Programmatic dependent launch: wait for the previous kernel on the stream
// (its completion and memory); a no-op when launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel's blocks be scheduled as soon as this grid's blocks
// have all started (they still wait in pdl_wait for this grid's results).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Bulk copies global -> shared memory through the tensor memory accelerator
// (cp.async.bulk, 1-D; source and destination 16-byte aligned, size a
// multiple of 16), completed on a shared-memory mbarrier. Local to the
// calling CTA: no cluster multicast.
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t arrivals) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(arrivals) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// One arrival that also announces `bytes` of bulk copies to come.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
               " selp.u32 %0, 1, 0, p;\n}"
               : "=r"(done)
               : "r"(smem_u32(bar)), "r"(parity)
               : "memory");
  return done != 0u;
}
// Bulk store of `bytes` from shared to global memory (TMA, bulk-group
// completion): both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_store_s2g(void *dst, const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)),
               "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until the committed bulk stores of this thread have read their
// shared-memory source (the buffer may be written again).
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Waits until the committed bulk stores of this thread are complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Orders this thread's shared-memory writes before later async-proxy (TMA)
// reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_inval(uint64_t *bar) {
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void raise_status(uint32_t *status, uint32_t bits) {
  atomicOr(status, bits);
}

// Loads that bypass L1 (directory words other blocks may be writing).
__device__ __forceinline__ uint64_t ld_cg(const uint64_t *p) { return __ldcg(p); }
__device__ __forceinline__ uint32_t ld_cg(const uint32_t *p) { return __ldcg(p); }

template <int G>
__device__ __forceinline__ unsigned group_mask() {
  if constexpr (G == 32) {
    return 0xffffffffu;
  } else {
    const unsigned lane = threadIdx.x & 31u;
    return ((1u << G) - 1u) << (lane & ~unsigned(G - 1));
  }
}

}  // namespace se_gpu
