// Reference shim: TEST INFRASTRUCTURE ONLY.
//
// Compiles the reference's own hot-path headers, unmodified and in place
// (include path -I<reference root>), into oracle/_ref/libse_ref.so, and exposes
// them through a C ABI so the tests can pin the oracle's restatement against
// the reference's real code on identical inputs:
//   - ModuloPartitioner / HashPartitioner / FastRangePartitioner
//     (sparse_embedding/src/ops/partitioner.hpp:72-406)
//   - simd_uniform_init (sparse_embedding/src/simd/uniform_init_ops.hpp:32-134)
//   - simd_sgd_update   (sparse_embedding/src/simd/sgd_ops.hpp:30-78)
//   - simd_adam_update  (sparse_embedding/src/simd/adam_ops.hpp:30-232)
//   - simd_accumulate   (sparse_embedding/src/simd/memory_ops.hpp:37-70)
// Nothing here is product code and nothing here is copied from the reference;
// the functions below only forward to it.

#include <cstdint>
#include <span>

#include "sparse_embedding/src/ops/partitioner.hpp"
#include "sparse_embedding/src/simd/adam_ops.hpp"
#include "sparse_embedding/src/simd/memory_ops.hpp"
#include "sparse_embedding/src/simd/sgd_ops.hpp"
#include "sparse_embedding/src/simd/uniform_init_ops.hpp"

namespace {

template <class Part, class K>
void run_partition(uint32_t n, const void *keys, size_t count, uint32_t *out) {
  Part p(n);
  p.template partition_span<K>(std::span<const K>(static_cast<const K *>(keys), count),
                               std::span<uint32_t>(out, count));
}

template <class Part>
int dispatch_key(uint32_t n, int key_dtype, const void *keys, size_t count, uint32_t *out) {
  switch (key_dtype) {
  case 0: run_partition<Part, int32_t>(n, keys, count, out); return 0;
  case 1: run_partition<Part, uint32_t>(n, keys, count, out); return 0;
  case 2: run_partition<Part, int64_t>(n, keys, count, out); return 0;
  case 3: run_partition<Part, uint64_t>(n, keys, count, out); return 0;
  }
  return -1;
}

template <class Part, class K>
void run_filter(uint32_t n, const void *keys, size_t count, uint32_t target, uint8_t *mask) {
  Part p(n);
  bool *tmp = new bool[count];
  p.template filter_span<K>(std::span<const K>(static_cast<const K *>(keys), count), target,
                            std::span<bool>(tmp, count));
  for (size_t i = 0; i < count; ++i) mask[i] = tmp[i] ? 1 : 0;
  delete[] tmp;
}

template <class Part>
int dispatch_filter(uint32_t n, int key_dtype, const void *keys, size_t count, uint32_t target,
                    uint8_t *mask) {
  switch (key_dtype) {
  case 0: run_filter<Part, int32_t>(n, keys, count, target, mask); return 0;
  case 1: run_filter<Part, uint32_t>(n, keys, count, target, mask); return 0;
  case 2: run_filter<Part, int64_t>(n, keys, count, target, mask); return 0;
  case 3: run_filter<Part, uint64_t>(n, keys, count, target, mask); return 0;
  }
  return -1;
}

}  // namespace

extern "C" {

int ref_simd_width() { return static_cast<int>(se::simd::kFloatSimdWidth); }

int ref_partition(int kind, uint32_t n, int key_dtype, const void *keys, size_t count,
                  uint32_t *out) {
  switch (kind) {
  case 0: return dispatch_key<se::ops::ModuloPartitioner>(n, key_dtype, keys, count, out);
  case 1: return dispatch_key<se::ops::HashPartitioner>(n, key_dtype, keys, count, out);
  case 2: return dispatch_key<se::ops::FastRangePartitioner>(n, key_dtype, keys, count, out);
  }
  return -1;
}

int ref_filter(int kind, uint32_t n, int key_dtype, const void *keys, size_t count,
               uint32_t target, uint8_t *mask) {
  switch (kind) {
  case 0: return dispatch_filter<se::ops::ModuloPartitioner>(n, key_dtype, keys, count, target, mask);
  case 1: return dispatch_filter<se::ops::HashPartitioner>(n, key_dtype, keys, count, target, mask);
  case 2: return dispatch_filter<se::ops::FastRangePartitioner>(n, key_dtype, keys, count, target, mask);
  }
  return -1;
}

void ref_uniform_init_f32(float *row, size_t dim, float mn, float mx, uint64_t key) {
  se::simd::simd_uniform_init<float>(row, dim, mn, mx, key);
}
void ref_uniform_init_bf16(void *row, size_t dim, float mn, float mx, uint64_t key) {
  se::simd::simd_uniform_init<se::bfloat16_t>(static_cast<se::bfloat16_t *>(row), dim, mn, mx, key);
}
void ref_uniform_init_f16(void *row, size_t dim, float mn, float mx, uint64_t key) {
  se::simd::simd_uniform_init<se::float16_t>(static_cast<se::float16_t *>(row), dim, mn, mx, key);
}

void ref_sgd_f32(float *p, const float *g, float lr, float wd, size_t dim) {
  se::simd::simd_sgd_update<float, float>(p, g, lr, wd, dim);
}

void ref_adam_f32(float *p, const float *g, float *m, float *v, float lr, float b1, float b2,
                  float eps, float bc1, float bc2, float wd, size_t dim) {
  se::simd::simd_adam_update<float, float, float>(p, g, m, v, lr, b1, b2, eps, bc1, bc2, wd, dim);
}

void ref_accumulate_f32(const float *src, float *dst, size_t dim) {
  se::simd::simd_accumulate<float>(src, dst, dim);
}

}  // extern "C"
