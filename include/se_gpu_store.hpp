// se_gpu_store.hpp - C++ store and partitioner types over the C ABI of
// libse_gpu.so (se_gpu.h), with the reference's facade conventions.
//
// GpuEmbeddingStore<ParamT, OptT> provides the hot-path conventions of
// EmbeddingTableFacade<ParamT, OptT>
// (sparse_embedding/src/interface/embedding_table_interface.hpp:214-248,
// 317-475): forward_lookup / lookup / lookup_or_insert / accumulate_gradients
// take std::span arguments and return std::error_code, optimizer_step takes
// the normalization step count, plus the mutation conventions (assign,
// contains, erase, erase_dimension) and the metadata queries (size, dim,
// reserve, internal_shard_count, entries_per_page). It is the second store
// type for make_store (sparse_embedding/src/backend/hogwild/store_factory_impl.inl:23-45).
//
// Errors follow the reference's exception classes: SE_ERR_INVALID_ARGUMENT
// throws std::invalid_argument, SE_ERR_OVERFLOW std::overflow_error, every
// other failure std::runtime_error, each with the library's message (the
// reference's wording where it has one). Success returns std::error_code{}.
//
// Spans may be host memory (staged to HBM inside the call, complete on
// return) or device memory on the store's device (used in place; the call is
// asynchronous on the store's stream argument, the legacy default stream
// here). Checkpoint, eviction and compaction conventions are not provided by
// the GPU store; the facade treats them as weak (embedding_table_interface.hpp:82-90).
//
// GpuPartitioner gives PartitionerFacade's partition_span / filter_span
// (sparse_embedding/src/ops/partitioner.hpp:48-70) for the registered
// algorithms, bit-identical to the CPU partitioners.
//
// Requires C++20 (std::span). Link with -lse_gpu.
#ifndef SE_GPU_STORE_HPP_
#define SE_GPU_STORE_HPP_

#include <cstddef>
#include <cstdint>
#include <span>
#include <stdexcept>
#include <string>
#include <system_error>
#include <type_traits>
#include <vector>

#include "se_gpu.h"

namespace se_gpu {

// Throws the reference's exception class for a failing status.
inline std::error_code check(int rc) {
  if (rc == SE_OK) return {};
  const std::string msg = se_last_error();
  if (rc == SE_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
  if (rc == SE_ERR_OVERFLOW) throw std::overflow_error(msg);
  throw std::runtime_error(msg);
}

template <typename K> constexpr int32_t key_code() {
  if constexpr (std::is_same_v<K, int32_t>) return SE_KEY_INT32;
  else if constexpr (std::is_same_v<K, uint32_t>) return SE_KEY_UINT32;
  else if constexpr (std::is_same_v<K, int64_t>) return SE_KEY_INT64;
  else {
    static_assert(std::is_same_v<K, uint64_t>, "keys are int32, uint32, int64 or uint64");
    return SE_KEY_UINT64;
  }
}

// Store dtype codes of a C++ value type: float, or a 16-bit storage type
// tagged by the caller (the reference's float16_t / bfloat16_t).
struct Float16 { uint16_t bits; };
struct BFloat16 { uint16_t bits; };
template <typename T> constexpr int32_t value_code() {
  if constexpr (std::is_same_v<T, float>) return SE_FLOAT32;
  else if constexpr (std::is_same_v<T, Float16>) return SE_FLOAT16;
  else {
    static_assert(std::is_same_v<T, BFloat16>, "values are float, Float16 or BFloat16");
    return SE_BFLOAT16;
  }
}

// A config with the reference's defaults (EmbeddingConfig,
// sparse_embedding/src/interface/embedding_config.hpp:31-43; Uniform(-0.05, 0.05)
// initializer and Adam when the optimizer is enabled, bindings/module.cpp:124-134).
template <typename ParamT, typename OptT = ParamT>
inline se_store_config default_config(const std::vector<int64_t> &dims, int32_t key_dtype) {
  se_store_config c{};
  c.dims = dims.data();
  c.num_dims = dims.size();
  c.key_dtype = key_dtype;
  c.value_dtype = value_code<ParamT>();
  c.optimizer_dtype = value_code<OptT>();
  c.gradient_dtype = value_code<ParamT>();
  c.gradient_scale = 1.0f;
  c.enable_optimizer = 1;
  c.init_kind = SE_INIT_UNIFORM;
  c.init_min = -0.05f;
  c.init_max = 0.05f;
  c.optimizer_kind = SE_OPT_ADAM;
  c.lr = 1e-3f;
  c.beta1 = 0.9f;
  c.beta2 = 0.999f;
  c.eps = 1e-8f;
  c.simd_width = 16;
  c.internal_shards = 1;
  c.accumulation = SE_ACCUM_ORDERED;
  return c;
}

template <typename ParamT, typename OptT = ParamT> class GpuEmbeddingStore {
 public:
  explicit GpuEmbeddingStore(const se_store_config &cfg)
      : dims_(cfg.dims, cfg.dims + cfg.num_dims), key_dtype_(cfg.key_dtype) {
    if (cfg.value_dtype != value_code<ParamT>() || cfg.optimizer_dtype != value_code<OptT>())
      throw std::invalid_argument("store config dtypes do not match the store's ParamT / OptT");
    check(se_store_create(&cfg, &h_));
  }
  ~GpuEmbeddingStore() {
    if (h_) se_store_destroy(h_);
  }
  GpuEmbeddingStore(const GpuEmbeddingStore &) = delete;
  GpuEmbeddingStore &operator=(const GpuEmbeddingStore &) = delete;

  se_store *handle() const { return h_; }

  template <typename K>
  std::error_code forward_lookup(std::span<const K> keys, std::span<ParamT> out_values,
                                 std::span<const int64_t> row_lengths) {
    check_keys<K>();
    return check(se_forward_lookup(h_, keys.data(), keys.size(), out_values.data(), out_values.size(),
                                   row_lengths.data(), row_lengths.size(), nullptr));
  }
  template <typename K>
  std::error_code lookup(std::span<const K> keys, std::span<ParamT> out_values,
                         std::span<const int64_t> row_lengths) {
    return forward_lookup<K>(keys, out_values, row_lengths);
  }
  template <typename K>
  std::error_code lookup_or_insert(std::span<const K> keys, std::span<ParamT> out_values,
                                   std::span<const int64_t> row_lengths) {
    check_keys<K>();
    return check(se_lookup_or_insert(h_, keys.data(), keys.size(), out_values.data(), out_values.size(),
                                     row_lengths.data(), row_lengths.size(), nullptr));
  }
  // GradT is the store's gradient dtype (gradient_dtype of the config).
  template <typename K, typename GradT>
  std::error_code accumulate_gradients(std::span<const K> keys, std::span<const GradT> grads,
                                       std::span<const int64_t> row_lengths) {
    check_keys<K>();
    return check(se_accumulate_gradients(h_, keys.data(), keys.size(), grads.data(), grads.size(),
                                         row_lengths.data(), row_lengths.size(), nullptr));
  }
  std::error_code optimizer_step(std::size_t normalization_steps) {
    return check(se_optimizer_step(h_, normalization_steps, nullptr));
  }

  // mutation conventions (hogwild_embedding_store.hpp:4838-5106)
  template <typename K>
  std::error_code assign(std::span<const K> keys, std::span<const ParamT> values,
                         std::span<const int64_t> row_lengths) {
    check_keys<K>();
    return check(se_assign(h_, keys.data(), keys.size(), values.data(), values.size(), row_lengths.data(),
                           row_lengths.size(), nullptr));
  }
  template <typename K> std::error_code contains(std::span<const K> keys, std::span<uint8_t> out_exists) {
    check_keys<K>();
    if (out_exists.size() < keys.size()) throw std::invalid_argument("contains output is shorter than the keys");
    return check(se_contains(h_, keys.data(), keys.size(), out_exists.data(), nullptr));
  }
  template <typename K> std::error_code erase(std::span<const K> keys) {
    check_keys<K>();
    return check(se_erase(h_, keys.data(), keys.size(), nullptr));
  }
  template <typename K> std::error_code erase_dimension(std::size_t dimension, std::span<const K> keys) {
    check_keys<K>();
    return check(se_erase_dimension(h_, static_cast<int64_t>(dimension), keys.data(), keys.size(), nullptr));
  }

  // metadata conventions
  std::size_t size() const {
    uint64_t n = 0;
    check(se_store_size(h_, &n));
    return n;
  }
  std::size_t size(std::size_t dimension) const {
    uint64_t n = 0;
    check(se_store_dim_size(h_, static_cast<int64_t>(dimension), &n));
    return n;
  }
  std::size_t dim() const {
    int64_t m = 0;
    for (int64_t d : dims_) m = d > m ? d : m;
    return static_cast<std::size_t>(m);
  }
  std::error_code reserve(std::size_t keys, std::size_t dimension) {
    return check(se_store_reserve(h_, keys, static_cast<int64_t>(dimension)));
  }
  std::size_t internal_shard_count() const {
    uint64_t n = 0;
    check(se_store_internal_shard_count(h_, &n));
    return n;
  }
  std::size_t entries_per_page() const {
    uint64_t n = 0;
    check(se_store_entries_per_page(h_, &n));
    return n;
  }
  std::size_t dropped_gradients() const {
    uint64_t n = 0;
    check(se_store_dropped_gradients(h_, &n));
    return n;
  }

 private:
  // keys must have the store's key dtype (the reference's "key dtype does
  // not match store", sparse_embedding/tests/test_embedding_table.py:147-148)
  template <typename K> void check_keys() const {
    if (key_code<K>() != key_dtype_) throw std::invalid_argument("key dtype does not match store");
  }

  se_store *h_ = nullptr;
  std::vector<int64_t> dims_;
  int32_t key_dtype_;
};

// PartitionerFacade over the GPU partition kernels (registered under
// sparse_embedding.{modulo,hash,fast_range}, partitioner_registry.cpp:24-83).
struct GpuPartitioner {
  int32_t kind;             // enum se_partitioner_kind
  uint32_t num_partitions;
  int32_t device = 0;

  template <typename K> void partition_span(std::span<const K> keys, std::span<uint32_t> out) const {
    if (out.size() < keys.size()) throw std::invalid_argument("partition output is shorter than the keys");
    check(se_partition(kind, num_partitions, key_code<K>(), keys.data(), keys.size(), out.data(), device, nullptr));
  }
  template <typename K>
  void filter_span(std::span<const K> keys, uint32_t target, std::span<bool> mask) const {
    if (mask.size() < keys.size()) throw std::invalid_argument("filter output is shorter than the keys");
    std::vector<uint8_t> m(keys.size());
    check(se_filter(kind, num_partitions, key_code<K>(), keys.data(), keys.size(), target, m.data(), device,
                    nullptr));
    for (std::size_t i = 0; i < keys.size(); ++i) mask[i] = m[i] != 0;
  }
};

}  // namespace se_gpu

#endif  // SE_GPU_STORE_HPP_
