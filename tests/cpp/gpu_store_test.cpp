// C++ test of the drop-in boundary: GpuEmbeddingStore / GpuPartitioner
// (include/se_gpu_store.hpp) over libse_gpu.so, driven with host spans the
// way the reference's own store test drives HogwildEmbeddingStore
// (sparse_embedding/src/backend/hogwild/hogwild_storage_test.cpp:27-103).
// Plain main(); a failed check throws, main prints it and returns 1.
//
//   g++ -std=c++20 -I include tests/cpp/gpu_store_test.cpp
//       -L sparse_embedding_b200/_lib -lse_gpu -Wl,-rpath,<lib dir> -o gpu_store_test
// (tests/test_cpp_boundary.py builds and runs it).
#include "se_gpu_store.hpp"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <numeric>
#include <string>
#include <vector>

namespace {

void require(bool condition, const char *message) {
  if (!condition) throw std::runtime_error(message);
}

// The call must throw exactly E, with `needle` in its message.
template <typename E, typename F> void require_throws(F &&f, const char *needle) {
  try {
    f();
  } catch (const E &e) {
    if (std::string(e.what()).find(needle) == std::string::npos)
      throw std::runtime_error(std::string("unexpected message: ") + e.what());
    return;
  } catch (const std::exception &e) {
    throw std::runtime_error(std::string("wrong exception class: ") + e.what());
  }
  throw std::runtime_error(std::string("expected an exception containing: ") + needle);
}

using Store = se_gpu::GpuEmbeddingStore<float, float>;

se_store_config sgd_config(const std::vector<int64_t> &dims, int32_t accumulation) {
  se_store_config c = se_gpu::default_config<float>(dims, SE_KEY_UINT64);
  c.init_kind = SE_INIT_ZEROS;
  c.optimizer_kind = SE_OPT_SGD;
  c.lr = 0.01f;
  c.accumulation = accumulation;
  return c;
}

// hogwild_storage_test.cpp:42-103: normalized SGD update of 4,096 keys.
void run_normalized_sgd(int32_t accumulation) {
  const std::vector<int64_t> dims{8};
  Store store(sgd_config(dims, accumulation));
  constexpr size_t key_count = 4096, dimension = 8, normalization_steps = 2;
  std::vector<uint64_t> keys(key_count);
  std::iota(keys.begin(), keys.end(), uint64_t{1});
  std::vector<int64_t> lengths(key_count, dimension);
  std::vector<float> values(key_count * dimension, 1.0f);
  require(!store.lookup_or_insert<uint64_t>(keys, values, lengths), "lookup_or_insert failed");
  require(std::all_of(values.begin(), values.end(), [](float v) { return v == 0.0f; }), "zeros init");
  require(store.size() == key_count, "size after insert");
  store.optimizer_step(1);  // empty window: no change
  const std::vector<float> gradients(values.size(), 1.0f);
  require(!store.accumulate_gradients<uint64_t, float>(keys, gradients, lengths), "accumulate failed");
  require(!store.optimizer_step(normalization_steps), "optimizer_step failed");
  require(!store.lookup<uint64_t>(keys, values, lengths), "lookup failed");
  const float expected = -0.01f * 1.0f / float(normalization_steps);
  require(std::all_of(values.begin(), values.end(), [&](float v) { return std::abs(v - expected) < 1e-6f; }),
          "normalized SGD update");
}

// Uniform init is a function of the key: two stores agree bit for bit,
// values lie in [-0.05, 0.05), absent keys read as zero rows.
void run_lookup_semantics() {
  const std::vector<int64_t> dims{32};
  const se_store_config c = se_gpu::default_config<float>(dims, SE_KEY_INT64);
  Store a(c), b(c);
  std::vector<int64_t> keys{-5, -1, 0, 1, 5, int64_t(1) << 40, -5};
  std::vector<int64_t> lengths(keys.size(), 32);
  std::vector<float> va(keys.size() * 32), vb(keys.size() * 32);
  a.lookup_or_insert<int64_t>(keys, va, lengths);
  b.lookup_or_insert<int64_t>(std::span<const int64_t>(keys).subspan(3), std::span<float>(vb).subspan(3 * 32),
                              std::span<const int64_t>(lengths).subspan(3));
  b.lookup_or_insert<int64_t>(std::span<const int64_t>(keys).first(3), std::span<float>(vb).first(3 * 32),
                              std::span<const int64_t>(lengths).first(3));
  require(std::memcmp(va.data(), vb.data(), va.size() * 4) == 0, "init is a function of the key");
  require(std::memcmp(va.data(), va.data() + 6 * 32, 32 * 4) == 0, "duplicate keys share one row");
  require(std::all_of(va.begin(), va.end(), [](float v) { return v >= -0.05f && v < 0.05f; }), "init range");
  require(a.size() == 6, "duplicates insert once");
  std::vector<int64_t> absent{7, 8};
  std::vector<float> out(2 * 32, 1.0f);
  std::vector<int64_t> l2(2, 32);
  a.lookup<int64_t>(absent, out, l2);
  require(std::all_of(out.begin(), out.end(), [](float v) { return v == 0.0f; }), "absent keys zero-filled");
  std::vector<uint8_t> exists(keys.size());
  a.contains<int64_t>(keys, exists);
  require(std::all_of(exists.begin(), exists.end(), [](uint8_t e) { return e == 1; }), "contains");
  a.erase<int64_t>(std::span<const int64_t>(keys).first(2));
  require(a.size() == 4, "erase");
  std::vector<float> assigned(32, 0.25f);
  std::vector<int64_t> one{-5};
  std::vector<int64_t> l1{32};
  a.assign<int64_t>(one, assigned, l1);
  std::vector<float> back(32);
  a.lookup<int64_t>(one, back, l1);
  require(std::all_of(back.begin(), back.end(), [](float v) { return v == 0.25f; }), "assign");
  require(a.dim() == 32 && a.internal_shard_count() >= 1 && a.entries_per_page() > 0, "metadata");
}

// The reference's exception classes and messages.
void run_error_mapping() {
  const std::vector<int64_t> dims{4};
  se_store_config c = se_gpu::default_config<float>(dims, SE_KEY_UINT64);
  c.value_dtype = SE_FLOAT16;
  c.gradient_dtype = SE_FLOAT32;
  c.optimizer_dtype = SE_FLOAT32;
  c.optimizer_kind = SE_OPT_SGD;
  c.lr = 1.0f;
  se_store *raw = nullptr;
  require(se_store_create(&c, &raw) == SE_OK, "create fp16 store");
  std::vector<uint64_t> key{1};
  std::vector<uint16_t> row(4);
  const int64_t len = 4;
  se_gpu::check(se_lookup_or_insert(raw, key.data(), 1, row.data(), 4, &len, 1, nullptr));
  std::vector<float> huge(4, 1e6f);  // above the float16 parameter range
  require_throws<std::overflow_error>(
      [&] { se_gpu::check(se_accumulate_gradients(raw, key.data(), 1, huge.data(), 4, &len, 1, nullptr)); },
      "gradient");
  require_throws<std::invalid_argument>([&] { se_gpu::check(se_optimizer_step(raw, 0, nullptr)); },
                                        "normalization_steps must be positive");
  const int64_t bad_len = 5;
  std::vector<float> g5(5, 0.0f);
  require_throws<std::runtime_error>(
      [&] { se_gpu::check(se_accumulate_gradients(raw, key.data(), 1, g5.data(), 5, &bad_len, 1, nullptr)); },
      "invalid dim access");
  se_store_destroy(raw);
  Store s(se_gpu::default_config<float>(dims, SE_KEY_UINT64));
  std::vector<int32_t> wrong_keys{1};
  std::vector<float> out(4);
  std::vector<int64_t> l{4};
  require_throws<std::invalid_argument>([&] { s.lookup<int32_t>(wrong_keys, out, l); }, "key dtype");
}

// Partition ids of the reference's compiled partitioners for these keys
// (modulo / hash / fast_range, ops/partitioner.hpp:72-406).
void run_partitioner() {
  const std::vector<int64_t> keys{-5, -1, 0, 1, 5, int64_t(1) << 30};
  std::vector<uint32_t> out(keys.size());
  se_gpu::GpuPartitioner{SE_PART_MODULO, 3}.partition_span<int64_t>(keys, out);
  require(out == std::vector<uint32_t>({1, 2, 0, 1, 2, 1}), "modulo/3");
  se_gpu::GpuPartitioner{SE_PART_HASH, 8}.partition_span<int64_t>(keys, out);
  require(out == std::vector<uint32_t>({6, 3, 0, 5, 4, 7}), "hash/8");
  se_gpu::GpuPartitioner{SE_PART_FAST_RANGE, 7}.partition_span<int64_t>(keys, out);
  require(out == std::vector<uint32_t>({6, 6, 0, 0, 0, 0}), "fast_range/7");
  bool mask[6];
  se_gpu::GpuPartitioner{SE_PART_HASH, 8}.filter_span<int64_t>(keys, 0, std::span<bool>(mask, 6));
  require(!mask[0] && !mask[1] && mask[2] && !mask[3], "filter");
}

}  // namespace

int main() {
  try {
    run_normalized_sgd(SE_ACCUM_ORDERED);
    run_normalized_sgd(SE_ACCUM_ATOMIC);
    run_lookup_semantics();
    run_error_mapping();
    run_partitioner();
  } catch (const std::exception &e) {
    std::fprintf(stderr, "FAILED: %s\n", e.what());
    return 1;
  }
  std::printf("gpu_store_test ok\n");
  return 0;
}
