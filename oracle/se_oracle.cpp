// CPU oracle for the sparse_embedding hot path.
//
// TEST INFRASTRUCTURE ONLY. This file restates, in plain scalar C++, the
// arithmetic and the store flow of the reference's CPU hot path so that the
// CUDA implementation can be checked against it. Only the tests, the smoke
// check and the bench's CPU-baseline leg load it; the product never does.
//
// Every function names the reference file:line it follows (paths are relative
// to the sparse_embedding project root). Compile with -ffp-contract=off: the
// only fused multiply-adds are the explicit fmaf() calls below. In the SIMD
// bodies they stand for _mm512_fmadd_ps / _mm512_fnmadd_ps. In the scalar
// tails they stand for the contractions GCC 13 makes when it compiles the
// reference with its release flags (-std=c++23 -O3 -march=native; for C++ GCC
// contracts a*b+c by default). Which product each tail fuses was read off the
// reference compiled in place (oracle/_ref) and is pinned by the tests.
//
// "simd_width" is the vector width of the reference build being mirrored (16
// for its AVX-512 build, 8 for AVX2): element j of a row goes through the
// vector formula when j < (dim / simd_width) * simd_width, else through the
// scalar-tail formula (sparse_embedding/src/simd/*_ops.hpp loop structure).

#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace {

thread_local std::string g_last_error;

// ---------------------------------------------------------------------------
// Scalar types and conversions
// ---------------------------------------------------------------------------

enum KeyDType { kInt32 = 0, kUInt32 = 1, kInt64 = 2, kUInt64 = 3 };
enum ValDType { kF32 = 0, kF16 = 1, kBF16 = 2 };
enum OptKind { kOptNone = 0, kOptSgd = 1, kOptAdam = 2, kOptAdagrad = 3 };
enum InitKind { kInitZeros = 0, kInitUniform = 1 };
enum PartKind { kModulo = 0, kHash = 1, kFastRange = 2 };

struct bf16 { uint16_t bits; };
struct f16 { _Float16 v; };

inline float to_f32(float x) { return x; }
inline float to_f32(bf16 x) {
  uint32_t u = uint32_t(x.bits) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
inline float to_f32(f16 x) { return float(x.v); }

template <class T> T from_f32(float f);
template <> inline float from_f32<float>(float f) { return f; }
// Round-to-nearest-even float -> bfloat16 (sparse_embedding/src/simd/intrinsics.hpp:42-45,
// _mm512_cvtneps_pbh; scalar tails use the compiler's RNE __bf16 conversion).
template <> inline bf16 from_f32<bf16>(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  bf16 r;
  if ((u & 0x7fffffffu) > 0x7f800000u) {  // NaN: keep sign, force quiet
    r.bits = uint16_t((u >> 16) | 0x0040u);
    return r;
  }
  u += 0x7fffu + ((u >> 16) & 1u);
  r.bits = uint16_t(u >> 16);
  return r;
}
// Round-to-nearest-even float -> binary16 (intrinsics.hpp:55-58, _mm512_cvtps_ph
// with _MM_FROUND_TO_NEAREST_INT).
template <> inline f16 from_f32<f16>(float f) {
  f16 r;
  r.v = static_cast<_Float16>(f);
  return r;
}

template <class T> constexpr float dtype_max();
template <> constexpr float dtype_max<float>() { return std::numeric_limits<float>::max(); }
template <> constexpr float dtype_max<f16>() { return 65504.0f; }
template <> constexpr float dtype_max<bf16>() { return 3.38953139e38f; }

// ---------------------------------------------------------------------------
// Hashes and partitioners
// ---------------------------------------------------------------------------

// SplitMix64 finalizer: sparse_embedding/src/backend/hogwild/hogwild_embedding_store.hpp:1272-1281
// and HashPartitioner::SplitMix64Hash, sparse_embedding/src/ops/partitioner.hpp:226-234.
inline uint64_t splitmix64(uint64_t z) {
  z ^= z >> 30;
  z *= 0xbf58476d1ce4e5b9ull;
  z ^= z >> 27;
  z *= 0x94d049bb133111ebull;
  z ^= z >> 31;
  return z;
}

// Murmur3 fmix32: partitioner.hpp:250-258 and uniform_init_ops.hpp:119-124.
inline uint32_t fmix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x85ebca6bu;
  x ^= x >> 13;
  x *= 0xc2b2ae35u;
  x ^= x >> 16;
  return x;
}

// partitioner.hpp:36-43
inline uint32_t fast_range_64(uint64_t word, uint32_t p) {
  return uint32_t((static_cast<unsigned __int128>(word) * p) >> 64);
}
inline uint32_t fast_range_32(uint32_t word, uint32_t p) {
  return uint32_t((uint64_t(word) * p) >> 32);
}

// Signed floor modulo: sparse_embedding/src/common/dtypes.hpp:97-111.
template <class K> uint32_t modulo_partition(K key, uint32_t count) {
  if constexpr (std::is_signed_v<K>) {
    __int128 r = static_cast<__int128>(key) % static_cast<__int128>(count);
    if (r < 0) r += count;
    return uint32_t(r);
  } else {
    return uint32_t(uint64_t(key) % count);
  }
}

// One key -> partition id, for the three registered algorithms
// (ModuloPartitioner 72-179, FastRangePartitioner 181-220, HashPartitioner 222-406).
template <class K> uint32_t partition_one(int kind, uint32_t n, K key) {
  const bool pow2 = (n & (n - 1)) == 0;
  switch (kind) {
  case kModulo:
    if (pow2) return uint32_t(uint64_t(key) & uint64_t(n - 1));
    return modulo_partition<K>(key, n);
  case kFastRange:
    if constexpr (sizeof(K) == 8) return fast_range_64(uint64_t(key), n);
    else return fast_range_32(uint32_t(key), n);
  case kHash:
    if constexpr (sizeof(K) == 8) {
      uint64_t h = splitmix64(uint64_t(key));
      return pow2 ? uint32_t(h & uint64_t(n - 1)) : fast_range_64(h, n);
    } else {
      uint32_t h = fmix32(uint32_t(key));
      return pow2 ? (h & (n - 1)) : fast_range_32(h, n);
    }
  }
  return 0;
}

template <class K>
void partition_keys(int kind, uint32_t n, const K *keys, size_t count, uint32_t *out) {
  for (size_t i = 0; i < count; ++i) out[i] = partition_one<K>(kind, n, keys[i]);
}

inline uint64_t key_at(int key_dtype, const void *keys, size_t i) {
  switch (key_dtype) {
  case kInt32: return uint64_t(int64_t(static_cast<const int32_t *>(keys)[i]));
  case kUInt32: return uint64_t(static_cast<const uint32_t *>(keys)[i]);
  case kInt64: return uint64_t(static_cast<const int64_t *>(keys)[i]);
  default: return static_cast<const uint64_t *>(keys)[i];
  }
}

// ---------------------------------------------------------------------------
// Row arithmetic
// ---------------------------------------------------------------------------

// simd_uniform_init: sparse_embedding/src/simd/uniform_init_ops.hpp:32-134.
// Vector body (47-80): fmadd(f - 1, max - min, min); the scalar tail (117-134)
// is contracted to the same fused form by the reference's compiler.
template <class P>
void uniform_init(P *row, size_t dim, float mn, float mx, uint64_t key, size_t) {
  const uint32_t seed = uint32_t(key ^ (key >> 32));
  const float diff = mx - mn;
  for (size_t i = 0; i < dim; ++i) {
    uint32_t h = fmix32(seed + uint32_t(i));
    uint32_t bits = (h >> 9) | 0x3f800000u;
    float f;
    std::memcpy(&f, &bits, 4);
    f = f - 1.0f;
    row[i] = from_f32<P>(std::fmaf(f, diff, mn));
  }
}

// simd_sgd_update: sparse_embedding/src/simd/sgd_ops.hpp:30-78. The vector
// body fuses both steps (fmadd, fnmadd); the scalar tail (73-77) is contracted
// to the same two fused operations.
template <class P>
void sgd_row(P *param, const P *grad, float lr, float wd, size_t dim, size_t) {
  for (size_t i = 0; i < dim; ++i) {
    float p = to_f32(param[i]);
    float g = to_f32(grad[i]);
    g = std::fmaf(wd, p, g);   // g + wd * p
    p = std::fmaf(-lr, g, p);  // p - lr * g
    param[i] = from_f32<P>(p);
  }
}

// simd_adam_update: sparse_embedding/src/simd/adam_ops.hpp:30-232.
template <class P, class O>
void adam_row(P *param, const P *grad, O *m, O *v, float lr, float b1, float b2, float eps,
              float bc1, float bc2, float wd, size_t dim, size_t simd_cut) {
  const float omb1 = 1.0f - b1;
  const float omb2 = 1.0f - b2;
  for (size_t i = 0; i < dim; ++i) {
    float g = to_f32(grad[i]);
    float p = to_f32(param[i]);
    float mi = to_f32(m[i]);
    float vi = to_f32(v[i]);
    if (i < simd_cut) {
      if (wd > 0.0f) g = std::fmaf(wd, p, g);
      mi = std::fmaf(b1, mi, omb1 * g);
      float gg = g * g;
      vi = std::fmaf(b2, vi, omb2 * gg);
      m[i] = from_f32<O>(mi);
      v[i] = from_f32<O>(vi);
      float m_hat = mi * bc1;
      float v_hat = vi * bc2;
      float denom = std::sqrt(v_hat) + eps;
      p = std::fmaf(-lr, m_hat / denom, p);
    } else {
      // Scalar tail (adam_ops.hpp:199-229) as contracted by the reference's
      // compiler: g += wd*p and m fuse like the vector body; v fuses b2*v with
      // the addend ((1-b2)*g)*g (left-to-right product, unlike the vector
      // body's (1-b2)*(g*g)); the parameter step is not fused.
      if (wd > 0.0f) g = std::fmaf(wd, p, g);
      mi = std::fmaf(b1, mi, omb1 * g);
      { float t2 = omb2 * g; t2 = t2 * g; vi = std::fmaf(b2, vi, t2); }
      m[i] = from_f32<O>(mi);
      v[i] = from_f32<O>(vi);
      float m_hat = mi * bc1;
      float v_hat = vi * bc2;
      float num = lr * m_hat;
      float denom = std::sqrt(v_hat) + eps;
      float q = num / denom;
      p = p - q;
    }
    param[i] = from_f32<P>(p);
  }
}

// Adagrad has no counterpart in the reference. Its contract, shared with the
// CUDA kernel: acc starts at initial_accumulator when the row is created; per
// update g = fma(wd, p, g) when wd > 0, acc = fma(g, g, acc),
// p = fma(-lr, g / (sqrt(acc) + eps), p).
template <class P, class O>
void adagrad_row(P *param, const P *grad, O *acc, float lr, float eps, float wd, size_t dim) {
  for (size_t i = 0; i < dim; ++i) {
    float g = to_f32(grad[i]);
    float p = to_f32(param[i]);
    float a = to_f32(acc[i]);
    if (wd > 0.0f) g = std::fmaf(wd, p, g);
    a = std::fmaf(g, g, a);
    float denom = std::sqrt(a) + eps;
    p = std::fmaf(-lr, g / denom, p);
    acc[i] = from_f32<O>(a);
    param[i] = from_f32<P>(p);
  }
}

// ---------------------------------------------------------------------------
// Key -> slot map (sentinel-free linear probing, erase by tombstone). Stands
// in for the FlatKeyDirectory + SegmentedLocatorTable pair; only its
// find/insert/erase semantics matter to the results.
// ---------------------------------------------------------------------------

struct KeyMap {
  std::vector<uint64_t> keys;
  std::vector<uint32_t> vals;
  std::vector<uint8_t> used;  // 0 empty, 1 live, 2 erased
  size_t count = 0;           // occupied slots (live + erased)
  size_t live = 0;
  size_t mask = 0;

  KeyMap() { rehash(64); }

  void rehash(size_t cap) {
    std::vector<uint64_t> ok;
    std::vector<uint32_t> ov;
    std::vector<uint8_t> ou;
    ok.swap(keys);
    ov.swap(vals);
    ou.swap(used);
    keys.assign(cap, 0);
    vals.assign(cap, 0);
    used.assign(cap, 0);
    mask = cap - 1;
    count = 0;
    live = 0;
    for (size_t i = 0; i < ou.size(); ++i)
      if (ou[i] == 1) insert_new(ok[i], ov[i]);
  }
  void insert_new(uint64_t k, uint32_t v) {
    size_t pos = splitmix64(k) & mask;
    while (used[pos]) pos = (pos + 1) & mask;
    used[pos] = 1;
    keys[pos] = k;
    vals[pos] = v;
    ++count;
    ++live;
  }
  bool find(uint64_t k, uint32_t *v) const {
    size_t pos = splitmix64(k) & mask;
    while (used[pos]) {
      if (used[pos] == 1 && keys[pos] == k) { *v = vals[pos]; return true; }
      pos = (pos + 1) & mask;
    }
    return false;
  }
  bool erase(uint64_t k) {
    size_t pos = splitmix64(k) & mask;
    while (used[pos]) {
      if (used[pos] == 1 && keys[pos] == k) {
        used[pos] = 2;
        --live;
        return true;
      }
      pos = (pos + 1) & mask;
    }
    return false;
  }
  void reserve(size_t n) {
    size_t cap = keys.size();
    while (cap < 2 * n) cap *= 2;
    if (cap != keys.size()) rehash(cap);
  }
  void insert(uint64_t k, uint32_t v) {
    if (2 * (count + 1) > keys.size()) rehash(4 * (live + 1) > keys.size() ? keys.size() * 2 : keys.size());
    insert_new(k, v);
  }
  void clear() {
    std::fill(used.begin(), used.end(), 0);
    count = 0;
    live = 0;
  }
};

// ---------------------------------------------------------------------------
// Store
// ---------------------------------------------------------------------------

struct Config {
  int key_dtype, value_dtype, optimizer_dtype, gradient_dtype;
  float gradient_scale;
  int enable_optimizer;
  int init_kind;
  float init_min, init_max;
  int optimizer_kind;
  float lr, beta1, beta2, eps, weight_decay, initial_accumulator;
  int simd_width;
  int threads;
  // scores and dynamic learning rates (score_policy.hpp:37; dynamic_lr_policy.hpp:32-124)
  int score_policy;          // 0 none, 1 lfu, 2 lru, 3 manual
  int lr_policy;             // 0 constant, 1 sqrt, 2 log, 3 inverse, 4 cosine, 5 custom LUT
  float lr_min_ratio;
  uint64_t lr_max_score;
  std::vector<float> lut;    // cosine table or custom LUT
};

// compute_lr of the reference's policies (dynamic_lr_policy.hpp:32-110). The
// reference's compiled cosine step fuses (base - min) * lut + min.
inline float policy_lr(const Config &c, uint64_t score) {
  const float base = c.lr;
  switch (c.lr_policy) {
  case 1: return score == 0 ? base : base / std::sqrt(static_cast<float>(score));
  case 2: return base / std::log2(2.0f + static_cast<float>(score));
  case 3: return score == 0 ? base : base / static_cast<float>(score);
  case 4: {
    const float min_lr = base * c.lr_min_ratio;
    if (score >= c.lr_max_score) return min_lr;
    return std::fma(base - min_lr, c.lut[size_t(score)], min_lr);
  }
  case 5: return base * c.lut[size_t(score >= c.lr_max_score ? c.lr_max_score : score)];
  default: return base;
  }
}

struct TableBase {
  virtual ~TableBase() = default;
  virtual int64_t dim() const = 0;
  virtual size_t size() const = 0;
  virtual void reserve(size_t n) = 0;
  virtual void lookup(const void *keys, size_t n, void *out, int threads) = 0;
  virtual void lookup_or_insert(const void *keys, size_t n, void *out) = 0;
  virtual int accumulate(const void *keys, size_t n, const void *grads) = 0;
  virtual void optimizer_step(size_t normalization_steps, uint64_t *dropped, int threads) = 0;
  virtual int read_row(uint64_t key, void *param, void *state, uint32_t *step) const = 0;
  virtual void contains(const void *keys, size_t n, uint8_t *out) const = 0;
  virtual void assign(const void *keys, size_t n, const void *values) = 0;
  virtual void erase(const void *keys, size_t n) = 0;
  virtual void touch(const void *keys, size_t n, uint64_t *clock) = 0;
  virtual bool set_score(uint64_t key, uint64_t score) = 0;
  virtual bool get_score(uint64_t key, uint64_t *score) const = 0;
};

template <class F> void parallel_for(size_t n, int threads, F &&f) {
  if (threads <= 1 || n < 4096) { f(size_t(0), n, 0); return; }
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) {
    size_t b = n * t / threads, e = n * (t + 1) / threads;
    pool.emplace_back([&, b, e, t] { f(b, e, t); });
  }
  for (auto &th : pool) th.join();
}

template <class P, class O, class G> struct Table final : TableBase {
  Config cfg;
  int64_t dim_;
  size_t simd_cut;
  KeyMap map;
  uint32_t nrows = 0;  // rows ever created (an erased key's row is not reused)
  std::vector<P> params;
  std::vector<O> s0, s1;    // Adam m, v  |  Adagrad acc (s0)
  std::vector<uint32_t> steps;
  std::vector<uint64_t> scores;  // per row, 0 at creation
  std::vector<float> bc1, bc2;
  // Transient accumulation (TransientArena), one shard per worker thread,
  // a key's shard = splitmix64(key) % shards: key -> slot, sums kept in G.
  struct Shard {
    KeyMap tmap;
    std::vector<uint64_t> tkeys;
    std::vector<uint64_t> trows;  // gradient rows accumulated into each slot
    std::vector<G> tgrads;
  };
  std::vector<Shard> shards;

  Table(const Config &c, int64_t d) : cfg(c), dim_(d), shards(size_t(c.threads > 1 ? c.threads : 1)) {
    const size_t w = size_t(c.simd_width > 0 ? c.simd_width : 1);
    simd_cut = (size_t(d) / w) * w;
  }
  int64_t dim() const override { return dim_; }
  size_t size() const override { return map.live; }
  void reserve(size_t n) override { map.reserve(n); }

  size_t nstate() const {
    if (!cfg.enable_optimizer) return 0;
    if (cfg.optimizer_kind == kOptAdam) return 2;
    if (cfg.optimizer_kind == kOptAdagrad) return 1;
    return 0;
  }

  uint32_t insert_row(uint64_t key) {
    const uint32_t row = nrows++;
    map.insert(key, row);
    const size_t d = size_t(dim_);
    params.resize(params.size() + d);
    P *p = params.data() + size_t(row) * d;
    // Initializer: Uniform (uniform_initializer.hpp:36-53) or Zeros.
    if (cfg.init_kind == kInitUniform) uniform_init<P>(p, d, cfg.init_min, cfg.init_max, key, simd_cut);
    else for (size_t i = 0; i < d; ++i) p[i] = from_f32<P>(0.0f);
    const size_t ns = nstate();
    if (ns >= 1) {
      const float init = cfg.optimizer_kind == kOptAdagrad ? cfg.initial_accumulator : 0.0f;
      s0.resize(s0.size() + d, from_f32<O>(init));
    }
    if (ns >= 2) s1.resize(s1.size() + d, from_f32<O>(0.0f));
    if (cfg.enable_optimizer && cfg.optimizer_kind == kOptAdam) steps.push_back(0);
    scores.push_back(0);
    return row;
  }

  // forward_lookup: hogwild_embedding_store.hpp:4358-4594 (copy row, zero on miss 4501-4503).
  void lookup(const void *keys, size_t n, void *out, int threads) override {
    P *o = static_cast<P *>(out);
    const size_t d = size_t(dim_);
    parallel_for(n, threads, [&](size_t b, size_t e, int) {
      for (size_t i = b; i < e; ++i) {
        uint32_t row;
        if (map.find(key_at(cfg.key_dtype, keys, i), &row))
          std::memcpy(o + i * d, params.data() + size_t(row) * d, d * sizeof(P));
        else
          for (size_t j = 0; j < d; ++j) o[i * d + j] = from_f32<P>(0.0f);
      }
    });
  }

  // lookup_or_insert: hogwild_embedding_store.hpp:4925-4980 and
  // SlotStore::find_or_insert_batch 3057-3353 (duplicate misses share one row).
  void lookup_or_insert(const void *keys, size_t n, void *out) override {
    P *o = static_cast<P *>(out);
    const size_t d = size_t(dim_);
    for (size_t i = 0; i < n; ++i) {
      const uint64_t key = key_at(cfg.key_dtype, keys, i);
      uint32_t row;
      if (!map.find(key, &row)) row = insert_row(key);
      std::memcpy(o + i * d, params.data() + size_t(row) * d, d * sizeof(P));
    }
  }

  // accumulate_gradients: hogwild_embedding_store.hpp:4607-4771 with
  // GradientAccumulator::validate_input / accumulate_hashed
  // (gradient_accumulator.hpp:88-128) and TransientArena zero-then-add
  // (transient_arena.hpp:234-269, memory_ops.hpp:37-70). Per key, rows are
  // summed in batch order starting from +0.0.
  int accumulate(const void *keys, size_t n, const void *grads) override {
    const G *g = static_cast<const G *>(grads);
    const size_t d = size_t(dim_);
    const float scale = cfg.gradient_scale;
    std::atomic<bool> bad{false};
    parallel_for(n * d, cfg.threads, [&](size_t b, size_t e, int) {
      for (size_t i = b; i < e; ++i) {
        const float scaled = to_f32(g[i]) / scale;
        if (!std::isfinite(scaled) || std::fabs(scaled) > dtype_max<G>() ||
            std::fabs(scaled) > dtype_max<P>())
          bad.store(true);
      }
    });
    if (bad.load()) {
      g_last_error = "gradient scale storage exceeds configured dtype";
      return -3;
    }
    const size_t ns = shards.size();
    auto work = [&](size_t sh) {
      Shard &S = shards[sh];
      for (size_t i = 0; i < n; ++i) {
        const uint64_t key = key_at(cfg.key_dtype, keys, i);
        if (ns > 1 && splitmix64(key) % ns != sh) continue;
        uint32_t slot;
        if (!S.tmap.find(key, &slot)) {
          slot = uint32_t(S.tkeys.size());
          S.tmap.insert(key, slot);
          S.tkeys.push_back(key);
          S.trows.push_back(0);
          S.tgrads.resize(S.tgrads.size() + d, from_f32<G>(0.0f));
        }
        S.trows[slot] += 1;
        G *dst = S.tgrads.data() + size_t(slot) * d;
        for (size_t j = 0; j < d; ++j) {
          float src = scale == 1.0f ? to_f32(g[i * d + j])
                                    : to_f32(from_f32<G>(to_f32(g[i * d + j]) / scale));
          dst[j] = from_f32<G>(to_f32(dst[j]) + src);
        }
      }
    };
    if (ns == 1 || n < 4096) {
      for (size_t sh = 0; sh < ns; ++sh) work(sh);
    } else {
      std::vector<std::thread> pool;
      for (size_t sh = 0; sh < ns; ++sh) pool.emplace_back(work, sh);
      for (auto &th : pool) th.join();
    }
    return 0;
  }

  // optimizer_step: hogwild_embedding_store.hpp:4777-4824 ->
  // GradientAccumulator::with_accumulated_batch (gradient_accumulator.hpp:130-152,
  // GradientBatchView::assign 38-53) -> SlotStore::update_batch (2799-2901) ->
  // AdamOptimizer::step (adam_optimizer.hpp:138-165) / SgdOptimizer::step
  // (sgd_optimizer.hpp:72-78). Gradients of a key absent at step time are
  // dropped; the count is of dropped gradient rows.
  void optimizer_step(size_t nsteps, uint64_t *dropped, int threads) override {
    const size_t d = size_t(dim_);
    const bool raw = std::is_same_v<G, P> && nsteps == 1 && cfg.gradient_scale == 1.0f;
    const float factor = cfg.gradient_scale / float(nsteps);
    std::atomic<uint64_t> drop{0};
    if (cfg.optimizer_kind == kOptAdam) {
      // Host bias-correction table (adam_optimizer.hpp:55-61), extended on demand.
      uint32_t maxstep = 0;
      for (uint32_t s : steps) maxstep = s > maxstep ? s : maxstep;
      extend_bc(size_t(maxstep) + 2);
    }
    auto work = [&](Shard &S) {
      std::vector<P> gbuf(d);
      for (size_t s = 0; s < S.tkeys.size(); ++s) {
        uint32_t row;
        if (!map.find(S.tkeys[s], &row)) { drop.fetch_add(S.trows[s]); continue; }
        const G *src = S.tgrads.data() + s * d;
        for (size_t j = 0; j < d; ++j)
          gbuf[j] = raw ? from_f32<P>(to_f32(src[j])) : from_f32<P>(to_f32(src[j]) * factor);
        P *p = params.data() + size_t(row) * d;
        switch (cfg.optimizer_kind) {
        case kOptSgd:
          sgd_row<P>(p, gbuf.data(), policy_lr(cfg, scores[row]), cfg.weight_decay, d, simd_cut);
          break;
        case kOptAdagrad:
          adagrad_row<P, O>(p, gbuf.data(), s0.data() + size_t(row) * d, policy_lr(cfg, scores[row]), cfg.eps,
                            cfg.weight_decay, d);
          break;
        case kOptAdam: {
          uint32_t t = ++steps[row];
          adam_row<P, O>(p, gbuf.data(), s0.data() + size_t(row) * d, s1.data() + size_t(row) * d,
                         policy_lr(cfg, scores[row]), cfg.beta1, cfg.beta2, cfg.eps, bc1[t], bc2[t],
                         cfg.weight_decay, d,
                         simd_cut);
          break;
        }
        default: break;
        }
      }
    };
    if (shards.size() == 1 || threads <= 1) {
      for (auto &S : shards) work(S);
    } else {
      std::vector<std::thread> pool;
      for (auto &S : shards) pool.emplace_back([&work, &S] { work(S); });
      for (auto &th : pool) th.join();
    }
    if (dropped) *dropped += drop.load();
    for (auto &S : shards) {
      S.tmap.clear();
      S.tkeys.clear();
      S.trows.clear();
      S.tgrads.clear();
    }
  }

  void extend_bc(size_t n) {
    while (bc1.size() < n) {
      const size_t t = bc1.size();
      if (t == 0) { bc1.push_back(1.0f); bc2.push_back(1.0f); continue; }
      const float tf = float(t);
      bc1.push_back(1.0f / (1.0f - std::pow(cfg.beta1, tf)));
      bc2.push_back(1.0f / (1.0f - std::pow(cfg.beta2, tf)));
    }
  }

  // contains: hogwild_embedding_store.hpp:4983-5009 (a key is present when
  // any table holds it: the caller ORs the tables).
  void contains(const void *keys, size_t n, uint8_t *out) const override {
    for (size_t i = 0; i < n; ++i) {
      uint32_t row;
      if (map.find(key_at(cfg.key_dtype, keys, i), &row)) out[i] = 1;
    }
  }

  // assign: hogwild_embedding_store.hpp:4838-4923. A present key's
  // parameters are overwritten (optimizer state kept); an absent key is
  // inserted (fresh optimizer state) with the given parameters.
  void assign(const void *keys, size_t n, const void *values) override {
    const P *v = static_cast<const P *>(values);
    const size_t d = size_t(dim_);
    for (size_t i = 0; i < n; ++i) {
      const uint64_t key = key_at(cfg.key_dtype, keys, i);
      uint32_t row;
      if (!map.find(key, &row)) row = insert_row(key);
      std::memcpy(params.data() + size_t(row) * d, v + i * d, d * sizeof(P));
    }
  }

  // ScorePolicyRuntime::on_access (score_policy.hpp:40-100) for every key a
  // lookup finds, in batch order: LFU counts, LRU stamps with the store's clock.
  void touch(const void *keys, size_t n, uint64_t *clock) override {
    if (cfg.score_policy != 1 && cfg.score_policy != 2) return;
    for (size_t i = 0; i < n; ++i) {
      uint32_t row;
      if (!map.find(key_at(cfg.key_dtype, keys, i), &row)) continue;
      if (cfg.score_policy == 1) {
        if (scores[row] != ~0ull) ++scores[row];
      } else {
        const uint64_t ts = (*clock)++;
        if (scores[row] < ts) scores[row] = ts;
      }
    }
  }
  bool set_score(uint64_t key, uint64_t score) override {
    uint32_t row;
    if (!map.find(key, &row)) return false;
    scores[row] = score;
    return true;
  }
  bool get_score(uint64_t key, uint64_t *score) const override {
    uint32_t row;
    if (!map.find(key, &row)) return false;
    *score = scores[row];
    return true;
  }

  // erase: hogwild_embedding_store.hpp:5011-5062 (absent keys are ignored).
  // Pending gradients stay keyed; optimizer_step resolves them then.
  void erase(const void *keys, size_t n) override {
    for (size_t i = 0; i < n; ++i) map.erase(key_at(cfg.key_dtype, keys, i));
  }

  int read_row(uint64_t key, void *param, void *state, uint32_t *step) const override {
    uint32_t row;
    if (!map.find(key, &row)) return 0;
    const size_t d = size_t(dim_);
    if (param) std::memcpy(param, params.data() + size_t(row) * d, d * sizeof(P));
    const size_t ns = nstate();
    if (state && ns >= 1) std::memcpy(state, s0.data() + size_t(row) * d, d * sizeof(O));
    if (state && ns >= 2)
      std::memcpy(static_cast<char *>(state) + d * sizeof(O), s1.data() + size_t(row) * d,
                  d * sizeof(O));
    if (step) *step = steps.empty() ? 0 : steps[row];
    return 1;
  }
};

template <class P, class O>
TableBase *make_table_g(const Config &c, int64_t d) {
  switch (c.gradient_dtype) {
  case kF16: return new Table<P, O, f16>(c, d);
  case kBF16: return new Table<P, O, bf16>(c, d);
  default: return new Table<P, O, float>(c, d);
  }
}
template <class P> TableBase *make_table_o(const Config &c, int64_t d) {
  switch (c.optimizer_dtype) {
  case kF16: return make_table_g<P, f16>(c, d);
  case kBF16: return make_table_g<P, bf16>(c, d);
  default: return make_table_g<P, float>(c, d);
  }
}
TableBase *make_table(const Config &c, int64_t d) {
  switch (c.value_dtype) {
  case kF16: return make_table_o<f16>(c, d);
  case kBF16: return make_table_o<bf16>(c, d);
  default: return make_table_o<float>(c, d);
  }
}

struct Store {
  Config cfg;
  std::vector<TableBase *> tables;
  uint64_t dropped = 0;
  uint64_t lru_clock = 1;  // the reference's clock starts at 1
  ~Store() { for (auto *t : tables) delete t; }
  TableBase *table(int64_t dim) {
    for (auto *t : tables) if (t->dim() == dim) return t;
    g_last_error = "invalid dim access: no physical table for dim " + std::to_string(dim);
    return nullptr;
  }
};

}  // namespace

extern "C" {

const char *or_last_error() { return g_last_error.c_str(); }

uint64_t or_splitmix64(uint64_t x) { return splitmix64(x); }
uint32_t or_fmix32(uint32_t x) { return fmix32(x); }

int or_partition(int kind, uint32_t n, int key_dtype, const void *keys, size_t count, uint32_t *out) {
  if (n == 0) { g_last_error = "num_shards must be > 0"; return -1; }
  switch (key_dtype) {
  case kInt32: partition_keys<int32_t>(kind, n, static_cast<const int32_t *>(keys), count, out); break;
  case kUInt32: partition_keys<uint32_t>(kind, n, static_cast<const uint32_t *>(keys), count, out); break;
  case kInt64: partition_keys<int64_t>(kind, n, static_cast<const int64_t *>(keys), count, out); break;
  case kUInt64: partition_keys<uint64_t>(kind, n, static_cast<const uint64_t *>(keys), count, out); break;
  default: g_last_error = "unsupported key dtype code"; return -1;
  }
  return 0;
}

int or_filter(int kind, uint32_t n, int key_dtype, const void *keys, size_t count, uint32_t target,
              uint8_t *mask) {
  std::vector<uint32_t> ids(count);
  int rc = or_partition(kind, n, key_dtype, keys, count, ids.data());
  if (rc) return rc;
  for (size_t i = 0; i < count; ++i) mask[i] = ids[i] == target;
  return 0;
}

// Row arithmetic entry points, float32 only, for known-answer checks.
void or_uniform_init_f32(float *row, size_t dim, float mn, float mx, uint64_t key, int simd_width) {
  const size_t w = size_t(simd_width > 0 ? simd_width : 1);
  uniform_init<float>(row, dim, mn, mx, key, (dim / w) * w);
}
void or_sgd_f32(float *p, const float *g, float lr, float wd, size_t dim, int simd_width) {
  const size_t w = size_t(simd_width > 0 ? simd_width : 1);
  sgd_row<float>(p, g, lr, wd, dim, (dim / w) * w);
}
void or_adam_f32(float *p, const float *g, float *m, float *v, float lr, float b1, float b2, float eps,
                 float bc1, float bc2, float wd, size_t dim, int simd_width) {
  const size_t w = size_t(simd_width > 0 ? simd_width : 1);
  adam_row<float, float>(p, g, m, v, lr, b1, b2, eps, bc1, bc2, wd, dim, (dim / w) * w);
}
void or_adagrad_f32(float *p, const float *g, float *acc, float lr, float eps, float wd, size_t dim) {
  adagrad_row<float, float>(p, g, acc, lr, eps, wd, dim);
}
uint16_t or_f32_to_bf16(float f) { return from_f32<bf16>(f).bits; }
uint16_t or_f32_to_f16(float f) {
  f16 h = from_f32<f16>(f);
  uint16_t u;
  std::memcpy(&u, &h, 2);
  return u;
}

void *or_store_create(const int64_t *dims, size_t ndims, int key_dtype, int value_dtype,
                      int optimizer_dtype, int gradient_dtype, float gradient_scale,
                      int enable_optimizer, int init_kind, float init_min, float init_max,
                      int optimizer_kind, float lr, float beta1, float beta2, float eps,
                      float weight_decay, float initial_accumulator, int simd_width, int threads,
                      int score_policy, int lr_policy, float lr_min_ratio, uint64_t lr_max_score,
                      const float *lut, size_t lut_len) {
  Store *s = new Store();
  s->cfg = Config{key_dtype, value_dtype, optimizer_dtype, gradient_dtype, gradient_scale,
                  enable_optimizer, init_kind, init_min, init_max, optimizer_kind, lr, beta1,
                  beta2, eps, weight_decay, initial_accumulator, simd_width, threads,
                  score_policy, lr_policy, lr_min_ratio, lr_max_score, {}};
  if (lr_policy == 4) {
    // CosineFrequencyLrPolicy's table (dynamic_lr_policy.hpp:70-80)
    s->cfg.lut.resize(size_t(lr_max_score) + 1);
    const float pi = static_cast<float>(3.14159265358979323846);
    for (uint64_t i = 0; i <= lr_max_score; ++i) {
      const float ratio = static_cast<float>(i) / static_cast<float>(lr_max_score);
      s->cfg.lut[size_t(i)] = (1.0f + std::cos(pi * ratio)) / 2.0f;
    }
  } else if (lr_policy == 5) {
    s->cfg.lut.assign(lut, lut + lut_len);
    s->cfg.lr_max_score = lut_len - 1;
  }
  for (size_t i = 0; i < ndims; ++i) {
    bool dup = false;
    for (auto *t : s->tables) dup |= t->dim() == dims[i];
    if (!dup) s->tables.push_back(make_table(s->cfg, dims[i]));
  }
  return s;
}

void or_store_destroy(void *h) { delete static_cast<Store *>(h); }

int or_store_reserve(void *h, int64_t dim, size_t n) {
  auto *t = static_cast<Store *>(h)->table(dim);
  if (!t) return -2;
  t->reserve(n);
  return 0;
}

int or_lookup(void *h, const void *keys, size_t n, int64_t dim, void *out) {
  Store *s = static_cast<Store *>(h);
  auto *t = s->table(dim);
  if (!t) return -2;
  t->lookup(keys, n, out, s->cfg.threads);
  t->touch(keys, n, &s->lru_clock);
  return 0;
}

int or_lookup_or_insert(void *h, const void *keys, size_t n, int64_t dim, void *out) {
  auto *t = static_cast<Store *>(h)->table(dim);
  if (!t) return -2;
  t->lookup_or_insert(keys, n, out);
  return 0;
}

int or_accumulate_gradients(void *h, const void *keys, size_t n, int64_t dim, const void *grads) {
  Store *s = static_cast<Store *>(h);
  if (dim <= 0) { g_last_error = "gradient row length must be positive"; return -1; }
  auto *t = s->table(dim);
  if (!t) return -2;
  return t->accumulate(keys, n, grads);
}

int or_optimizer_step(void *h, size_t normalization_steps) {
  Store *s = static_cast<Store *>(h);
  if (normalization_steps == 0) { g_last_error = "normalization_steps must be positive"; return -1; }
  for (auto *t : s->tables) t->optimizer_step(normalization_steps, &s->dropped, s->cfg.threads);
  return 0;
}

uint64_t or_store_size(void *h, int64_t dim) {
  Store *s = static_cast<Store *>(h);
  uint64_t total = 0;
  for (auto *t : s->tables) if (dim <= 0 || t->dim() == dim) total += t->size();
  return total;
}

uint64_t or_store_dropped(void *h) { return static_cast<Store *>(h)->dropped; }

// assign_scores (hogwild_embedding_store.hpp:5202-5250): first table holding the key.
void or_assign_scores(void *h, const void *keys, size_t n, const uint64_t *scores) {
  Store *s = static_cast<Store *>(h);
  for (size_t i = 0; i < n; ++i) {
    const uint64_t key = key_at(s->cfg.key_dtype, keys, i);
    for (auto *t : s->tables)
      if (t->set_score(key, scores[i])) break;
  }
}

void or_read_scores(void *h, const void *keys, size_t n, uint64_t *out) {
  Store *s = static_cast<Store *>(h);
  for (size_t i = 0; i < n; ++i) {
    out[i] = 0;
    const uint64_t key = key_at(s->cfg.key_dtype, keys, i);
    for (auto *t : s->tables)
      if (t->get_score(key, &out[i])) break;
  }
}

void or_contains(void *h, const void *keys, size_t n, uint8_t *out) {
  Store *s = static_cast<Store *>(h);
  std::memset(out, 0, n);
  for (auto *t : s->tables) t->contains(keys, n, out);
}

int or_assign(void *h, const void *keys, size_t n, int64_t dim, const void *values) {
  auto *t = static_cast<Store *>(h)->table(dim);
  if (!t) return -2;
  t->assign(keys, n, values);
  return 0;
}

// dim 0: every table (erase); else the table of dim (erase_dimension).
int or_erase(void *h, const void *keys, size_t n, int64_t dim) {
  Store *s = static_cast<Store *>(h);
  if (dim != 0 && !s->table(dim)) { g_last_error = "erase dimension is not configured"; return -1; }
  for (auto *t : s->tables) if (dim == 0 || t->dim() == dim) t->erase(keys, n);
  return 0;
}

int or_read_row(void *h, int64_t dim, uint64_t key, void *param, void *state, uint32_t *step) {
  auto *t = static_cast<Store *>(h)->table(dim);
  if (!t) return -2;
  return t->read_row(key, param, state, step);
}

}  // extern "C"
