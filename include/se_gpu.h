/*
 * se_gpu.h — C ABI of the B200 sparse-embedding store (libse_gpu.so).
 *
 * This is the drop-in boundary for the reference's hot path. Each entry point
 * names the reference interface it replaces (paths relative to the
 * sparse_embedding project root). Signatures use plain pointers and sizes
 * only; no C++ or torch types cross the boundary.
 *
 * Memory spaces. Every data pointer (keys, values, gradients, partition ids)
 * may point to host memory (pageable or pinned) or to device memory on the
 * store's device. Host inputs are staged to the device inside the call; host
 * outputs are complete when the call returns. With device pointers the call is
 * asynchronous on `stream` (a cudaStream_t; NULL is the legacy default
 * stream) and results are ready when that stream reaches the call.
 *
 * Errors. Every function returns 0 on success or a negative SE_ERR_* code,
 * one per C++ exception class the reference throws for the same condition;
 * se_last_error() returns the message (the reference's own wording where it
 * has one) for the calling thread.
 */
#ifndef SE_GPU_H_
#define SE_GPU_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define SE_OK 0
#define SE_ERR_INVALID_ARGUMENT (-1) /* std::invalid_argument -> Python ValueError   */
#define SE_ERR_RUNTIME (-2)          /* std::runtime_error    -> Python RuntimeError */
#define SE_ERR_OVERFLOW (-3)         /* std::overflow_error   -> Python OverflowError*/
#define SE_ERR_CUDA (-4)             /* CUDA runtime failure                          */
#define SE_ERR_OUT_OF_MEMORY (-5)    /* device allocation failed                     */
#define SE_ERR_TABLE_FULL (-6)       /* bounded probe or row allocation exhausted    */
#define SE_ERR_NOT_IMPLEMENTED (-7)  /* convention not provided by the GPU store     */

/* Key dtypes, in the order of se::KeyDType (sparse_embedding/src/common/dtypes.hpp:21-26). */
enum se_key_dtype { SE_KEY_INT32 = 0, SE_KEY_UINT32 = 1, SE_KEY_INT64 = 2, SE_KEY_UINT64 = 3 };
/* Value dtypes, in the order of se::ValueDType (dtypes.hpp:117-121). */
enum se_value_dtype { SE_FLOAT32 = 0, SE_FLOAT16 = 1, SE_BFLOAT16 = 2 };
enum se_optimizer_kind { SE_OPT_NONE = 0, SE_OPT_SGD = 1, SE_OPT_ADAM = 2, SE_OPT_ADAGRAD = 3 };
enum se_init_kind { SE_INIT_ZEROS = 0, SE_INIT_UNIFORM = 1 };
/* Score policies (ScorePolicyKind, sparse_embedding/src/eviction/score_policy.hpp:37):
 * LFU counts lookups of a key, LRU stamps it with a store-wide access clock,
 * manual scores change only through se_assign_scores. */
enum se_score_policy { SE_SCORE_NONE = 0, SE_SCORE_LFU = 1, SE_SCORE_LRU = 2, SE_SCORE_MANUAL = 3 };
/* Dynamic learning-rate policies (sparse_embedding/src/optimizer/dynamic_lr_policy.hpp:32-124):
 * the row's learning rate as a function of its score. */
enum se_lr_policy {
  SE_LR_CONSTANT = 0, SE_LR_SQRT_DECAY = 1, SE_LR_LOG_DECAY = 2, SE_LR_INVERSE_DECAY = 3,
  SE_LR_COSINE_FREQUENCY = 4, SE_LR_CUSTOM_LUT = 5
};
/* How accumulate_gradients sums a key's gradient rows until optimizer_step.
 * ORDERED: rows are kept and each key's rows are summed in arrival order
 * from +0.0, rounding to the gradient dtype after each add - the reference's
 * TransientArena order (sparse_embedding/src/arena/transient_arena.hpp:234-269),
 * bit-exact for keys with at most 64 rows per window.
 * ATOMIC: rows are added on arrival into fp32 per-key sums with vector
 * reductions (a hash table keyed by key, like TransientArena::accumulate_hashed,
 * transient_arena.hpp:119-145); the order of the adds varies, so updates
 * match ORDERED within the rounding of a reassociated fp32 sum. Tables whose
 * row exceeds 8,192 values use ORDERED. */
enum se_accumulation_mode { SE_ACCUM_ORDERED = 0, SE_ACCUM_ATOMIC = 1 };
/* Registered partitioners: sparse_embedding.{modulo,hash,fast_range}. */
enum se_partitioner_kind { SE_PART_MODULO = 0, SE_PART_HASH = 1, SE_PART_FAST_RANGE = 2 };

/*
 * Store configuration: the fields of se::EmbeddingConfig
 * (sparse_embedding/src/interface/embedding_config.hpp:31-43) plus the
 * initializer and optimizer configs the Python constructor takes
 * (sparse_embedding/src/bindings/module.cpp:103-190, optimizer_config.hpp:28-44).
 */
typedef struct se_store_config {
  const int64_t *dims;       /* one table per distinct dim                         */
  size_t num_dims;
  int32_t key_dtype;         /* enum se_key_dtype                                  */
  int32_t value_dtype;       /* enum se_value_dtype (ParamT)                       */
  int32_t optimizer_dtype;   /* OptT (optimizer state)                             */
  int32_t gradient_dtype;    /* accumulated gradient storage type                  */
  float gradient_scale;      /* finite, > 0                                        */
  int32_t enable_optimizer;
  int32_t init_kind;         /* enum se_init_kind                                  */
  float init_min, init_max;  /* Uniform bounds (default -0.05, 0.05)               */
  int32_t optimizer_kind;    /* enum se_optimizer_kind                             */
  float lr, beta1, beta2, eps, weight_decay;
  float initial_accumulator; /* Adagrad accumulator value for a new row            */
  uint64_t initial_capacity; /* rows reserved per table at creation (0: default)   */
  int32_t device;            /* CUDA device ordinal                                */
  int32_t simd_width;        /* float lanes of the mirrored CPU build: 16 or 8     */
  int32_t internal_shards;   /* value reported by se_store_internal_shard_count    */
  int32_t score_policy;      /* enum se_score_policy                               */
  int32_t lr_policy;         /* enum se_lr_policy (needs a score policy unless constant) */
  float lr_min_ratio;        /* cosine: learning rate at max_score, as a ratio     */
  uint64_t lr_max_score;     /* cosine: score where the decay ends                 */
  const float *lr_lut;       /* custom LUT: multiplier per score (last one beyond) */
  size_t lr_lut_len;
  int32_t accumulation;      /* enum se_accumulation_mode                          */
} se_store_config;

typedef struct se_store se_store;

/* Message of the last failing call on this thread ("" after success). */
const char *se_last_error(void);
/* Library build identifier. */
const char *se_version(void);
/* Number of CUDA kernels this library has launched in this process. */
uint64_t se_kernel_launch_count(void);

/* Replaces make_store / create_hogwild_store
 * (sparse_embedding/src/backend/hogwild/store_factory_impl.inl:23-45,
 *  store_construction.cpp:21-67) for the GPU store. */
int se_store_create(const se_store_config *config, se_store **out_store);
int se_store_destroy(se_store *store);

/* EmbeddingTableFacade::forward_lookup / lookup
 * (sparse_embedding/src/interface/embedding_table_interface.hpp:214-216, 242-244;
 *  HogwildEmbeddingStoreCore::forward_lookup, hogwild_embedding_store.hpp:4358-4594).
 * out_values holds num_keys rows of row_lengths[i] ParamT values; rows of keys
 * that are absent are zero-filled. row_lengths is a host array. */
int se_forward_lookup(se_store *store, const void *keys, size_t num_keys, void *out_values,
                      size_t num_out_values, const int64_t *row_lengths, size_t num_row_lengths,
                      void *stream);

/* EmbeddingTableFacade::lookup_or_insert (embedding_table_interface.hpp:218-220;
 * hogwild_embedding_store.hpp:4925-4980): absent keys are inserted once each
 * (duplicates in one batch share one row), initialized from the key, and
 * every position receives its row. */
int se_lookup_or_insert(se_store *store, const void *keys, size_t num_keys, void *out_values,
                        size_t num_out_values, const int64_t *row_lengths,
                        size_t num_row_lengths, void *stream);

/* Uniform-row-length forms of the two calls above (the Python binding's path,
 * sparse_embedding/src/bindings/typed/module_typed_sync.inl:12-89). */
int se_forward_lookup_dim(se_store *store, const void *keys, size_t num_keys, int64_t dim,
                          void *out_values, void *stream);
int se_lookup_or_insert_dim(se_store *store, const void *keys, size_t num_keys, int64_t dim,
                            void *out_values, void *stream);

/* EmbeddingTableFacade::accumulate_gradients (embedding_table_interface.hpp:246-248;
 * hogwild_embedding_store.hpp:4607-4771). grads are in the store's gradient
 * dtype, num_keys rows of row_lengths[i] values. Gradients are validated
 * (GradientAccumulator::validate_input) before anything is accumulated. */
int se_accumulate_gradients(se_store *store, const void *keys, size_t num_keys, const void *grads,
                            size_t num_grad_scalars, const int64_t *row_lengths,
                            size_t num_row_lengths, void *stream);
int se_accumulate_gradients_dim(se_store *store, const void *keys, size_t num_keys, int64_t dim,
                                const void *grads, void *stream);

/* EmbeddingTableFacade::optimizer_step (hogwild_embedding_store.hpp:4777-4824):
 * sums each key's accumulated gradients in arrival order, scales them by
 * gradient_scale / normalization_steps and applies the optimizer once per
 * key present in the store. */
int se_optimizer_step(se_store *store, size_t normalization_steps, void *stream);

/* EmbeddingTableFacade::contains (hogwild_embedding_store.hpp:4983-5009):
 * out_exists[i] = 1 when any table of the store holds keys[i], else 0.
 * out_exists is host or device memory (num_keys bytes). */
int se_contains(se_store *store, const void *keys, size_t num_keys, uint8_t *out_exists, void *stream);

/* EmbeddingTableFacade::assign (hogwild_embedding_store.hpp:4838-4923): each
 * key's parameters are set to its row of values (ParamT, row_lengths[i]
 * each); a present key keeps its optimizer state, an absent key is inserted
 * with fresh optimizer state. Keys must be distinct
 * (validate_unique_mutation_batch, 5278-5305). */
int se_assign(se_store *store, const void *keys, size_t num_keys, const void *values,
              size_t num_values, const int64_t *row_lengths, size_t num_row_lengths, void *stream);
int se_assign_dim(se_store *store, const void *keys, size_t num_keys, int64_t dim, const void *values,
                  void *stream);

/* EmbeddingTableFacade::erase (hogwild_embedding_store.hpp:5011-5062): removes
 * the keys from every table; absent keys are ignored. Gradients accumulated
 * for an erased key are dropped at the next optimizer_step unless the key is
 * inserted again before it. erase_dimension (5064-5106) removes them from the
 * table of one dim only. */
int se_erase(se_store *store, const void *keys, size_t num_keys, void *stream);
int se_erase_dimension(se_store *store, int64_t dim, const void *keys, size_t num_keys, void *stream);

/* Checkpoint export (EmbeddingTableFacade::export_batch / export_opt_state_batch,
 * embedding_table_interface.hpp:259-267, 293-298; hogwild_embedding_store.hpp:6112-6300):
 * se_export_snapshot lists the present keys of the table of `dim` in
 * directory order (replacing an earlier list of that table) and returns
 * their number; se_export_read copies entries [offset, offset + count) of the
 * list: keys (key dtype), parameter rows (ParamT, dim each), optimizer state
 * rows (OptT, dim x states each: Adam m then v, Adagrad accumulator; none
 * for SGD) and Adam steps. Any output may be null; outputs are host or
 * device memory. The list reflects the table when it was taken; rows are
 * read when se_export_read runs. */
int se_export_snapshot(se_store *store, int64_t dim, uint64_t *num_keys_out, void *stream);
int se_export_read(se_store *store, int64_t dim, uint64_t offset, uint64_t count, void *keys_out,
                   void *values_out, void *opt_states_out, uint32_t *steps_out, void *stream);
/* assign_opt_states (hogwild_embedding_store.hpp:6278-6351): sets the optimizer
 * state rows (num_keys x dim x states values of OptT, laid out as exported)
 * and, when steps is not null, the Adam steps of present keys. Every key
 * must be present ("assign_opt_states key is absent from dimension table");
 * nothing is written otherwise. */
int se_assign_opt_states(se_store *store, int64_t dim, const void *keys, size_t num_keys,
                         const void *opt_states, size_t num_state_values, const uint32_t *steps,
                         void *stream);

/* Embedding bag (no counterpart in the reference, whose DLRM users pool the
 * rows of lookup / lookup_or_insert themselves): sum pooling of multi-hot
 * bags. Bag b holds keys [offsets[b], offsets[b+1]) (int64 CSR offsets,
 * num_bags + 1 entries); out_pooled[b] (dim values of ParamT) is the sum of
 * their parameter rows in key order, in fp32 from +0.0, rounded once to
 * ParamT. Absent keys add a zero row, or with insert != 0 are inserted first
 * as lookup_or_insert does. Offsets in host memory must start at 0, be
 * non-decreasing and end at num_keys; device offsets are clamped to
 * [0, num_keys]. */
int se_embedding_bag(se_store *store, const void *keys, size_t num_keys, const int64_t *offsets,
                     size_t num_bags, int64_t dim, void *out_pooled, int32_t insert, void *stream);
/* Backward of se_embedding_bag: every key of bag b accumulates pooled_grads[b]
 * (dim values of the gradient dtype) - the same result as
 * se_accumulate_gradients with the pooled gradient repeated for each key,
 * without building the repeated rows. */
int se_embedding_bag_backward(se_store *store, const void *keys, size_t num_keys, const int64_t *offsets,
                              size_t num_bags, int64_t dim, const void *pooled_grads, void *stream);

/* assign_scores (hogwild_embedding_store.hpp:5202-5250): each key's score is
 * set in the first table that holds it; absent keys are skipped. Needs a
 * score policy. se_read_scores reads them back (0 for absent keys). */
int se_assign_scores(se_store *store, const void *keys, size_t num_keys, const uint64_t *scores,
                     void *stream);
int se_read_scores(se_store *store, const void *keys, size_t num_keys, uint64_t *scores_out, void *stream);

/* Metadata conventions (embedding_table_interface.hpp:317-396). */
int se_store_size(se_store *store, uint64_t *out_size);
int se_store_dim_size(se_store *store, int64_t dim, uint64_t *out_size);
int se_store_reserve(se_store *store, size_t keys, int64_t dim);
int se_store_internal_shard_count(se_store *store, uint64_t *out_count);
int se_store_entries_per_page(se_store *store, uint64_t *out_entries);
/* Gradient rows dropped at optimizer_step because their key was absent. */
int se_store_dropped_gradients(se_store *store, uint64_t *out_count);
/* Optimizer state of one key, for checks: state holds the optimizer's state
 * rows (Adam m then v, or the Adagrad accumulator) in OptT; *found is 0 if the
 * key is absent. Host pointers. */
int se_store_read_state(se_store *store, int64_t dim, uint64_t key, void *param_out,
                        void *state_out, uint32_t *step_out, int32_t *found);
/* EmbeddingTableFacade::clear (hogwild_embedding_store.hpp:5107-5154; Python
 * EmbeddingStore.clear, sparse_embedding/src/bindings/module.cpp:640):
 * removes every key of every table and discards the gradients accumulated
 * since the last optimizer_step; reserved capacity is kept. Waits for the
 * stream. */
int se_store_clear(se_store *store, void *stream);
/* Waits for all work the store has queued. */
int se_store_synchronize(se_store *store);
/* CUDA-event timing of the store's kernels: enable, then read the summed
 * device time and launch count of kernels whose name contains `name`. */
int se_store_profile_enable(se_store *store, int32_t enable);
int se_store_profile_read(se_store *store, const char *name, double *out_ms, uint64_t *out_launches);

/* PartitionerFacade::partition_span (sparse_embedding/src/ops/partitioner.hpp:48-70,
 * 72-406) for the three registered algorithms: out[i] = partition of keys[i]. */
int se_partition(int32_t kind, uint32_t num_partitions, int32_t key_dtype, const void *keys,
                 size_t num_keys, uint32_t *out_partition_ids, int32_t device, void *stream);
/* PartitionerFacade::filter_span: out_mask[i] = (partition of keys[i] == target). */
int se_filter(int32_t kind, uint32_t num_partitions, int32_t key_dtype, const void *keys,
              size_t num_keys, uint32_t target_partition, uint8_t *out_mask, int32_t device,
              void *stream);

/* se::ops::unique_keys_inverse (sparse_embedding/src/ops/unique_ops.hpp:73-418;
 * Python async_unique, sparse_embedding/src/bindings/module.cpp:959-1072):
 * the distinct keys of keys[0, num_keys) in order of first appearance (the
 * reference leaves the order unspecified; its sequential path uses this
 * one), with int32 inverse indices (unique_keys_out[inverse[i]] == keys[i]),
 * the position of each key's first appearance and its number of
 * appearances. unique_keys_out (key_dtype), first_indices_out and counts_out
 * need room for num_keys entries, inverse_out for num_keys; any of the last
 * three may be null (not computed). *num_unique_out receives the count.
 * Host or device pointers; the call waits for its results. num_keys must be
 * below 2^31 (validate_unique_input_size, unique_ops.hpp:42-47). */
int se_unique(int32_t key_dtype, const void *keys, size_t num_keys, void *unique_keys_out,
              int32_t *inverse_out, int32_t *first_indices_out, int32_t *counts_out,
              uint64_t *num_unique_out, int32_t device, void *stream);

/*
 * Exchange routing (no reference counterpart: the reference leaves routing to
 * the caller, sparse_embedding/partitioner.py:84-100). Device pointers only.
 * Partitions keys and groups them by destination, stably: send_keys holds the
 * keys of partition 0 first, each partition in input order; send_positions[j]
 * is the input position of send_keys[j]; counts[p] is the number of keys of
 * partition p. Keys are num_keys values of key_dtype; send_keys has the same dtype.
 */
int se_partition_route(int32_t kind, uint32_t num_partitions, int32_t key_dtype, const void *keys,
                       size_t num_keys, void *send_keys, uint32_t *send_positions,
                       uint32_t *counts, int32_t device, void *stream);
/*
 * se_partition_route without any device allocation. It has no counterpart in
 * the reference. Same arguments, results and errors as se_partition_route,
 * for callers that cannot allocate device memory during a step: a host
 * framework whose own allocator has reserved (nearly) all device memory, or a
 * serving loop that must not fail or stall on an allocation mid-batch.
 * Its scratch (per-tile partition counts and offsets) is a fixed array
 * compiled into the library and held by every GPU that loads it until the
 * process exits: 2 x 256 KiB. Limit: ceil(num_keys / 2048) * num_partitions
 * <= 65536 (e.g. up to 16,777,216 keys over 8 partitions) and
 * num_partitions <= 1024; larger inputs fail with SE_ERR_INVALID_ARGUMENT.
 * The first call on a device looks up the scratch array's device address on
 * that device; make that first call before any stream capture. All calls share
 * the one array, so calls that overlap on the GPU (different streams, or
 * different host threads, on one device) race; serialise them.
 */
int se_partition_route_noalloc(int32_t kind, uint32_t num_partitions, int32_t key_dtype,
                               const void *keys, size_t num_keys, void *send_keys,
                               uint32_t *send_positions, uint32_t *counts, int32_t device,
                               void *stream);
/* Moves rows between the routed order and the input order. row_bytes per row.
 * scatter=0: out[positions[j]] = in[j]  (routed -> input order)
 * scatter=1: out[j] = in[positions[j]]  (input -> routed order) */
int se_permute_rows(const void *in_rows, void *out_rows, const uint32_t *positions, size_t num_rows,
                    size_t row_bytes, int32_t scatter, int32_t device, void *stream);

/*
 * Peer-memory exchange of a key-sharded store: one process per GPU, rank r
 * owns the keys partitioner `kind` maps to r (no reference counterpart: the
 * reference leaves cross-worker routing to its caller,
 * sparse_embedding/partitioner.py:84-100). Each rank's batch goes to the
 * owners and back through CUDA IPC mappings of every rank's exchange arena
 * (NVLink peer stores, no collective library); the owner applies
 * lookup_or_insert / forward_lookup / accumulate_gradients to its local store
 * with the received keys in sender-rank order, so results equal one store fed
 * the concatenation of the ranks' batches. optimizer_step stays per-rank
 * (se_optimizer_step on the local store).
 *
 * Collective use: every rank makes the same sequence of exchange calls on one
 * stream each. Waits inside the kernels give up after timeout_ms and mark the
 * exchange failed; se_exchange_check raises that (SE_ERR_RUNTIME) and the
 * exchange must then be recreated. Device pointers only; calls are
 * asynchronous on `stream`.
 */
typedef struct se_exchange se_exchange;
/* This rank's end over `store` (which must outlive it) for rows of length
 * dim: world_size <= 64 ranks, at most max_keys_per_rank keys per rank per
 * call. Allocates the arena on the store's device. */
int se_exchange_create(se_store *store, int32_t partitioner_kind, uint32_t world_size, uint32_t rank,
                       uint64_t max_keys_per_rank, int64_t dim, uint32_t timeout_ms, se_exchange **out);
/* Writes this rank's arena handle (a CUDA IPC handle, 64 bytes) to handle_out. */
int se_exchange_handle(se_exchange *ex, void *handle_out, size_t handle_bytes);
/* Maps every peer's arena: handles holds world_size handles in rank order
 * (this rank's entry is ignored). Call once, after every rank created its end. */
int se_exchange_connect(se_exchange *ex, const void *handles, size_t handles_bytes);
/* Connects the ends of all ranks when they live in this one process
 * (exchanges[r] is rank r; count == world_size). */
int se_exchange_connect_local(se_exchange *const *exchanges, uint32_t count);
/* Rows (value dtype, n x dim, batch order) of this rank's keys from their
 * owners: insert != 0 is lookup_or_insert (hogwild_embedding_store.hpp:4925-4980),
 * insert == 0 is forward_lookup with zero rows for absent keys (4406-4534). */
int se_exchange_lookup(se_exchange *ex, const void *keys, size_t n, void *out, int32_t insert, void *stream);
/* accumulate_gradients (hogwild_embedding_store.hpp:4536-4680) at the owners:
 * grads holds n x dim values of the gradient dtype. Device-side validation
 * (see se_accumulate_gradients with device inputs). */
int se_exchange_accumulate(se_exchange *ex, const void *keys, size_t n, const void *grads, void *stream);
/* accumulate_gradients for the keys of this rank's last se_exchange_lookup,
 * in that batch's order (grads: n x dim, n = that batch's size). The rows
 * follow the lookup's route and the owners reuse the keys it delivered, so no
 * keys cross NVLink again. Every rank must make the same choice of call. */
int se_exchange_accumulate_routed(se_exchange *ex, const void *grads, size_t n, void *stream);
/* Synchronises `stream`; raises a timed-out wait, then the owner table's errors. */
int se_exchange_check(se_exchange *ex, void *stream);
/* Sender-side dedupe (no reference counterpart): with enable != 0, each
 * se_exchange_lookup routes every distinct key of the rank's batch once and
 * expands the returned rows to the batch's positions (rows are identical to
 * the plain route), and se_exchange_accumulate_routed sums each distinct
 * key's gradient rows on the sender (fp32) before sending one row per key
 * (the order of the adds changes: updates match the plain route within
 * fp32 reassociation). Every rank of the exchange must make the same
 * choice; rows of at most 8,192 values. */
int se_exchange_set_dedupe(se_exchange *ex, int32_t enable);
/* Frees this rank's end. Call only after every rank finished its last
 * exchange call (peers store into this arena). */
int se_exchange_destroy(se_exchange *ex);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* SE_GPU_H_ */
