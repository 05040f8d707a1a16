/*
 * lgbm_b200 — C ABI of the B200 histogram tree learner.
 *
 * This ABI replaces the reference's compute seam, `trait Backend` of
 * BectorVoom/lightgbm_rs (crates/lgbm-compute/src/lib.rs:1092-2782), and the
 * whole-tree / whole-iteration device paths behind it. Each entry point names
 * the reference interface it stands in for.
 *
 * Conventions
 *  - Every function returns an int status (LGBM_B200_*). On failure,
 *    lgbm_b200_last_error() returns a thread-local message. No C++ exception,
 *    abort or device trap crosses this boundary.
 *  - Host pointers are borrowed for the duration of the call only.
 *  - Device state is owned by opaque handles with create/destroy pairs.
 *  - Histograms are interleaved [g0, h0, g1, h1, ...] f64 cells, as in the
 *    reference (GET_GRAD(i) = hist[2i], GET_HESS(i) = hist[2i+1]).
 */
#ifndef LGBM_B200_H
#define LGBM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. 1..5 mirror lgbm_compute::error::ComputeError
 * (crates/lgbm-compute/src/error.rs:19-80). */
#define LGBM_B200_OK 0
#define LGBM_B200_BIN_OUT_OF_RANGE 1
#define LGBM_B200_LENGTH_MISMATCH 2
#define LGBM_B200_CAPABILITY_UNAVAILABLE 3
#define LGBM_B200_RUNTIME 4
#define LGBM_B200_NON_FINITE 5
#define LGBM_B200_INVALID_ARGUMENT 6

/* Missing-value handling of a feature (lgbm-dataset/src/bin_mapper.rs:15-20). */
#define LGBM_B200_MISSING_NONE 0
#define LGBM_B200_MISSING_ZERO 1
#define LGBM_B200_MISSING_NAN 2

/* Objectives on the path (lgbm-objective/src/binary.rs, regression.rs, rank.rs). */
#define LGBM_B200_OBJECTIVE_BINARY 0
#define LGBM_B200_OBJECTIVE_L2 1
#define LGBM_B200_OBJECTIVE_LAMBDARANK 2

/* Largest query a lambdarank objective accepts: the DCG discount table's length
 * (K_MAX_POSITION, lgbm-metric/src/dcg_calculator.rs:32). */
#define LGBM_B200_MAX_QUERY_ROWS 10000

/* Gradient-pair encodings accepted by lgbm_b200_learner_grow_tree. */
#define LGBM_B200_GH_F32 0       /* float g[N], float h[N] */
#define LGBM_B200_GH_INT8_PAIR 1 /* int8 (qg, qh) per row + grad/hess scales */

/* lgbm_compute::gain::GainConfig (crates/lgbm-compute/src/gain.rs:904-960). */
typedef struct lgbm_b200_gain_config {
  int32_t min_data_in_leaf;
  int32_t _reserved;
  double min_sum_hessian_in_leaf;
  double max_delta_step;
  double lambda_l1;
  double lambda_l2;
  double min_gain_to_split;
  double path_smooth;
  double parent_output;
  /* categorical splits (feature_histogram_categorical.rs; LightGBM defaults 100, 32,
   * 4, 10, 10) */
  int32_t min_data_per_group;
  int32_t max_cat_threshold;
  int32_t max_cat_to_onehot;
  int32_t _reserved2;
  double cat_l2;
  double cat_smooth;
} lgbm_b200_gain_config;

/* lgbm_compute::gain::SplitInfo (crates/lgbm-compute/src/gain.rs:1040-1065).
 * gain == -inf means "no split". */
typedef struct lgbm_b200_split_info {
  uint32_t threshold;
  int32_t default_left;
  int32_t left_count;
  int32_t right_count;
  double gain;
  double left_sum_gradient;
  double left_sum_hessian;
  double right_sum_gradient;
  double right_sum_hessian;
  double left_output;
  double right_output;
} lgbm_b200_split_info;

/* The per-feature fields of lgbm_treelearner::FeatureColumn the learner reads
 * (crates/lgbm-treelearner/src/learner.rs:87-140). offset is derived:
 * 1 iff most_freq_bin == 0 (crates/lgbm-treelearner/src/lib.rs:89-95). */
typedef struct lgbm_b200_feature_meta {
  int32_t num_bin;
  int32_t default_bin;
  int32_t most_freq_bin;
  int32_t missing_type;
  int32_t bin_type; /* 0 numerical, 1 categorical (BinType, bin_mapper.rs:22-26) */
} lgbm_b200_feature_meta;

/* lgbm_compute::BatchedSplitFeature (crates/lgbm-compute/src/kernels/split.rs:77). */
typedef struct lgbm_b200_batched_feature {
  int64_t slot_off;
  uint32_t num_bin;
  int32_t offset;
  uint32_t default_bin;
  uint32_t most_freq_bin;
  int32_t skip_default_bin;
  int32_t na_as_missing;
  int32_t run_forward;
  int32_t _reserved;
} lgbm_b200_batched_feature;

/* Tree node arrays (crates/lgbm-model/src/tree.rs:94-160). Caller-owned host
 * arrays sized for max_leaves leaves / max_leaves-1 internal nodes. */
typedef struct lgbm_b200_tree {
  int32_t num_leaves;
  int32_t max_leaves;
  int32_t* left_child;
  int32_t* right_child;
  int32_t* split_feature;
  uint32_t* threshold_bin;
  float* split_gain;
  int8_t* decision_type;
  double* leaf_value;
  double* leaf_weight;
  int32_t* leaf_count;
  double* internal_value;
  int32_t* internal_count;
  /* per internal node, 8 words: the set of bins a categorical node sends left
   * (decision_type bit 0; threshold_bin is the categorical-node index); may be
   * NULL. The category bitsets of the model text follow from the feature's
   * bin_to_category (Tree::split_categorical, lgbm-model/src/tree.rs:710-770). */
  uint32_t* cat_bins;
} lgbm_b200_tree;

/* SerialTreeLearner construction parameters
 * (crates/lgbm-treelearner/src/learner.rs:627). */
typedef struct lgbm_b200_learner_config {
  int32_t num_leaves;
  int32_t max_depth;
  lgbm_b200_gain_config gain;
} lgbm_b200_learner_config;

/* The Gbdt training knobs the path reads (crates/lgbm-boosting/src/gbdt.rs:691-1300). */
typedef struct lgbm_b200_train_config {
  lgbm_b200_learner_config learner;
  int32_t objective;
  int32_t use_quantized_grad;
  int32_t num_grad_quant_bins;
  int32_t boost_from_average;
  double sigmoid;
  double learning_rate;
  /* Lambdarank only (Lambdarank::new, lgbm-objective/src/rank.rs:152-227): the query
   * boundaries of this device's rows (num_queries + 1 ascending prefix sums from 0 to
   * num_data; borrowed for the call), lambdarank_truncation_level, lambdarank_norm,
   * and the label gains (num_label_gain = 0: the default 2^i - 1 for i < 31). A
   * ranking objective has no boost-from-average score. */
  const int32_t* query_boundaries;
  int32_t num_queries;
  int32_t lambdarank_truncation_level;
  int32_t lambdarank_norm;
  int32_t num_label_gain;
  const double* label_gain;
  /* use_quantized_grad only: stochastic rounding (the reference's default,
   * crates/lgbm-core/src/config/mod.rs:485): rounding offsets from the reference's
   * seeded xorshift64 (crates/lgbm-treelearner/src/gradient_discretizer.rs:252-262),
   * seed ((iteration << 20) ^ 0x51702010) per iteration (crates/lgbm-boosting/src/
   * gbdt.rs:950), drawn over the rows of the whole job in row order (a data-parallel
   * job: rank 0's rows first). 0: deterministic rounding (offset 0.5). */
  int32_t stochastic_rounding;
  int32_t _reserved0;
} lgbm_b200_train_config;

/* BinMapper::find_bin_from_column parameters (crates/lgbm-dataset/src/bin_mapper.rs:642-675). */
typedef struct lgbm_b200_bin_config {
  int32_t max_bin;
  int32_t min_data_in_bin;
  int32_t min_data_in_leaf;
  int32_t pre_filter;
  int32_t use_missing;
  int32_t zero_as_missing;
  int32_t bin_construct_sample_cnt;
  int32_t data_random_seed;
} lgbm_b200_bin_config;

/* BinMapper result fields (crates/lgbm-dataset/src/bin_mapper.rs:45-60). */
typedef struct lgbm_b200_bin_mapper {
  int32_t num_bin;
  int32_t missing_type;
  int32_t default_bin;
  int32_t most_freq_bin;
  int32_t is_trivial;
  int32_t _reserved;
  double min_val;
  double max_val;
  double sparse_rate;
} lgbm_b200_bin_mapper;

typedef struct lgbm_b200_dataset lgbm_b200_dataset;
typedef struct lgbm_b200_learner lgbm_b200_learner;
typedef struct lgbm_b200_booster lgbm_b200_booster;

/* Thread-local message of the last failed call on this thread ("" if none). */
const char* lgbm_b200_last_error(void);

/* ABI version of this header (major * 100 + minor). */
int32_t lgbm_b200_abi_version(void);

/* Number of CUDA devices visible (0 when none; never an error). */
int lgbm_b200_device_count(int32_t* out);

/* Frees the device blocks (1 MB and larger) that destroyed datasets and
 * boosters left in this library's per-process cache, on `device` (-1: every
 * device), and reports the bytes freed (may be NULL). No counterpart in the
 * reference, whose CubeCL runtime keeps its own memory pool. The cache is
 * also trimmed on its own before a cudaMalloc is reported as failed. */
int lgbm_b200_release_cached_memory(int32_t device, int64_t* released_bytes);

/* ------------------------------------------------------------------ binning */

/* BinMapper::find_bin_from_column + value_to_bin
 * (crates/lgbm-dataset/src/bin_mapper.rs:642-675, :148-199, :201-415).
 * upper_bounds receives num_bin values (capacity upper_cap); bins_out (may be
 * NULL) receives value_to_bin of every row. Host-only; needs no GPU. */
int lgbm_b200_bin_column(const double* column, int64_t n, const lgbm_b200_bin_config* cfg,
                         lgbm_b200_bin_mapper* mapper_out, double* upper_bounds,
                         int32_t upper_cap, uint32_t* bins_out);

/* BinMapper::find_bin_categorical + value_to_bin for a categorical column
 * (crates/lgbm-dataset/src/bin_mapper.rs:416-641, :148-199): categories by
 * descending count, bin 0 the dummy bin of NaN / negative / unseen values.
 * bin_to_category receives num_bin category values (bin 0: -1; capacity cap);
 * mapper_out->_reserved is 1 (categorical). Host-only; needs no GPU. */
int lgbm_b200_bin_column_categorical(const double* column, int64_t n,
                                     const lgbm_b200_bin_config* cfg,
                                     lgbm_b200_bin_mapper* mapper_out, int32_t* bin_to_category,
                                     int32_t cap, uint32_t* bins_out);

/* BinMapper::find_bin_from_column of many numerical columns at once, on the device
 * (crates/lgbm-dataset/src/bin_mapper.rs:642-675 with find_bin_numeric :201-415): every
 * column's sample (the same rows for every column: create_sample_indices, :92-95) is
 * gathered on the host, then sorted and binned on the device; the mappers and bounds
 * equal lgbm_b200_bin_column's. columns: feature-major host arrays of n f32
 * (value_width 4) or f64 (8) values. mappers_out[f] and upper_bounds[f * upper_cap ...]
 * (num_bin values; upper_cap >= max_bin + 2) receive the results. Categorical columns
 * go through lgbm_b200_bin_column_categorical. */
int lgbm_b200_find_bins(int32_t device, const void* const* columns, int32_t value_width,
                        int64_t n, int32_t num_features, const lgbm_b200_bin_config* cfg,
                        lgbm_b200_bin_mapper* mappers_out, double* upper_bounds,
                        int32_t upper_cap);

/* ------------------------------------------------------ per-op Backend mirror */

/* Backend::construct_histograms (crates/lgbm-compute/src/lib.rs:1119-1126):
 * histogram of one feature over all rows. out has 2*num_bin cells.
 * f32 g/h accumulate in 64-bit fixed point (relative error ~1e-11 of the
 * reference's f64 fold). num_bin <= 256. */
int lgbm_b200_construct_histograms(const uint32_t* binned, const float* gradients,
                                   const float* hessians, int64_t n, uint32_t num_bin,
                                   double* out);

/* Backend::find_best_split (crates/lgbm-compute/src/lib.rs:1174-1189), computed
 * by the device threshold-scan kernel; bit-exact with the reference CPU scan. */
int lgbm_b200_find_best_split(const double* hist, const lgbm_b200_gain_config* cfg,
                              uint32_t num_bin, int32_t offset, uint32_t default_bin,
                              uint32_t most_freq_bin, int32_t skip_default_bin,
                              int32_t na_as_missing, int32_t run_forward, double sum_gradient,
                              double sum_hessian, int32_t num_data, lgbm_b200_split_info* out);

/* Backend::find_best_splits_batched (crates/lgbm-compute/src/lib.rs:1500-1509). */
int lgbm_b200_find_best_splits_batched(const double* buf, int64_t buf_len,
                                       const lgbm_b200_batched_feature* feats, int32_t n_feats,
                                       const lgbm_b200_gain_config* cfg, double sum_gradient,
                                       double sum_hessian, int32_t num_data,
                                       lgbm_b200_split_info* out);

/* Backend::data_partition (crates/lgbm-compute/src/lib.rs:1206-1215): stable
 * partition of rows 0..n-1; order_out = [left ascending | right ascending]. */
int lgbm_b200_data_partition(const uint32_t* bins, int64_t n, uint32_t num_bin, uint32_t min_bin,
                             uint32_t max_bin, uint32_t threshold, uint32_t most_freq_bin,
                             uint32_t* order_out, int64_t* split_point_out);

/* The kernel-level partition with the whole missing-value routing fan-out:
 * partition_leaf_stable / partition_on_device (crates/lgbm-compute/src/kernels/
 * data_partition.rs:487-520, routing RouteFlags::derive + route_to_left :325-406,
 * :64-138). Arguments as lgbm_b200_data_partition plus default_bin, missing_type
 * (0 None, 1 Zero, 2 NaN) and default_left. missing_type 1 routes the zero bin
 * (min_bin + default_bin - [most_freq_bin == 0]) and 2 the NA bin (max_bin) by
 * default_left, unless the most frequent bin is that bin; min_bin == max_bin is the
 * degenerate one-bin feature. Host buffers; result [left ascending | right
 * ascending]. */
int lgbm_b200_data_partition_missing(const uint32_t* bins, int64_t n, uint32_t num_bin,
                                     uint32_t min_bin, uint32_t max_bin, uint32_t threshold,
                                     uint32_t most_freq_bin, uint32_t default_bin,
                                     int32_t missing_type, int32_t default_left,
                                     uint32_t* order_out, int64_t* split_point_out);

/* Allocation-free variant of lgbm_b200_data_partition. No counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc when they
 * partition rows. Examples are a host engine whose device memory belongs to its
 * own pool allocator, which has reserved the HBM up front so that a cudaMalloc
 * can fail or fragment its reservation, and a latency-bound loop that cannot
 * pay for cudaMalloc/cudaFree, which synchronise the whole device.
 *
 * Same argument meaning and result as lgbm_b200_data_partition, except that
 * `bins` (n bytes, one bin per row), `order_out` (n words) and
 * `split_point_out` (one int64) are DEVICE pointers on the current device, and
 * the work is enqueued on `stream` (a cudaStream_t; NULL is the legacy default
 * stream) without waiting for it: the outputs are ready once the stream
 * reaches that point. Bins are not range-checked on this path; a bin outside
 * [min_bin, max_bin] goes where the most frequent bin goes.
 *
 * Scratch: the partition's look-back status words (one per 2048-row tile), two
 * counters and the routing descriptor live in a fixed array compiled into the
 * library, one per device, 256 B + 8 B per tile = 262,400 B at the limit. The
 * function allocates nothing. n above LGBM_B200_NOALLOC_MAX_ROWS fails with
 * LGBM_B200_CAPABILITY_UNAVAILABLE and enqueues no work. Each call first
 * clears, on `stream`, the status words and counters it uses; they must start
 * at zero. Every call on a device shares the one array, so calls that overlap
 * on the GPU (different streams, or different host threads) race and return
 * wrong results: serialise them. The first call on each device looks the
 * array up with cudaGetSymbolAddress (with that device current); make that
 * first call before any stream capture. A failed lookup returns
 * LGBM_B200_RUNTIME and is tried again by the next call.
 *
 * The partition's look-back waits are bounded. If one runs out (a tile whose
 * predecessor never published, e.g. under heavy preemption), `order_out` is
 * left incomplete and *split_point_out is set to the sentinel -1 on the
 * stream: check it before using the order. The allocating entry point
 * returns LGBM_B200_RUNTIME in the same case. */
#define LGBM_B200_NOALLOC_MAX_ROWS 67108864 /* 2^26 rows */
int lgbm_b200_data_partition_noalloc(const uint8_t* bins, int64_t n, uint32_t num_bin,
                                     uint32_t min_bin, uint32_t max_bin, uint32_t threshold,
                                     uint32_t most_freq_bin, uint32_t* order_out,
                                     int64_t* split_point_out, void* stream);

/* Backend::subtract_histograms (crates/lgbm-compute/src/lib.rs:1314-1319). */
int lgbm_b200_subtract_histograms(const double* parent, const double* child, int64_t len,
                                  double* out);

/* ---------------------------------------------------- device-resident dataset */

/* Backend::upload_resident_bins (crates/lgbm-compute/src/lib.rs:1564): take
 * feature-major bin columns (bin_width 1, 2 or 4 bytes per bin) and keep a
 * row-major u8 bin matrix resident on `device`. Validates bin < num_bin once
 * (the learner's bin-range gate, learner.rs:1161-1187). */
int lgbm_b200_dataset_create(int32_t device, const void* const* columns, int32_t bin_width,
                             int64_t num_data, int32_t num_features,
                             const lgbm_b200_feature_meta* meta, lgbm_b200_dataset** out);
int lgbm_b200_dataset_destroy(lgbm_b200_dataset* ds);

/* The device dataset from raw feature values: BinMapper::value_to_bin
 * (crates/lgbm-dataset/src/bin_mapper.rs:148-199) runs on the device with the mappers
 * found on the host from each column's sample (lgbm_b200_bin_column /
 * lgbm_b200_bin_column_categorical with bins_out = NULL). columns: feature-major host
 * arrays of f32 (value_width 4) or f64 (8). upper_bounds[f] (numerical features) and
 * bin_to_category[f] (categorical features) hold num_bin values each. Replaces the
 * host binning loop of the reference's dataset construction
 * (crates/lgbm/src/booster.rs:381-540). */
int lgbm_b200_dataset_create_from_values(int32_t device, const void* const* columns,
                                         int32_t value_width, int64_t num_data,
                                         int32_t num_features,
                                         const lgbm_b200_feature_meta* meta,
                                         const double* const* upper_bounds,
                                         const int32_t* const* bin_to_category,
                                         lgbm_b200_dataset** out);
/* Copies the device bin matrix back: row-major u8 [num_data][stride], stride =
 * num_features rounded up to a multiple of 16. */
int lgbm_b200_dataset_copy_bins(const lgbm_b200_dataset* ds, uint8_t* out);
int lgbm_b200_dataset_num_data(const lgbm_b200_dataset* ds, int64_t* out);

/* ------------------------------------------------------------ tree learner */

/* SerialTreeLearner::new (crates/lgbm-treelearner/src/learner.rs:627). */
int lgbm_b200_learner_create(lgbm_b200_dataset* ds, const lgbm_b200_learner_config* cfg,
                             lgbm_b200_learner** out);
int lgbm_b200_learner_destroy(lgbm_b200_learner* learner);

/* Backend::grow_tree_on_device_with_cfg (crates/lgbm-compute/src/lib.rs:2771-2781):
 * grow one tree from host gradients. gh_kind LGBM_B200_GH_F32: gh = float[2][N]
 * (g then h); LGBM_B200_GH_INT8_PAIR: gh = int8 (qg, qh) per row and
 * quant_scales = {grad_scale, hess_scale, is_constant_hessian, num_grad_quant_bins}
 * as produced by GradientDiscretizer (gradient_discretizer.rs:145-191), in which
 * case the tree is bit-identical to the reference learner on the dequantized
 * gradients. indices_out (N), leaf_begin_out / leaf_count_out (num_leaves) may
 * be NULL; rows inside a leaf are a permutation of the reference's order. */
int lgbm_b200_learner_grow_tree(lgbm_b200_learner* learner, int32_t gh_kind, const void* gh,
                                const double* quant_scales, lgbm_b200_tree* tree_out,
                                uint32_t* indices_out, int32_t* leaf_begin_out,
                                int32_t* leaf_count_out);

/* ------------------------------------------------------------------ booster */

/* Gbdt (crates/lgbm-boosting/src/gbdt.rs:691-1300) with the score kept resident:
 * gradients, quantization, tree growth, shrinkage and score update all run on
 * the device; labels are copied once. */
int lgbm_b200_booster_create(lgbm_b200_dataset* ds, const float* labels,
                             const lgbm_b200_train_config* cfg, lgbm_b200_booster** out);
int lgbm_b200_booster_destroy(lgbm_b200_booster* b);
/* Run up to num_iterations boosting iterations; *done_out receives how many
 * produced a tree before training stopped (a 1-leaf tree after the first). */
int lgbm_b200_booster_train(lgbm_b200_booster* b, int32_t num_iterations, int32_t* done_out);
int lgbm_b200_booster_num_trees(const lgbm_b200_booster* b, int32_t* out);
/* Trees after shrinkage; the init score of boost_from_average is reported separately. */
int lgbm_b200_booster_get_tree(lgbm_b200_booster* b, int32_t index, lgbm_b200_tree* out);
int lgbm_b200_booster_init_score(const lgbm_b200_booster* b, double* out);
int lgbm_b200_booster_get_scores(lgbm_b200_booster* b, double* out);
/* The gradients of the most recent iteration (f32, before quantization). */
int lgbm_b200_booster_get_gradients(lgbm_b200_booster* b, float* g, float* h);
/* Device time of the last lgbm_b200_booster_train call in ms (out3[1]; the other
 * two entries are 0). */
int lgbm_b200_booster_phase_ms(const lgbm_b200_booster* b, double* out3);
/* Run ONE more boosting iteration outside the CUDA graph with CUDA events around
 * every kernel launch. ms_out[7] receives the summed device time per kernel class
 * {prepare, histogram build, fix+scan, partition, tree init, gradients, finish};
 * counts_out[8] = {kernel launches, histogram builds, rows streamed by the builds,
 * splits, parent rows streamed by the partitions, 1 if the partition kernel also
 * builds the child histogram, look-ahead partitions run, look-ahead partitions whose
 * leaf was the next split}. Builds and rows count the partitions whose result the tree
 * used. The iteration counts as a normal boosting iteration. */
int lgbm_b200_booster_profile_iteration(lgbm_b200_booster* b, double* ms_out,
                                        int64_t* counts_out);
/* Run `iterations` more boosting iterations through a CUDA graph of the same launch
 * sequence as lgbm_b200_booster_train (look-ahead stream included), whose tree kernels
 * stamp their device-time spans (%globaltimer at each CTA's entry and exit): a span is
 * first entry to last exit of one launch, as it ran in the pipeline. span_ms_out[7]
 * receives the mean per iteration of the summed spans per kernel class (same order as
 * profile_iteration; partition = the main-stream partitions). iter_ms_out[2] = {mean
 * device ms per iteration, mean summed spans of the look-ahead partitions, which run
 * beside the control steps}. counts_out[10] receives the same eight counters as
 * profile_iteration, summed over the iterations (counts_out[0]: stamped tree-kernel
 * launches), then the parent rows of the main partitions that ran inside control steps
 * (one device: a control step partitions the previous split's leaf itself when the
 * look-ahead did not) and the rows their child builds accumulated. No counterpart in the
 * reference (a profiling aid). */
int lgbm_b200_booster_profile_pipeline(lgbm_b200_booster* b, int32_t iterations,
                                       double* span_ms_out, double* iter_ms_out,
                                       int64_t* counts_out);
/* The raw spans of the last iteration lgbm_b200_booster_profile_pipeline ran: per slot
 * (0: the root build; 1 + 4*s + kind for split step s, kind 0 control step, 1 main-stream
 * partition, 2 look-ahead partition, 3 separate build) the earliest CTA entry and latest
 * CTA exit in %globaltimer ns; a slot not launched holds start = UINT64_MAX. phase_out
 * (optional, cap * 20 entries): for split step s, twenty marks at phase_out[20*s] (latest
 * CTA time, 0 when not reached). Eight control-step marks: pending split applied, feature
 * cells loaded, FixHistogram and child stores done, scans done, every feature of the CTA
 * done, pick inputs staged, pick made, control block written. Then six marks of the
 * step's look-ahead partition and six of its main partition, raised by the CTAs that hold
 * a tile: entry, setup done, first tile's rows routed, its prefix known, last tile
 * written, histogram flushed. *n_out receives the slot
 * count; at most cap entries of each span array are written. No counterpart in the
 * reference (a profiling aid). */
int lgbm_b200_booster_profile_spans(const lgbm_b200_booster* b, int32_t cap,
                                    uint64_t* start_out, uint64_t* end_out, uint64_t* phase_out,
                                    int32_t* n_out);
/* The launches timed by the last lgbm_b200_booster_profile_iteration, in launch order:
 * kernel class (the ms_out order of that call) and device ms of each timed span; *n_out
 * receives the count, at most cap entries are written. */
int lgbm_b200_booster_profile_launches(const lgbm_b200_booster* b, int32_t cap,
                                       int32_t* class_out, float* ms_out, int32_t* n_out);

/* ---------------------------------------------------- data-parallel training */

/* Several GPUs train one model on a dataset sharded by rows, one process (or
 * thread) per GPU: LightGBM's data-parallel tree learner. The reference has no
 * counterpart: it maps tree_learner=data/feature/voting back to serial
 * (crates/lgbm-core/src/config/set.rs:592-600). Every rank keeps its own rows;
 * after each histogram build the ranks sum the integer child histogram and its
 * left-row count over NCCL (one all-reduce per split), so all ranks take the
 * same decisions and hold the same trees. With quantized gradients the trees
 * are bit-identical to single-GPU training on all rows.
 *
 * NCCL is loaded at run time (libnccl.so.2); without it these calls return
 * LGBM_B200_CAPABILITY_UNAVAILABLE. Rank 0 makes the id with
 * lgbm_b200_comm_unique_id and hands the bytes to every rank out of band. */
typedef struct lgbm_b200_comm lgbm_b200_comm;
#define LGBM_B200_COMM_ID_BYTES 128
int lgbm_b200_comm_unique_id(uint8_t* id_out);
int lgbm_b200_comm_create(int32_t device, int32_t nranks, int32_t rank, const uint8_t* id,
                          lgbm_b200_comm** out);
int lgbm_b200_comm_destroy(lgbm_b200_comm* comm);

/* Gbdt over this rank's shard. `labels` are the shard's rows in the dataset's
 * order; the global row order is the shards in rank order (the init score is
 * computed from all labels, gathered once). Every rank must call
 * lgbm_b200_booster_train with the same iteration counts. Tree and score
 * accessors work as for lgbm_b200_booster_create; scores are this shard's. */
int lgbm_b200_booster_create_distributed(lgbm_b200_dataset* ds, const float* labels,
                                         const lgbm_b200_train_config* cfg,
                                         lgbm_b200_comm* comm, lgbm_b200_booster** out);

/* ---- Batch prediction from raw feature values (Tree::predict / GetLeaf,
 * lgbm-model/src/tree.rs:193-300; GbdtModel predict, lgbm-model/src/predict.rs) ---- */

/* A tree ensemble: every tree's internal nodes and leaves concatenated, in tree order
 * (borrowed for the create call). Child indices are tree-local: >= 0 an internal node
 * (always greater than its parent's index, as LightGBM numbers nodes), < 0 the leaf ~c.
 * A categorical node's threshold is its index into cat_boundaries over ALL trees;
 * cat_threshold holds the bitsets of real category values (LightGBM model text). */
typedef struct lgbm_b200_model {
  int32_t num_trees;
  int32_t num_features;          /* row width: max_feature_idx + 1 */
  const int32_t* node_offset;    /* [num_trees + 1] */
  const int32_t* leaf_offset;    /* [num_trees + 1] */
  const int32_t* split_feature;  /* [nodes] */
  const double* threshold;       /* [nodes] */
  const int8_t* decision_type;   /* [nodes] bit0 categorical, bit1 default left, bits 2-3 missing type */
  const int32_t* left_child;     /* [nodes] */
  const int32_t* right_child;    /* [nodes] */
  const double* leaf_value;      /* [leaves] */
  int32_t num_cat;
  int32_t transform;             /* 0 identity, 1 sigmoid (binary objective) */
  const int32_t* cat_boundaries; /* [num_cat + 1] */
  const uint32_t* cat_threshold; /* [cat_boundaries[num_cat]] */
  double sigmoid;
} lgbm_b200_model;

typedef struct lgbm_b200_predictor lgbm_b200_predictor;

/* Uploads the ensemble to `device` after checking every index in it. */
int lgbm_b200_predictor_create(int32_t device, const lgbm_b200_model* model,
                               lgbm_b200_predictor** out);
int lgbm_b200_predictor_destroy(lgbm_b200_predictor* p);
/* rows: host row-major f64 [num_rows][num_features]; out: host f64 [num_rows], the sum
 * of the trees' leaf values in tree order, then the model's transform unless raw_score. */
int lgbm_b200_predict(lgbm_b200_predictor* p, const double* rows, int64_t num_rows,
                      int32_t raw_score, double* out);

#ifdef __cplusplus
}
#endif

#endif /* LGBM_B200_H */
