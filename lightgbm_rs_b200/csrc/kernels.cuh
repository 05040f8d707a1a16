// Kernel entry points and the device-state bundle shared by the host runtime.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "common.cuh"

namespace lgbm_b200 {

// A contiguous run of features whose bins share one shared-memory accumulator
// in the histogram build. f_begin is a multiple of 16 so every block reads the
// row with aligned 16-byte vector loads.
struct DevFeatureGroup {
  int32_t f_begin;
  int32_t f_end;
  int32_t bin_base;  // first global bin of the group
  int32_t num_bins;  // bins in the group (packed layout) or (f_end-f_begin) << shift
  int32_t shift;     // quantized kernel: log2 of the per-feature bin stride in shared memory
  int32_t _pad;
};

// The 4-bin quantized build kernel keeps per-CTA accumulators for at most this many
// shared-memory cells (features x power-of-two bin stride): 4 x 4 B x 7168 = 112 KB,
// two CTAs per SM.
constexpr int kQ4MaxCells = 7168;

// Rows per tile of the row-partition kernel (one look-back status word per tile).
constexpr int kPartitionTileRows = 2048;

// Look-ahead slots: the kernel of step s uses slot s % kLaSlots. Step s + 2 may consume
// it and step s + 3 clears it; with several devices every rank has read it by then.
constexpr int kLaSlots = 4;

// Splits of up to this many partition tiles store per-tile partial histograms.
constexpr int kMaxPrivateTiles = 16;

// Most ranks of the peer-memory exchange (one node).
constexpr int kMaxXRanks = 8;

// One look-ahead partition: the leaf that ranks second at a control step's pick (the
// runner-up) is partitioned, with its child histogram, while the next control step runs.
// When the following pick chooses that leaf, its partition is already done. Written by
// the control step that picks (its last CTA), read by the look-ahead kernel of that
// step; the kernel adds the counters below.
struct LookAhead {
  int32_t active;      // a runner-up leaf with a positive gain was recorded
  int32_t leaf;
  int32_t feature;
  int32_t build;       // accumulate the child histogram
  int32_t build_left;  // ... of the left rows (else the right rows)
  uint32_t epoch;      // status-word epoch of the partition
  uint32_t ticket;     // tile tickets
  int32_t left_total;  // left rows
  int32_t failed;      // a look-back gave up (spin limit)
  int32_t ran;         // the kernel partitioned the leaf
  int32_t cancel;      // the next pick took another leaf: the kernel takes no more tiles
  uint32_t done;       // tiles finished (the fused control step's main partition record)
  uint32_t _pad;
  long long rows;      // parent rows streamed
  long long built;     // rows accumulated into the child histogram
  DevSplitInfo split;
  uint32_t cat[kCatWords];  // left bins of a categorical split
};

// Everything the per-split kernels touch, passed by value.
struct GrowDev {
  GrowCtrl* ctrl;
  const int32_t* stopped;  // booster-level stop flag (may be null)
  const DevFeature* feat;
  const DevFeatureGroup* groups;
  int32_t F;
  int32_t num_groups;
  const uint8_t* bins;  // row-major [N][stride]
  int32_t stride;
  int32_t L;
  int64_t N;
  int32_t max_depth;
  int32_t slot_len;  // cells per histogram slot
  DevGainConfig gain;
  // per-leaf state [L]
  int32_t* leaf_begin;
  int32_t* leaf_count;    // rows of the leaf on this device
  int32_t* leaf_count_g;  // rows of the leaf on all devices
  int32_t* leaf_is_right;  // the leaf is its parent node's right child
  int32_t* leaf_buf;  // 0/1 = index buffer, 2 = identity (root)
  int32_t* slot_of_leaf;
  DevLeafSplits* ls;
  DevSplitInfo* best;
  int32_t* best_feature;
  uint8_t* splittable;  // [L][F]
  // tree arrays [L]
  int32_t* t_left;
  int32_t* t_right;
  int32_t* t_split_feature;
  uint32_t* t_threshold;
  float* t_split_gain;
  int8_t* t_decision;
  double* t_leaf_value;
  double* t_leaf_weight;
  int32_t* t_leaf_count;
  double* t_internal_value;
  int32_t* t_internal_count;
  int32_t* t_leaf_depth;
  int32_t* t_leaf_parent;
  // work buffers
  uint32_t* idx0;
  uint32_t* idx1;
  unsigned long long* part_status;
  int32_t max_tiles;
  double* pool;            // [L][slot_len]
  long long* raw;          // [raw_len + 2]: the accumulated child, then its left-row count
  long long* rawpool;      // [L][raw_len]: integer histogram of every leaf
  int32_t raw_len;         // 2 * total_bins
  int32_t fused;           // the partition kernel accumulates the child histogram
  int32_t private_tiles;   // fused: splits of up to this many tiles store per-tile partials
  long long* partials;     // [private_tiles][raw_len]
  int64_t n_global;        // rows on all devices
  DevSplitInfo* scan_out;  // [2][F]
  uint32_t* scan_cat;      // [2][F][kCatWords] left bins of categorical scan results
  uint32_t* best_cat;      // [L][kCatWords] left bins of each leaf's best split
  uint32_t* t_cat;         // [L][kCatWords] left bins of each categorical tree node
  uint32_t* split_cat;     // [kCatWords] left bins of the pending split (categorical)
  int32_t packed4;         // the bin matrix holds two 4-bit bins per byte (row_bin)
  int32_t has_cat;         // some feature is categorical: the control step's CAT variant
  int32_t narrow_scan;     // numeric features of at most 64 bins: 256-thread control CTAs
  uint8_t* scan_ok;        // [2] leaf scanned flags
  // Data-parallel exchange of the accumulated child over peer memory (xranks > 1). Every
  // rank holds two accumulators [2][raw_len + 2]; producer k of a tree (the root build,
  // then split k-1's partition or build) adds into its own buffer k % 2 and publishes a
  // sequence number into every rank's flags; its consumer waits for all ranks' numbers,
  // sums buffer xpar over the ranks and clears its own other buffer (`raw` in a consumer
  // launch). With xranks <= 1 `raw` is the one accumulator of every launch.
  int32_t xranks;
  int32_t xrank;
  int32_t xpar;
  int32_t _xpad;
  long long* xlocal;                          // this rank's two accumulators
  long long* const* xbuf;                     // [xranks] each rank's accumulators (device)
  unsigned long long* xflags;                 // this rank's flags, one per rank
  unsigned long long* const* peer_xflags;     // [xranks] each rank's flags (device)
  unsigned long long* xseq;                   // exchanges this rank has published
  // Producer launches over peer memory publish their own exchange at the end (set on the
  // launch's copy): 1 the accumulator exchange (xflags / xseq), 2 the look-ahead slot
  // (la_flags / la_seq); 0 none (one device, or a separate signal kernel). arrive: the
  // two kinds' CTA arrival counters (zero between launches).
  int32_t self_signal;
  uint32_t* arrive;
  // Histogram builds with warp-aggregated atomics (LGBM_B200_WARP_AGG=1; the C1 layout only).
  int32_t warp_agg;
  // Placeholder warps of every control-step CTA run the pick's code on placeholder inputs
  // into scratch records while the prep runs, so that the code is in the SM's instruction
  // cache when the last CTA runs the pick for real.
  int32_t warm_pick;
  // One device, fused partition: the control step runs the main partition of the previous
  // split itself when the look-ahead did not (k_fixscan_part); else a launch of its own.
  int32_t fuse_main;
  // A look-ahead whose leaf the next pick did not take is cancelled (LookAhead.cancel).
  int32_t la_cancel;
  long long xwait_ns;                         // wait limit, then the spin-timeout error
  // Look-ahead partitions (fused partition): control step s records slot s % kLaSlots and
  // its look-ahead kernel fills it; control step s + 2 consumes it (when step s + 1 picked
  // the recorded leaf) and step s + 3 clears it. With the peer exchange (xranks > 1) the
  // accumulators are exchanged like the main one: each look-ahead kernel is followed by a
  // signal (la_seq) into every rank's la_flags, and the consumer sums all ranks' slot.
  int32_t lookahead;
  int32_t _lapad;
  LookAhead* la;                  // [kLaSlots]
  // [2] the split each fused control step partitions when the look-ahead did not, written
  // by the control step before it (record (s & 1) for step s; null when not fused)
  LookAhead* mainrec;
  long long* la_raw;              // [kLaSlots][raw_len + 2] accumulated child, left-row count
  long long* la_partials;         // [kLaSlots][private_tiles][raw_len]
  unsigned long long* la_status;  // [max_tiles] look-back words of the look-ahead kernel
  long long* const* la_xbuf;                // [xranks] each rank's la_raw (device)
  unsigned long long* la_flags;             // this rank's look-ahead flags, one per rank
  unsigned long long* const* peer_la_flags; // [xranks] each rank's la_flags (device)
  unsigned long long* la_seq;               // look-ahead signals this rank has published
  // gradients
  int32_t gh_mode;
  int32_t q4_shift;  // quantized build: log2 bin stride
  int32_t q4_nch;    // quantized build: 16-feature chunks per group
  const void* gh;  // float2[N] (GH_FLOAT) or uint16 int8 pairs (quantized)
  const DevGhParams* ghp;
  // Device-time spans of the tree's launches as the pipeline runs them (null: off). Each
  // CTA's thread 0 lowers span_start[span_slot] to its entry time and raises
  // span_end[span_slot] to its exit time (%globaltimer, ns). Slots: kSpanRootBuild, then
  // span_slot_of(s, kind) for split step s.
  unsigned long long* span_start;
  unsigned long long* span_end;
  int32_t span_slot;
  // Phase marks of split step s (null: off), kStepMarks words per step: word p is raised
  // to the latest CTA's %globaltimer at control-step phase p (CtlPhase), word
  // kCtlPhases + p at phase p of the step's look-ahead partition and word
  // kCtlPhases + kPartPhases + p at phase p of its main partition (PartPhase).
  unsigned long long* ctl_phase;
  // Feature slices of a data-parallel job over peer memory (sliced = 1): this rank's
  // control step decodes and scans features [slice_begin, slice_end) only, then the ranks
  // exchange their slices' best split of each scanned leaf (XPick records, pushed into
  // every rank's pick area, a flag per rank) and every rank reduces them in split_gt order
  // to the same pick. Otherwise the slice is every feature.
  int32_t sliced;
  int32_t slice_begin;
  int32_t slice_end;
  unsigned long long* pick_local;               // [2][kMaxXRanks][kXPickWords] records
  unsigned long long* const* peer_pick;         // [xranks] each rank's pick area (device)
  unsigned long long* pick_flags;               // this rank's pick flags, one per rank
  unsigned long long* const* peer_pick_flags;   // [xranks] each rank's pick flags (device)
  unsigned long long* pick_seq;                 // picks this rank has published
};

// One rank's contribution to a sliced pick: its slice's best split of each scanned leaf
// (feature -1: none) and their categorical left bins.
struct XPick {
  DevSplitInfo si[2];
  int32_t bf[2];
  uint32_t cat[2][kCatWords];
};
constexpr int kXPickWords = (int)((sizeof(XPick) + 15) / 16 * 2);

// Span slots of one tree: the root build, then four per split step.
enum SpanKind { SPAN_FIXSCAN = 0, SPAN_PARTITION = 1, SPAN_LOOKAHEAD = 2, SPAN_BUILD = 3 };
constexpr int kSpanRootBuild = 0;
__host__ __device__ inline int span_slot_of(int s, int kind) { return 1 + 4 * s + kind; }
inline int span_slots(int L) { return 1 + 4 * (L > 1 ? L - 1 : 1); }

// Phase marks of one control step: the pending split applied (every CTA), the feature's
// cells loaded and decoded, FixHistogram / compaction / child stores done, the scans done,
// every feature of the CTA done; then, in the last CTA only, the pick's inputs staged, the
// pick made, and the control block written.
enum CtlPhase {
  CP_PREP = 0, CP_LOADED = 1, CP_FIXED = 2, CP_SCANNED = 3, CP_FEATURES = 4, CP_STAGED = 5,
  CP_PICKED = 6, CP_WRITTEN = 7
};
constexpr int kCtlPhases = 8;

// Phase marks of a partition launch, raised by each CTA that holds a tile: its entry, its
// setup done (leaf range, feature mask, cleared accumulators), its first tile's rows loaded
// and routed, that tile's prefix known (look-back), its last tile written, its histogram
// flushed.
enum PartPhase {
  PP_START = 0, PP_READY = 1, PP_LOADED = 2, PP_PREFIX = 3, PP_TILES = 4, PP_FLUSHED = 5
};
constexpr int kPartPhases = 6;
constexpr int kStepMarks = kCtlPhases + 2 * kPartPhases;  // control, look-ahead, main

// Optional per-kernel timing of a launch sequence: events recorded around each kernel.
enum KernelClass { KC_PREPARE = 0, KC_BUILD = 1, KC_FIXSCAN = 2, KC_PARTITION = 3, KC_INIT = 4,
                   KC_GRAD = 5, KC_FINISH = 6, KC_COUNT = 7 };
struct LaunchProfiler {
  cudaEvent_t (*ev)[2];
  int* cls;
  int cap;
  int n;
  int begin(cudaStream_t st, int c);
  void end(cudaStream_t st, int slot);
};

// Reductions over the devices of a data-parallel job, enqueued on the caller's stream
// (and captured into its CUDA graph). Every device issues the same calls in the same
// order. A null DeviceComm means one device.
struct DeviceComm {
  void* ctx;
  void (*sum_i64)(void* ctx, long long* buf, int64_t n, cudaStream_t st);
  void (*max_u32)(void* ctx, uint32_t* buf, int64_t n, cudaStream_t st);
  void (*min_u32)(void* ctx, uint32_t* buf, int64_t n, cudaStream_t st);
};

// The second stream of the look-ahead partitions and its events (owned by the learner).
struct LookAheadStreams {
  cudaStream_t st;
  cudaEvent_t fork;     // after control step s, on the main stream
  cudaEvent_t done[kLaSlots];  // after the look-ahead kernel of step s, slot s % kLaSlots
  int blocks;           // CTAs of a look-ahead kernel (the control step keeps the rest) ...
  int blocks_fused;     // ... when the control step runs the main partition (all SMs)
  int main_blocks;      // CTAs of the main-stream partition while look-aheads run ...
  int main_late_blocks; // ... and from split step main_early_steps on, where its leaf is
  int main_early_steps; //     almost always partitioned already by the look-ahead
};

// Host-side launch helpers (kernels.cu).
void launch_tree(const GrowDev& d, int build_blocks, size_t build_smem, cudaStream_t st,
                 LaunchProfiler* prof = nullptr, const DeviceComm* comm = nullptr,
                 const LookAheadStreams* las = nullptr);
bool fused_partition_supported(int gh_mode, int num_features, int shift, int nch, bool pack4);
int build_smem_bytes_per_bin(int gh_mode);

// Objective / score kernels (objective.cu).
struct ObjDev {
  int64_t N;         // rows on this device
  int64_t n_global;  // rows on all devices
  int32_t objective;  // 0 binary, 1 l2
  int32_t gh_mode;
  double sigmoid;
  const float* label;
  double* score;
  void* gh;  // float2 (FLOAT) or uint16 (quantized)
  DevGhParams* ghp;
  int32_t num_quant_bins;
  const int32_t* stopped;
  // lambdarank (objective 2): per-query tables built once on the host
  const int32_t* qb;          // [num_queries + 1] query boundaries
  int32_t num_queries;
  int32_t trunc;              // lambdarank_truncation_level
  int32_t norm;               // lambdarank_norm
  int32_t _pad;
  const double* sig_table;    // [kRankSigmoidBins] 1 / (1 + exp(sigmoid * x))
  double sig_min, sig_max, sig_factor;
  const double* discount;     // [LGBM_B200_MAX_QUERY_ROWS] 1 / log2(2 + rank)
  const double* label_gain;   // gain of each integer label
  const double* inv_max_dcg;  // [num_queries] 1 / max DCG at the truncation level
  int32_t* order;             // [N] each query's rows by descending score
  // Stochastic rounding of the quantized gradients (stochastic_rounding=true): the
  // reference's xorshift64 stream over the rows of the whole job in row order, seeded per
  // iteration from *iter_counter. xs_pow[64 j + k] is column k of T^(2^j), T the 64x64
  // bit matrix of one xorshift step, for jumping to a row's place in the stream.
  int32_t stochastic;
  int32_t _sr_pad;
  const int32_t* iter_counter;
  int64_t row_offset;  // global index of this device's first row
  const unsigned long long* xs_pow;
};
void xorshift_pow_table(unsigned long long* out /* [64 * 64] */);
constexpr int64_t kRankSigmoidBins = 1 << 20;  // LambdarankNDCG::_sigmoid_bins
void launch_gradients(const ObjDev& o, cudaStream_t st, LaunchProfiler* prof = nullptr,
                      const DeviceComm* comm = nullptr);
void launch_fill_f64(double* p, int64_t n, double v, cudaStream_t st);

// Per-iteration tree finish: shrinkage + score update + tree record.
struct FinishDev {
  const GrowDev* gd_host;  // unused on device
  int32_t* stopped;
  int32_t* iter_counter;
  int32_t max_iters;
  double learning_rate;
  double* score;
  // tree record storage [max_iters][L] per array, + num_leaves per iter
  int32_t* rec_num_leaves;
  int32_t* rec_left;
  int32_t* rec_right;
  int32_t* rec_split_feature;
  uint32_t* rec_threshold;
  float* rec_split_gain;
  int8_t* rec_decision;
  double* rec_leaf_value;
  double* rec_leaf_weight;
  int32_t* rec_leaf_count;
  double* rec_internal_value;
  int32_t* rec_internal_count;
  uint32_t* rec_cat;  // [max_iters][L][kCatWords]
};
void launch_finish_iteration(const GrowDev& d, const FinishDev& f, cudaStream_t st,
                             LaunchProfiler* prof = nullptr);

// Row-major bin matrix from feature-major columns (bin_rows.cu).
struct DevBinFeature {
  int32_t num_bin;
  int32_t missing_type;
  int32_t bin_type;  // 0 numerical, 1 categorical
  int32_t n_cat;     // categorical: categories in cat_keys
  int64_t off;       // first bound in `upper` (numerical) or key in `cat_keys` (categorical)
};
// Bin of feature f in one row of the bin matrix: one byte per bin, or (packed4, every
// feature with at most 16 bins) two 4-bit bins per byte, feature 2k in the low nibble of
// byte k and 2k + 1 in the high nibble.
__device__ __forceinline__ uint32_t row_bin(const uint8_t* row, int f, bool packed4) {
  return packed4 ? ((uint32_t)row[f >> 1] >> ((f & 1) << 2)) & 15u : (uint32_t)row[f];
}

struct BinRowsDev {
  const DevBinFeature* feats;
  int32_t num_features;
  int32_t packed4;                  // write two 4-bit bins per byte
  int32_t stride;                   // bytes per row (a multiple of 16)
  const double* upper;              // numerical bin upper bounds, concatenated
  const int32_t* cat_keys;          // categorical: ascending categories, concatenated
  const uint8_t* cat_bins;          // their bins
  unsigned long long* first_bad;    // pre-binned input: smallest row * F + feature out of range
};
enum BinRowsKind { kBinRowsU8 = 1, kBinRowsU16 = 2, kBinRowsU32 = 4, kBinRowsF32 = 5,
                   kBinRowsF64 = 8 };

// Bin finding of a batch of numerical features on the device (find_bin.cu): the sampled
// values in, each feature's mapper fields and bin upper bounds out.
struct FindBinsDev {
  double* vals_a;                 // [nf][k] sampled values (sorted in place, or into b)
  double* vals_b;                 // [nf][k]
  unsigned long long* keys_a;     // [nf][k]
  unsigned long long* keys_b;     // [nf][k]
  int32_t* which;                 // [nf]
  int32_t* na_cnt;                // [nf] (zeroed by the caller)
  int64_t k;
  int32_t nf;
  int32_t max_bin;
  int32_t min_data_in_bin;
  int32_t filter_cnt;
  int32_t pre_filter;
  int32_t use_missing;
  int32_t zero_as_missing;
  int32_t cap;                    // >= max_bin + 2
  double* dv;                     // [nf][k + 2]
  int32_t* cnt;                   // [nf][k + 2]
  uint8_t* big;                   // [nf][k + 2]
  double* edges;                  // [nf][2][max_bin]
  double* side;                   // [nf][max_bin + 1]
  int32_t* cnt_in_bin;            // [nf][cap]
  double* upper;                  // [nf][cap]
  int32_t* meta;                  // [nf][6]
  double* meta_f;                 // [nf][3]
};
void launch_find_bins(const FindBinsDev& d, cudaStream_t st);
void launch_bin_rows(const BinRowsDev& d, int kind, const void* cols, int64_t col_stride,
                     int64_t n, int64_t row0, uint8_t* out, cudaStream_t st);

// Batch prediction (predict.cu). One internal node of a flattened ensemble.
struct PredNode {
  double threshold;  // numerical threshold
  int32_t left;      // tree-local: >= 0 node, < 0 ~leaf
  int32_t right;
  int32_t feature;
  int32_t cat;       // categorical: index into cat_boundaries over all trees
  int32_t dt;        // decision_type
  int32_t _pad;
};
struct PredModelDev {
  int32_t num_trees;
  int32_t num_features;
  int32_t transform;  // 0 identity, 1 sigmoid
  int32_t _pad;
  double sigmoid;
  const int32_t* node_offset;  // [num_trees + 1]
  const int32_t* leaf_offset;  // [num_trees + 1]
  const PredNode* nodes;
  const double* leaf_value;
  const int32_t* cat_boundaries;
  const uint32_t* cat_threshold;
};
void launch_predict(const PredModelDev& m, const double* rows, int64_t n, int32_t raw,
                    double* out, cudaStream_t st);

// Standalone per-op launches (the Backend-trait entry points).
void launch_construct_histogram_f32(const uint8_t* bins_rm, int32_t stride, int64_t n,
                                    const float2* gh, int32_t num_bin, double scale_g,
                                    double scale_h, long long* raw, cudaStream_t st);
void launch_scan_features(const double* hist, const DevFeature* feats, int32_t n_feats,
                          DevGainConfig cfg, DevLeafSplits ls, DevSplitInfo* out,
                          cudaStream_t st);
void launch_partition_rows(const uint8_t* bins_rm, int32_t stride, int32_t feature,
                           const DevFeature* feat, uint32_t threshold, int32_t default_left,
                           int64_t count, uint32_t* dst, unsigned long long* status,
                           int32_t* left_total, uint32_t* ticket, uint32_t* error,
                           cudaStream_t st);
void launch_subtract(const double* parent, const double* child, double* out, int64_t len,
                     cudaStream_t st);

}  // namespace lgbm_b200
