// Shared device-side definitions for the B200 histogram tree learner.
//
// Numerics: the library is compiled with --fmad=false so that every f64
// expression rounds exactly as the reference's Rust code does (Rust never
// contracts a*b+c). The only fused multiply-add is the explicit one of the
// given-output gain (lgbm-compute/src/gain.rs:201-218), written as fma().
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "lgbm_b200.h"

namespace lgbm_b200 {

constexpr int kMaxBins = 256;  // u8 bin matrix
constexpr double kNegInf = -__builtin_huge_val();

// lgbm-core/src/types.rs:31 kEpsilon = 1e-15f widened to double.
__host__ __device__ inline double k_eps() { return (double)1e-15f; }

// Per-feature metadata resident on the device.
struct DevFeature {
  int32_t num_bin;
  int32_t offset;        // 1 iff most_freq_bin == 0 (lgbm-treelearner/src/lib.rs:89-95)
  int32_t default_bin;
  int32_t most_freq_bin;
  int32_t missing_type;  // 0 None, 1 Zero, 2 NaN
  int32_t slot_off;      // first cell of this feature in a histogram slot (cells = 2*num_bin)
  int32_t bin_off;       // first bin of this feature in the raw accumulator (bins)
  int32_t flags;         // bit0 skip_default_bin, bit1 na_as_missing, bit2 run_forward,
                         // bit3 categorical
  int32_t route_min;     // partition min_bin (learner.rs:3957: min_bin + offset)
  int32_t route_max;     // partition max_bin (num_bin - 1)
};

struct DevGainConfig {
  int32_t min_data_in_leaf;
  int32_t use_l1;
  int32_t use_smoothing;
  int32_t use_full;
  double min_sum_hessian_in_leaf;
  double max_delta_step;
  double lambda_l1;
  double lambda_l2;
  double min_gain_to_split;
  double path_smooth;
  int32_t min_data_per_group;
  int32_t max_cat_threshold;
  int32_t max_cat_to_onehot;
  int32_t _pad;
  double cat_l2;
  double cat_smooth;
};

constexpr int32_t kFeatCategorical = 8;  // DevFeature::flags bit of categorical features
constexpr int kCatWords = 8;             // bins sent left by a categorical split (<= 256)

// lgbm_compute::gain::SplitInfo (gain.rs:1040-1065) in a flat layout.
struct DevSplitInfo {
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
};

// LeafSplits (lgbm-treelearner/src/leaf_splits.rs:43-60).
struct DevLeafSplits {
  int32_t num_data;
  int32_t _pad;
  double sum_g;
  double sum_h;
  double weight;
};

// How per-row gradient pairs enter the histogram accumulator.
enum GhMode : int32_t {
  GH_FLOAT = 0,  // f32 g/h, int64 fixed point with per-iteration power-of-two scales
  GH_QLUT = 1,   // int8 quantized pairs, int64 per-level LUT (exact)
  GH_QPACK = 2,  // int8 quantized pairs with num_grad_quant_bins <= 4, one packed int64
};

// Per-iteration gradient encoding parameters (written on device by the objective
// kernels, read by the histogram build and its finalizer).
struct DevGhParams {
  int32_t mode;
  int32_t is_const_hess;
  int32_t num_quant_bins;
  int32_t _pad;
  double scale_g;      // FLOAT: 2^kg ; QLUT/QPACK: unused
  double scale_h;
  double unit_g;       // decode multiplier for the g accumulator (FLOAT: 2^-kg; QLUT: ulp unit; QPACK: v1g)
  double unit_h;       // FLOAT: 2^-kh ; QLUT: ulp unit ; QPACK: v1h
  double v3h;          // QPACK: dequantized hessian of level 3
  double grad_scale;   // GradientDiscretizer grad_scale / hess_scale (gradient_discretizer.rs:145-165)
  double hess_scale;
  double inv_grad_scale;
  double inv_hess_scale;
  uint32_t max_abs_g_bits;  // running max |g| (f32 bits, non-negative floats order as ints)
  uint32_t max_abs_h_bits;
  uint32_t min_h_key_inv;   // ordered-int keys for the constant-hessian check: the minimum
  uint32_t max_h_key;       // is kept complemented, so all four reduce with one max
  long long root_g;         // root sums in accumulator units
  long long root_h;
  long long lut_g[256];     // QLUT: per-level accumulator value, index q + 128
  long long lut_h[256];
};

// Device control block of one tree grower.
struct GrowCtrl {
  int32_t done;
  int32_t num_leaves;      // leaves in the tree so far
  int32_t left_leaf;
  int32_t right_leaf;
  int32_t smaller_leaf;
  int32_t larger_leaf;
  int32_t do_find;
  int32_t use_subtract;
  int32_t smaller_slot;
  int32_t larger_slot;
  int32_t next_slot;
  int32_t pending;         // a split decided but not yet applied
  int32_t split_leaf;
  int32_t split_feature;
  int32_t part_left_total;
  uint32_t part_ticket;
  uint32_t scan_counter;
  uint32_t epoch;
  uint32_t error;
  int32_t num_splits;
  int32_t num_builds;      // histogram builds in this tree
  int32_t build_left;      // the pending split's left rows are accumulated (else right)
  long long rows_built;    // rows streamed by those builds
  long long rows_parted;   // parent rows streamed by the partitions
  int32_t num_cat;         // categorical nodes in the tree so far
  int32_t pend_la;         // 0: the pending split's rows were partitioned by the main
                           // partition; 1 + k: by the look-ahead partition of slot k
  long long la_rows;       // parent rows streamed by look-ahead partitions (used or not)
  unsigned long long la_base;  // look-ahead signals published before this tree
  int32_t la_runs;         // look-ahead partitions run in this tree
  int32_t la_hits;         // ... whose leaf was the next split
  DevSplitInfo split;
  long long rows_parted_ctl;  // parent rows of main partitions run inside control steps
  long long rows_built_ctl;   // ... and the rows their fused child builds accumulated
};

// Error bits reported through GrowCtrl::error.
constexpr uint32_t kErrSpinTimeout = 1u;
constexpr uint32_t kErrNoParentHistogram = 2u;
constexpr uint32_t kErrRootHessian = 4u;

// ---------------- gain primitives: lgbm-compute/src/gain.rs ----------------

__device__ __forceinline__ double d_threshold_l1(double s, double l1) {  // gain.rs:108-117
  double reg = fmax(0.0, fabs(s) - l1);
  double pos = s > 0.0 ? 1.0 : 0.0;
  double neg = s < 0.0 ? 1.0 : 0.0;
  return (pos - neg) * reg;
}

__device__ __forceinline__ double d_leaf_gain(bool use_l1, double g, double h, double l1,
                                              double l2) {  // gain.rs:133-140
  if (use_l1) {
    double t = d_threshold_l1(g, l1);
    return (t * t) / (h + l2);
  }
  return (g * g) / (h + l2);
}

__device__ __forceinline__ double d_leaf_output(bool use_l1, double g, double h, double l1,
                                                double l2) {  // gain.rs:233-244
  if (use_l1) return -d_threshold_l1(g, l1) / (h + l2);
  return -g / (h + l2);
}

__device__ __forceinline__ double d_leaf_output_full(const DevGainConfig& c, bool use_smoothing,
                                                     double g, double h, int32_t num_data,
                                                     double parent_output) {  // gain.rs:494-539
  double base = d_leaf_output(c.use_l1, g, h, c.lambda_l1, c.lambda_l2);
  const double mds = c.max_delta_step;
  bool clamp = mds > 0.0 && fabs(base) > mds;
  double pos = base > 0.0 ? 1.0 : 0.0;
  double neg = base < 0.0 ? 1.0 : 0.0;
  double clamped = clamp ? (pos - neg) * mds : base;
  if (use_smoothing) {
    double n = (double)num_data / c.path_smooth;
    return clamped * n / (n + 1.0) + parent_output / (n + 1.0);
  }
  return clamped;
}

__device__ __forceinline__ double d_leaf_gain_full(const DevGainConfig& c, double g, double h,
                                                   int32_t num_data, double parent_output) {
  // gain.rs:557-596; given-output form gain.rs:201-218 (first multiply fused)
  if (c.use_full) {
    double o = d_leaf_output_full(c, c.use_smoothing, g, h, num_data, parent_output);
    double sg = c.use_l1 ? d_threshold_l1(g, c.lambda_l1) : g;
    return -fma(2.0 * sg, o, (h + c.lambda_l2) * o * o);
  }
  return d_leaf_gain(c.use_l1, g, h, c.lambda_l1, c.lambda_l2);
}

__device__ __forceinline__ double d_split_gain(const DevGainConfig& c, double slg, double slh,
                                               double srg, double srh, int32_t lc, int32_t rc,
                                               double po) {
  if (c.use_full)
    return d_leaf_gain_full(c, slg, slh, lc, po) + d_leaf_gain_full(c, srg, srh, rc, po);
  return d_leaf_gain(c.use_l1, slg, slh, c.lambda_l1, c.lambda_l2) +
         d_leaf_gain(c.use_l1, srg, srh, c.lambda_l1, c.lambda_l2);
}

// Common::RoundInt (kernels/split.rs:9056-9058)
__device__ __forceinline__ int32_t d_round_int(double x) { return (int32_t)(x + (double)0.5f); }

// split_info.rs:28-36 split_gt, as a total order key (gain desc, feature asc, -1 last).
__device__ __forceinline__ bool d_split_gt(double ga, int32_t fa, double gb, int32_t fb) {
  if (ga != gb) return ga > gb;
  int32_t x = fa == -1 ? 0x7fffffff : fa;
  int32_t y = fb == -1 ? 0x7fffffff : fb;
  return x < y;
}

__device__ __forceinline__ DevSplitInfo d_split_none() {
  DevSplitInfo s;
  s.threshold = 0;
  s.default_left = 1;
  s.left_count = 0;
  s.right_count = 0;
  s.gain = kNegInf;
  s.left_sum_gradient = 0.0;
  s.left_sum_hessian = 0.0;
  s.right_sum_gradient = 0.0;
  s.right_sum_hessian = 0.0;
  s.left_output = 0.0;
  s.right_output = 0.0;
  return s;
}

// Row-to-child routing of DataPartition::split (lgbm-treelearner/src/data_partition.rs:360-432).
// Row routing of a categorical split: the chosen bins go left
// (DataPartition::split_categorical, data_partition.rs:636-688).
__device__ __forceinline__ bool d_cat_go_right(const uint32_t* cat, int32_t bin) {
  return !((cat[bin >> 5] >> (bin & 31)) & 1u);
}

// DevFeature::flags bit 5: route with the kernel partition's whole missing-value fan-out
// (d_route_left_missing) instead of the learner's rule (d_go_right).
constexpr int32_t kFeatMissingRoute = 32;

// The kernel-level router of partition_leaf_stable (RouteFlags::derive + route_left_host,
// lgbm-compute/src/kernels/data_partition.rs:325-406): true = left. missing_type 1 sends
// the zero bin (route_min + default_bin - [mfb == 0]) and 2 the NA bin (route_max) the
// default_left way unless the most frequent bin is that bin; then out-of-range bins take
// the missing direction instead of the most frequent bin's. route_min == route_max is
// the degenerate one-bin case.
__device__ __forceinline__ bool d_route_left_missing(const DevFeature& f, uint32_t threshold,
                                                    bool default_left, int32_t bin) {
  const int32_t lo = f.route_min, hi = f.route_max, mfb = f.most_freq_bin;
  const bool zm = f.missing_type == 1, nm = f.missing_type == 2;
  const bool mfb_zero = zm && f.default_bin == mfb;
  const bool mfb_na = nm && hi == mfb + lo && mfb > 0;
  const int32_t shift = mfb == 0 ? 1 : 0;
  const int32_t th = (int32_t)threshold + lo - shift;
  const bool miss_left = (zm || nm) && default_left;
  const bool mfb_left = mfb <= (int32_t)threshold;
  const bool oor_missing = (nm && mfb_na) || (zm && mfb_zero);
  const bool oor_left = oor_missing ? miss_left : mfb_left;
  if (zm && !mfb_zero && bin == lo + f.default_bin - shift) return miss_left;
  if (lo == hi) {
    if (bin != hi) return oor_left;
    return (nm && !mfb_na) ? miss_left : hi <= th;
  }
  if (nm && !mfb_na && bin == hi) return miss_left;
  if (bin < lo || bin > hi) return oor_left;
  return bin <= th;
}

__device__ __forceinline__ bool d_go_right(const DevFeature& f, uint32_t threshold,
                                           bool default_left, int32_t bin) {
  int32_t th = (int32_t)threshold + f.route_min;
  if (f.most_freq_bin == 0) th -= 1;
  const bool default_to_right = f.most_freq_bin > (int32_t)threshold;
  if ((f.flags & 2) && bin == f.num_bin - 1) return !default_left;
  if (bin < f.route_min || bin > f.route_max) return default_to_right;
  return bin > th;
}

}  // namespace lgbm_b200
