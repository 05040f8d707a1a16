// CPU restatement of the lightgbm_rs histogram tree-learner path.
//
// TEST INFRASTRUCTURE ONLY. This file is the parity checker for the B200
// library in lightgbm_rs_b200/: only tests/, __graft_entry__.smoke() and
// bench.py's cpu_baseline leg may load it, and only to check or time the
// reference algorithm. The product never links, loads or calls it.
//
// Every function restates the reference's CPU behaviour (the Rust crates of
// BectorVoom/lightgbm_rs, themselves a bit-exact transcription of LightGBM
// C++ 4.6.0.99 @195c26fc). Citations are path:line inside the reference
// project. Parity of this restatement is pinned against the reference's own
// golden vectors (crates/oracle-harness/tests/fixtures/...) by tests/.
//
// Numerics: compile with -ffp-contract=off. Rust never contracts a*b+c into
// an FMA; the only fused multiply-add on the path is the explicit
// `fused_mul_add` of the given-output gain (lgbm-compute/src/gain.rs:62-64),
// restated below with std::fma.

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// lgbm-core/src/types.rs:31 — `const score_t kEpsilon = 1e-15f;`
const double kEps = (double)1e-15f;
// lgbm-core/src/types.rs:35 — kZeroThreshold (the Rust reference stores the
// f64 literal 1e-35).
const double kZeroThreshold = 1e-35;
const double kMinScore = -std::numeric_limits<double>::infinity();

struct GainCfg {
  int32_t min_data_in_leaf;
  double min_sum_hessian_in_leaf;
  double max_delta_step;
  double lambda_l1;
  double lambda_l2;
  double min_gain_to_split;
  double path_smooth;
  double parent_output;
  int32_t min_data_per_group = 100;
  int32_t max_cat_threshold = 32;
  int32_t max_cat_to_onehot = 4;
  double cat_l2 = 10.0;
  double cat_smooth = 10.0;
  bool use_l1() const { return lambda_l1 > 0.0; }          // gain.rs:1000-1003
  bool use_smoothing() const { return path_smooth > kEps; } // gain.rs:1018-1020
};

}  // namespace

extern "C" {

// Flat C layout of lgbm_compute::gain::SplitInfo (gain.rs:1040-1065).
typedef struct {
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
} OSplitInfo;

typedef struct {
  int32_t min_data_in_leaf;
  int32_t _pad;
  double min_sum_hessian_in_leaf;
  double max_delta_step;
  double lambda_l1;
  double lambda_l2;
  double min_gain_to_split;
  double path_smooth;
  double parent_output;
  // categorical split parameters (gain.rs GainConfig; config defaults 100, 32, 4, 10, 10)
  int32_t min_data_per_group;
  int32_t max_cat_threshold;
  int32_t max_cat_to_onehot;
  int32_t _pad2;
  double cat_l2;
  double cat_smooth;
} OGainConfig;

// Per-feature metadata the learner reads (lgbm-treelearner/src/learner.rs:87-140).
typedef struct {
  int32_t num_bin;
  int32_t offset;          // 1 iff most_freq_bin == 0 (lgbm-treelearner/src/lib.rs:89-95)
  int32_t default_bin;
  int32_t most_freq_bin;
  int32_t missing_type;    // 0 None, 1 Zero, 2 NaN
  int32_t is_categorical;  // BinType::Categorical (learner.rs:130-140)
} OFeatureMeta;

typedef struct {
  int32_t num_leaves;
  int32_t max_depth;
  OGainConfig gain;
} OLearnerConfig;

// Tree node arrays (lgbm-model/src/tree.rs:94-160). Arrays are caller-owned and
// sized for cfg.num_leaves leaves (num_leaves - 1 internal nodes).
typedef struct {
  int32_t num_leaves;
  int32_t _pad;
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
  int32_t* leaf_depth;
  int32_t* leaf_parent;
  // categorical nodes: the bins sent left, a 256-bit set per internal node (may be NULL)
  uint32_t* cat_bins;
} OTree;

}  // extern "C"

namespace {

// ---------------- gain primitives: lgbm-compute/src/gain.rs ----------------

// gain.rs:108-117 threshold_l1
inline double threshold_l1(double s, double l1) {
  double reg = std::max(0.0, std::fabs(s) - l1);
  double pos = s > 0.0 ? 1.0 : 0.0;
  double neg = s < 0.0 ? 1.0 : 0.0;
  return (pos - neg) * reg;
}

// gain.rs:133-140 get_leaf_gain (closed form)
inline double leaf_gain(bool use_l1, double g, double h, double l1, double l2) {
  if (use_l1) {
    double t = threshold_l1(g, l1);
    return (t * t) / (h + l2);
  }
  return (g * g) / (h + l2);
}

// gain.rs:233-244 calculate_splitted_leaf_output
inline double leaf_output(bool use_l1, double g, double h, double l1, double l2) {
  if (use_l1) return -threshold_l1(g, l1) / (h + l2);
  return -g / (h + l2);
}

// gain.rs:201-218 get_leaf_gain_given_output (first multiply fused)
inline double leaf_gain_given_output(bool use_l1, double g, double h, double l1, double l2,
                                     double o) {
  double sg = use_l1 ? threshold_l1(g, l1) : g;
  return -std::fma(2.0 * sg, o, (h + l2) * o * o);
}

// gain.rs:494-539 calculate_splitted_leaf_output_full
inline double leaf_output_full(bool use_l1, double g, double h, double l1, double l2,
                               double mds, bool use_smoothing, double path_smooth,
                               int32_t num_data, double parent_output) {
  double base = leaf_output(use_l1, g, h, l1, l2);
  bool clamp = mds > 0.0 && std::fabs(base) > mds;
  double pos = base > 0.0 ? 1.0 : 0.0;
  double neg = base < 0.0 ? 1.0 : 0.0;
  double clamped = clamp ? (pos - neg) * mds : base;
  if (use_smoothing) {
    double n = (double)num_data / path_smooth;
    return clamped * n / (n + 1.0) + parent_output / (n + 1.0);
  }
  return clamped;
}

// gain.rs:557-596 get_leaf_gain_full
inline double leaf_gain_full(bool use_l1, double g, double h, double l1, double l2, double mds,
                             bool use_smoothing, double path_smooth, int32_t num_data,
                             double parent_output) {
  if (mds > 0.0 || use_smoothing) {
    double o = leaf_output_full(use_l1, g, h, l1, l2, mds, use_smoothing, path_smooth, num_data,
                                parent_output);
    return leaf_gain_given_output(use_l1, g, h, l1, l2, o);
  }
  return leaf_gain(use_l1, g, h, l1, l2);
}

GainCfg to_cfg(const OGainConfig& c) {
  GainCfg g;
  g.min_data_in_leaf = c.min_data_in_leaf;
  g.min_sum_hessian_in_leaf = c.min_sum_hessian_in_leaf;
  g.max_delta_step = c.max_delta_step;
  g.lambda_l1 = c.lambda_l1;
  g.lambda_l2 = c.lambda_l2;
  g.min_gain_to_split = c.min_gain_to_split;
  g.path_smooth = c.path_smooth;
  g.parent_output = c.parent_output;
  g.min_data_per_group = c.min_data_per_group;
  g.max_cat_threshold = c.max_cat_threshold;
  g.max_cat_to_onehot = c.max_cat_to_onehot;
  g.cat_l2 = c.cat_l2;
  g.cat_smooth = c.cat_smooth;
  return g;
}

OSplitInfo split_none() {
  OSplitInfo s;
  std::memset(&s, 0, sizeof(s));
  s.gain = kMinScore;
  s.default_left = 1;  // gain.rs:1079-1093 SplitInfo::none
  return s;
}

// Common::RoundInt: (int)(x + 0.5f) (kernels/split.rs:9056-9058)
inline int32_t round_int(double x) { return (int32_t)(x + (double)0.5f); }

// ------------- find_best_split_cpu_native: kernels/split.rs:8970-9329 -------------
OSplitInfo find_best_split(const double* hist, const GainCfg& cfg, int32_t num_bin, int32_t offset,
                           int32_t default_bin, bool skip_default_bin, bool na_as_missing,
                           bool run_forward, double sum_gradient, double sum_hessian,
                           int32_t num_data) {
  const double sum_hessian_bumped = sum_hessian + 2.0 * kEps;  // :9020-9021
  const bool use_l1 = cfg.use_l1();
  const bool use_smoothing = cfg.use_smoothing();
  const double mds = cfg.max_delta_step;
  const double po = cfg.parent_output;
  const bool use_full = use_smoothing || mds > 0.0;  // :9037
  const double l1 = cfg.lambda_l1, l2 = cfg.lambda_l2, ps = cfg.path_smooth;
  const double gain_shift =
      leaf_gain_full(use_l1, sum_gradient, sum_hessian_bumped, l1, l2, mds, use_smoothing, ps,
                     num_data, po);  // :9043-9054
  const double min_gain_shift = gain_shift + cfg.min_gain_to_split;

  const int32_t rev_count = std::max(num_bin - 1 - (na_as_missing ? 1 : 0), 0);
  const bool na_preamble = na_as_missing && offset == 1;
  int32_t fwd_count = 0;
  if (run_forward) {
    int32_t base = std::max(num_bin - 1 - offset, 0);
    fwd_count = na_preamble ? base + 1 : base;
  }
  const double cnt_factor = (double)num_data / sum_hessian_bumped;
  const double min_hess = cfg.min_sum_hessian_in_leaf;
  const int32_t min_data = cfg.min_data_in_leaf;

  auto split_gain = [&](double slg, double slh, double srg, double srh, int32_t lc,
                        int32_t rc) -> double {
    if (use_full)
      return leaf_gain_full(use_l1, slg, slh, l1, l2, mds, use_smoothing, ps, lc, po) +
             leaf_gain_full(use_l1, srg, srh, l1, l2, mds, use_smoothing, ps, rc, po);
    return leaf_gain(use_l1, slg, slh, l1, l2) + leaf_gain(use_l1, srg, srh, l1, l2);
  };

  double best_slg = 0.0, best_slh = 0.0, best_gain = kMinScore;
  int32_t best_lc = 0, best_thr = 0;
  bool splittable = false, best_default_left = true;

  // REVERSE (:9078-9165)
  {
    double srg = 0.0, srh = kEps;
    int32_t rc = 0;
    const int32_t t_start = num_bin - 1 - offset - (na_as_missing ? 1 : 0);
    bool done = false;
    for (int32_t k = 0; k < rev_count; ++k) {
      if (done) break;
      const int32_t t = t_start - k;
      const bool in_range = t >= (1 - offset);
      const bool skip = skip_default_bin && (t + offset) == default_bin;
      const bool active = in_range && !skip;
      if (active) {
        double hg = hist[2 * t], hh = hist[2 * t + 1];
        srg += hg;
        srh += hh;
        rc += round_int(hh * cnt_factor);
      }
      const int32_t lc = num_data - rc;
      const double slh = sum_hessian_bumped - srh;
      const double slg = sum_gradient - srg;
      const bool cont = rc < min_data || srh < min_hess;
      const bool brk = lc < min_data || slh < min_hess;
      done = done || (active && !cont && brk);
      if (active && !cont && !done) {
        double g = split_gain(slg, slh, srg, srh, lc, rc);
        if (g > min_gain_shift) {
          splittable = true;
          if (g > best_gain) {
            best_lc = lc;
            best_slg = slg;
            best_slh = slh;
            best_thr = t - 1 + offset;
            best_gain = g;
            best_default_left = true;
          }
        }
      }
    }
  }
  // FORWARD (:9167-9265)
  {
    double slg = 0.0, slh = kEps;
    int32_t lc = 0;
    int32_t fwd_start = 0;
    if (na_preamble) {
      slg = sum_gradient;
      slh = sum_hessian_bumped - kEps;
      lc = num_data;
      for (int32_t i = 0; i < num_bin - offset; ++i) {
        slg -= hist[2 * i];
        slh -= hist[2 * i + 1];
        lc -= round_int(hist[2 * i + 1] * cnt_factor);
      }
      fwd_start = -1;
    }
    bool done = false;
    for (int32_t k = 0; k < fwd_count; ++k) {
      if (done) break;
      const int32_t t = fwd_start + k;
      const bool skip = skip_default_bin && (t + offset) == default_bin;
      const bool active = !skip;
      if (active && t >= 0) {
        double hg = hist[2 * t], hh = hist[2 * t + 1];
        slg += hg;
        slh += hh;
        lc += round_int(hh * cnt_factor);
      }
      const int32_t rc = num_data - lc;
      const double srh = sum_hessian_bumped - slh;
      const double srg = sum_gradient - slg;
      const bool cont = lc < min_data || slh < min_hess;
      const bool brk = rc < min_data || srh < min_hess;
      done = done || (active && !cont && brk);
      if (active && !cont && !done) {
        double g = split_gain(slg, slh, srg, srh, lc, rc);
        if (g > min_gain_shift) {
          splittable = true;
          if (g > best_gain) {
            best_lc = lc;
            best_slg = slg;
            best_slh = slh;
            best_thr = t + offset;
            best_gain = g;
            best_default_left = false;
          }
        }
      }
    }
  }
  // finalization (:9267-9326)
  const int32_t best_rc = num_data - best_lc;
  const double lo = leaf_output_full(use_l1, best_slg, best_slh, l1, l2, mds, use_smoothing, ps,
                                     best_lc, po);
  const double rsg = sum_gradient - best_slg;
  const double rsh = sum_hessian_bumped - best_slh;
  const double ro =
      leaf_output_full(use_l1, rsg, rsh, l1, l2, mds, use_smoothing, ps, best_rc, po);
  if (splittable && best_gain > kMinScore) {
    OSplitInfo s;
    s.threshold = (uint32_t)best_thr;
    s.gain = best_gain - min_gain_shift;
    s.left_count = best_lc;
    s.right_count = num_data - best_lc;
    s.left_sum_gradient = best_slg;
    s.left_sum_hessian = best_slh - kEps;
    s.right_sum_gradient = rsg;
    s.right_sum_hessian = rsh - kEps;
    s.left_output = lo;
    s.right_output = ro;
    s.default_left = best_default_left ? 1 : 0;
    return s;
  }
  return split_none();
}

// ---------------- FixHistogram: lgbm-treelearner/src/fix_histogram.rs:50-81 ----------------
void fix_histogram(double* hist, int32_t num_bin, int32_t mfb, double sum_g, double sum_h) {
  if (mfb == 0 || mfb >= num_bin) return;
  double g = sum_g, h = sum_h;
  for (int32_t i = 0; i < num_bin; ++i) {
    if (i != mfb) {
      g -= hist[2 * i];
      h -= hist[2 * i + 1];
    }
  }
  hist[2 * mfb] = g;
  hist[2 * mfb + 1] = h;
}

// ---------------- compact_histogram: learner.rs:4460-4486 ----------------
void compact_histogram(double* hist, int32_t num_bin, int32_t offset) {
  if (offset <= 0) return;
  if (offset >= num_bin) {
    std::fill(hist, hist + 2 * num_bin, 0.0);
    return;
  }
  for (int32_t c = 0; c < num_bin - offset; ++c) {
    hist[2 * c] = hist[2 * (c + offset)];
    hist[2 * c + 1] = hist[2 * (c + offset) + 1];
  }
  std::fill(hist + 2 * (num_bin - offset), hist + 2 * num_bin, 0.0);
}

// split_info.rs:28-36 split_gt
inline bool split_gt(const OSplitInfo& a, int32_t af, const OSplitInfo& b, int32_t bf) {
  if (a.gain != b.gain) return a.gain > b.gain;
  int32_t x = af == -1 ? INT32_MAX : af;
  int32_t y = bf == -1 ? INT32_MAX : bf;
  return x < y;
}

// Bin-column accessor: columns are feature-major, `bytes` wide.
// ------- categorical split finder: feature_histogram_categorical.rs:96-490 -------
// (LightGBM FeatureHistogram::FindBestThresholdCategoricalInner). `sum_hessian` is the
// leaf sum already bumped by 2 kEpsilon, as at the numeric call site. `bins_out` gets
// the set of (uncompacted) bins sent left; the split's threshold is 0 and default_left
// false.
OSplitInfo find_best_categorical(const double* hist, const GainCfg& cfg, int32_t num_bin,
                                 int32_t offset, double sum_gradient, double sum_hessian,
                                 int32_t num_data, uint32_t bins_out[8]) {
  for (int i = 0; i < 8; ++i) bins_out[i] = 0;
  const bool use_l1 = cfg.use_l1();
  const double l1 = cfg.lambda_l1, mds = cfg.max_delta_step, ps = cfg.path_smooth;
  const bool smoothing = cfg.use_smoothing();
  const double parent = cfg.parent_output;
  // gain_shift with the original l2 (the deliberate asymmetry, :140-160)
  const double gain_shift =
      smoothing ? leaf_gain_given_output(use_l1, sum_gradient, sum_hessian, l1, cfg.lambda_l2,
                                         parent)
                : leaf_gain_full(use_l1, sum_gradient, sum_hessian, l1, cfg.lambda_l2, mds, false,
                                 0.0, num_data, 0.0);
  const double min_gain_shift = gain_shift + cfg.min_gain_to_split;
  const int32_t bin_start = 1 - offset, bin_end = num_bin - offset;
  const double cnt_factor = (double)num_data / sum_hessian;
  auto gains = [&](double lg, double lh, double rg, double rh, int32_t lc, int32_t rc,
                   double l2) {
    return leaf_gain_full(use_l1, lg, lh, l1, l2, mds, smoothing, ps, lc, parent) +
           leaf_gain_full(use_l1, rg, rh, l1, l2, mds, smoothing, ps, rc, parent);
  };
  bool splittable = false;
  double best_gain = kMinScore, best_slg = 0.0, best_slh = 0.0;
  int32_t best_lc = 0, best_thr = -1, best_dir = 1;
  const bool onehot = num_bin <= cfg.max_cat_to_onehot;
  double l2 = cfg.lambda_l2;
  std::vector<int32_t> order;
  int32_t used = 0;
  if (onehot) {
    for (int32_t t = bin_start; t < bin_end; ++t) {
      const double gr = hist[2 * t], he = hist[2 * t + 1];
      const int32_t cnt = round_int(he * cnt_factor);
      if (cnt < cfg.min_data_in_leaf || he < cfg.min_sum_hessian_in_leaf) continue;
      const int32_t other = num_data - cnt;
      if (other < cfg.min_data_in_leaf) continue;
      const double soh = sum_hessian - he - kEps;
      if (soh < cfg.min_sum_hessian_in_leaf) continue;
      const double sog = sum_gradient - gr;
      const double g = gains(sog, soh, gr, he + kEps, other, cnt, l2);
      if (g <= min_gain_shift) continue;
      splittable = true;
      if (g > best_gain) {
        best_thr = t;
        best_slg = gr;
        best_slh = he + kEps;
        best_lc = cnt;
        best_gain = g;
      }
    }
  } else {
    // many-vs-many: categories with enough rows, in ascending order of the smoothed
    // gradient ratio (a stable sort), scanned from both ends (:300-420)
    for (int32_t t = bin_start; t < bin_end; ++t)
      if ((double)round_int(hist[2 * t + 1] * cnt_factor) >= cfg.cat_smooth) order.push_back(t);
    used = (int32_t)order.size();
    l2 += cfg.cat_l2;
    auto ctr = [&](int32_t t) { return hist[2 * t] / (hist[2 * t + 1] + cfg.cat_smooth); };
    // Stable ascending sort by ctr as the reference's sort_by(partial_cmp, unordered as
    // Equal) runs it on up to 20 elements: an insertion sort that moves a category left
    // while its ctr is strictly below its neighbour's. A NaN ctr (0/0: cat_smooth 0 and a
    // category without rows in the leaf) is below nothing and nothing is below it, so it
    // keeps its place and the categories on either side are sorted apart.
    for (size_t i = 1; i < order.size(); ++i) {
      const int32_t t = order[i];
      const double c = ctr(t);
      size_t j = i;
      for (; j > 0 && c < ctr(order[j - 1]); --j) order[j] = order[j - 1];
      order[j] = t;
    }
    const int32_t max_num_cat = std::min(cfg.max_cat_threshold, (used + 1) / 2);
    for (int dir_i = 0; dir_i < 2; ++dir_i) {
      const int32_t dir = dir_i == 0 ? 1 : -1;
      int32_t pos = dir_i == 0 ? 0 : used - 1;
      int32_t cnt_group = 0, lc = 0;
      double slg = 0.0, slh = kEps;
      for (int32_t i = 0; i < used && i < max_num_cat; ++i) {
        const int32_t t = order[pos];
        pos += dir;
        const double gr = hist[2 * t], he = hist[2 * t + 1];
        const int32_t cnt = round_int(he * cnt_factor);
        slg += gr;
        slh += he;
        lc += cnt;
        cnt_group += cnt;
        if (lc < cfg.min_data_in_leaf || slh < cfg.min_sum_hessian_in_leaf) continue;
        const int32_t rc = num_data - lc;
        if (rc < cfg.min_data_in_leaf || rc < cfg.min_data_per_group) break;
        const double srh = sum_hessian - slh;
        if (srh < cfg.min_sum_hessian_in_leaf) break;
        if (cnt_group < cfg.min_data_per_group) continue;
        cnt_group = 0;
        const double srg = sum_gradient - slg;
        const double g = gains(slg, slh, srg, srh, lc, rc, l2);
        if (g <= min_gain_shift) continue;
        splittable = true;
        if (g > best_gain) {
          best_lc = lc;
          best_slg = slg;
          best_slh = slh;
          best_thr = i;
          best_gain = g;
          best_dir = dir;
        }
      }
    }
  }
  OSplitInfo s = split_none();
  s.default_left = 0;
  if (!splittable) return s;
  const int32_t rc = num_data - best_lc;
  s.threshold = 0;
  s.gain = best_gain - min_gain_shift;
  s.left_count = best_lc;
  s.right_count = rc;
  s.left_output = leaf_output_full(use_l1, best_slg, best_slh, l1, l2, mds, smoothing, ps,
                                   best_lc, parent);
  s.left_sum_gradient = best_slg;
  s.left_sum_hessian = best_slh - kEps;
  s.right_output = leaf_output_full(use_l1, sum_gradient - best_slg, sum_hessian - best_slh, l1,
                                    l2, mds, smoothing, ps, rc, parent);
  s.right_sum_gradient = sum_gradient - best_slg;
  s.right_sum_hessian = sum_hessian - best_slh - kEps;
  auto put = [&](int32_t bin) { bins_out[bin >> 5] |= 1u << (bin & 31); };
  if (onehot) {
    put(best_thr + offset);
  } else {
    for (int32_t i = 0; i <= best_thr; ++i)
      put((best_dir == 1 ? order[i] : order[used - 1 - i]) + offset);
  }
  return s;
}

struct Bins {
  const void* const* cols;
  int bytes;
  inline uint32_t get(int32_t f, int64_t row) const {
    switch (bytes) {
      case 1: return ((const uint8_t*)cols[f])[row];
      case 2: return ((const uint16_t*)cols[f])[row];
      default: return ((const uint32_t*)cols[f])[row];
    }
  }
};

// LeafSplits (lgbm-treelearner/src/leaf_splits.rs:43-178)
struct LeafSplits {
  int32_t num_data = 0;
  double sum_g = 0.0, sum_h = 0.0, weight = 0.0;
};

// leaf_splits.rs:128-145 self_output (root: max_delta_step clamps, no smoothing)
double self_output(double sg, double sh, const GainCfg& c) {
  return leaf_output_full(c.use_l1(), sg, sh, c.lambda_l1, c.lambda_l2, c.max_delta_step, false,
                          c.path_smooth, 0, 0.0);
}

inline bool is_zero(double v) { return v >= -kZeroThreshold && v <= kZeroThreshold; }

// Serial tree learner state for one tree (learner.rs:980-1562).
struct Learner {
  const Bins bins;
  int64_t num_data;
  int32_t F;
  const OFeatureMeta* meta;
  const float* g;
  const float* h;
  GainCfg cfg;
  int32_t num_leaves;
  int32_t max_depth;
  int nthreads;

  std::vector<size_t> slot_off;
  size_t slot_len = 0;
  // DataPartition (data_partition.rs:16-70)
  std::vector<uint32_t> indices, part_left, part_right;
  std::vector<int32_t> leaf_begin, leaf_count;
  // HistogramPool with one slot per leaf (histogram_pool.rs: cache_size == num_leaves
  // never evicts, so Get/Move reduce to a per-leaf slot map).
  std::vector<std::vector<double>> pool;
  std::vector<int32_t> slot_of_leaf;  // -1 = no histogram
  int32_t next_slot = 0;

  std::vector<OSplitInfo> best_split;
  std::vector<int32_t> best_feature;
  std::vector<std::vector<uint8_t>> feature_splittable;
  // bins sent left by each leaf's best split when its feature is categorical
  // (learner.rs:1356-1357 best_cat_threshold, as a bin set)
  std::vector<std::array<uint32_t, 8>> best_cat;
  int32_t num_cat = 0;

  Learner(Bins b, int64_t n, int32_t f, const OFeatureMeta* m, const float* gg, const float* hh,
          const OLearnerConfig& lc, int nt)
      : bins(b), num_data(n), F(f), meta(m), g(gg), h(hh), cfg(to_cfg(lc.gain)),
        num_leaves(lc.num_leaves), max_depth(lc.max_depth), nthreads(nt) {}

  bool skip_default_bin(int32_t f) const {  // learner.rs:167-169
    return meta[f].num_bin > 2 && meta[f].missing_type == 1;
  }
  bool na_as_missing(int32_t f) const {  // learner.rs:173-175
    return meta[f].num_bin > 2 && meta[f].missing_type == 2;
  }
  bool run_forward(int32_t f) const {  // learner.rs:191-193
    return meta[f].num_bin > 2 && meta[f].missing_type != 0;
  }

  // build_leaf_histogram_into (learner.rs:2464-2566) with the ordered per-feature
  // fold of build_histograms_into / fold_one_feature (lgbm-compute/src/lib.rs:223-390).
  void build_leaf(int32_t leaf, const LeafSplits& ls, double* buf, const uint8_t* used) {
    const bool buildable = ls.sum_h > 0.0 && ls.num_data > 0;
    std::fill(buf, buf + slot_len, 0.0);
    if (!buildable) return;
    const uint32_t* rows = indices.data() + leaf_begin[leaf];
    const int32_t cnt = leaf_count[leaf];
    std::vector<float> og(cnt), oh(cnt);
    for (int32_t k = 0; k < cnt; ++k) {
      og[k] = g[rows[k]];
      oh[k] = h[rows[k]];
    }
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads) if (cnt >= 2048 && nthreads > 1)
    for (int32_t f = 0; f < F; ++f) {
      if (used && !used[f]) continue;
      double* hf = buf + slot_off[f];
      for (int32_t k = 0; k < cnt; ++k) {
        uint32_t b = bins.get(f, rows[k]);
        hf[2 * b] += (double)og[k];
        hf[2 * b + 1] += (double)oh[k];
      }
      fix_histogram(hf, meta[f].num_bin, meta[f].most_freq_bin, ls.sum_g, ls.sum_h);
      compact_histogram(hf, meta[f].num_bin, meta[f].offset);
    }
  }

  // scan_leaf_histogram (learner.rs:2708-3354), spine path.
  void scan_leaf(int32_t leaf, const LeafSplits& ls, const double* buf,
                 const std::vector<uint8_t>* parent_splittable) {
    std::vector<uint8_t> this_splittable(F, 0);
    if (!(ls.sum_h > 0.0) || ls.num_data <= 0) {
      best_split[leaf] = split_none();
      best_feature[leaf] = -1;
      // feature_splittable is left untouched on this early return (:2740-2745).
      return;
    }
    GainCfg lc = cfg;
    lc.parent_output = ls.weight;
    std::vector<OSplitInfo> per(F);
    std::vector<std::array<uint32_t, 8>> cat_bits(F);
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads) if (nthreads > 1 && F >= 8)
    for (int32_t f = 0; f < F; ++f) {
      if (parent_splittable && !(*parent_splittable)[f]) continue;
      if (meta[f].is_categorical) {
        // bin_type dispatch (learner.rs:3099-3149): the leaf hessian is bumped here
        per[f] = find_best_categorical(buf + slot_off[f], lc, meta[f].num_bin, meta[f].offset,
                                       ls.sum_g, ls.sum_h + 2.0 * kEps, ls.num_data,
                                       cat_bits[f].data());
        continue;
      }
      per[f] = find_best_split(buf + slot_off[f], lc, meta[f].num_bin, meta[f].offset,
                               meta[f].default_bin, skip_default_bin(f), na_as_missing(f),
                               run_forward(f), ls.sum_g, ls.sum_h, ls.num_data);
    }
    OSplitInfo leaf_best = split_none();
    int32_t leaf_best_feature = -1;
    for (int32_t f = 0; f < F; ++f) {
      if (parent_splittable && !(*parent_splittable)[f]) continue;
      const OSplitInfo& s = per[f];
      this_splittable[f] = s.gain > kMinScore ? 1 : 0;
      if (s.gain > kMinScore && split_gt(s, f, leaf_best, leaf_best_feature)) {
        leaf_best = s;
        leaf_best_feature = f;
      }
    }
    best_split[leaf] = leaf_best;
    best_feature[leaf] = leaf_best_feature;
    if (leaf_best_feature >= 0 && meta[leaf_best_feature].is_categorical)
      best_cat[leaf] = cat_bits[leaf_best_feature];
    feature_splittable[leaf] = this_splittable;
  }

  int32_t get_slot(int32_t leaf, bool* existed) {
    if (slot_of_leaf[leaf] >= 0) {
      *existed = true;
      return slot_of_leaf[leaf];
    }
    *existed = false;
    slot_of_leaf[leaf] = next_slot++;
    return slot_of_leaf[leaf];
  }

  // DataPartition::split -> split_fused_host_impl (data_partition.rs:192-487)
  void partition(int32_t leaf, int32_t right_leaf, int32_t f, uint32_t threshold,
                 bool default_left) {
    const int32_t begin = leaf_begin[leaf], count = leaf_count[leaf];
    const int32_t num_bin = meta[f].num_bin;
    const int32_t min_b = 0 + std::max(meta[f].offset, 0);  // learner.rs:3957
    const int32_t max_b = num_bin - 1;
    const int32_t mfb = meta[f].most_freq_bin;
    int32_t th = (int32_t)threshold + min_b;
    if (mfb == 0) th -= 1;
    const bool default_to_right = mfb > (int32_t)threshold;
    const bool na = na_as_missing(f);
    const int32_t na_bin = num_bin - 1;
    int32_t lc = 0, rc = 0;
    const bool cat = meta[f].is_categorical != 0;
    const std::array<uint32_t, 8> cb = best_cat[leaf];
    for (int32_t i = 0; i < count; ++i) {
      const uint32_t row = indices[begin + i];
      const int32_t b = (int32_t)bins.get(f, row);
      bool gr;
      if (cat)  // DataPartition::split_categorical (data_partition.rs:636-688)
        gr = !((cb[b >> 5] >> (b & 31)) & 1u);
      else if (na && b == na_bin)
        gr = !default_left;
      else if (b < min_b || b > max_b)
        gr = default_to_right;
      else
        gr = b > th;
      if (gr)
        part_right[rc++] = row;
      else
        part_left[lc++] = row;
    }
    std::copy(part_left.begin(), part_left.begin() + lc, indices.begin() + begin);
    std::copy(part_right.begin(), part_right.begin() + rc, indices.begin() + begin + lc);
    leaf_count[leaf] = lc;
    leaf_begin[right_leaf] = begin + lc;
    leaf_count[right_leaf] = rc;
  }

  int grow(OTree* tree, uint32_t* idx_out, int32_t* lb_out, int32_t* lc_out, int32_t* trace) {
    // feature_slot_layout (learner.rs:4438-4447)
    slot_off.resize(F);
    slot_len = 0;
    for (int32_t f = 0; f < F; ++f) {
      slot_off[f] = slot_len;
      slot_len += 2 * (size_t)meta[f].num_bin;
    }
    indices.resize(num_data);
    for (int64_t i = 0; i < num_data; ++i) indices[i] = (uint32_t)i;
    part_left.resize(num_data);
    part_right.resize(num_data);
    leaf_begin.assign(num_leaves, 0);
    leaf_count.assign(num_leaves, 0);
    leaf_count[0] = (int32_t)num_data;
    pool.assign(num_leaves, std::vector<double>(slot_len, 0.0));
    slot_of_leaf.assign(num_leaves, -1);
    next_slot = 0;
    best_split.assign(num_leaves, split_none());
    best_feature.assign(num_leaves, -1);
    feature_splittable.assign(num_leaves, std::vector<uint8_t>(F, 1));
    best_cat.assign(num_leaves, std::array<uint32_t, 8>{});
    num_cat = 0;
    for (int32_t f = 0; f < F; ++f)
      if (meta[f].is_categorical && meta[f].num_bin > 256) return -2;

    // root LeafSplits::init: ordered f64 fold over all rows (leaf_splits.rs:75-92)
    LeafSplits smaller, larger;
    {
      double sg = 0.0, sh = 0.0;
      for (int64_t i = 0; i < num_data; ++i) {
        sg += (double)g[i];
        sh += (double)h[i];
      }
      smaller.num_data = (int32_t)num_data;
      smaller.sum_g = sg;
      smaller.sum_h = sh;
      smaller.weight = self_output(sg, sh, cfg);
    }
    if (!(smaller.sum_h > 0.0)) return -1;  // InvalidLeafHessian (learner.rs:1330-1336)

    // root tree (learner.rs:5398-5424)
    int32_t nl = 1;
    tree->leaf_value[0] = smaller.weight;
    tree->leaf_weight[0] = 0.0;
    tree->leaf_count[0] = (int32_t)num_data;
    tree->leaf_depth[0] = 0;
    tree->leaf_parent[0] = -1;

    int32_t left_leaf = 0, right_leaf = -1;
    int32_t nsplit_trace = 0;
    for (int32_t s = 0; s < num_leaves - 1; ++s) {
      // before_find_best_split (learner.rs:1808-1839)
      bool did = true;
      {
        const int32_t num_left = leaf_count[left_leaf];
        const int32_t min2 = cfg.min_data_in_leaf * 2;
        if (max_depth > 0 && tree->leaf_depth[left_leaf] >= max_depth) {
          best_split[left_leaf].gain = kMinScore;
          if (right_leaf >= 0) best_split[right_leaf].gain = kMinScore;
          did = false;
        } else if (right_leaf >= 0) {
          const int32_t num_right = leaf_count[right_leaf];
          if (num_right < min2 && num_left < min2) {
            best_split[left_leaf].gain = kMinScore;
            best_split[right_leaf].gain = kMinScore;
            did = false;
          }
        } else if (num_left < min2) {
          best_split[left_leaf].gain = kMinScore;
          did = false;
        }
      }
      if (did) {
        // find_best_splits (learner.rs:1851-2453): pool slot dance.
        int32_t smaller_leaf, larger_leaf;
        if (right_leaf < 0) {
          smaller_leaf = left_leaf;
          larger_leaf = -1;
        } else if (leaf_count[left_leaf] < leaf_count[right_leaf]) {
          smaller_leaf = left_leaf;
          larger_leaf = right_leaf;
        } else {
          smaller_leaf = right_leaf;
          larger_leaf = left_leaf;
        }
        int32_t smaller_slot, larger_slot = -1;
        bool use_subtract = false;
        if (right_leaf < 0) {
          bool e;
          smaller_slot = get_slot(left_leaf, &e);
        } else if (smaller_leaf == left_leaf) {
          bool existed;
          int32_t parent = get_slot(left_leaf, &existed);
          use_subtract = existed;
          slot_of_leaf[right_leaf] = parent;  // Move(left -> right)
          slot_of_leaf[left_leaf] = -1;
          bool e;
          smaller_slot = get_slot(left_leaf, &e);
          larger_slot = parent;
        } else {
          bool existed;
          int32_t parent = get_slot(left_leaf, &existed);
          use_subtract = existed;
          bool e;
          smaller_slot = get_slot(right_leaf, &e);
          larger_slot = parent;
        }
        std::vector<uint8_t> parent_splittable;
        const std::vector<uint8_t>* ps = nullptr;
        if (use_subtract) {
          parent_splittable = feature_splittable[left_leaf];
          ps = &parent_splittable;
        }
        const LeafSplits& sls = smaller;
        const LeafSplits& lls = right_leaf < 0 ? smaller : larger;
        build_leaf(smaller_leaf, sls, pool[smaller_slot].data(), ps ? ps->data() : nullptr);
        if (larger_leaf >= 0) {
          double* lb = pool[larger_slot].data();
          if (use_subtract) {
            // HistogramPool::subtract_into (histogram_pool.rs:249-283)
            const double* sb = pool[smaller_slot].data();
            for (size_t i = 0; i < slot_len; ++i) lb[i] = lb[i] - sb[i];
          } else {
            build_leaf(larger_leaf, lls, lb, ps ? ps->data() : nullptr);
          }
        }
        scan_leaf(smaller_leaf, sls, pool[smaller_slot].data(), ps);
        if (larger_leaf >= 0) scan_leaf(larger_leaf, lls, pool[larger_slot].data(), ps);
      }
      // arg_max (learner.rs:4537-4551)
      int32_t best_leaf = 0;
      for (int32_t i = 1; i < num_leaves; ++i)
        if (split_gt(best_split[i], best_feature[i], best_split[best_leaf], best_feature[best_leaf]))
          best_leaf = i;
      const OSplitInfo best = best_split[best_leaf];
      if (best.gain <= 0.0) break;
      const int32_t f = best_feature[best_leaf];
      const int32_t new_left = best_leaf, new_right = nl;
      partition(best_leaf, new_right, f, best.threshold, best.default_left != 0);
      // Tree::split (lgbm-model/src/tree.rs:614-690)
      {
        const int32_t node = nl - 1;
        const int32_t parent = tree->leaf_parent[best_leaf];
        if (parent >= 0) {
          if (tree->right_child[parent] == ~best_leaf)
            tree->right_child[parent] = node;
          else
            tree->left_child[parent] = node;
        }
        tree->split_feature[node] = f;
        tree->split_gain[node] = (float)(best.gain + cfg.min_gain_to_split);
        tree->threshold_bin[node] = best.threshold;
        const bool cat = meta[f].is_categorical != 0;
        tree->internal_value[node] = tree->leaf_value[best_leaf];
        tree->internal_count[node] = leaf_count[new_left] + leaf_count[new_right];
        tree->left_child[node] = ~best_leaf;
        tree->right_child[node] = ~new_right;
        int8_t dt = 0;
        if (cat) {
          // Tree::split_categorical (lgbm-model/src/tree.rs:710-770): the threshold
          // is the categorical-node index, default_left is not encoded
          dt |= 1;
          tree->threshold_bin[node] = (uint32_t)num_cat++;
          if (tree->cat_bins)
            for (int k = 0; k < 8; ++k) tree->cat_bins[8 * node + k] = best_cat[best_leaf][k];
        } else if (best.default_left) {
          dt |= 2;
        }
        dt |= (int8_t)((meta[f].missing_type & 3) << 2);
        tree->decision_type[node] = dt;
        tree->leaf_value[best_leaf] = best.left_output;
        tree->leaf_weight[best_leaf] = best.left_sum_hessian;
        tree->leaf_count[best_leaf] = leaf_count[new_left];
        tree->leaf_value[new_right] = best.right_output;
        tree->leaf_weight[new_right] = best.right_sum_hessian;
        tree->leaf_count[new_right] = leaf_count[new_right];
        tree->leaf_depth[new_right] = tree->leaf_depth[best_leaf] + 1;
        tree->leaf_depth[best_leaf] += 1;
        tree->leaf_parent[best_leaf] = node;
        tree->leaf_parent[new_right] = node;
        nl += 1;
      }
      if (trace) {
        trace[4 * nsplit_trace + 0] = best_leaf;
        trace[4 * nsplit_trace + 1] = f;
        trace[4 * nsplit_trace + 2] = (int32_t)best.threshold;
        trace[4 * nsplit_trace + 3] = best.default_left;
        nsplit_trace++;
      }
      // seed children (learner.rs:4061-4089): smaller = fewer partition rows, tie -> right
      const int32_t pl = leaf_count[new_left], pr = leaf_count[new_right];
      if (pl < pr) {
        smaller = {pl, best.left_sum_gradient, best.left_sum_hessian, best.left_output};
        larger = {pr, best.right_sum_gradient, best.right_sum_hessian, best.right_output};
      } else {
        smaller = {pr, best.right_sum_gradient, best.right_sum_hessian, best.right_output};
        larger = {pl, best.left_sum_gradient, best.left_sum_hessian, best.left_output};
      }
      best_split[best_leaf] = split_none();
      best_feature[best_leaf] = -1;
      best_split[new_left] = split_none();
      best_feature[new_left] = -1;
      best_split[new_right] = split_none();
      best_feature[new_right] = -1;
      left_leaf = new_left;
      right_leaf = new_right;
    }
    tree->num_leaves = nl;
    if (idx_out) std::copy(indices.begin(), indices.end(), idx_out);
    if (lb_out) std::copy(leaf_begin.begin(), leaf_begin.end(), lb_out);
    if (lc_out) std::copy(leaf_count.begin(), leaf_count.end(), lc_out);
    return nsplit_trace;
  }
};

}  // namespace

extern "C" {

// Backend::construct_histograms on the CPU backend: ordered f64 fold of f32 g/h
// over every row (lgbm-compute/src/kernels/histogram.rs:207-233).
void oracle_construct_histogram(const uint32_t* bins, const float* g, const float* h, int64_t n,
                                uint32_t num_bin, double* out) {
  std::fill(out, out + 2 * (size_t)num_bin, 0.0);
  for (int64_t i = 0; i < n; ++i) {
    out[2 * bins[i]] += (double)g[i];
    out[2 * bins[i] + 1] += (double)h[i];
  }
}

// Fold over an explicit ascending row list (Backend::build_leaf_histograms_raw_into
// for one feature, lgbm-compute/src/lib.rs:1422-1469).
void oracle_construct_leaf_histogram(const uint32_t* bins, const uint32_t* rows, int64_t n_rows,
                                     const float* g, const float* h, uint32_t num_bin,
                                     double* out) {
  std::fill(out, out + 2 * (size_t)num_bin, 0.0);
  for (int64_t k = 0; k < n_rows; ++k) {
    uint32_t r = rows[k];
    out[2 * bins[r]] += (double)g[r];
    out[2 * bins[r] + 1] += (double)h[r];
  }
}

int oracle_find_best_split(const double* hist, const OGainConfig* cfg, int32_t num_bin,
                           int32_t offset, int32_t default_bin, int32_t skip_default_bin,
                           int32_t na_as_missing, int32_t run_forward, double sum_gradient,
                           double sum_hessian, int32_t num_data, OSplitInfo* out) {
  if (num_bin <= 0 || !(sum_hessian > 0.0)) return -1;  // split.rs:8993-9016
  *out = find_best_split(hist, to_cfg(*cfg), num_bin, offset, default_bin, skip_default_bin != 0,
                         na_as_missing != 0, run_forward != 0, sum_gradient, sum_hessian,
                         num_data);
  return 0;
}

// kernels/subtract.rs:204-227: derived[i] = parent[i] - child[i]
void oracle_subtract(const double* parent, const double* child, int64_t len, double* out) {
  for (int64_t i = 0; i < len; ++i) out[i] = parent[i] - child[i];
}

void oracle_fix_histogram(double* hist, int32_t num_bin, int32_t mfb, double sum_g, double sum_h) {
  fix_histogram(hist, num_bin, mfb, sum_g, sum_h);
}

void oracle_compact_histogram(double* hist, int32_t num_bin, int32_t offset) {
  compact_histogram(hist, num_bin, offset);
}

// DataPartition routing over one leaf (data_partition.rs:360-487). `bins` holds
// the split feature's bin for each of the `count` rows in `rows` (in place).
// Returns the left count; rows are reordered [left asc | right asc].
int64_t oracle_partition(const uint32_t* bins_of_rows, uint32_t* rows, int64_t count,
                         uint32_t num_bin, uint32_t min_bin, uint32_t max_bin, uint32_t threshold,
                         uint32_t most_freq_bin, int32_t na_as_missing, int32_t default_left) {
  std::vector<uint32_t> L, R;
  const int32_t min_b = (int32_t)min_bin, max_b = (int32_t)max_bin, thr = (int32_t)threshold;
  int32_t th = thr + min_b;
  if (most_freq_bin == 0) th -= 1;
  const bool default_to_right = (int32_t)most_freq_bin > thr;
  const int32_t na_bin = (int32_t)num_bin - 1;
  for (int64_t i = 0; i < count; ++i) {
    const int32_t b = (int32_t)bins_of_rows[i];
    bool gr;
    if (na_as_missing && b == na_bin)
      gr = !default_left;
    else if (b < min_b || b > max_b)
      gr = default_to_right;
    else
      gr = b > th;
    (gr ? R : L).push_back(rows[i]);
  }
  std::copy(L.begin(), L.end(), rows);
  std::copy(R.begin(), R.end(), rows + L.size());
  return (int64_t)L.size();
}

// The kernel-level partition with the whole missing-value fan-out: RouteFlags::derive
// and route_left_host (lgbm-compute/src/kernels/data_partition.rs:325-406), driven by
// partition_leaf_stable (:487-520). missing_type 1 routes the zero bin
// (min_bin + default_bin - [mfb == 0]) and 2 the NA bin (max_bin) by default_left,
// unless the most frequent bin coincides with it, in which case out-of-range rows
// follow default_left instead; min_bin == max_bin is the degenerate one-bin feature.
int64_t oracle_partition_missing(const uint32_t* bins_of_rows, uint32_t* rows, int64_t count,
                                 uint32_t min_bin, uint32_t max_bin, uint32_t threshold,
                                 uint32_t most_freq_bin, uint32_t default_bin,
                                 int32_t missing_type, int32_t default_left) {
  const bool zero_missing = missing_type == 1, na_missing = missing_type == 2;
  const bool mfb_zero = zero_missing && default_bin == most_freq_bin;
  const bool mfb_na = na_missing && max_bin == most_freq_bin + min_bin && most_freq_bin > 0;
  const int32_t lo = (int32_t)min_bin, hi = (int32_t)max_bin;
  const int32_t shift = most_freq_bin == 0 ? 1 : 0;
  const int32_t th = (int32_t)threshold + lo - shift;
  const int32_t zero_bin = lo + (int32_t)default_bin - shift;
  // 0 = left, 1 = right
  const int mfb_side = most_freq_bin <= threshold ? 0 : 1;
  const int missing_side = ((zero_missing || na_missing) && default_left) ? 0 : 1;
  const bool oor_is_missing = (na_missing && mfb_na) || (zero_missing && mfb_zero);
  const bool zero_sentinel = zero_missing && !mfb_zero;
  const bool na_sentinel = na_missing && !mfb_na;
  std::vector<uint32_t> L, R;
  for (int64_t i = 0; i < count; ++i) {
    const int32_t b = (int32_t)bins_of_rows[i];
    int side;
    if (zero_sentinel && b == zero_bin) {
      side = missing_side;
    } else if (lo == hi) {
      if (b != hi)
        side = oor_is_missing ? missing_side : mfb_side;
      else
        side = na_sentinel ? missing_side : (hi <= th ? 0 : 1);
    } else if (na_sentinel && b == hi) {
      side = missing_side;
    } else if (b < lo || b > hi) {
      side = oor_is_missing ? missing_side : mfb_side;
    } else {
      side = b > th ? 1 : 0;
    }
    (side ? R : L).push_back(rows[i]);
  }
  std::copy(L.begin(), L.end(), rows);
  std::copy(R.begin(), R.end(), rows + L.size());
  return (int64_t)L.size();
}

// SerialTreeLearner::train (spine path). Returns the number of splits made, or
// a negative code. `cols` are feature-major bin columns of `bin_bytes` width.
int32_t oracle_grow_tree(const void* const* cols, int32_t bin_bytes, int64_t num_data,
                         int32_t num_features, const OFeatureMeta* meta, const float* g,
                         const float* h, const OLearnerConfig* cfg, int32_t nthreads,
                         OTree* tree, uint32_t* indices_out, int32_t* leaf_begin_out,
                         int32_t* leaf_count_out, int32_t* trace) {
  if (num_data <= 0 || num_features <= 0 || cfg->num_leaves < 1) return -2;
  Bins b{cols, bin_bytes};
  Learner L(b, num_data, num_features, meta, g, h, *cfg, nthreads < 1 ? 1 : nthreads);
  return L.grow(tree, indices_out, leaf_begin_out, leaf_count_out, trace);
}

// Binary::get_gradients (lgbm-objective/src/binary.rs:134-171), label weights 1.
void oracle_binary_gradients(const double* score, const float* label, int64_t n, double sigmoid,
                             float* g, float* h, int32_t nthreads) {
#pragma omp parallel for schedule(static) num_threads(nthreads) if (nthreads > 1 && n >= 50000)
  for (int64_t i = 0; i < n; ++i) {
    const bool is_pos = label[i] > 0.0f;
    const double lv = is_pos ? 1.0 : -1.0;
    const double resp = -lv * sigmoid / (1.0 + std::exp(lv * sigmoid * score[i]));
    const double ar = std::fabs(resp);
    g[i] = (float)(resp * 1.0);
    h[i] = (float)(ar * (sigmoid - ar) * 1.0);
  }
}

// Regression (L2) get_gradients (lgbm-objective/src/regression.rs:429-433).
void oracle_l2_gradients(const double* score, const float* label, int64_t n, float* g, float* h,
                         int32_t nthreads) {
#pragma omp parallel for schedule(static) num_threads(nthreads) if (nthreads > 1 && n >= 50000)
  for (int64_t i = 0; i < n; ++i) {
    g[i] = (float)(score[i] - (double)label[i]);
    h[i] = 1.0f;
  }
}

// Lambdarank::new + get_gradients (lgbm-objective/src/rank.rs:152-366; LightGBM
// rank_objective.hpp:140-294), unweighted, no position bias. Per query: a stable sort
// by descending score, then for every pair with its upper document above the
// truncation level and different labels, the sigmoid-table lambda and hessian scaled
// by the pair's NDCG change, accumulated into the f32 outputs in loop order; with
// `norm`, a final rescale by log2(1 + sum_lambdas) / sum_lambdas. The DCG tables follow
// DcgCalculator (lgbm-metric/src/dcg_calculator.rs:48-162): gains 2^i - 1 (31 entries)
// unless given, discount 1 / log2(2 + rank) for 10000 ranks. Returns 0, or -1 when the
// query boundaries or labels are invalid.
int32_t oracle_lambdarank_gradients(const double* score, const float* label, int64_t n,
                                    const int32_t* qb, int32_t nq, double sigmoid,
                                    int32_t norm, int32_t trunc, const double* label_gain_in,
                                    int32_t n_gain_in, float* g, float* h, int32_t nthreads) {
  if (nq < 1 || qb[0] != 0 || qb[nq] != n || !(sigmoid > 0.0)) return -1;
  for (int32_t q = 0; q < nq; ++q)
    if (qb[q + 1] < qb[q]) return -1;
  std::vector<double> gain;
  if (n_gain_in > 0) {
    gain.assign(label_gain_in, label_gain_in + n_gain_in);
  } else {
    gain.push_back(0.0);
    for (int i = 1; i < 31; ++i) gain.push_back((double)((1ll << i) - 1));
  }
  for (int64_t i = 0; i < n; ++i) {
    const float l = label[i];
    if (std::fabs(l - (float)(int32_t)l) > 1e-15f || l < 0.0f || (int64_t)l >= (int64_t)gain.size())
      return -1;
  }
  constexpr int kMaxPosition = 10000;
  static std::vector<double> discount;
  if (discount.empty())
    for (int i = 0; i < kMaxPosition; ++i) discount.push_back(1.0 / std::log2(2.0 + (double)i));
  // ConstructSigmoidTable: 2^20 bins over [-50 / sigmoid / 2, +50 / sigmoid / 2]
  constexpr int64_t kBins = 1024 * 1024;
  static std::vector<double> table;
  static double table_sigmoid = 0.0;
  const double min_in = -50.0 / sigmoid / 2.0, max_in = -min_in;
  const double idx_factor = (double)kBins / (max_in - min_in);
  if (table.empty() || table_sigmoid != sigmoid) {
    table.resize(kBins);
    for (int64_t i = 0; i < kBins; ++i) {
      const double s = (double)i / idx_factor + min_in;
      table[i] = 1.0 / (1.0 + std::exp(s * sigmoid));
    }
    table_sigmoid = sigmoid;
  }
  auto sig = [&](double s) {
    if (s <= min_in) return table[0];
    if (s >= max_in) return table[kBins - 1];
    const size_t i = (size_t)((s - min_in) * idx_factor);
    return table[std::min<size_t>(i, (size_t)kBins - 1)];
  };
  const double kMinScore = -std::numeric_limits<double>::infinity();
#pragma omp parallel for schedule(dynamic, 16) num_threads(nthreads) if (nthreads > 1 && nq >= 64)
  for (int32_t q = 0; q < nq; ++q) {
    const int64_t b = qb[q];
    const int64_t cnt = qb[q + 1] - b;
    const double* s = score + b;
    const float* lab = label + b;
    float* lam = g + b;
    float* hes = h + b;
    for (int64_t i = 0; i < cnt; ++i) lam[i] = hes[i] = 0.0f;
    if (cnt == 0) continue;
    // DcgCalculator::cal_max_dcg_at_k(trunc) -> inverse
    std::vector<int64_t> lc(gain.size(), 0);
    for (int64_t i = 0; i < cnt; ++i) lc[(size_t)lab[i]] += 1;
    double maxdcg = 0.0;
    int64_t top = (int64_t)gain.size() - 1;
    const int64_t kk = std::min<int64_t>(trunc, cnt);
    for (int64_t j = 0; j < kk; ++j) {
      while (top > 0 && lc[top] <= 0) --top;
      if (top < 0) break;
      maxdcg += discount[j] * gain[top];
      lc[top] -= 1;
    }
    const double inv_max = maxdcg > 0.0 ? 1.0 / maxdcg : maxdcg;
    std::vector<int64_t> order(cnt);
    for (int64_t i = 0; i < cnt; ++i) order[i] = i;
    std::stable_sort(order.begin(), order.end(),
                     [&](int64_t a, int64_t c) { return s[a] > s[c]; });
    const double best = s[order[0]];
    int64_t wi = cnt - 1;
    if (wi > 0 && s[order[wi]] == kMinScore) --wi;
    const double worst = s[order[wi]];
    double sum_lambdas = 0.0;
    for (int64_t i = 0; i + 1 < cnt && i < trunc; ++i) {
      if (s[order[i]] == kMinScore) continue;
      for (int64_t j = i + 1; j < cnt; ++j) {
        if (s[order[j]] == kMinScore) continue;
        if (lab[order[i]] == lab[order[j]]) continue;
        const bool i_high = lab[order[i]] > lab[order[j]];
        const int64_t hr = i_high ? i : j, lr = i_high ? j : i;
        const int64_t hi = order[hr], lo = order[lr];
        const double ds = s[hi] - s[lo];
        const double gap = gain[(size_t)lab[hi]] - gain[(size_t)lab[lo]];
        const double pd = std::fabs(discount[hr] - discount[lr]);
        double dndcg = gap * pd * inv_max;
        if (norm && best != worst) dndcg /= (double)0.01f + std::fabs(ds);
        double pl = sig(ds);
        double ph = pl * (1.0 - pl);
        pl *= -sigmoid * dndcg;
        ph *= sigmoid * sigmoid * dndcg;
        lam[lo] -= (float)pl;
        hes[lo] += (float)ph;
        lam[hi] += (float)pl;
        hes[hi] += (float)ph;
        sum_lambdas -= 2.0 * pl;
      }
    }
    if (norm && sum_lambdas > 0.0) {
      const double nf = std::log2(1.0 + sum_lambdas) / sum_lambdas;
      for (int64_t i = 0; i < cnt; ++i) {
        lam[i] = (float)((double)lam[i] * nf);
        hes[i] = (float)((double)hes[i] * nf);
      }
    }
  }
  return 0;
}

// GbdtModel raw prediction (lgbm-model/src/predict.rs) over a flattened ensemble:
// Tree::get_leaf with numerical_decision / categorical_decision
// (lgbm-model/src/tree.rs:173-300), leaf values summed in tree order. Child indices are
// tree-local (< 0: leaf ~c); a categorical node's threshold indexes cat_boundaries over
// all trees.
void oracle_predict_raw(int32_t num_trees, int32_t num_features, const int32_t* node_offset,
                        const int32_t* leaf_offset, const int32_t* split_feature,
                        const double* threshold, const int8_t* decision_type,
                        const int32_t* left_child, const int32_t* right_child,
                        const double* leaf_value, const int32_t* cat_boundaries,
                        const uint32_t* cat_threshold, const double* rows, int64_t n,
                        double* out) {
  for (int64_t r = 0; r < n; ++r) {
    const double* x = rows + r * num_features;
    double acc = 0.0;
    for (int32_t t = 0; t < num_trees; ++t) {
      const int32_t nb = node_offset[t];
      int32_t node = node_offset[t + 1] > nb ? 0 : -1;
      while (node >= 0) {
        const int32_t k = nb + node;
        double fval = x[split_feature[k]];
        const int8_t dt = decision_type[k];
        if (dt & 1) {
          if (std::isnan(fval)) {
            node = right_child[k];
            continue;
          }
          const int32_t iv = (int32_t)std::max(-2147483648.0, std::min(2147483647.0, fval));
          if (iv < 0) {
            node = right_child[k];
            continue;
          }
          const int32_t c = (int32_t)threshold[k];
          const int32_t lo = cat_boundaries[c], nw = cat_boundaries[c + 1] - lo;
          const int32_t w = iv / 32;
          const bool in = w < nw && ((cat_threshold[lo + w] >> (iv % 32)) & 1u);
          node = in ? left_child[k] : right_child[k];
          continue;
        }
        const int mt = (dt >> 2) & 3;
        if (std::isnan(fval) && mt != 2) fval = 0.0;
        if ((mt == 1 && fval >= -kZeroThreshold && fval <= kZeroThreshold) ||
            (mt == 2 && std::isnan(fval))) {
          node = (dt & 2) ? left_child[k] : right_child[k];
          continue;
        }
        node = fval <= threshold[k] ? left_child[k] : right_child[k];
      }
      acc += leaf_value[leaf_offset[t] + ~node];
    }
    out[r] = acc;
  }
}

// Binary::boost_from_score (binary.rs:178-194)
double oracle_binary_boost_from_score(const float* label, int64_t n, double sigmoid) {
  if (n == 0) return 0.0;
  const double sumw = (double)n;
  double suml = 0.0;
  for (int64_t i = 0; i < n; ++i) suml += label[i] > 0.0f ? 1.0 : 0.0;
  double pavg = suml / sumw;
  pavg = std::min(pavg, 1.0 - kEps);
  pavg = std::max(pavg, kEps);
  return std::log(pavg / (1.0 - pavg)) / sigmoid;
}

// Regression::boost_from_score (regression.rs:563-577): ordered label mean.
double oracle_l2_boost_from_score(const float* label, int64_t n) {
  if (n == 0) return 0.0;
  double s = 0.0;
  for (int64_t i = 0; i < n; ++i) s += (double)label[i];
  return s / (double)n;
}

// quantize_grad_hess_in_place (lgbm-boosting/src/gbdt.rs:43-62) with
// GradientDiscretizer::{compute_scales, quantize_pair}
// (lgbm-treelearner/src/gradient_discretizer.rs:126-191), deterministic rounding.
// Writes the int8 pair (qg, qh) per row when q_out != NULL and the dequantized f32
// values back into g/h. scales_out = {grad_scale, hess_scale, is_constant_hessian}.
// GradientDiscretizer with stochastic rounding (gradient_discretizer.rs:83-90,167-191,
// 252-262): a seeded xorshift64, one draw for the gradient then one for the hessian of
// every row in row order, each draw the top 53 bits over 2^53.
struct Xorshift64 {
  uint64_t s;
  double next_u01() {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    return (double)(s >> 11) / (double)(1ull << 53);
  }
};

void oracle_quantize_ex(float* g, float* h, int64_t n, int32_t num_grad_quant_bins,
                        int8_t* q_out, double* scales_out, int32_t stochastic, uint64_t seed);

void oracle_quantize(float* g, float* h, int64_t n, int32_t num_grad_quant_bins,
                     int8_t* q_out, double* scales_out) {
  oracle_quantize_ex(g, h, n, num_grad_quant_bins, q_out, scales_out, 0, 0);
}

// stochastic != 0: the rounding offsets come from the xorshift stream seeded with
// seed ^ 0x9E3779B97F4A7C15 (new_stochastic); the caller passes the per-iteration seed
// of gbdt.rs:950, ((iter << 20) ^ class ^ 0x51702010).
void oracle_quantize_ex(float* g, float* h, int64_t n, int32_t num_grad_quant_bins,
                        int8_t* q_out, double* scales_out, int32_t stochastic, uint64_t seed) {
  if (n == 0) return;
  Xorshift64 rng{seed ^ 0x9E3779B97F4A7C15ull};
  bool is_const = true;
  for (int64_t i = 0; i < n; ++i)
    if (!(h[i] == h[0])) {
      is_const = false;
      break;
    }
  double max_g = std::fabs((double)g[0]), max_h = std::fabs((double)h[0]);
  for (int64_t i = 0; i < n; ++i) {
    max_g = std::max(max_g, std::fabs((double)g[i]));
    max_h = std::max(max_h, std::fabs((double)h[i]));
  }
  const double half_bins = (double)(num_grad_quant_bins / 2);
  const double gs = max_g / half_bins;
  const double hs = is_const ? max_h : max_h / (double)num_grad_quant_bins;
  const double igs = 1.0 / gs, ihs = 1.0 / hs;
  for (int64_t i = 0; i < n; ++i) {
    double bg = 0.5, bh = 0.5;
    if (stochastic) {
      bg = rng.next_u01();
      bh = rng.next_u01();
    }
    const double gv = (double)g[i] * igs;
    const int8_t qg = (int8_t)(int32_t)(g[i] >= 0.0f ? gv + bg : gv - bg);
    const int8_t qh = is_const ? (int8_t)1 : (int8_t)(int32_t)((double)h[i] * ihs + bh);
    if (q_out) {
      q_out[2 * i] = qg;
      q_out[2 * i + 1] = qh;
    }
    g[i] = (float)((double)qg * gs);
    h[i] = (float)((double)qh * hs);
  }
  if (scales_out) {
    scales_out[0] = gs;
    scales_out[1] = hs;
    scales_out[2] = is_const ? 1.0 : 0.0;
  }
}

// Tree::shrinkage (lgbm-model/src/tree.rs:1074-1100) on leaf and internal values.
void oracle_tree_shrinkage(double* leaf_value, int32_t num_leaves, double* internal_value,
                           double rate) {
  for (int32_t i = 0; i < num_leaves; ++i) {
    double v = leaf_value[i] * rate;
    leaf_value[i] = is_zero(v) ? 0.0 : v;
  }
  for (int32_t i = 0; i + 1 < num_leaves; ++i) {
    double v = internal_value[i] * rate;
    internal_value[i] = is_zero(v) ? 0.0 : v;
  }
}

// SerialTreeLearner::add_prediction_to_score (learner.rs:4380-4395).
void oracle_add_prediction_to_score(const double* leaf_value, int32_t num_leaves,
                                    const uint32_t* indices, const int32_t* leaf_begin,
                                    const int32_t* leaf_count, double* score) {
  if (num_leaves <= 1) return;
  for (int32_t l = 0; l < num_leaves; ++l) {
    const double v = leaf_value[l];
    for (int32_t k = 0; k < leaf_count[l]; ++k) score[indices[leaf_begin[l] + k]] += v;
  }
}

int32_t oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

}  // extern "C"
