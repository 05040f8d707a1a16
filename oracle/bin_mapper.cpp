// TEST INFRASTRUCTURE ONLY -- the CPU oracle's own restatement of the reference's
// feature binning, used by tests/ and by bench.py's CPU arms (`--impl reference`,
// `cpu_baseline`) so that those processes bin their data without loading the product
// library. The product path never links or calls this file.
//
// Restated from the reference (paths inside the lightgbm_rs project):
//   Random (LCG, rand16/rand32, next_float, next_int, sample)   crates/lgbm-core/src/random.rs
//   create_sample_indices / sample_count                        crates/lgbm-dataset/src/bin_mapper.rs:80-95
//   value_to_bin (numeric binary search, categorical lookup)    bin_mapper.rs:148-199
//   find_bin_numeric                                            bin_mapper.rs:201-415
//   find_bin_categorical                                        bin_mapper.rs:416-641
//   find_bin_from_column, scaled_filter_cnt, need_filter         bin_mapper.rs:642-746
//   greedy_find_bin                                             bin_mapper.rs:749-835
//   find_bin_with_zero_as_one_bin                               bin_mapper.rs:938-1013
// kZeroThreshold is the double 1e-35 (crates/lgbm-core/src/types.rs:35).
// Forced bin bounds (find_bin_with_predefined_bin) are not restated: no caller here
// passes them.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <limits>
#include <map>
#include <set>
#include <utility>
#include <vector>

namespace {

constexpr double kZeroThr = 1e-35;
constexpr double kInf = std::numeric_limits<double>::infinity();

// ---------------------------------------------------------------- LCG (random.rs)
class Lcg {
 public:
  explicit Lcg(int32_t seed) : state_((uint32_t)seed) {}
  int32_t next_int(int32_t lo, int32_t hi) { return step31() % (hi - lo) + lo; }
  float next_float() { return (float)step15() / 32768.0f; }

  // Random::sample: k of n indices, ascending.
  std::vector<int32_t> sample(int32_t n, int32_t k) {
    std::vector<int32_t> out;
    if (k <= 0 || k > n) return out;
    if (k == n) {
      for (int32_t i = 0; i < n; ++i) out.push_back(i);
      return out;
    }
    if (k > 1 && (double)k > (double)n / std::log2((double)k)) {
      // sequential selection: keep i with probability (still needed) / (still left)
      for (int32_t i = 0; i < n; ++i) {
        const double p = (double)(k - (int32_t)out.size()) / (double)(n - i);
        if ((double)next_float() < p) out.push_back(i);
      }
      return out;
    }
    // Floyd's selection over the last k positions
    std::set<int32_t> chosen;
    for (int32_t r = n - k; r < n; ++r) {
      const int32_t v = next_int(0, r + 1);
      if (!chosen.insert(v).second) chosen.insert(r);
    }
    out.assign(chosen.begin(), chosen.end());
    return out;
  }

 private:
  uint32_t advance() { return state_ = state_ * 214013u + 2531011u; }
  int32_t step15() { return (int32_t)((advance() >> 16) & 0x7fffu); }
  int32_t step31() { return (int32_t)(advance() & 0x7fffffffu); }
  uint32_t state_;
};

double next_up(double a) { return std::nextafter(a, kInf); }
bool equal_ordered(double a, double b) { return b <= next_up(a); }

// ---------------------------------------------------------------- mapper
struct Mapper {
  bool categorical = false;
  int32_t num_bin = 0;
  int32_t missing = 0;  // 0 none, 1 zero, 2 NaN
  std::vector<double> upper;
  std::vector<int32_t> bin_to_cat;
  std::map<int32_t, uint32_t> cat_to_bin;
  bool trivial = false;
  double sparse_rate = 0.0;
  uint32_t default_bin = 0, most_freq_bin = 0;
  double min_val = 0.0, max_val = 0.0;

  uint32_t bin_of(double v) const {
    if (std::isnan(v)) {
      if (categorical) return 0;
      if (missing == 2) return (uint32_t)(num_bin - 1);
      v = 0.0;
    }
    if (!categorical) {
      int32_t lo = 0, hi = num_bin - 1 - (missing == 2 ? 1 : 0);
      while (lo < hi) {
        const int32_t mid = (hi + lo - 1) / 2;  // the reference's midpoint
        if (v <= upper[mid])
          hi = mid;
        else
          lo = mid + 1;
      }
      return (uint32_t)lo;
    }
    const int32_t code = (int32_t)v;
    if (code < 0) return 0;
    auto it = cat_to_bin.find(code);
    return it == cat_to_bin.end() ? 0u : it->second;
  }
};

// Sorted non-NaN sample values folded into distinct values and their counts, with the
// zero pseudo-value placed where the sample's zeros (rows the sample did not hold as
// nonzero values) belong.
struct Distinct {
  std::vector<double> value;
  std::vector<int32_t> count;
};

Distinct fold_distinct(std::vector<double>& v, int32_t zero_cnt) {
  Distinct d;
  std::stable_sort(v.begin(), v.end());
  const size_t n = v.size();
  auto push = [&](double x, int32_t c) {
    d.value.push_back(x);
    d.count.push_back(c);
  };
  if (n == 0 || (v[0] > 0.0 && zero_cnt > 0)) push(0.0, zero_cnt);
  if (n > 0) push(v[0], 1);
  for (size_t i = 1; i < n; ++i) {
    if (equal_ordered(v[i - 1], v[i])) {
      d.value.back() = v[i];  // keep the larger value
      d.count.back() += 1;
      continue;
    }
    if (v[i - 1] < 0.0 && v[i] > 0.0) push(0.0, zero_cnt);
    push(v[i], 1);
  }
  if (n > 0 && v[n - 1] < 0.0 && zero_cnt > 0) push(0.0, zero_cnt);
  return d;
}

// greedy_find_bin over the first `nd` entries of (vals, cnts).
std::vector<double> greedy(const double* vals, const int32_t* cnts, int32_t nd, int32_t max_bin,
                           int64_t total_cnt, int32_t min_data_in_bin) {
  std::vector<double> bounds;
  auto add_bound = [&](double x) {
    if (bounds.empty() || !equal_ordered(bounds.back(), x)) {
      bounds.push_back(x);
      return true;
    }
    return false;
  };
  if (nd <= max_bin) {
    int32_t run = 0;
    for (int32_t i = 0; i + 1 < nd; ++i) {
      run += cnts[i];
      if (run >= min_data_in_bin && add_bound(next_up((vals[i] + vals[i + 1]) / 2.0))) run = 0;
    }
    bounds.push_back(kInf);
    return bounds;
  }
  if (min_data_in_bin > 0) {
    max_bin = std::min(max_bin, (int32_t)(total_cnt / (int64_t)min_data_in_bin));
    max_bin = std::max(max_bin, 1);
  }
  double mean = (double)total_cnt / (double)max_bin;
  int32_t bins_left = max_bin;
  int32_t samples_left = (int32_t)total_cnt;
  std::vector<char> big(nd, 0);
  for (int32_t i = 0; i < nd; ++i) {
    if ((double)cnts[i] >= mean) {
      big[i] = 1;
      --bins_left;
      samples_left -= cnts[i];
    }
  }
  mean = (double)samples_left / (double)bins_left;
  std::vector<double> hi_edge(max_bin, kInf), lo_edge(max_bin, kInf);
  size_t nb = 0;
  lo_edge[0] = vals[0];
  int32_t run = 0;
  for (int32_t i = 0; i + 1 < nd; ++i) {
    if (!big[i]) samples_left -= cnts[i];
    run += cnts[i];
    // the reference multiplies the running mean by the float literal 0.5f
    const bool cut = big[i] || (double)run >= mean ||
                     (big[i + 1] && (double)run >= std::max(1.0, mean * (double)0.5f));
    if (!cut) continue;
    hi_edge[nb] = vals[i];
    ++nb;
    lo_edge[nb] = vals[i + 1];
    if ((int32_t)nb >= max_bin - 1) break;
    run = 0;
    if (!big[i]) {
      --bins_left;
      mean = (double)samples_left / (double)bins_left;
    }
  }
  ++nb;
  for (size_t i = 0; i + 1 < nb; ++i) add_bound(next_up((hi_edge[i] + lo_edge[i + 1]) / 2.0));
  bounds.push_back(kInf);
  return bounds;
}

// find_bin_with_zero_as_one_bin: negatives and positives binned apart, zero its own bin.
std::vector<double> zero_as_one_bin(const Distinct& d, int32_t max_bin, int64_t total_cnt,
                                    int32_t min_data_in_bin) {
  const int32_t nd = (int32_t)d.value.size();
  int32_t neg_cnt = 0, zero_cnt = 0, pos_cnt = 0;
  for (int32_t i = 0; i < nd; ++i) {
    const double x = d.value[i];
    if (x <= -kZeroThr)
      neg_cnt += d.count[i];
    else if (x > kZeroThr)
      pos_cnt += d.count[i];
    else
      zero_cnt += d.count[i];
  }
  int32_t first_nonneg = nd;
  for (int32_t i = 0; i < nd; ++i)
    if (d.value[i] > -kZeroThr) {
      first_nonneg = i;
      break;
    }
  std::vector<double> bounds;
  if (first_nonneg > 0 && max_bin > 1) {
    int32_t neg_bins = (int32_t)((double)neg_cnt / (double)((int32_t)total_cnt - zero_cnt) *
                                 (double)(max_bin - 1));
    neg_bins = std::max(neg_bins, 1);
    bounds = greedy(d.value.data(), d.count.data(), first_nonneg, neg_bins, neg_cnt,
                    min_data_in_bin);
    if (!bounds.empty()) bounds.back() = -kZeroThr;
  }
  int32_t first_pos = -1;
  for (int32_t i = first_nonneg; i < nd; ++i)
    if (d.value[i] > kZeroThr) {
      first_pos = i;
      break;
    }
  const int32_t pos_bins = max_bin - 1 - (int32_t)bounds.size();
  if (first_pos >= 0 && pos_bins > 0) {
    std::vector<double> right = greedy(d.value.data() + first_pos, d.count.data() + first_pos,
                                       nd - first_pos, pos_bins, pos_cnt, min_data_in_bin);
    bounds.push_back(kZeroThr);
    bounds.insert(bounds.end(), right.begin(), right.end());
  } else {
    bounds.push_back(kInf);
  }
  return bounds;
}

int32_t first_max(const std::vector<int32_t>& v) {
  int32_t best = 0;
  for (int32_t i = 1; i < (int32_t)v.size(); ++i)
    if (v[i] > v[best]) best = i;
  return best;
}

// need_filter: no cut of the sample leaves filter_cnt rows on both sides.
bool filtered(const std::vector<int32_t>& cnt_in_bin, int32_t total, int32_t filter_cnt,
              bool categorical) {
  if (categorical && cnt_in_bin.size() > 2) return false;
  int32_t left = 0;
  for (size_t i = 0; i + 1 < cnt_in_bin.size(); ++i) {
    left = categorical ? cnt_in_bin[i] : left + cnt_in_bin[i];
    if (left >= filter_cnt && total - left >= filter_cnt) return false;
  }
  return true;
}

// The tail shared by both kinds: triviality, pre-filter, default and most frequent bin.
void finish(Mapper& m, const std::vector<int32_t>& cnt_in_bin, int64_t total, int32_t filter_cnt,
            bool pre_filter) {
  m.trivial = m.num_bin <= 1;
  if (!m.trivial && pre_filter && filtered(cnt_in_bin, (int32_t)total, filter_cnt, m.categorical))
    m.trivial = true;
  if (m.trivial) {
    m.sparse_rate = 1.0;
    return;
  }
  m.default_bin = m.bin_of(0.0);
  uint32_t mfb = (uint32_t)first_max(cnt_in_bin);
  const double top_rate = (double)cnt_in_bin[mfb] / (double)total;
  if (mfb != m.default_bin && top_rate < 0.7) mfb = m.default_bin;  // kSparseThreshold
  m.most_freq_bin = mfb;
  m.sparse_rate = (double)cnt_in_bin[mfb] / (double)total;
}

Mapper bin_numeric(std::vector<double> v, int32_t max_bin, int32_t min_data_in_bin,
                   int32_t filter_cnt, bool pre_filter, bool use_missing, bool zero_as_missing,
                   int64_t total) {
  Mapper m;
  const int32_t n_in = (int32_t)v.size();
  v.erase(std::remove_if(v.begin(), v.end(), [](double x) { return std::isnan(x); }), v.end());
  int32_t na_cnt = 0;
  if (!use_missing)
    m.missing = 0;
  else if (zero_as_missing)
    m.missing = 1;
  else if ((int32_t)v.size() == n_in)
    m.missing = 0;
  else {
    na_cnt = n_in - (int32_t)v.size();
    m.missing = 2;
  }
  const int32_t zero_cnt = (int32_t)(total - (int64_t)v.size() - na_cnt);
  Distinct d = fold_distinct(v, zero_cnt);
  m.min_val = d.value.empty() ? 0.0 : d.value.front();
  m.max_val = d.value.empty() ? 0.0 : d.value.back();
  if (m.missing == 2) {
    m.upper = zero_as_one_bin(d, max_bin - 1, total - na_cnt, min_data_in_bin);
    m.upper.push_back(std::numeric_limits<double>::quiet_NaN());
  } else {
    m.upper = zero_as_one_bin(d, max_bin, total, min_data_in_bin);
    if (m.missing == 1 && m.upper.size() == 2) m.missing = 0;
  }
  m.num_bin = (int32_t)m.upper.size();
  std::vector<int32_t> cnt_in_bin(m.num_bin, 0);
  int32_t b = 0;
  for (size_t i = 0; i < d.value.size(); ++i) {
    while (b < m.num_bin - 1 && d.value[i] > m.upper[b]) ++b;
    cnt_in_bin[b] += d.count[i];
  }
  if (m.missing == 2) cnt_in_bin[m.num_bin - 1] = na_cnt;
  finish(m, cnt_in_bin, total, filter_cnt, pre_filter);
  return m;
}

Mapper bin_categorical(std::vector<double> v, int32_t max_bin, int32_t min_data_in_bin,
                       int32_t filter_cnt, bool pre_filter, bool use_missing, bool zero_as_missing,
                       int64_t total) {
  Mapper m;
  m.categorical = true;
  const int32_t n_in = (int32_t)v.size();
  v.erase(std::remove_if(v.begin(), v.end(), [](double x) { return std::isnan(x); }), v.end());
  int32_t na_cnt = 0;
  if (!use_missing)
    m.missing = 0;
  else if (zero_as_missing)
    m.missing = 1;
  else if ((int32_t)v.size() == n_in)
    m.missing = 0;
  else {
    na_cnt = n_in - (int32_t)v.size();
    m.missing = 2;
  }
  const int32_t zero_cnt = (int32_t)(total - (int64_t)v.size() - na_cnt);
  Distinct d = fold_distinct(v, zero_cnt);
  m.min_val = d.value.empty() ? 0.0 : d.value.front();
  m.max_val = d.value.empty() ? 0.0 : d.value.back();
  // integer codes; negative codes count as missing; equal neighbours merge
  std::vector<std::pair<int32_t, int32_t>> cats;  // (count, code)
  for (size_t i = 0; i < d.value.size(); ++i) {
    const int32_t code = (int32_t)d.value[i];
    if (code < 0)
      na_cnt += d.count[i];
    else if (cats.empty() || cats.back().second != code)
      cats.push_back({d.count[i], code});
    else
      cats.back().first += d.count[i];
  }
  m.num_bin = 1;
  std::vector<int32_t> cnt_in_bin;
  const int32_t rest = (int32_t)(total - na_cnt);
  if (rest > 0) {
    std::stable_sort(cats.begin(), cats.end(),
                     [](const std::pair<int32_t, int32_t>& a,
                        const std::pair<int32_t, int32_t>& b) { return a.first > b.first; });
    // (int)(float(rest) * 0.99f + 0.5f): float product, then RoundInt in double
    const float scaled = (float)rest * 0.99f;
    const int32_t cut = (int32_t)((double)scaled + (double)0.5f);
    int32_t distinct = (int32_t)cats.size() + (na_cnt > 0 ? 1 : 0);
    max_bin = std::min(max_bin, distinct);
    m.bin_to_cat.push_back(-1);  // bin 0: the missing-value dummy
    m.cat_to_bin[-1] = 0;
    cnt_in_bin.push_back(0);
    int32_t used = 0;
    size_t c = 0;
    while (c < cats.size() && (used < cut || m.num_bin < max_bin)) {
      if (cats[c].first < min_data_in_bin && c > 1) break;
      m.bin_to_cat.push_back(cats[c].second);
      m.cat_to_bin[cats[c].second] = (uint32_t)m.num_bin;
      used += cats[c].first;
      cnt_in_bin.push_back(cats[c].first);
      ++m.num_bin;
      ++c;
    }
    m.missing = (c == cats.size() && na_cnt == 0) ? 0 : 2;
    cnt_in_bin[0] = (int32_t)(total - used);
  }
  finish(m, cnt_in_bin, total, filter_cnt, pre_filter);
  return m;
}

}  // namespace

extern "C" {

struct OracleBinMapper {
  int32_t num_bin;
  int32_t missing_type;
  int32_t default_bin;
  int32_t most_freq_bin;
  int32_t is_trivial;
  int32_t is_categorical;
  double min_val;
  double max_val;
  double sparse_rate;
};

// BinMapper::find_bin_from_column (numeric) or its categorical counterpart, then
// value_to_bin of every row. upper_out (numeric) or bin_to_cat_out (categorical)
// receive num_bin entries (capacity `cap`); bins_out may be null. Returns 0, or -1
// when `cap` is too small.
int oracle_bin_column(const double* column, int64_t n, int32_t max_bin, int32_t min_data_in_bin,
                      int32_t min_data_in_leaf, int32_t pre_filter, int32_t use_missing,
                      int32_t zero_as_missing, int32_t sample_cnt, int32_t seed,
                      int32_t categorical, OracleBinMapper* out, double* upper_out,
                      int32_t* bin_to_cat_out, int32_t cap, uint32_t* bins_out) {
  const int32_t rows = (int32_t)n;
  const int32_t k = rows < sample_cnt ? rows : sample_cnt;
  Lcg rng(seed);
  const std::vector<int32_t> idx = rng.sample(rows, k);
  std::vector<double> sample(idx.size());
  for (size_t i = 0; i < idx.size(); ++i) sample[i] = column[idx[i]];
  const int64_t total = (int64_t)sample.size();
  // scaled_filter_cnt: min_data_in_leaf scaled from all rows to the sample
  const int32_t filter_cnt =
      rows == 0 ? min_data_in_leaf
                : (int32_t)(((int64_t)min_data_in_leaf * total) / (int64_t)rows);
  Mapper m = categorical
                 ? bin_categorical(std::move(sample), max_bin, min_data_in_bin, filter_cnt,
                                   pre_filter != 0, use_missing != 0, zero_as_missing != 0, total)
                 : bin_numeric(std::move(sample), max_bin, min_data_in_bin, filter_cnt,
                               pre_filter != 0, use_missing != 0, zero_as_missing != 0, total);
  if (m.num_bin > cap) return -1;
  out->num_bin = m.num_bin;
  out->missing_type = m.missing;
  out->default_bin = (int32_t)m.default_bin;
  out->most_freq_bin = (int32_t)m.most_freq_bin;
  out->is_trivial = m.trivial ? 1 : 0;
  out->is_categorical = categorical ? 1 : 0;
  out->min_val = m.min_val;
  out->max_val = m.max_val;
  out->sparse_rate = m.sparse_rate;
  if (categorical) {
    if (bin_to_cat_out) std::copy(m.bin_to_cat.begin(), m.bin_to_cat.end(), bin_to_cat_out);
  } else if (upper_out) {
    std::copy(m.upper.begin(), m.upper.end(), upper_out);
  }
  if (bins_out)
    for (int64_t i = 0; i < n; ++i) bins_out[i] = m.bin_of(column[i]);
  return 0;
}

}  // extern "C"
