// Host-side feature binning: raw f64 column -> bin upper bounds + per-row bins.
//
// Restates BinMapper::find_bin_from_column / find_bin_numeric / value_to_bin of
// the reference (crates/lgbm-dataset/src/bin_mapper.rs:45-1043) and its row
// sampler Random::sample (crates/lgbm-core/src/random.rs). Binning runs once
// per dataset on the host, exactly as in the reference facade
// (crates/lgbm/src/booster.rs:381-540); the bins then live on the device.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <limits>
#include <memory>
#include <mutex>
#include <set>
#include <vector>

#include "binning.h"

namespace lgbm_b200 {
namespace {

const double kZeroThreshold = 1e-35;  // lgbm-core/src/types.rs:35

// C++ LightGBM's LCG (lgbm-core/src/random.rs).
struct Random {
  uint32_t x;
  explicit Random(int32_t seed) : x((uint32_t)seed) {}
  int32_t rand_int16() {
    x = x * 214013u + 2531011u;
    return (int32_t)((x >> 16) & 0x7FFF);
  }
  int32_t rand_int32() {
    x = x * 214013u + 2531011u;
    return (int32_t)(x & 0x7FFFFFFF);
  }
  int32_t next_int(int32_t lo, int32_t hi) { return rand_int32() % (hi - lo) + lo; }
  float next_float() { return (float)rand_int16() / 32768.0f; }
  std::vector<int32_t> sample(int32_t n, int32_t k) {
    std::vector<int32_t> ret;
    if (k > n || k <= 0) return ret;
    if (k == n) {
      for (int32_t i = 0; i < n; ++i) ret.push_back(i);
      return ret;
    }
    if (k > 1 && (double)k > ((double)n / std::log2((double)k))) {
      for (int32_t i = 0; i < n; ++i) {
        double prob = (double)(k - (int32_t)ret.size()) / (double)(n - i);
        if ((double)next_float() < prob) ret.push_back(i);
      }
      return ret;
    }
    std::set<int32_t> s;
    for (int32_t r = n - k; r < n; ++r) {
      int32_t v = next_int(0, r + 1);
      if (!s.insert(v).second) s.insert(r);
    }
    ret.assign(s.begin(), s.end());
    return ret;
  }
};

inline double next_up(double a) { return std::nextafter(a, std::numeric_limits<double>::infinity()); }
inline double upper_bound_of(double a) { return next_up(a); }                // bin_mapper.rs:22-25
inline bool check_equal_ordered(double a, double b) { return b <= next_up(a); }  // :27-30

// Every column of a dataset draws the same sample (same row count, sample size and seed:
// create_sample_indices, bin_mapper.rs:92-95), so the indices of the last (n, k, seed) are
// kept and shared by the columns instead of being drawn again for each one.
std::shared_ptr<const std::vector<int32_t>> sample_indices(int32_t n, int32_t k, int32_t seed) {
  static std::mutex mu;
  static int32_t key_n = -1, key_k = -1, key_seed = 0;
  static std::shared_ptr<const std::vector<int32_t>> cached;
  std::lock_guard<std::mutex> lock(mu);
  if (!cached || key_n != n || key_k != k || key_seed != seed) {
    Random rnd(seed);
    cached = std::make_shared<const std::vector<int32_t>>(rnd.sample(n, k));
    key_n = n;
    key_k = k;
    key_seed = seed;
  }
  return cached;
}

// greedy_find_bin (bin_mapper.rs:711-790)
std::vector<double> greedy_find_bin(const double* dv, const int32_t* cnt, int32_t nd,
                                    int32_t max_bin, int64_t total_cnt, int32_t min_data_in_bin) {
  std::vector<double> ub;
  if (nd <= max_bin) {
    int32_t cur = 0;
    for (int32_t i = 0; i < nd - 1; ++i) {
      cur += cnt[i];
      if (cur >= min_data_in_bin) {
        double val = upper_bound_of((dv[i] + dv[i + 1]) / 2.0);
        if (ub.empty() || !check_equal_ordered(ub.back(), val)) {
          ub.push_back(val);
          cur = 0;
        }
      }
    }
    ub.push_back(std::numeric_limits<double>::infinity());
    return ub;
  }
  if (min_data_in_bin > 0) {
    max_bin = std::min(max_bin, (int32_t)(total_cnt / (int64_t)min_data_in_bin));
    max_bin = std::max(max_bin, 1);
  }
  double mean_bin_size = (double)total_cnt / (double)max_bin;
  int32_t rest_bin_cnt = max_bin;
  int32_t rest_sample_cnt = (int32_t)total_cnt;
  std::vector<char> big(nd, 0);
  for (int32_t i = 0; i < nd; ++i) {
    if ((double)cnt[i] >= mean_bin_size) {
      big[i] = 1;
      rest_bin_cnt -= 1;
      rest_sample_cnt -= cnt[i];
    }
  }
  mean_bin_size = (double)rest_sample_cnt / (double)rest_bin_cnt;
  std::vector<double> upper(max_bin, std::numeric_limits<double>::infinity());
  std::vector<double> lower(max_bin, std::numeric_limits<double>::infinity());
  size_t bin_cnt = 0;
  lower[bin_cnt] = dv[0];
  int32_t cur = 0;
  for (int32_t i = 0; i < nd - 1; ++i) {
    if (!big[i]) rest_sample_cnt -= cnt[i];
    cur += cnt[i];
    if (big[i] || (double)cur >= mean_bin_size ||
        (big[i + 1] && (double)cur >= std::max(1.0, mean_bin_size * (double)0.5f))) {
      upper[bin_cnt] = dv[i];
      bin_cnt += 1;
      lower[bin_cnt] = dv[i + 1];
      if ((int32_t)bin_cnt >= max_bin - 1) break;
      cur = 0;
      if (!big[i]) {
        rest_bin_cnt -= 1;
        mean_bin_size = (double)rest_sample_cnt / (double)rest_bin_cnt;
      }
    }
  }
  bin_cnt += 1;
  for (size_t i = 0; i + 1 < bin_cnt; ++i) {
    double val = upper_bound_of((upper[i] + lower[i + 1]) / 2.0);
    if (ub.empty() || !check_equal_ordered(ub.back(), val)) ub.push_back(val);
  }
  ub.push_back(std::numeric_limits<double>::infinity());
  return ub;
}

// find_bin_with_zero_as_one_bin (bin_mapper.rs:944-1015)
std::vector<double> find_bin_zero_as_one(const std::vector<double>& dv,
                                         const std::vector<int32_t>& cnt, int32_t max_bin,
                                         int64_t total_sample_cnt, int32_t min_data_in_bin) {
  const int32_t nd = (int32_t)dv.size();
  std::vector<double> ub;
  int32_t left_cnt_data = 0, cnt_zero = 0, right_cnt_data = 0;
  for (int32_t i = 0; i < nd; ++i) {
    if (dv[i] <= -kZeroThreshold)
      left_cnt_data += cnt[i];
    else if (dv[i] > kZeroThreshold)
      right_cnt_data += cnt[i];
    else
      cnt_zero += cnt[i];
  }
  int32_t left_cnt = -1;
  for (int32_t i = 0; i < nd; ++i)
    if (dv[i] > -kZeroThreshold) {
      left_cnt = i;
      break;
    }
  if (left_cnt < 0) left_cnt = nd;
  if (left_cnt > 0 && max_bin > 1) {
    int32_t left_max_bin = (int32_t)((double)left_cnt_data /
                                     (double)((int32_t)total_sample_cnt - cnt_zero) *
                                     (double)(max_bin - 1));
    left_max_bin = std::max(left_max_bin, 1);
    ub = greedy_find_bin(dv.data(), cnt.data(), left_cnt, left_max_bin, left_cnt_data,
                         min_data_in_bin);
    if (!ub.empty()) ub.back() = -kZeroThreshold;
  }
  int32_t right_start = -1;
  for (int32_t i = left_cnt; i < nd; ++i)
    if (dv[i] > kZeroThreshold) {
      right_start = i;
      break;
    }
  const int32_t right_max_bin = max_bin - 1 - (int32_t)ub.size();
  if (right_start >= 0 && right_max_bin > 0) {
    std::vector<double> rb =
        greedy_find_bin(dv.data() + right_start, cnt.data() + right_start, nd - right_start,
                        right_max_bin, right_cnt_data, min_data_in_bin);
    ub.push_back(kZeroThreshold);
    ub.insert(ub.end(), rb.begin(), rb.end());
  } else {
    ub.push_back(std::numeric_limits<double>::infinity());
  }
  return ub;
}

// need_filter (bin_mapper.rs:690-709), numerical case.
bool need_filter(const std::vector<int32_t>& cnt_in_bin, int32_t total_cnt, int32_t filter_cnt) {
  int32_t sum_left = 0;
  for (size_t i = 0; i + 1 < cnt_in_bin.size(); ++i) {
    sum_left += cnt_in_bin[i];
    if (sum_left >= filter_cnt && total_cnt - sum_left >= filter_cnt) return false;
  }
  return true;
}

}  // namespace

uint32_t BinMapperHost::value_to_bin(double value) const {  // bin_mapper.rs:148-199
  if (std::isnan(value)) {
    if (bin_type == 1) return 0;
    if (missing_type == 2) return (uint32_t)(num_bin - 1);
    value = 0.0;
  }
  if (bin_type == 1) {
    // categorical: truncate to int; negatives and unseen categories -> bin 0
    const int32_t iv = (int32_t)value;
    if (iv < 0) return 0;
    auto it = category_to_bin.find(iv);
    return it == category_to_bin.end() ? 0u : it->second;
  }
  int32_t l = 0, r = num_bin - 1;
  if (missing_type == 2) r -= 1;
  while (l < r) {
    int32_t m = (r + l - 1) / 2;
    if (value <= upper[m])
      r = m;
    else
      l = m + 1;
  }
  return (uint32_t)l;
}

namespace {

// Sorted distinct values with counts, plus the zero pseudo-value for the rows the
// sample did not hold (bin_mapper.rs:339-375 numeric prefix, shared with categorical).
void distinct_with_zero(std::vector<double>& values, int32_t zero_cnt, std::vector<double>* dv,
                        std::vector<int32_t>* counts) {
  const size_t ns = values.size();
  // stable, as the reference's sort_by (bin_mapper.rs:250): -0.0 and 0.0 keep input order
  std::stable_sort(values.begin(), values.end());
  if (ns == 0 || (values[0] > 0.0 && zero_cnt > 0)) {
    dv->push_back(0.0);
    counts->push_back(zero_cnt);
  }
  if (ns > 0) {
    dv->push_back(values[0]);
    counts->push_back(1);
  }
  for (size_t i = 1; i < ns; ++i) {
    if (!check_equal_ordered(values[i - 1], values[i])) {
      if (values[i - 1] < 0.0 && values[i] > 0.0) {
        dv->push_back(0.0);
        counts->push_back(zero_cnt);
      }
      dv->push_back(values[i]);
      counts->push_back(1);
    } else {
      dv->back() = values[i];
      counts->back() += 1;
    }
  }
  if (ns > 0 && values[ns - 1] < 0.0 && zero_cnt > 0) {
    dv->push_back(0.0);
    counts->push_back(zero_cnt);
  }
}

// need_filter (bin_mapper.rs:724-746), categorical case: only one- or two-bin
// features can be filtered.
bool need_filter_categorical(const std::vector<int32_t>& cnt_in_bin, int32_t total_cnt,
                             int32_t filter_cnt) {
  if (cnt_in_bin.size() > 2) return false;
  for (size_t i = 0; i + 1 < cnt_in_bin.size(); ++i) {
    const int32_t left = cnt_in_bin[i];
    if (left >= filter_cnt && total_cnt - left >= filter_cnt) return false;
  }
  return true;
}

}  // namespace

// find_bin_numeric (bin_mapper.rs:201-415)
BinMapperHost find_bin_numeric(std::vector<double> values, int32_t max_bin,
                               int32_t min_data_in_bin, int32_t min_split_data, bool pre_filter,
                               bool use_missing, bool zero_as_missing, int64_t total_sample_cnt) {
  const int32_t num_in = (int32_t)values.size();
  size_t non_na = 0;
  for (size_t i = 0; i < values.size(); ++i)
    if (!std::isnan(values[i])) values[non_na++] = values[i];
  int32_t na_cnt = 0;
  int32_t missing_type;
  if (!use_missing)
    missing_type = 0;
  else if (zero_as_missing)
    missing_type = 1;
  else if ((int32_t)non_na == num_in)
    missing_type = 0;
  else {
    na_cnt = num_in - (int32_t)non_na;
    missing_type = 2;
  }
  const size_t ns = non_na;
  values.resize(ns);
  const int32_t zero_cnt = (int32_t)(total_sample_cnt - (int64_t)ns - na_cnt);
  std::vector<double> dv;
  std::vector<int32_t> counts;
  distinct_with_zero(values, zero_cnt, &dv, &counts);
  BinMapperHost m;
  m.min_val = dv.empty() ? 0.0 : dv.front();
  m.max_val = dv.empty() ? 0.0 : dv.back();
  if (missing_type == 1) {
    m.upper = find_bin_zero_as_one(dv, counts, max_bin, total_sample_cnt, min_data_in_bin);
    if (m.upper.size() == 2) missing_type = 0;
  } else if (missing_type == 0) {
    m.upper = find_bin_zero_as_one(dv, counts, max_bin, total_sample_cnt, min_data_in_bin);
  } else {
    m.upper = find_bin_zero_as_one(dv, counts, max_bin - 1, total_sample_cnt - na_cnt,
                                   min_data_in_bin);
    m.upper.push_back(std::numeric_limits<double>::quiet_NaN());
  }
  m.missing_type = missing_type;
  m.num_bin = (int32_t)m.upper.size();
  std::vector<int32_t> cnt_in_bin(m.num_bin, 0);
  {
    size_t ib = 0;
    for (size_t i = 0; i < dv.size(); ++i) {
      while (dv[i] > m.upper[ib] && ib < (size_t)(m.num_bin - 1)) ++ib;
      cnt_in_bin[ib] += counts[i];
    }
    if (missing_type == 2) cnt_in_bin[m.num_bin - 1] = na_cnt;
  }
  bool trivial = m.num_bin <= 1;
  if (!trivial && pre_filter && need_filter(cnt_in_bin, (int32_t)total_sample_cnt, min_split_data))
    trivial = true;
  if (!trivial) {
    const uint32_t default_bin = m.value_to_bin(0.0);
    size_t best = 0;
    for (size_t i = 1; i < cnt_in_bin.size(); ++i)
      if (cnt_in_bin[i] > cnt_in_bin[best]) best = i;
    uint32_t mfb = (uint32_t)best;
    const double max_sparse = (double)cnt_in_bin[mfb] / (double)total_sample_cnt;
    if (mfb != default_bin && max_sparse < 0.7) mfb = default_bin;
    m.sparse_rate = (double)cnt_in_bin[mfb] / (double)total_sample_cnt;
    m.default_bin = (int32_t)default_bin;
    m.most_freq_bin = (int32_t)mfb;
  } else {
    m.sparse_rate = 1.0;
    m.default_bin = 0;
    m.most_freq_bin = 0;
  }
  m.is_trivial = trivial;
  return m;
}

// find_bin_categorical (bin_mapper.rs:416-641): categories by descending sample count
// (stable: ties keep ascending category order), kept until 99 % of the non-missing
// sample is covered and max_bin is reached; rare categories stop the fold at
// min_data_in_bin. Bin 0 is the dummy bin of NaN, negative and unseen values.
BinMapperHost find_bin_categorical(std::vector<double> values, int32_t max_bin,
                                   int32_t min_data_in_bin, int32_t min_split_data,
                                   bool pre_filter, bool use_missing, bool zero_as_missing,
                                   int64_t total_sample_cnt) {
  const int32_t num_in = (int32_t)values.size();
  size_t non_na = 0;
  for (size_t i = 0; i < values.size(); ++i)
    if (!std::isnan(values[i])) values[non_na++] = values[i];
  int32_t na_cnt = 0;
  int32_t missing_type;
  if (!use_missing)
    missing_type = 0;
  else if (zero_as_missing)
    missing_type = 1;
  else if ((int32_t)non_na == num_in)
    missing_type = 0;
  else {
    na_cnt = num_in - (int32_t)non_na;
    missing_type = 2;
  }
  values.resize(non_na);
  const int32_t zero_cnt = (int32_t)(total_sample_cnt - (int64_t)non_na - na_cnt);
  std::vector<double> dv;
  std::vector<int32_t> counts;
  distinct_with_zero(values, zero_cnt, &dv, &counts);
  BinMapperHost m;
  m.bin_type = 1;
  m.min_val = dv.empty() ? 0.0 : dv.front();
  m.max_val = dv.empty() ? 0.0 : dv.back();
  // integer categories (negatives count as missing), equal neighbours merged
  std::vector<int32_t> cats, cat_cnt;
  for (size_t i = 0; i < dv.size(); ++i) {
    const int32_t v = (int32_t)dv[i];
    if (v < 0) {
      na_cnt += counts[i];
    } else if (cats.empty() || v != cats.back()) {
      cats.push_back(v);
      cat_cnt.push_back(counts[i]);
    } else {
      cat_cnt.back() += counts[i];
    }
  }
  m.num_bin = 1;
  std::vector<int32_t> cnt_in_bin;
  int32_t used_cnt = 0;
  const int32_t rest_cnt = (int32_t)(total_sample_cnt - na_cnt);
  if (rest_cnt > 0) {
    std::vector<size_t> order(cats.size());
    for (size_t i = 0; i < order.size(); ++i) order[i] = i;
    std::stable_sort(order.begin(), order.end(),
                     [&](size_t a, size_t b) { return cat_cnt[a] > cat_cnt[b]; });
    std::vector<int32_t> sc(cats.size()), sn(cats.size());
    for (size_t i = 0; i < order.size(); ++i) {
      sc[i] = cats[order[i]];
      sn[i] = cat_cnt[order[i]];
    }
    // cut_cnt = RoundInt((total - na) * 0.99f): the multiply is in f32
    const float scaled = (float)rest_cnt * 0.99f;
    const int32_t cut_cnt = (int32_t)((double)scaled + (double)0.5f);
    int32_t distinct_cnt = (int32_t)sc.size() + (na_cnt > 0 ? 1 : 0);
    max_bin = std::min(max_bin, distinct_cnt);
    m.bin_to_category.push_back(-1);
    m.category_to_bin[-1] = 0;
    cnt_in_bin.push_back(0);
    size_t idx = 0;
    while (idx < sc.size() && (used_cnt < cut_cnt || m.num_bin < max_bin)) {
      if (sn[idx] < min_data_in_bin && idx > 1) break;
      m.bin_to_category.push_back(sc[idx]);
      m.category_to_bin[sc[idx]] = (uint32_t)m.num_bin;
      used_cnt += sn[idx];
      cnt_in_bin.push_back(sn[idx]);
      m.num_bin += 1;
      ++idx;
    }
    missing_type = (idx == sc.size() && na_cnt == 0) ? 0 : 2;
    cnt_in_bin[0] = (int32_t)(total_sample_cnt - used_cnt);
  }
  m.missing_type = missing_type;
  bool trivial = m.num_bin <= 1;
  if (!trivial && pre_filter &&
      need_filter_categorical(cnt_in_bin, (int32_t)total_sample_cnt, min_split_data))
    trivial = true;
  if (!trivial) {
    const uint32_t default_bin = m.value_to_bin(0.0);
    size_t best = 0;
    for (size_t i = 1; i < cnt_in_bin.size(); ++i)
      if (cnt_in_bin[i] > cnt_in_bin[best]) best = i;
    uint32_t mfb = (uint32_t)best;
    const double max_sparse = (double)cnt_in_bin[mfb] / (double)total_sample_cnt;
    if (mfb != default_bin && max_sparse < 0.7) mfb = default_bin;
    m.sparse_rate = (double)cnt_in_bin[mfb] / (double)total_sample_cnt;
    m.default_bin = (int32_t)default_bin;
    m.most_freq_bin = (int32_t)mfb;
  } else {
    m.sparse_rate = 1.0;
  }
  m.is_trivial = trivial;
  return m;
}

std::shared_ptr<const std::vector<int32_t>> shared_sample_indices(int32_t n, int32_t k,
                                                                  int32_t seed) {
  return sample_indices(n, k, seed);
}

// find_bin_from_column (bin_mapper.rs:642-675)
BinMapperHost find_bin_from_column(const double* column, int64_t n, int32_t max_bin,
                                   int32_t min_data_in_bin, int32_t min_data_in_leaf,
                                   bool pre_filter, bool use_missing, bool zero_as_missing,
                                   int32_t bin_construct_sample_cnt, int32_t data_random_seed,
                                   bool categorical) {
  const int32_t total = (int32_t)n;
  const int32_t k = total < bin_construct_sample_cnt ? total : bin_construct_sample_cnt;
  const std::shared_ptr<const std::vector<int32_t>> ip = sample_indices(total, k, data_random_seed);
  const std::vector<int32_t>& idx = *ip;
  std::vector<double> sampled(idx.size());
  for (size_t i = 0; i < idx.size(); ++i) sampled[i] = column[idx[i]];
  const int64_t total_sample_cnt = (int64_t)sampled.size();
  // scaled_filter_cnt (bin_mapper.rs:684-689)
  const int32_t filter_cnt =
      total == 0 ? min_data_in_leaf
                 : (int32_t)(((int64_t)min_data_in_leaf * total_sample_cnt) / (int64_t)total);
  if (categorical)
    return find_bin_categorical(std::move(sampled), max_bin, min_data_in_bin, filter_cnt,
                                pre_filter, use_missing, zero_as_missing, total_sample_cnt);
  return find_bin_numeric(std::move(sampled), max_bin, min_data_in_bin, filter_cnt, pre_filter,
                          use_missing, zero_as_missing, total_sample_cnt);
}

}  // namespace lgbm_b200
