#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <vector>

namespace lgbm_b200 {

struct BinMapperHost {
  int32_t num_bin = 0;
  int32_t missing_type = 0;
  int32_t default_bin = 0;
  int32_t most_freq_bin = 0;
  int32_t bin_type = 0;  // 0 numerical, 1 categorical
  bool is_trivial = false;
  double sparse_rate = 0.0;
  double min_val = 0.0;
  double max_val = 0.0;
  std::vector<double> upper;               // numerical: bin upper bounds
  std::vector<int32_t> bin_to_category;    // categorical: bin -> category (bin 0: -1)
  std::map<int32_t, uint32_t> category_to_bin;
  uint32_t value_to_bin(double value) const;
};

BinMapperHost find_bin_numeric(std::vector<double> values, int32_t max_bin,
                               int32_t min_data_in_bin, int32_t min_split_data, bool pre_filter,
                               bool use_missing, bool zero_as_missing, int64_t total_sample_cnt);

BinMapperHost find_bin_categorical(std::vector<double> values, int32_t max_bin,
                                   int32_t min_data_in_bin, int32_t min_split_data,
                                   bool pre_filter, bool use_missing, bool zero_as_missing,
                                   int64_t total_sample_cnt);

// The bin-construction sample of a column of n rows (create_sample_indices,
// bin_mapper.rs:92-95): ascending row indices, shared by every column of that size.
std::shared_ptr<const std::vector<int32_t>> shared_sample_indices(int32_t n, int32_t k,
                                                                  int32_t seed);

BinMapperHost find_bin_from_column(const double* column, int64_t n, int32_t max_bin,
                                   int32_t min_data_in_bin, int32_t min_data_in_leaf,
                                   bool pre_filter, bool use_missing, bool zero_as_missing,
                                   int32_t bin_construct_sample_cnt, int32_t data_random_seed,
                                   bool categorical = false);

}  // namespace lgbm_b200
