// Bin finding on the device for numerical features: BinMapper::find_bin_numeric
// (lgbm-dataset/src/bin_mapper.rs:201-415) of every column's sample, the same sample the
// host draws (create_sample_indices, :92-95; Random::sample, lgbm-core/src/random.rs).
//
//  k_sample_keys   each sampled value -> a 64-bit key in IEEE order (-0.0 as +0.0, every
//                  NaN last), the value riding along; NaNs counted per feature.
//  k_sort_samples  one CTA per feature: stable LSD radix sort of its keys, 8 bits per pass
//                  (passes whose byte is the same for every key are skipped). A stable sort
//                  on keys that equate -0.0 and +0.0 orders the values as the reference's
//                  stable sort_by(partial_cmp) does.
//  k_find_bins     one thread per feature, sequential as the reference: the NaN strip,
//                  distinct values with the zero pseudo-value (bin_mapper.rs:339-375),
//                  find_bin_with_zero_as_one_bin (:938-1013) with greedy_find_bin
//                  (:749-835), the bin counts, need_filter (:690-709), default and most
//                  frequent bin. Every f64 operation is the reference's, in its order
//                  (compiled without contraction), so the bounds are bit-identical to the
//                  host's.
#include <cfloat>
#include <cmath>

#include "kernels.cuh"

namespace lgbm_b200 {

namespace {

constexpr int kSortThreads = 1024;
constexpr double kZeroThr = 1e-35;  // lgbm-core/src/types.rs:35

__device__ __forceinline__ unsigned long long sort_key(double v) {
  if (isnan(v)) return ~0ull;
  if (v == 0.0) v = 0.0;  // -0.0 sorts as +0.0 (they compare equal)
  const unsigned long long b = (unsigned long long)__double_as_longlong(v);
  return (b >> 63) ? ~b : (b | (1ull << 63));
}

__global__ void k_sample_keys(const double* vals, int64_t k, int32_t nf,
                              unsigned long long* keys, int32_t* na_cnt) {
  const int64_t total = k * nf;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const double v = vals[i];
    keys[i] = sort_key(v);
    if (isnan(v)) atomicAdd(&na_cnt[i / k], 1);
  }
}

// Feature blockIdx.x: keys/vals [k] in buffer a (the result ends in a or b; which[] says).
__global__ void __launch_bounds__(kSortThreads, 1)
    k_sort_samples(unsigned long long* keys_a, double* vals_a, unsigned long long* keys_b,
                   double* vals_b, int64_t k, int32_t* which) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t base[256];
  __shared__ uint32_t tcount[256];
  __shared__ uint16_t whist[kSortThreads / 32][256];
  __shared__ int s_skip;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t off = (size_t)blockIdx.x * (size_t)k;
  unsigned long long* ks[2] = {keys_a + off, keys_b + off};
  double* vs[2] = {vals_a + off, vals_b + off};
  int cur = 0;
  const unsigned lt = (1u << lane) - 1u;
  for (int pass = 0; pass < 8; ++pass) {
    const int shift = 8 * pass;
    const unsigned long long* sk = ks[cur];
    const double* sv = vs[cur];
    unsigned long long* dk = ks[cur ^ 1];
    double* dv = vs[cur ^ 1];
    for (int i = tid; i < 256; i += kSortThreads) hist[i] = 0u;
    __syncthreads();
    for (int64_t i = tid; i < k; i += kSortThreads) atomicAdd(&hist[(sk[i] >> shift) & 255u], 1u);
    __syncthreads();
    if (tid == 0) {
      uint32_t run = 0;
      int skip = 0;
      for (int d = 0; d < 256; ++d) {
        base[d] = run;
        run += hist[d];
        if (hist[d] == (uint32_t)k) skip = 1;  // one digit for every key: order unchanged
      }
      s_skip = skip;
    }
    __syncthreads();
    if (s_skip) continue;
    for (int64_t t0 = 0; t0 < k; t0 += kSortThreads) {
      const int64_t i = t0 + tid;
      const bool valid = i < k;
      const unsigned long long key = valid ? sk[i] : 0ull;
      const double val = valid ? sv[i] : 0.0;
      const uint32_t d = valid ? (uint32_t)((key >> shift) & 255u) : 256u;
      uint16_t* wh = &whist[0][0];
      for (int j = tid; j < (kSortThreads / 32) * 256; j += kSortThreads) wh[j] = 0;
      __syncthreads();
      const unsigned peers = __match_any_sync(0xffffffffu, d);
      const int lower = __popc(peers & lt);
      if (valid && lane == __ffs(peers) - 1) whist[warp][d] = (uint16_t)__popc(peers);
      __syncthreads();
      if (tid < 256) {  // exclusive prefix of this digit over the warps, in warp order
        uint32_t run = 0;
        for (int w = 0; w < kSortThreads / 32; ++w) {
          const uint32_t c = whist[w][tid];
          whist[w][tid] = (uint16_t)run;
          run += c;
        }
        tcount[tid] = run;
      }
      __syncthreads();
      if (valid) {
        const uint32_t pos = base[d] + whist[warp][d] + (uint32_t)lower;
        dk[pos] = key;
        dv[pos] = val;
      }
      __syncthreads();
      if (tid < 256) base[tid] += tcount[tid];
      __syncthreads();
    }
    cur ^= 1;
  }
  if (tid == 0) which[blockIdx.x] = cur;
}

__device__ __forceinline__ double next_up(double a) { return nextafter(a, (double)INFINITY); }
__device__ __forceinline__ bool equal_ordered(double a, double b) { return b <= next_up(a); }

// greedy_find_bin (bin_mapper.rs:749-835) over dv[0, nd): its bounds, appended at out[0..),
// count returned. hi / lo: scratch of max_bin entries; big: scratch of nd flags.
// The sequential per-feature loops read one lane's arrays kSeqBlock elements at a time: a
// block's loads are issued together, so a loop waits on memory once per block, not once
// per element (one thread walks ~200k elements per feature).
constexpr int kSeqBlock = 16;

__device__ int greedy_bins(const double* dv, const int32_t* cnt, int32_t nd, int32_t max_bin,
                           int64_t total_cnt, int32_t min_data_in_bin, double* hi, double* lo,
                           uint8_t* big, double* out) {
  int n = 0;
  if (nd <= max_bin) {
    int32_t run = 0;
    for (int32_t i = 0; i + 1 < nd; ++i) {
      run += cnt[i];
      if (run >= min_data_in_bin) {
        const double val = next_up((dv[i] + dv[i + 1]) / 2.0);
        if (n == 0 || !equal_ordered(out[n - 1], val)) {
          out[n++] = val;
          run = 0;
        }
      }
    }
    out[n++] = (double)INFINITY;
    return n;
  }
  if (min_data_in_bin > 0) {
    max_bin = min(max_bin, (int32_t)(total_cnt / (int64_t)min_data_in_bin));
    max_bin = max(max_bin, 1);
  }
  double mean = (double)total_cnt / (double)max_bin;
  int32_t bins_left = max_bin;
  int32_t samples_left = (int32_t)total_cnt;
  for (int32_t i0 = 0; i0 < nd; i0 += kSeqBlock) {
    int32_t c[kSeqBlock];
#pragma unroll
    for (int j = 0; j < kSeqBlock; ++j) c[j] = i0 + j < nd ? cnt[i0 + j] : 0;
#pragma unroll
    for (int j = 0; j < kSeqBlock; ++j) {
      if (i0 + j >= nd) break;
      const bool bg = (double)c[j] >= mean;
      big[i0 + j] = bg ? 1 : 0;
      if (bg) {
        --bins_left;
        samples_left -= c[j];
      }
    }
  }
  mean = (double)samples_left / (double)bins_left;
  for (int32_t b = 0; b < max_bin; ++b) {
    hi[b] = (double)INFINITY;
    lo[b] = (double)INFINITY;
  }
  int32_t nb = 0;
  lo[0] = dv[0];
  int32_t run = 0;
  bool stop = false;
  for (int32_t i0 = 0; i0 + 1 < nd && !stop; i0 += kSeqBlock) {
    // elements i0 .. i0 + kSeqBlock: one past the block for big[i + 1] and dv[i + 1]
    int32_t c[kSeqBlock];
    uint8_t bg[kSeqBlock + 1];
    double v[kSeqBlock + 1];
#pragma unroll
    for (int j = 0; j <= kSeqBlock; ++j) {
      const bool in = i0 + j < nd;
      if (j < kSeqBlock) c[j] = in ? cnt[i0 + j] : 0;
      bg[j] = in ? big[i0 + j] : 0;
      v[j] = in ? dv[i0 + j] : 0.0;
    }
#pragma unroll
    for (int j = 0; j < kSeqBlock; ++j) {
      if (i0 + j + 1 >= nd) break;
      if (!bg[j]) samples_left -= c[j];
      run += c[j];
      // mean * 0.5f: the reference's float literal, exactly 0.5
      if (bg[j] || (double)run >= mean || (bg[j + 1] && (double)run >= fmax(1.0, mean * 0.5))) {
        hi[nb] = v[j];
        ++nb;
        lo[nb] = v[j + 1];
        if (nb >= max_bin - 1) {
          stop = true;
          break;
        }
        run = 0;
        if (!bg[j]) {
          --bins_left;
          mean = (double)samples_left / (double)bins_left;
        }
      }
    }
  }
  ++nb;
  for (int32_t i = 0; i + 1 < nb; ++i) {
    const double val = next_up((hi[i] + lo[i + 1]) / 2.0);
    if (n == 0 || !equal_ordered(out[n - 1], val)) out[n++] = val;
  }
  out[n++] = (double)INFINITY;
  return n;
}

struct FindBinArgs {
  const unsigned long long* keys_a;
  const double* vals_a;
  const double* vals_b;
  const int32_t* which;   // [nf] buffer holding the sorted sample (0: a, 1: b)
  const int32_t* na_cnt;  // [nf]
  int64_t k;              // sample size (every feature)
  int32_t nf;
  int32_t max_bin;
  int32_t min_data_in_bin;
  int32_t filter_cnt;
  int32_t pre_filter;
  int32_t use_missing;
  int32_t zero_as_missing;
  int32_t cap;            // bound slots per feature in `upper`
  double* dv;             // [nf][k + 2] distinct values (scratch)
  int32_t* cnt;           // [nf][k + 2] their counts (scratch)
  uint8_t* big;           // [nf][k + 2] greedy scratch
  double* edges;          // [nf][2][max_bin] greedy scratch
  double* side;           // [nf][max_bin + 1] the positive side's bounds (scratch)
  int32_t* cnt_in_bin;    // [nf][cap] (scratch)
  double* upper;          // [nf][cap] result bounds
  int32_t* meta;          // [nf][6] num_bin, missing_type, default_bin, most_freq_bin, trivial, error
  double* meta_f;         // [nf][3] min_val, max_val, sparse_rate
};

__global__ void k_find_bins(FindBinArgs a) {
  const int f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= a.nf) return;
  const int64_t k = a.k;
  const double* vals = (a.which[f] ? a.vals_b : a.vals_a) + (size_t)f * k;
  double* dv = a.dv + (size_t)f * (k + 2);
  int32_t* cnt = a.cnt + (size_t)f * (k + 2);
  int32_t* m = a.meta + (size_t)f * 6;
  double* up = a.upper + (size_t)f * a.cap;
  // NaN strip and missing type (bin_mapper.rs:213-234); NaNs sorted last
  const int32_t na_in = a.na_cnt[f];
  const int32_t ns = (int32_t)k - na_in;
  int32_t na_cnt = 0, missing;
  if (!a.use_missing)
    missing = 0;
  else if (a.zero_as_missing)
    missing = 1;
  else if (na_in == 0)
    missing = 0;
  else {
    na_cnt = na_in;
    missing = 2;
  }
  const int64_t total = k;
  const int32_t zero_cnt = (int32_t)(total - (int64_t)ns - na_cnt);
  // distinct values with the zero pseudo-value (bin_mapper.rs:339-375)
  int32_t nd = 0;
  if (ns == 0 || (vals[0] > 0.0 && zero_cnt > 0)) {
    dv[nd] = 0.0;
    cnt[nd++] = zero_cnt;
  }
  if (ns > 0) {
    // the open run (its last value and its count) stays in registers and is stored when
    // the next distinct value starts; the sorted values are read a block at a time
    double prev = vals[0], rv = vals[0];
    int32_t rc = 1;
    for (int32_t i0 = 1; i0 < ns; i0 += kSeqBlock) {
      double x[kSeqBlock];
#pragma unroll
      for (int j = 0; j < kSeqBlock; ++j) x[j] = i0 + j < ns ? vals[i0 + j] : 0.0;
#pragma unroll
      for (int j = 0; j < kSeqBlock; ++j) {
        if (i0 + j >= ns) break;
        const double v = x[j];
        if (!equal_ordered(prev, v)) {
          dv[nd] = rv;
          cnt[nd++] = rc;
          if (prev < 0.0 && v > 0.0) {
            dv[nd] = 0.0;
            cnt[nd++] = zero_cnt;
          }
          rc = 0;
        }
        rv = v;
        ++rc;
        prev = v;
      }
    }
    dv[nd] = rv;
    cnt[nd++] = rc;
  }
  if (ns > 0 && vals[ns - 1] < 0.0 && zero_cnt > 0) {
    dv[nd] = 0.0;
    cnt[nd++] = zero_cnt;
  }
  const double min_val = nd > 0 ? dv[0] : 0.0;
  const double max_val = nd > 0 ? dv[nd - 1] : 0.0;
  // find_bin_with_zero_as_one_bin (bin_mapper.rs:938-1013)
  const int32_t mb = missing == 2 ? a.max_bin - 1 : a.max_bin;
  const int64_t tc = missing == 2 ? total - na_cnt : total;
  double* hi = a.edges + (size_t)f * 2 * a.max_bin;
  double* lo = hi + a.max_bin;
  uint8_t* big = a.big + (size_t)f * (k + 2);
  double* side = a.side + (size_t)f * (a.max_bin + 1);
  int32_t neg = 0, zc = 0, pos = 0;
  for (int32_t i0 = 0; i0 < nd; i0 += kSeqBlock) {
    double x[kSeqBlock];
    int32_t c[kSeqBlock];
#pragma unroll
    for (int j = 0; j < kSeqBlock; ++j) {
      x[j] = i0 + j < nd ? dv[i0 + j] : 0.0;
      c[j] = i0 + j < nd ? cnt[i0 + j] : 0;
    }
#pragma unroll
    for (int j = 0; j < kSeqBlock; ++j) {
      if (x[j] <= -kZeroThr)
        neg += c[j];
      else if (x[j] > kZeroThr)
        pos += c[j];
      else
        zc += c[j];
    }
  }
  int32_t first_nonneg = nd;  // dv ascends: the first entry above -kZeroThr, by bisection
  {
    int32_t l = 0, r = nd;
    while (l < r) {
      const int32_t m = (l + r) / 2;
      if (dv[m] > -kZeroThr)
        r = m;
      else
        l = m + 1;
    }
    first_nonneg = l;
  }
  int nu = 0;
  if (first_nonneg > 0 && mb > 1) {
    int32_t neg_bins = (int32_t)((double)neg / (double)((int32_t)tc - zc) * (double)(mb - 1));
    neg_bins = max(neg_bins, 1);
    nu = greedy_bins(dv, cnt, first_nonneg, neg_bins, neg, a.min_data_in_bin, hi, lo, big, up);
    if (nu > 0) up[nu - 1] = -kZeroThr;
  }
  int32_t first_pos = -1;
  {
    int32_t l = first_nonneg, r = nd;  // the first entry above kZeroThr, by bisection
    while (l < r) {
      const int32_t m = (l + r) / 2;
      if (dv[m] > kZeroThr)
        r = m;
      else
        l = m + 1;
    }
    if (l < nd) first_pos = l;
  }
  const int32_t pos_bins = mb - 1 - nu;
  if (first_pos >= 0 && pos_bins > 0) {
    const int ns2 = greedy_bins(dv + first_pos, cnt + first_pos, nd - first_pos, pos_bins, pos,
                                a.min_data_in_bin, hi, lo, big, side);
    up[nu++] = kZeroThr;
    for (int i = 0; i < ns2; ++i) up[nu++] = side[i];
  } else {
    up[nu++] = (double)INFINITY;
  }
  if (missing == 1 && nu == 2) missing = 0;
  if (missing == 2) up[nu++] = (double)NAN;
  const int32_t num_bin = nu;
  // bin counts of the sample (bin_mapper.rs:396-408)
  int32_t* cib = a.cnt_in_bin + (size_t)f * a.cap;
  for (int b = 0; b < num_bin; ++b) cib[b] = 0;
  {
    // the current bin's count in a register, stored when the bin advances
    int32_t b = 0, acc = 0;
    double ub = up[0];
    for (int32_t i0 = 0; i0 < nd; i0 += kSeqBlock) {
      double x[kSeqBlock];
      int32_t c[kSeqBlock];
#pragma unroll
      for (int j = 0; j < kSeqBlock; ++j) {
        x[j] = i0 + j < nd ? dv[i0 + j] : 0.0;
        c[j] = i0 + j < nd ? cnt[i0 + j] : 0;
      }
#pragma unroll
      for (int j = 0; j < kSeqBlock; ++j) {
        if (i0 + j >= nd) break;
        if (x[j] > ub && b < num_bin - 1) {
          cib[b] += acc;
          acc = 0;
          while (x[j] > up[b] && b < num_bin - 1) ++b;
          ub = up[b];
        }
        acc += c[j];
      }
    }
    cib[b] += acc;
    if (missing == 2) cib[num_bin - 1] = na_cnt;
  }
  bool trivial = num_bin <= 1;
  if (!trivial && a.pre_filter) {  // need_filter (bin_mapper.rs:690-709)
    bool filt = true;
    int32_t left = 0;
    for (int b = 0; b + 1 < num_bin; ++b) {
      left += cib[b];
      if (left >= a.filter_cnt && (int32_t)total - left >= a.filter_cnt) {
        filt = false;
        break;
      }
    }
    trivial = filt;
  }
  int32_t default_bin = 0, mfb = 0;
  double sparse = 1.0;
  if (!trivial) {
    // value_to_bin(0.0) (bin_mapper.rs:148-199)
    int32_t l = 0, r = num_bin - 1 - (missing == 2 ? 1 : 0);
    while (l < r) {
      const int32_t mid = (r + l - 1) / 2;
      if (0.0 <= up[mid])
        r = mid;
      else
        l = mid + 1;
    }
    default_bin = l;
    int32_t best = 0;
    for (int b = 1; b < num_bin; ++b)
      if (cib[b] > cib[best]) best = b;
    mfb = best;
    if (mfb != default_bin && (double)cib[mfb] / (double)total < 0.7) mfb = default_bin;
    sparse = (double)cib[mfb] / (double)total;
  }
  m[0] = num_bin;
  m[1] = missing;
  m[2] = default_bin;
  m[3] = mfb;
  m[4] = trivial ? 1 : 0;
  m[5] = 0;
  a.meta_f[(size_t)f * 3 + 0] = min_val;
  a.meta_f[(size_t)f * 3 + 1] = max_val;
  a.meta_f[(size_t)f * 3 + 2] = sparse;
}

}  // namespace

void launch_find_bins(const FindBinsDev& d, cudaStream_t st) {
  const int grid_keys = 1024;
  k_sample_keys<<<grid_keys, 256, 0, st>>>(d.vals_a, d.k, d.nf, d.keys_a, d.na_cnt);
  k_sort_samples<<<d.nf, kSortThreads, 0, st>>>(d.keys_a, d.vals_a, d.keys_b, d.vals_b, d.k,
                                                d.which);
  FindBinArgs a;
  a.keys_a = d.keys_a;
  a.vals_a = d.vals_a;
  a.vals_b = d.vals_b;
  a.which = d.which;
  a.na_cnt = d.na_cnt;
  a.k = d.k;
  a.nf = d.nf;
  a.max_bin = d.max_bin;
  a.min_data_in_bin = d.min_data_in_bin;
  a.filter_cnt = d.filter_cnt;
  a.pre_filter = d.pre_filter;
  a.use_missing = d.use_missing;
  a.zero_as_missing = d.zero_as_missing;
  a.cap = d.cap;
  a.dv = d.dv;
  a.cnt = d.cnt;
  a.big = d.big;
  a.edges = d.edges;
  a.side = d.side;
  a.cnt_in_bin = d.cnt_in_bin;
  a.upper = d.upper;
  a.meta = d.meta;
  a.meta_f = d.meta_f;
  k_find_bins<<<(d.nf + 63) / 64, 64, 0, st>>>(a);
}

}  // namespace lgbm_b200
