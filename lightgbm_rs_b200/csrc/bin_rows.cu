// Device construction of the row-major u8 bin matrix from feature-major columns: either
// bins already computed (range-checked here), or raw feature values binned here with
// the host-found bin mappers (BinMapper::value_to_bin, lgbm-dataset/src/bin_mapper.rs:
// 148-199). One thread handles one row and 16 consecutive features (32 in a 4-bit
// matrix): coalesced column reads (consecutive threads hold consecutive rows) and one
// 16-byte store of the row's bins.
#include <cmath>
#include <type_traits>

#include "kernels.cuh"

namespace lgbm_b200 {

namespace {

constexpr int kBinRowThreads = 256;

__device__ __forceinline__ uint32_t numeric_bin(const DevBinFeature& bf, const double* upper,
                                                double v) {
  if (isnan(v)) {
    if (bf.missing_type == 2) return (uint32_t)(bf.num_bin - 1);
    v = 0.0;
  }
  int32_t l = 0, r = bf.num_bin - 1;
  if (bf.missing_type == 2) r -= 1;
  const double* up = upper + bf.off;
  while (l < r) {
    const int32_t m = (r + l - 1) / 2;
    if (v <= __ldg(up + m))
      r = m;
    else
      l = m + 1;
  }
  return (uint32_t)l;
}

// categorical value_to_bin: the integer category's bin; NaN, negative and unseen
// categories go to bin 0. cat_keys holds the feature's categories in ascending order.
__device__ __forceinline__ uint32_t categorical_bin(const DevBinFeature& bf,
                                                    const int32_t* cat_keys,
                                                    const uint8_t* cat_bins, double v) {
  if (isnan(v)) return 0;
  const int32_t iv = (int32_t)v;  // truncation toward zero, saturating
  if (iv < 0) return 0;
  int32_t l = 0, r = bf.n_cat;
  const int32_t* k = cat_keys + bf.off;
  while (l < r) {
    const int32_t m = (l + r) >> 1;
    if (__ldg(k + m) < iv)
      l = m + 1;
    else
      r = m;
  }
  return (l < bf.n_cat && __ldg(k + l) == iv) ? cat_bins[bf.off + l] : 0u;
}

template <typename T>
__device__ __forceinline__ uint32_t to_bin(const BinRowsDev& d, int f, T v, int64_t row,
                                           unsigned long long* first_bad) {
  const DevBinFeature bf = d.feats[f];
  if constexpr (sizeof(T) <= 4 && !std::is_floating_point<T>::value) {
    const uint32_t b = (uint32_t)v;
    if (b >= (uint32_t)bf.num_bin) {
      atomicMin(first_bad, (unsigned long long)row * (unsigned long long)d.num_features + f);
      return 0;
    }
    return b;
  } else {
    const double x = (double)v;
    return bf.bin_type == 1 ? categorical_bin(bf, d.cat_keys, d.cat_bins, x)
                            : numeric_bin(bf, d.upper, x);
  }
}

template <typename T>
__global__ void __launch_bounds__(kBinRowThreads) k_bin_rows(BinRowsDev d, const T* cols,
                                                            int64_t col_stride, int64_t n,
                                                            int64_t row0, uint8_t* out) {
  const int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (r >= n) return;
  const int g = blockIdx.y;
  uint32_t w[4] = {0u, 0u, 0u, 0u};
  if (d.packed4) {  // 32 features per 16-byte chunk, two 4-bit bins per byte
    for (int j = 0; j < 32; ++j) {
      const int f = g * 32 + j;
      if (f >= d.num_features) break;
      const uint32_t b = to_bin<T>(d, f, cols[(int64_t)f * col_stride + r], row0 + r,
                                   d.first_bad);
      w[j >> 3] |= (b & 0xfu) << (4 * (j & 7));
    }
  } else {
    for (int j = 0; j < 16; ++j) {
      const int f = g * 16 + j;
      if (f >= d.num_features) break;
      const uint32_t b = to_bin<T>(d, f, cols[(int64_t)f * col_stride + r], row0 + r,
                                   d.first_bad);
      w[j >> 2] |= (b & 0xffu) << (8 * (j & 3));
    }
  }
  *reinterpret_cast<uint4*>(out + r * d.stride + g * 16) = make_uint4(w[0], w[1], w[2], w[3]);
}

}  // namespace

void launch_bin_rows(const BinRowsDev& d, int kind, const void* cols, int64_t col_stride,
                     int64_t n, int64_t row0, uint8_t* out, cudaStream_t st) {
  if (n <= 0) return;
  const dim3 grid((unsigned)((n + kBinRowThreads - 1) / kBinRowThreads), d.stride / 16);
  switch (kind) {
    case kBinRowsU8:
      k_bin_rows<uint8_t><<<grid, kBinRowThreads, 0, st>>>(
          d, (const uint8_t*)cols, col_stride, n, row0, out);
      break;
    case kBinRowsU16:
      k_bin_rows<uint16_t><<<grid, kBinRowThreads, 0, st>>>(
          d, (const uint16_t*)cols, col_stride, n, row0, out);
      break;
    case kBinRowsU32:
      k_bin_rows<uint32_t><<<grid, kBinRowThreads, 0, st>>>(
          d, (const uint32_t*)cols, col_stride, n, row0, out);
      break;
    case kBinRowsF32:
      k_bin_rows<float><<<grid, kBinRowThreads, 0, st>>>(d, (const float*)cols, col_stride, n,
                                                         row0, out);
      break;
    default:
      k_bin_rows<double><<<grid, kBinRowThreads, 0, st>>>(d, (const double*)cols, col_stride,
                                                          n, row0, out);
      break;
  }
}

}  // namespace lgbm_b200
