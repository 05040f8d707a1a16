// Batch prediction from raw feature values: one thread per row walks every tree of the
// ensemble in order (GbdtModel predict, lgbm-model/src/predict.rs; Tree::get_leaf and its
// decisions, lgbm-model/src/tree.rs:173-300).
#include <cmath>

#include "kernels.cuh"

namespace lgbm_b200 {

namespace {

constexpr int kPredThreads = 256;

// tree.rs:173-176 is_zero: |fval| <= kZeroThreshold
__device__ __forceinline__ bool pred_is_zero(double v) { return v >= -1e-35 && v <= 1e-35; }

// The next node from `node` for feature value `fval` (tree.rs:193-246): numerical
// decisions send missing values (NaN under missing type NaN, zero under missing type
// Zero) to the default side and otherwise compare fval <= threshold; categorical
// decisions send NaN and negative values right and look the integer category up in the
// node's bitset of real categories.
__device__ __forceinline__ int32_t pred_decide(const PredModelDev& m, const PredNode& nd,
                                               double fval) {
  if (nd.dt & 1) {
    if (isnan(fval)) return nd.right;
    const int32_t iv = (int32_t)fval;
    if (iv < 0) return nd.right;
    const int32_t c = nd.cat;
    const int32_t lo = m.cat_boundaries[c], hi = m.cat_boundaries[c + 1];
    const int32_t w = iv >> 5;
    const bool in = w < hi - lo && ((m.cat_threshold[lo + w] >> (iv & 31)) & 1u);
    return in ? nd.left : nd.right;
  }
  const int mt = (nd.dt >> 2) & 3;
  if (isnan(fval) && mt != 2) fval = 0.0;
  if ((mt == 1 && pred_is_zero(fval)) || (mt == 2 && isnan(fval)))
    return (nd.dt & 2) ? nd.left : nd.right;
  return fval <= nd.threshold ? nd.left : nd.right;
}

__global__ void __launch_bounds__(kPredThreads) k_predict(PredModelDev m, const double* rows,
                                                          int64_t n, int32_t raw,
                                                          double* out) {
  const int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (r >= n) return;
  const double* x = rows + r * m.num_features;
  double acc = 0.0;
  for (int32_t t = 0; t < m.num_trees; ++t) {
    const int32_t nb = m.node_offset[t];
    const int32_t nn = m.node_offset[t + 1] - nb;
    int32_t node = nn > 0 ? 0 : -1;  // a one-leaf tree is its leaf 0
    // children always have larger indices than their parent, so at most nn steps
    for (int32_t step = 0; node >= 0 && step < nn; ++step) {
      const PredNode nd = m.nodes[nb + node];
      node = pred_decide(m, nd, __ldg(x + nd.feature));
    }
    acc += m.leaf_value[m.leaf_offset[t] + ~node];
  }
  if (!raw && m.transform == 1) acc = 1.0 / (1.0 + exp(-m.sigmoid * acc));
  out[r] = acc;
}

}  // namespace

void launch_predict(const PredModelDev& m, const double* rows, int64_t n, int32_t raw,
                    double* out, cudaStream_t st) {
  if (n <= 0) return;
  const int64_t blocks = (n + kPredThreads - 1) / kPredThreads;
  k_predict<<<(unsigned)blocks, kPredThreads, 0, st>>>(m, rows, n, raw, out);
}

}  // namespace lgbm_b200
