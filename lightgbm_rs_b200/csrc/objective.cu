// Gradient/hessian, quantization, root sums, shrinkage and score update kernels.
#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstddef>

#include "kernels.cuh"

namespace lgbm_b200 {

namespace {

constexpr int kObjThreads = 256;
static_assert(offsetof(DevGhParams, max_h_key) == offsetof(DevGhParams, max_abs_g_bits) + 12,
              "the four gradient maxima are reduced over devices as one array");

__device__ __forceinline__ uint32_t f32_key(float x) {
  x = x + 0.0f;  // -0.0 -> +0.0: the reference compares hessians with ==
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Binary::get_gradients (lgbm-objective/src/binary.rs:134-171), label weights 1.
// Regression L2 (lgbm-objective/src/regression.rs:429-433).
__device__ __forceinline__ float2 grad_hess(int objective, double sigmoid, double s, float l) {
  if (objective == LGBM_B200_OBJECTIVE_BINARY) {
    const bool is_pos = l > 0.0f;
    const double lv = is_pos ? 1.0 : -1.0;
    const double resp = -lv * sigmoid / (1.0 + exp(lv * sigmoid * s));
    const double ar = fabs(resp);
    return make_float2((float)(resp * 1.0), (float)(ar * (sigmoid - ar) * 1.0));
  }
  return make_float2((float)(s - (double)l), 1.0f);
}

// Rust `f64 as i8`: truncation toward zero, saturating, NaN -> 0.
__device__ __forceinline__ int as_i8(double x) {
  if (x != x) return 0;
  if (x >= 127.0) return 127;
  if (x <= -128.0) return -128;
  return (int)x;
}

__global__ void k_fill_f64(double* p, int64_t n, double v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

__global__ void k_gh_reset(DevGhParams* p, const int32_t* stopped) {
  if (stopped && *stopped) return;
  p->max_abs_g_bits = 0u;
  p->max_abs_h_bits = 0u;
  p->min_h_key_inv = 0u;
  p->max_h_key = 0u;
  p->root_g = 0;
  p->root_h = 0;
}

__global__ void __launch_bounds__(kObjThreads) k_grad_pass1(ObjDev o) {
  if (o.stopped && *o.stopped) return;
  uint32_t mg = 0, mh = 0, kmin = 0xffffffffu, kmax = 0u;
  float2* gh = reinterpret_cast<float2*>(o.gh);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < o.N;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float2 v = grad_hess(o.objective, o.sigmoid, o.score[i], o.label[i]);
    gh[i] = v;
    mg = max(mg, __float_as_uint(fabsf(v.x)));
    mh = max(mh, __float_as_uint(fabsf(v.y)));
    const uint32_t k = f32_key(v.y);
    kmin = min(kmin, k);
    kmax = max(kmax, k);
  }
  for (int off = 16; off > 0; off >>= 1) {
    mg = max(mg, __shfl_xor_sync(0xffffffffu, mg, off));
    mh = max(mh, __shfl_xor_sync(0xffffffffu, mh, off));
    kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, off));
    kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, off));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMax(&o.ghp->max_abs_g_bits, mg);
    atomicMax(&o.ghp->max_abs_h_bits, mh);
    atomicMax(&o.ghp->min_h_key_inv, ~kmin);
    atomicMax(&o.ghp->max_h_key, kmax);
  }
}

// ------------------------------------------------------------------------------------
// LambdarankNDCG gradients (Lambdarank::get_gradients, lgbm-objective/src/rank.rs:264-366;
// LightGBM rank_objective.hpp:180-266), one warp per query. The reference walks the
// document pairs (i, j) of each query in the order of its score-sorted positions,
// outer i below the truncation level, and adds every pair's f32 lambda and hessian into
// both documents, so each document receives its terms in a fixed order: first the
// pairs in which it is the inner j (outer i ascending), then those in which it is the
// outer i (inner j ascending). One lane per document replays exactly that order, so
// the f32 sums are the reference's. The f64 sum of all lambdas, which the norm needs,
// depends on the whole pair order: the warp computes 32 pairs at a time and every lane
// folds them sequentially.
// ------------------------------------------------------------------------------------

// LambdarankNDCG::GetSigmoid (rank.rs:230-241): the table lookup.
__device__ __forceinline__ double rank_sigmoid(const ObjDev& o, double x) {
  if (x <= o.sig_min) return o.sig_table[0];
  if (x >= o.sig_max) return o.sig_table[kRankSigmoidBins - 1];
  // (x - min) * factor can round up to the table length just below max: clamp
  const size_t i = (size_t)((x - o.sig_min) * o.sig_factor);
  return o.sig_table[i < (size_t)kRankSigmoidBins ? i : (size_t)kRankSigmoidBins - 1];
}

// One pair's lambda and hessian (rank.rs:326-351). hr / lr are the sorted positions of
// the higher- and lower-labelled documents.
__device__ __forceinline__ void rank_pair(const ObjDev& o, double hs, double ls, float hl,
                                          float ll, int hr, int lr, double inv_max,
                                          bool scale, double* pl, double* ph) {
  const double ds = hs - ls;
  const double gap = o.label_gain[(int)hl] - o.label_gain[(int)ll];
  const double pd = fabs(o.discount[hr] - o.discount[lr]);
  double dn = gap * pd * inv_max;
  if (scale) dn /= (double)0.01f + fabs(ds);
  double p = rank_sigmoid(o, ds);
  double h = p * (1.0 - p);
  p *= -o.sigmoid * dn;
  h *= o.sigmoid * o.sigmoid * dn;
  *pl = p;
  *ph = h;
}

// Total order of scores for the stable descending sort: -0.0 and +0.0 share a key, so
// equal scores keep row order as in the reference's sort.
__device__ __forceinline__ unsigned long long score_key(double x) {
  x = x + 0.0;
  const unsigned long long b = (unsigned long long)__double_as_longlong(x);
  return (b >> 63) ? ~b : (b | 0x8000000000000000ull);
}

__global__ void __launch_bounds__(kObjThreads) k_lambdarank(ObjDev o) {
  if (o.stopped && *o.stopped) return;
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const double kMinScore = -INFINITY;
  float2* gh = reinterpret_cast<float2*>(o.gh);
  uint32_t mg = 0, mh = 0, kmin = 0xffffffffu, kmax = 0u;
  for (int64_t q = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; q < o.num_queries;
       q += nwarps) {
    const int32_t b = o.qb[q];
    const int32_t cnt = o.qb[q + 1] - b;
    const double* s = o.score + b;
    const float* lab = o.label + b;
    int32_t* ord = o.order + b;
    // stable sort by descending score: position = rows ahead of this one
    for (int i = lane; i < cnt; i += 32) {
      const unsigned long long ki = score_key(s[i]);
      int r = 0;
      for (int e = 0; e < cnt; ++e) {
        const unsigned long long ke = score_key(s[e]);
        r += (ke > ki || (ke == ki && e < i)) ? 1 : 0;
      }
      ord[r] = i;
    }
    __syncwarp();
    if (cnt == 0) continue;
    const double best = s[ord[0]];
    int wi = cnt - 1;
    if (wi > 0 && s[ord[wi]] == kMinScore) --wi;
    const double worst = s[ord[wi]];
    const bool scale = o.norm && best != worst;
    const double inv_max = o.inv_max_dcg[q];
    const int I = min(o.trunc, cnt - 1);  // outer positions: i + 1 < cnt && i < trunc
    // the f64 sum of the lambdas, in the reference's pair order
    double sum = 0.0;
    if (o.norm) {
      for (int i = 0; i < I; ++i) {
        const int ei = ord[i];
        const double si = s[ei];
        if (si == kMinScore) continue;
        const float li = lab[ei];
        for (int j0 = i + 1; j0 < cnt; j0 += 32) {
          const int j = j0 + lane;
          double t = 0.0;
          bool valid = false;
          if (j < cnt) {
            const int ej = ord[j];
            const double sj = s[ej];
            const float lj = lab[ej];
            if (sj != kMinScore && lj != li) {
              double pl, ph;
              if (li > lj)
                rank_pair(o, si, sj, li, lj, i, j, inv_max, scale, &pl, &ph);
              else
                rank_pair(o, sj, si, lj, li, j, i, inv_max, scale, &pl, &ph);
              t = 2.0 * pl;
              valid = true;
            }
          }
          const unsigned vm = __ballot_sync(full, valid);
          for (int k = 0; k < 32; ++k) {
            const double tk = __shfl_sync(full, t, k);
            if ((vm >> k) & 1u) sum -= tk;
          }
        }
      }
    }
    const bool rescale = o.norm && sum > 0.0;
    const double nf = rescale ? log2(1.0 + sum) / sum : 1.0;
    // per-document f32 sums in the reference's order
    for (int r = lane; r < cnt; r += 32) {
      const int d = ord[r];
      const double sd = s[d];
      const float ld = lab[d];
      float lam = 0.0f, hes = 0.0f;
      if (sd != kMinScore) {
        const int n_in = min(r, I);
        for (int i = 0; i < n_in; ++i) {  // pairs (i, r): this document is the inner one
          const int e = ord[i];
          const double se = s[e];
          const float le = lab[e];
          if (se == kMinScore || le == ld) continue;
          double pl, ph;
          if (le > ld) {
            rank_pair(o, se, sd, le, ld, i, r, inv_max, scale, &pl, &ph);
            lam -= (float)pl;
          } else {
            rank_pair(o, sd, se, ld, le, r, i, inv_max, scale, &pl, &ph);
            lam += (float)pl;
          }
          hes += (float)ph;
        }
        if (r < I) {
          for (int j = r + 1; j < cnt; ++j) {  // pairs (r, j): this document is the outer one
            const int e = ord[j];
            const double se = s[e];
            const float le = lab[e];
            if (se == kMinScore || le == ld) continue;
            double pl, ph;
            if (ld > le) {
              rank_pair(o, sd, se, ld, le, r, j, inv_max, scale, &pl, &ph);
              lam += (float)pl;
            } else {
              rank_pair(o, se, sd, le, ld, j, r, inv_max, scale, &pl, &ph);
              lam -= (float)pl;
            }
            hes += (float)ph;
          }
        }
      }
      if (rescale) {
        lam = (float)((double)lam * nf);
        hes = (float)((double)hes * nf);
      }
      gh[b + d] = make_float2(lam, hes);
      mg = max(mg, __float_as_uint(fabsf(lam)));
      mh = max(mh, __float_as_uint(fabsf(hes)));
      const uint32_t k = f32_key(hes);
      kmin = min(kmin, k);
      kmax = max(kmax, k);
    }
    __syncwarp();
  }
  for (int off = 16; off > 0; off >>= 1) {
    mg = max(mg, __shfl_xor_sync(full, mg, off));
    mh = max(mh, __shfl_xor_sync(full, mh, off));
    kmin = min(kmin, __shfl_xor_sync(full, kmin, off));
    kmax = max(kmax, __shfl_xor_sync(full, kmax, off));
  }
  if (lane == 0) {
    atomicMax(&o.ghp->max_abs_g_bits, mg);
    atomicMax(&o.ghp->max_abs_h_bits, mh);
    atomicMax(&o.ghp->min_h_key_inv, ~kmin);
    atomicMax(&o.ghp->max_h_key, kmax);
  }
}

// Quantized decode units for given grad/hess scales (see GhMode).
__device__ void set_quant_units(DevGhParams* p, int mode, double gs, double hs) {
  if (mode == GH_QPACK) {
    p->unit_g = (double)(float)(1.0 * gs);
    p->unit_h = (double)(float)(1.0 * hs);
    p->v3h = (double)(float)(3.0 * hs);
    return;
  }
  // QLUT: every dequantized level (f32)(q * scale) is an integer multiple of the
  // f32 ulp of the level-1 value; accumulate those integers.
  auto unit_of = [](double v1) -> double {
    if (!(v1 > 0.0)) return 1.0;
    int e;
    frexp(v1, &e);
    return ldexp(1.0, e - 24);
  };
  const double ug = unit_of((double)(float)gs);
  const double uh = unit_of((double)(float)hs);
  p->unit_g = ug;
  p->unit_h = uh;
  for (int q = -128; q < 128; ++q) {
    p->lut_g[q + 128] = (long long)((double)(float)((double)q * gs) / ug);
    p->lut_h[q + 128] = (long long)((double)(float)((double)q * hs) / uh);
  }
}

// Per-iteration encoding parameters. Quantized: GradientDiscretizer::compute_scales
// (lgbm-treelearner/src/gradient_discretizer.rs:145-165).
__global__ void k_gh_scales(ObjDev o) {
  if (o.stopped && *o.stopped) return;
  DevGhParams* p = o.ghp;
  const double max_g = (double)__uint_as_float(p->max_abs_g_bits);
  const double max_h = (double)__uint_as_float(p->max_abs_h_bits);
  p->mode = o.gh_mode;
  p->num_quant_bins = o.num_quant_bins;
  p->root_g = 0;
  p->root_h = 0;
  if (o.gh_mode == GH_FLOAT) {
    int lg = 0;
    while (lg < 62 && ((int64_t)1 << lg) < o.n_global) ++lg;
    auto kscale = [&](double m) -> int {
      if (!(m > 0.0) || !isfinite(m)) return 0;
      int e;
      frexp(m, &e);  // m < 2^e
      int k = 62 - e - lg;
      if (k > 1000) k = 1000;
      if (k < -1000) k = -1000;
      return k;
    };
    const int kg = kscale(max_g), kh = kscale(max_h);
    p->scale_g = ldexp(1.0, kg);
    p->unit_g = ldexp(1.0, -kg);
    p->scale_h = ldexp(1.0, kh);
    p->unit_h = ldexp(1.0, -kh);
    p->is_const_hess = 0;
    return;
  }
  const int bins = o.num_quant_bins;
  const bool is_const = ~p->min_h_key_inv == p->max_h_key;
  const double half_bins = (double)(bins / 2);
  const double gs = max_g / half_bins;
  const double hs = is_const ? max_h : max_h / (double)bins;
  p->is_const_hess = is_const ? 1 : 0;
  p->grad_scale = gs;
  p->hess_scale = hs;
  p->inv_grad_scale = 1.0 / gs;
  p->inv_hess_scale = 1.0 / hs;
  set_quant_units(p, o.gh_mode, gs, hs);
}

// Scales handed in by the caller (learner entry point with int8 pairs).
__global__ void k_gh_given_scales(ObjDev o) {
  DevGhParams* p = o.ghp;
  p->root_g = 0;
  p->root_h = 0;
  p->inv_grad_scale = 1.0 / p->grad_scale;
  p->inv_hess_scale = 1.0 / p->hess_scale;
  set_quant_units(p, p->mode, p->grad_scale, p->hess_scale);
}

__global__ void k_maxabs(ObjDev o) {
  uint32_t mg = 0, mh = 0;
  const float2* gh = reinterpret_cast<const float2*>(o.gh);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < o.N;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float2 v = gh[i];
    mg = max(mg, __float_as_uint(fabsf(v.x)));
    mh = max(mh, __float_as_uint(fabsf(v.y)));
  }
  for (int off = 16; off > 0; off >>= 1) {
    mg = max(mg, __shfl_xor_sync(0xffffffffu, mg, off));
    mh = max(mh, __shfl_xor_sync(0xffffffffu, mh, off));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMax(&o.ghp->max_abs_g_bits, mg);
    atomicMax(&o.ghp->max_abs_h_bits, mh);
  }
}

// Root sums of caller-provided int8 pairs.
__global__ void __launch_bounds__(kObjThreads) k_root_sums_q(ObjDev o) {
  const DevGhParams& p = *o.ghp;
  const uint16_t* q = reinterpret_cast<const uint16_t*>(reinterpret_cast<const float2*>(o.gh) + o.N);
  long long sa = 0, sb = 0;
  const bool pack = p.mode == GH_QPACK;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < o.N;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint16_t v = q[i];
    const int qg = (int)(int8_t)(v & 0xff);
    const int qh = (int)(int8_t)(v >> 8);
    if (pack) {
      sa += qg;
      sb += qh == 3 ? (1ll << 32) : (long long)qh;
    } else {
      sa += p.lut_g[qg + 128];
      sb += p.lut_h[qh + 128];
    }
  }
  for (int off = 16; off > 0; off >>= 1) {
    sa += __shfl_xor_sync(0xffffffffu, sa, off);
    sb += __shfl_xor_sync(0xffffffffu, sb, off);
  }
  if ((threadIdx.x & 31) == 0) {
    atomicAdd((unsigned long long*)&o.ghp->root_g, (unsigned long long)sa);
    atomicAdd((unsigned long long*)&o.ghp->root_h, (unsigned long long)sb);
  }
}

// GradientDiscretizer::quantize_pair, deterministic rounding
// (gradient_discretizer.rs:167-191), plus the exact integer root sums.
__global__ void __launch_bounds__(kObjThreads) k_quantize(ObjDev o) {
  if (o.stopped && *o.stopped) return;
  const DevGhParams& p = *o.ghp;
  const float2* gh = reinterpret_cast<const float2*>(o.gh);
  // int8 pairs live right after the f32 pairs
  uint16_t* q = reinterpret_cast<uint16_t*>(reinterpret_cast<float2*>(o.gh) + o.N);
  long long sa = 0, sb = 0;
  const bool pack = p.mode == GH_QPACK;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < o.N;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float2 v = gh[i];
    const double gv = (double)v.x * p.inv_grad_scale;
    const int qg = as_i8(v.x >= 0.0f ? gv + 0.5 : gv - 0.5);
    const int qh = p.is_const_hess ? 1 : as_i8((double)v.y * p.inv_hess_scale + 0.5);
    q[i] = (uint16_t)((qg & 0xff) | ((qh & 0xff) << 8));
    if (pack) {
      sa += qg;
      sb += qh == 3 ? (1ll << 32) : (long long)qh;
    } else {
      sa += p.lut_g[qg + 128];
      sb += p.lut_h[qh + 128];
    }
  }
  for (int off = 16; off > 0; off >>= 1) {
    sa += __shfl_xor_sync(0xffffffffu, sa, off);
    sb += __shfl_xor_sync(0xffffffffu, sb, off);
  }
  if ((threadIdx.x & 31) == 0) {
    atomicAdd((unsigned long long*)&o.ghp->root_g, (unsigned long long)sa);
    atomicAdd((unsigned long long*)&o.ghp->root_h, (unsigned long long)sb);
  }
}

// ------------------------------------------------------------------------------------
// GradientDiscretizer::quantize_pair with stochastic rounding
// (lgbm-treelearner/src/gradient_discretizer.rs:167-191, 252-262; seed per iteration
// gbdt.rs:950). The offsets are one xorshift64 stream over every row of the job in row
// order, a gradient draw then a hessian draw per row. The stream is linear over GF(2),
// so a warp jumps to its segment's place with bit-matrix products (one per set bit of
// 2 x the segment's first global row), then hands each lane the state 64 draws further
// on; each lane then runs the sequential stream over its 32 consecutive rows. Rows are
// staged through shared memory so that global loads and stores stay coalesced.
// ------------------------------------------------------------------------------------
constexpr int kSrLaneRows = 32;
constexpr int kSrWarpRows = 32 * kSrLaneRows;
constexpr int kSrThreads = 128;
constexpr int kSrLanePow = 6;  // 2 draws x kSrLaneRows rows = 2^6 steps per lane
static_assert(2 * kSrLaneRows == (1 << kSrLanePow), "lane stride is a power of two");

__device__ __forceinline__ unsigned long long xs_step_warp(const unsigned long long* cols,
                                                           unsigned long long s, int lane) {
  // y = M s over GF(2): lane l folds columns 2l and 2l+1, then the warp XOR-reduces
  const unsigned long long c0 = cols[2 * lane], c1 = cols[2 * lane + 1];
  unsigned long long y = (((s >> (2 * lane)) & 1ull) ? c0 : 0ull) ^
                         (((s >> (2 * lane + 1)) & 1ull) ? c1 : 0ull);
  for (int o = 16; o > 0; o >>= 1) y ^= __shfl_xor_sync(0xffffffffu, y, o);
  return y;
}

__device__ __forceinline__ double xs_next_u01(unsigned long long& x) {
  x ^= x << 13;
  x ^= x >> 7;
  x ^= x << 17;
  return (double)(x >> 11) / 9007199254740992.0;  // 2^53
}

__global__ void __launch_bounds__(kSrThreads) k_quantize_sr(ObjDev o) {
  if (o.stopped && *o.stopped) return;
  constexpr int kWarps = kSrThreads / 32;
  constexpr int kPad = kSrWarpRows + kSrWarpRows / 32;
  __shared__ float s_g[kWarps][kPad];
  __shared__ float s_h[kWarps][kPad];
  const DevGhParams& p = *o.ghp;
  const float2* gh = reinterpret_cast<const float2*>(o.gh);
  uint16_t* q = reinterpret_cast<uint16_t*>(reinterpret_cast<float2*>(o.gh) + o.N);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t warps_total = (int64_t)gridDim.x * kWarps;
  const int64_t gw = (int64_t)blockIdx.x * kWarps + w;
  const unsigned long long seed =
      ((unsigned long long)(uint32_t)*o.iter_counter << 20) ^ 0x51702010ull;
  const unsigned long long s0 = seed ^ 0x9E3779B97F4A7C15ull;
  const double igs = p.inv_grad_scale, ihs = p.inv_hess_scale;
  const bool cst = p.is_const_hess != 0;
  const bool pack = p.mode == GH_QPACK;
  long long sa = 0, sb = 0;
  for (int64_t seg = gw * kSrWarpRows; seg < o.N; seg += warps_total * kSrWarpRows) {
    const int nrows = (int)min((int64_t)kSrWarpRows, o.N - seg);
    for (int k = lane; k < nrows; k += 32) {
      const float2 v = gh[seg + k];
      s_g[w][k + (k >> 5)] = v.x;
      s_h[w][k + (k >> 5)] = v.y;
    }
    __syncwarp();
    unsigned long long st = s0;
    unsigned long long e = 2ull * (unsigned long long)(o.row_offset + seg);
    for (int j = 0; e != 0ull; ++j, e >>= 1)
      if (e & 1ull) st = xs_step_warp(o.xs_pow + 64 * j, st, lane);
    unsigned long long mine = st;
    for (int l = 1; l < 32; ++l) {
      st = xs_step_warp(o.xs_pow + 64 * kSrLanePow, st, lane);
      if (lane == l) mine = st;
    }
    for (int k = 0; k < kSrLaneRows; ++k) {
      const int r = lane * kSrLaneRows + k;
      const double bg = xs_next_u01(mine);
      const double bh = xs_next_u01(mine);
      if (r >= nrows) continue;
      const int pr = r + (r >> 5);
      const float gv32 = s_g[w][pr], hv32 = s_h[w][pr];
      const double gv = (double)gv32 * igs;
      const int qg = as_i8(gv32 >= 0.0f ? gv + bg : gv - bg);
      const int qh = cst ? 1 : as_i8((double)hv32 * ihs + bh);
      s_g[w][pr] = __uint_as_float((uint32_t)((qg & 0xff) | ((qh & 0xff) << 8)));
      if (pack) {
        sa += qg;
        sb += qh == 3 ? (1ll << 32) : (long long)qh;
      } else {
        sa += p.lut_g[qg + 128];
        sb += p.lut_h[qh + 128];
      }
    }
    __syncwarp();
    for (int k = lane; k < nrows; k += 32)
      q[seg + k] = (uint16_t)__float_as_uint(s_g[w][k + (k >> 5)]);
    __syncwarp();
  }
  for (int off = 16; off > 0; off >>= 1) {
    sa += __shfl_xor_sync(0xffffffffu, sa, off);
    sb += __shfl_xor_sync(0xffffffffu, sb, off);
  }
  if (lane == 0) {
    atomicAdd((unsigned long long*)&o.ghp->root_g, (unsigned long long)sa);
    atomicAdd((unsigned long long*)&o.ghp->root_h, (unsigned long long)sb);
  }
}

__global__ void __launch_bounds__(kObjThreads) k_root_sums_float(ObjDev o) {
  if (o.stopped && *o.stopped) return;
  const DevGhParams& p = *o.ghp;
  const float2* gh = reinterpret_cast<const float2*>(o.gh);
  long long sa = 0, sb = 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < o.N;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float2 v = gh[i];
    sa += __double2ll_rn((double)v.x * p.scale_g);
    sb += __double2ll_rn((double)v.y * p.scale_h);
  }
  for (int off = 16; off > 0; off >>= 1) {
    sa += __shfl_xor_sync(0xffffffffu, sa, off);
    sb += __shfl_xor_sync(0xffffffffu, sb, off);
  }
  if ((threadIdx.x & 31) == 0) {
    atomicAdd((unsigned long long*)&o.ghp->root_g, (unsigned long long)sa);
    atomicAdd((unsigned long long*)&o.ghp->root_h, (unsigned long long)sb);
  }
}

__device__ __forceinline__ bool is_zero(double v) { return v >= -1e-35 && v <= 1e-35; }

// Tree::shrinkage (lgbm-model/src/tree.rs:1074-1100) and the record of the tree.
__global__ void k_finish_tree(GrowDev d, FinishDev f) {
  if (*f.stopped) return;
  const int nl = d.ctrl->num_leaves;
  const int it = *f.iter_counter;
  __shared__ int s_skip;
  if (threadIdx.x == 0) {
    s_skip = 0;
    if (nl <= 1 && it > 0) {
      // no split after the first iteration: training stops (gbdt.rs:1272-1283)
      *f.stopped = 1;
      s_skip = 1;
    } else if (it >= f.max_iters) {
      s_skip = 1;
    }
  }
  __syncthreads();
  if (s_skip) return;
  const int L = d.L;
  for (int i = threadIdx.x; i < L; i += blockDim.x) {
    double lv = d.t_leaf_value[i];
    if (nl > 1 && i < nl) {
      lv = lv * f.learning_rate;
      lv = is_zero(lv) ? 0.0 : lv;
      d.t_leaf_value[i] = lv;
    }
    double iv = d.t_internal_value[i];
    if (nl > 1 && i + 1 < nl) {
      iv = iv * f.learning_rate;
      iv = is_zero(iv) ? 0.0 : iv;
      d.t_internal_value[i] = iv;
    }
    const size_t o = (size_t)it * L + i;
    f.rec_left[o] = d.t_left[i];
    f.rec_right[o] = d.t_right[i];
    f.rec_split_feature[o] = d.t_split_feature[i];
    f.rec_threshold[o] = d.t_threshold[i];
    f.rec_split_gain[o] = d.t_split_gain[i];
    f.rec_decision[o] = d.t_decision[i];
    f.rec_leaf_value[o] = nl > 1 ? lv : 0.0;
    f.rec_leaf_weight[o] = d.t_leaf_weight[i];
    f.rec_leaf_count[o] = d.t_leaf_count[i];
    f.rec_internal_value[o] = iv;
    f.rec_internal_count[o] = d.t_internal_count[i];
#pragma unroll
    for (int k = 0; k < kCatWords; ++k) f.rec_cat[o * kCatWords + k] = d.t_cat[i * kCatWords + k];
  }
  if (threadIdx.x == 0) {
    f.rec_num_leaves[it] = nl;
    *f.iter_counter = it + 1;
  }
}

// score[row] += leaf_value[leaf(row)] (learner.rs:4380-4395), walking the tree on the
// row's bins in row order so the score array streams instead of scattering.
__global__ void __launch_bounds__(256) k_score_update(GrowDev d, double* score,
                                                      const int32_t* stopped,
                                                      const int32_t* iter_counter,
                                                      const int32_t* rec_num_leaves) {
  if (*stopped) return;
  const int it = *iter_counter - 1;
  if (it < 0 || rec_num_leaves[it] <= 1) return;
  __shared__ int32_t s_left[256], s_right[256], s_feat[256];
  __shared__ uint32_t s_thr[256];
  __shared__ int8_t s_dec[256];
  __shared__ double s_val[256];
  __shared__ uint32_t s_cat[256][kCatWords];
  const int nl = d.ctrl->num_leaves;
  for (int i = threadIdx.x; i < nl; i += blockDim.x) {
    s_val[i] = d.t_leaf_value[i];
    if (i + 1 < nl) {
      s_left[i] = d.t_left[i];
      s_right[i] = d.t_right[i];
      s_feat[i] = d.t_split_feature[i];
      s_thr[i] = d.t_threshold[i];
      s_dec[i] = d.t_decision[i];
      if (d.t_decision[i] & 1)
        for (int k = 0; k < kCatWords; ++k) s_cat[i][k] = d.t_cat[i * kCatWords + k];
    }
  }
  __syncthreads();
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < d.N;
       r += (int64_t)gridDim.x * blockDim.x) {
    const uint8_t* rp = d.bins + (size_t)r * d.stride;
    int node = 0;
    while (node >= 0) {
      const int f = s_feat[node];
      const int8_t dec = s_dec[node];
      const int32_t bin = (int32_t)row_bin(rp, f, d.packed4 != 0);
      const bool right = (dec & 1) ? d_cat_go_right(s_cat[node], bin)
                                   : d_go_right(d.feat[f], s_thr[node], (dec & 2) != 0, bin);
      node = right ? s_right[node] : s_left[node];
    }
    score[r] += s_val[~node];
  }
}

int num_sms_obj() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

}  // namespace

void launch_fill_f64(double* p, int64_t n, double v, cudaStream_t st) {
  if (n <= 0) return;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms_obj() * 8);
  k_fill_f64<<<blocks, 256, 0, st>>>(p, n, v);
}

// With several devices: the scales come from the maxima over all devices' rows, and the
// root sums are summed over devices (integers, so exact in any order).
void launch_gradients(const ObjDev& o, cudaStream_t st, LaunchProfiler* prof,
                      const DeviceComm* comm) {
  const int grid = num_sms_obj() * 8;
  const int slot = prof ? prof->begin(st, KC_GRAD) : -1;
  k_gh_reset<<<1, 1, 0, st>>>(o.ghp, o.stopped);
  if (o.objective == LGBM_B200_OBJECTIVE_LAMBDARANK) {
    const int64_t warps_needed = o.num_queries > 0 ? o.num_queries : 1;
    const int64_t blocks = (warps_needed + kObjThreads / 32 - 1) / (kObjThreads / 32);
    k_lambdarank<<<(int)std::min<int64_t>(blocks, (int64_t)grid * 4), kObjThreads, 0, st>>>(o);
  } else {
    k_grad_pass1<<<grid, kObjThreads, 0, st>>>(o);
  }
  if (comm) {
    // max |g|, max |h|, ~min key, max key: one max over four words
    comm->max_u32(comm->ctx, &o.ghp->max_abs_g_bits, 4, st);
  }
  k_gh_scales<<<1, 1, 0, st>>>(o);
  if (o.gh_mode == GH_FLOAT) {
    k_root_sums_float<<<grid, kObjThreads, 0, st>>>(o);
  } else if (o.stochastic) {
    const int64_t segs = (o.N + kSrWarpRows - 1) / kSrWarpRows;
    const int64_t blocks = (segs + kSrThreads / 32 - 1) / (kSrThreads / 32);
    k_quantize_sr<<<(int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)grid * 2)),
                    kSrThreads, 0, st>>>(o);
  } else {
    k_quantize<<<grid, kObjThreads, 0, st>>>(o);
  }
  if (comm) comm->sum_i64(comm->ctx, &o.ghp->root_g, 2, st);
  if (prof) prof->end(st, slot);
}

// Columns of T^(2^j), j = 0..63, for T the bit matrix of one xorshift64 step (the
// reference's next_u01 shifts 13, 7, 17): out[64 j + k] = T^(2^j) e_k.
void xorshift_pow_table(unsigned long long* out) {
  auto step = [](unsigned long long x) {
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    return x;
  };
  for (int k = 0; k < 64; ++k) out[k] = step(1ull << k);
  for (int j = 1; j < 64; ++j) {
    const unsigned long long* m = out + 64 * (j - 1);
    for (int k = 0; k < 64; ++k) {
      unsigned long long x = m[k], y = 0ull;  // M (M e_k)
      for (int b = 0; b < 64; ++b)
        if ((x >> b) & 1ull) y ^= m[b];
      out[64 * j + k] = y;
    }
  }
}

void launch_learner_gradients(const ObjDev& o, int32_t kind, cudaStream_t st) {
  const int grid = num_sms_obj() * 8;
  if (kind == LGBM_B200_GH_F32) {
    k_gh_reset<<<1, 1, 0, st>>>(o.ghp, nullptr);
    k_maxabs<<<grid, kObjThreads, 0, st>>>(o);
    k_gh_scales<<<1, 1, 0, st>>>(o);
    k_root_sums_float<<<grid, kObjThreads, 0, st>>>(o);
  } else {
    k_gh_given_scales<<<1, 1, 0, st>>>(o);
    k_root_sums_q<<<grid, kObjThreads, 0, st>>>(o);
  }
}

void launch_finish_iteration(const GrowDev& d, const FinishDev& f, cudaStream_t st,
                             LaunchProfiler* prof) {
  const int slot = prof ? prof->begin(st, KC_FINISH) : -1;
  k_finish_tree<<<1, 256, 0, st>>>(d, f);
  k_score_update<<<num_sms_obj() * 8, 256, 0, st>>>(d, f.score, f.stopped, f.iter_counter,
                                                    f.rec_num_leaves);
  if (prof) prof->end(st, slot);
}

}  // namespace lgbm_b200
