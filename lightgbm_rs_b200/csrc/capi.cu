// Host runtime behind the C ABI (include/lgbm_b200.h): device-resident datasets,
// the tree learner, the boosting loop and the per-op Backend mirror.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <limits>
#include <map>
#include <memory>
#include <atomic>
#include <mutex>
#include <thread>
#include <string>
#include <vector>

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>  // types only: the library is loaded at run time

#include "binning.h"
#include "common.cuh"
#include "host_copy.h"
#include "kernels.cuh"
#include "lgbm_b200.h"

namespace lgbm_b200 {
void set_build_smem_limit(size_t bytes);
int q4_max_cells();
bool q4_supported(int shift, int nch, bool pack4);
void launch_learner_gradients(const ObjDev& o, int32_t kind, cudaStream_t st);
void launch_gather_partition(const GrowDev& d, uint32_t* out, cudaStream_t st);
}  // namespace lgbm_b200

using namespace lgbm_b200;

namespace {

// Splits of leaves with at most this many 2048-row tiles (this device's rows) hand the
// accumulated child to the next control step as one partial histogram per tile.
constexpr int kPrivateTiles = kMaxPrivateTiles;

thread_local std::string g_last_error;

struct Error {
  int code;
  std::string msg;
};

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define CUDA_TRY(expr)                                                                     \
  do {                                                                                     \
    cudaError_t _e = (expr);                                                               \
    if (_e != cudaSuccess)                                                                 \
      return fail(LGBM_B200_RUNTIME, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), \
                  __FILE__, __LINE__);                                                     \
  } while (0)

// Large device blocks are kept after release and handed out again for the same size on
// the same device: a booster built after another was destroyed (the same data, the same
// sizes) maps no new memory. A cudaMalloc of hundreds of MB after a cudaFree cost tens
// of milliseconds. Releasing a kept block waits for the device, as cudaFree does.
struct BlockCache {
  std::mutex mu;
  std::multimap<std::pair<int, size_t>, void*> blocks;
  size_t bytes = 0;
};

BlockCache& block_cache() {
  static BlockCache* c = new BlockCache;  // never destroyed: no teardown-order hazards
  return *c;
}

constexpr size_t kCacheMinBytes = 1ull << 20;
constexpr size_t kCacheMaxBytes = 16ull << 30;

// Frees every kept block of `device` (-1: of every device); returns the bytes freed.
size_t release_cached_blocks(int device) {
  BlockCache& c = block_cache();
  std::lock_guard<std::mutex> lk(c.mu);
  size_t freed = 0;
  int prev = -1;
  cudaGetDevice(&prev);
  for (auto it = c.blocks.begin(); it != c.blocks.end();) {
    if (device >= 0 && it->first.first != device) {
      ++it;
      continue;
    }
    if (it->first.first != prev) cudaSetDevice(it->first.first);
    cudaFree(it->second);
    freed += it->first.second;
    c.bytes -= it->first.second;
    it = c.blocks.erase(it);
  }
  if (prev >= 0) cudaSetDevice(prev);
  return freed;
}

cudaError_t dev_malloc(void** p, size_t bytes, bool cacheable) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (cacheable && bytes >= kCacheMinBytes) {
    BlockCache& c = block_cache();
    std::lock_guard<std::mutex> lk(c.mu);
    auto it = c.blocks.find({dev, bytes});
    if (it != c.blocks.end()) {
      *p = it->second;
      c.bytes -= bytes;
      c.blocks.erase(it);
      return cudaSuccess;
    }
  }
  cudaError_t e = cudaMalloc(p, bytes);
  if (e == cudaErrorMemoryAllocation && release_cached_blocks(dev) > 0) {
    // idle kept blocks of other sizes stood in the way: give them back and retry once
    cudaGetLastError();
    e = cudaMalloc(p, bytes);
  }
  return e;
}

void dev_free(void* p, size_t bytes, bool cacheable) {
  if (cacheable && bytes >= kCacheMinBytes) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) == cudaSuccess && a.type == cudaMemoryTypeDevice) {
      int prev = -1;
      cudaGetDevice(&prev);
      if (prev != a.device) cudaSetDevice(a.device);
      const bool idle = cudaDeviceSynchronize() == cudaSuccess;
      if (prev >= 0 && prev != a.device) cudaSetDevice(prev);
      BlockCache& c = block_cache();
      std::lock_guard<std::mutex> lk(c.mu);
      if (idle && c.bytes + bytes <= kCacheMaxBytes) {
        c.blocks.insert({{a.device, bytes}, p});
        c.bytes += bytes;
        return;
      }
    }
    cudaGetLastError();
  }
  cudaFree(p);
}

// RAII device buffer (large blocks through the cache above unless `nocache`).
template <typename T>
struct DevBuf {
  T* p = nullptr;
  size_t n = 0;
  bool nocache = false;  // memory shared with other processes (CUDA IPC)
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  ~DevBuf() { release(); }
  void release() {
    if (p) dev_free(p, n * sizeof(T), !nocache);
    p = nullptr;
    n = 0;
  }
  cudaError_t alloc(size_t count) {
    release();
    n = count;
    if (count == 0) return cudaSuccess;
    return dev_malloc((void**)&p, count * sizeof(T), !nocache);
  }
};

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

DevGainConfig to_dev_gain(const lgbm_b200_gain_config& g) {
  DevGainConfig c;
  c.min_data_in_leaf = g.min_data_in_leaf;
  c.use_l1 = g.lambda_l1 > 0.0 ? 1 : 0;                  // gain.rs:1000-1003
  c.use_smoothing = g.path_smooth > (double)1e-15f ? 1 : 0;  // gain.rs:1018-1020
  c.use_full = (c.use_smoothing || g.max_delta_step > 0.0) ? 1 : 0;
  c.min_sum_hessian_in_leaf = g.min_sum_hessian_in_leaf;
  c.max_delta_step = g.max_delta_step;
  c.lambda_l1 = g.lambda_l1;
  c.lambda_l2 = g.lambda_l2;
  c.min_gain_to_split = g.min_gain_to_split;
  c.path_smooth = g.path_smooth;
  c.min_data_per_group = g.min_data_per_group;
  c.max_cat_threshold = g.max_cat_threshold;
  c.max_cat_to_onehot = g.max_cat_to_onehot;
  c._pad = 0;
  c.cat_l2 = g.cat_l2;
  c.cat_smooth = g.cat_smooth;
  return c;
}

DevFeature make_feature(int32_t num_bin, int32_t default_bin, int32_t mfb, int32_t missing_type) {
  DevFeature f{};
  f.num_bin = num_bin;
  f.offset = mfb == 0 ? 1 : 0;
  f.default_bin = default_bin;
  f.most_freq_bin = mfb;
  f.missing_type = missing_type;
  int flags = 0;
  if (num_bin > 2 && missing_type == LGBM_B200_MISSING_ZERO) flags |= 1;  // learner.rs:167-169
  if (num_bin > 2 && missing_type == LGBM_B200_MISSING_NAN) flags |= 2;   // learner.rs:173-175
  if (num_bin > 2 && missing_type != LGBM_B200_MISSING_NONE) flags |= 4;  // learner.rs:191-193
  f.flags = flags;
  f.route_min = f.offset;
  f.route_max = num_bin - 1;
  return f;
}

lgbm_b200_split_info to_abi(const DevSplitInfo& s) {
  lgbm_b200_split_info o;
  o.threshold = s.threshold;
  o.default_left = s.default_left;
  o.left_count = s.left_count;
  o.right_count = s.right_count;
  o.gain = s.gain;
  o.left_sum_gradient = s.left_sum_gradient;
  o.left_sum_hessian = s.left_sum_hessian;
  o.right_sum_gradient = s.right_sum_gradient;
  o.right_sum_hessian = s.right_sum_hessian;
  o.left_output = s.left_output;
  o.right_output = s.right_output;
  return o;
}

int sm_count(int device) {
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
  return n > 0 ? n : 148;
}

bool have_device() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return n > 0;
}

}  // namespace

// ----------------------------------------------------------------------------------
// Dataset
// ----------------------------------------------------------------------------------

struct lgbm_b200_dataset {
  int device = 0;
  int64_t num_data = 0;
  int32_t num_features = 0;
  int32_t stride = 0;   // bytes per row of the bin matrix
  int32_t packed4 = 0;  // two 4-bit bins per byte
  int32_t total_bins = 0;
  std::vector<DevFeature> feats;
  DevBuf<uint8_t> bins;
  DevBuf<DevFeature> d_feats;
};

// ----------------------------------------------------------------------------------
// Learner
// ----------------------------------------------------------------------------------

struct lgbm_b200_learner {
  lgbm_b200_dataset* ds = nullptr;
  lgbm_b200_learner_config cfg{};
  int device = 0;
  cudaStream_t stream = nullptr;
  int32_t L = 0;
  int32_t slot_len = 0;
  int32_t max_tiles = 0;
  int gh_mode = GH_FLOAT;
  int q4_shift = 0;
  int q4_nch = 0;
  int build_blocks = 0;
  size_t build_smem = 0;
  std::vector<DevFeatureGroup> groups;
  DevBuf<DevFeatureGroup> d_groups;
  DevBuf<GrowCtrl> ctrl;
  DevBuf<int32_t> leaf_i32;  // leaf_begin, leaf_count, leaf_buf, slot_of_leaf, best_feature,
                             // leaf_count_g, leaf_is_right
  DevBuf<DevLeafSplits> ls;
  DevBuf<DevSplitInfo> best;
  DevBuf<uint8_t> splittable;
  DevBuf<int32_t> tree_i32;  // left, right, split_feature, leaf_count, internal_count, depth, parent
  DevBuf<uint32_t> tree_thr;
  DevBuf<float> tree_gain;
  DevBuf<int8_t> tree_dec;
  DevBuf<double> tree_f64;  // leaf_value, leaf_weight, internal_value
  DevBuf<uint32_t> idx;     // 2 * N
  DevBuf<unsigned long long> part_status;
  DevBuf<double> pool;
  DevBuf<long long> raw;
  DevBuf<long long*> xtab;  // one-device exchange table: {raw}
  DevBuf<long long> rawpool;
  DevBuf<long long> partials;
  DevBuf<DevSplitInfo> scan_out;
  DevBuf<uint32_t> cat_words;  // scan_cat [2F][8] | best_cat [L][8] | t_cat [L][8] | split_cat [8]
  DevBuf<uint8_t> scan_ok;
  // look-ahead partitions: two slots and the second stream they run on
  DevBuf<LookAhead> la;
  DevBuf<LookAhead> mainrec;  // [2] the fused control step's main-partition records
  DevBuf<long long> la_raw;
  DevBuf<long long> la_partials;
  DevBuf<unsigned long long> la_status;
  LookAheadStreams las{};
  bool la_enabled = true;  // LGBM_B200_LOOKAHEAD=0 turns the look-ahead off
  // gradients owned by a standalone learner (the booster owns its own)
  DevBuf<uint8_t> gh;
  DevBuf<DevGhParams> ghp;
  GrowDev d{};

  int configure_groups(int mode);
  int init(lgbm_b200_dataset* dataset, const lgbm_b200_learner_config& c);
  void bind(const void* gh_ptr, const DevGhParams* ghp_ptr, const int32_t* stopped);
  ~lgbm_b200_learner() {
    if (las.st) cudaStreamDestroy(las.st);
    if (las.fork) cudaEventDestroy(las.fork);
    for (cudaEvent_t e : las.done)
      if (e) cudaEventDestroy(e);
  }
};

int lgbm_b200_learner::configure_groups(int mode) {
  // Feature groups: runs of 16-feature blocks whose bins fit the shared-memory
  // budget of one build CTA.
  const int bpb = build_smem_bytes_per_bin(mode);
  const size_t budget = 112 * 1024;
  groups.clear();
  const int F = ds->num_features;
  if (mode == GH_QPACK) {
    // One power-of-two bin stride for every group: cell = (feature << shift) + bin.
    // Groups hold whole 16-feature blocks (aligned 16-byte row loads) except the last.
    int shift = 4;
    for (int f = 0; f < F; ++f)
      while ((1 << shift) < ds->feats[f].num_bin) ++shift;
    const int max_nf = std::min(128, kQ4MaxCells >> shift);
    // groups start on a 16-byte boundary of the row: 16 features, or 32 in a 4-bit matrix
    const int align = ds->packed4 ? 32 : 16;
    int per_group = F <= max_nf ? F : (max_nf / align) * align;
    // Wide data: groups of 48 features rather than the widest the shared layout holds. A
    // child's build splits its rows over the CTAs of each group and every CTA flushes its
    // group's cells with global atomics, so narrower groups (more groups, fewer CTAs per
    // group) flush fewer cells in total (C2, 2,000 features of 63 bins: builds 5.8 -> 4.4
    // ms per tree with 112 -> 48 features per group; 16 gave 4.6).
    constexpr int kWideGroup = 48;
    if (F > max_nf && per_group > kWideGroup && kWideGroup % align == 0) per_group = kWideGroup;
    if (const char* e = std::getenv("LGBM_B200_Q4_GROUP")) {  // tuning: features per group
      const int g = (std::atoi(e) / align) * align;
      if (g >= align && g < per_group) per_group = g;
    }
    for (int f0 = 0; f0 < F; f0 += per_group) {
      const int f1 = std::min(F, f0 + per_group);
      groups.push_back(DevFeatureGroup{f0, f1, ds->feats[f0].bin_off, (f1 - f0) << shift, shift,
                                       0});
    }
    const int nch = (per_group + 15) / 16;
    if (!q4_supported(shift, nch, ds->packed4 != 0))
      return fail(LGBM_B200_CAPABILITY_UNAVAILABLE,
                  "quantized build: no kernel for bin stride 2^%d with %d feature chunks", shift,
                  nch);
    q4_shift = shift;
    q4_nch = nch;
    build_smem = (size_t)4 * sizeof(uint32_t) * q4_max_cells();
    gh_mode = mode;
    CUDA_TRY(d_groups.alloc(groups.size()));
    CUDA_TRY(cudaMemcpy(d_groups.p, groups.data(), groups.size() * sizeof(DevFeatureGroup),
                        cudaMemcpyHostToDevice));
    set_build_smem_limit(build_smem);
    CUDA_TRY(cudaGetLastError());
    const int sms = sm_count(device);
    build_blocks = sms * 2;
    // Several feature groups (wide data): about two waves of CTAs over all groups. A build
    // CTA holds most of an SM's shared memory, so CTAs of a small child that find no rows
    // would otherwise take SMs wave after wave.
    const int ng = (int)groups.size();
    if (ng > 1) build_blocks = std::max(1, (2 * sms + ng - 1) / ng);
    // per-CTA row ranges stay below 65536 rows (level-3 counters and cold sums)
    const int64_t need = (ds->num_data + 65535 - 1) / 65535;
    if (build_blocks < need) build_blocks = (int)need;
    return LGBM_B200_OK;
  }
  DevFeatureGroup cur{0, 0, 0, 0, 0, 0};
  const int blk = ds->packed4 ? 32 : 16;  // a group starts on a 16-byte boundary of the row
  for (int b0 = 0; b0 < F; b0 += blk) {
    const int b1 = std::min(F, b0 + blk);
    int nb = 0;
    for (int f = b0; f < b1; ++f) nb += ds->feats[f].num_bin;
    const bool fits = (size_t)(cur.num_bins + nb) * bpb <= budget && (b1 - cur.f_begin) <= 128;
    if (cur.f_end > cur.f_begin && !fits) {
      groups.push_back(cur);
      cur = DevFeatureGroup{b0, b0, ds->feats[b0].bin_off, 0, 0, 0};
    }
    if (cur.f_end == cur.f_begin) {
      cur.f_begin = b0;
      cur.bin_base = ds->feats[b0].bin_off;
    }
    cur.f_end = b1;
    cur.num_bins += nb;
  }
  if (cur.f_end > cur.f_begin) groups.push_back(cur);
  size_t max_bins = 0;
  for (auto& g : groups) max_bins = std::max(max_bins, (size_t)g.num_bins);
  build_smem = max_bins * bpb;
  gh_mode = mode;
  CUDA_TRY(d_groups.alloc(groups.size()));
  CUDA_TRY(cudaMemcpy(d_groups.p, groups.data(), groups.size() * sizeof(DevFeatureGroup),
                      cudaMemcpyHostToDevice));
  set_build_smem_limit(build_smem);
  CUDA_TRY(cudaGetLastError());
  // grid: resident CTAs of the build kernel, and enough CTAs to keep <= 2^18 rows each
  int per_sm = std::max(1, (int)((228 * 1024) / (build_smem + 4096)));
  per_sm = std::min(per_sm, 4);
  const int sms = sm_count(device);
  build_blocks = sms * per_sm;
  if (groups.size() > 1)  // about two waves over all groups (see the quantized build)
    build_blocks = std::max(1, (2 * sms * per_sm + (int)groups.size() - 1) / (int)groups.size());
  const int64_t need = (ds->num_data + (1 << 18) - 1) >> 18;
  if (build_blocks < need) build_blocks = (int)need;
  // the fused partition's cell layout (feature << shift) + bin, for f32 gradients
  int shift = 4;
  for (int f = 0; f < F; ++f)
    while ((1 << shift) < ds->feats[f].num_bin) ++shift;
  q4_shift = shift;
  q4_nch = (F + 15) / 16;
  return LGBM_B200_OK;
}

int lgbm_b200_learner::init(lgbm_b200_dataset* dataset, const lgbm_b200_learner_config& c) {
  ds = dataset;
  cfg = c;
  device = ds->device;
  L = c.num_leaves;
  if (L < 2) L = 2;
  if (L > 256)
    return fail(LGBM_B200_CAPABILITY_UNAVAILABLE,
                "num_leaves %d: the device learner supports at most 256 leaves", L);
  slot_len = 2 * ds->total_bins;
  const int64_t N = ds->num_data;
  max_tiles = (int32_t)((N + 2047) / 2048) + 1;
  // The main stream at the highest priority and the look-ahead stream at the lowest: when
  // both have CTAs waiting for an SM, the main-stream partition of the pick goes first
  // (graphs keep each kernel's capture-stream priority: cudaGraphInstantiateFlagUseNodePriority).
  int prio_lo = 0, prio_hi = 0;
  CUDA_TRY(cudaDeviceGetStreamPriorityRange(&prio_lo, &prio_hi));
  if (const char* e = std::getenv("LGBM_B200_STREAM_PRIORITY"))
    if (e[0] == '0') prio_lo = prio_hi = 0;
  CUDA_TRY(cudaStreamCreateWithPriority(&stream, cudaStreamNonBlocking, prio_hi));
  CUDA_TRY(ctrl.alloc(1));
  CUDA_TRY(cudaMemset(ctrl.p, 0, sizeof(GrowCtrl)));
  CUDA_TRY(leaf_i32.alloc((size_t)7 * L));
  CUDA_TRY(ls.alloc(L));
  CUDA_TRY(best.alloc(L));
  CUDA_TRY(splittable.alloc((size_t)L * ds->num_features));
  CUDA_TRY(tree_i32.alloc((size_t)7 * L));
  CUDA_TRY(tree_thr.alloc(L));
  CUDA_TRY(tree_gain.alloc(L));
  CUDA_TRY(tree_dec.alloc(L));
  CUDA_TRY(tree_f64.alloc((size_t)3 * L));
  CUDA_TRY(idx.alloc((size_t)2 * N));
  CUDA_TRY(part_status.alloc(max_tiles));
  CUDA_TRY(pool.alloc((size_t)L * slot_len));
  CUDA_TRY(raw.alloc((size_t)slot_len + 2));
  CUDA_TRY(cudaMemset(raw.p, 0, ((size_t)slot_len + 2) * sizeof(long long)));
  CUDA_TRY(rawpool.alloc((size_t)L * slot_len));
  CUDA_TRY(partials.alloc((size_t)kPrivateTiles * slot_len));

  CUDA_TRY(scan_out.alloc((size_t)2 * ds->num_features));
  CUDA_TRY(cat_words.alloc((size_t)kCatWords * (2 * ds->num_features + 2 * L + 1)));
  CUDA_TRY(cudaMemset(cat_words.p, 0,
                      sizeof(uint32_t) * kCatWords * (2 * ds->num_features + 2 * L + 1)));
  CUDA_TRY(scan_ok.alloc(2));
  CUDA_TRY(la.alloc(kLaSlots));
  CUDA_TRY(mainrec.alloc(2));
  CUDA_TRY(cudaMemset(mainrec.p, 0, 2 * sizeof(LookAhead)));
  CUDA_TRY(cudaMemset(la.p, 0, kLaSlots * sizeof(LookAhead)));
  CUDA_TRY(la_raw.alloc(kLaSlots * ((size_t)slot_len + 2)));
  CUDA_TRY(la_partials.alloc((size_t)kLaSlots * kPrivateTiles * slot_len));
  CUDA_TRY(la_status.alloc(max_tiles));
  CUDA_TRY(cudaStreamCreateWithPriority(&las.st, cudaStreamNonBlocking, prio_lo));
  CUDA_TRY(cudaEventCreateWithFlags(&las.fork, cudaEventDisableTiming));
  for (cudaEvent_t& e : las.done) CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  {
    const int sms = sm_count(device);
    las.blocks = std::max(sms / 2, sms - std::min(ds->num_features, sms));
    las.main_blocks = sms;
    // Past the first splits the main partition almost always finds its leaf done by the
    // look-ahead. A smaller grid then costs less (fewer CTAs to place and retire) and leaves
    // the SMs to the look-ahead launched next to it; the few leaves it does partition there
    // are small.
    las.main_late_blocks = std::max(1, sms * 7 / 16);
    las.main_early_steps = 16;
    // launch-shape overrides (tuning): look-ahead and main-partition CTAs
    // With the main partition inside the control step the look-ahead does better with every
    // SM: its idle CTAs return at once, and the control step's CTAs are placed as they do.
    las.blocks_fused = sms;
    if (const char* e = std::getenv("LGBM_B200_LA_BLOCKS"))
      las.blocks = las.blocks_fused = std::max(1, std::atoi(e));
    if (const char* e = std::getenv("LGBM_B200_MAIN_BLOCKS"))
      las.main_blocks = std::max(1, std::atoi(e));
    if (const char* e = std::getenv("LGBM_B200_MAIN_LATE_BLOCKS"))
      las.main_late_blocks = std::max(1, std::atoi(e));
    if (const char* e = std::getenv("LGBM_B200_MAIN_EARLY_STEPS"))
      las.main_early_steps = std::max(0, std::atoi(e));
  }
  if (const char* e = std::getenv("LGBM_B200_LOOKAHEAD")) la_enabled = std::strcmp(e, "0") != 0;
  d = GrowDev{};
  d.ctrl = ctrl.p;
  d.feat = ds->d_feats.p;
  d.F = ds->num_features;
  d.packed4 = ds->packed4;
  d.sliced = 0;  // every feature on this device (a data-parallel job may slice them)
  if (const char* e = std::getenv("LGBM_B200_WARP_AGG")) d.warp_agg = std::strcmp(e, "1") == 0;
  d.warm_pick = 1;
  if (const char* e = std::getenv("LGBM_B200_WARM_PICK")) d.warm_pick = std::strcmp(e, "0") != 0;
  d.fuse_main = 1;
  if (const char* e = std::getenv("LGBM_B200_FUSE_MAIN")) d.fuse_main = std::strcmp(e, "0") != 0;
  d.la_cancel = 1;
  if (const char* e = std::getenv("LGBM_B200_LA_CANCEL")) d.la_cancel = std::strcmp(e, "0") != 0;
  d.slice_begin = 0;
  d.slice_end = d.F;
  d.bins = ds->bins.p;
  d.stride = ds->stride;
  d.L = L;
  d.N = N;
  d.max_depth = c.max_depth;
  d.slot_len = slot_len;
  d.gain = to_dev_gain(c.gain);
  d.leaf_begin = leaf_i32.p;
  d.leaf_count = leaf_i32.p + L;
  d.leaf_buf = leaf_i32.p + 2 * L;
  d.slot_of_leaf = leaf_i32.p + 3 * L;
  d.best_feature = leaf_i32.p + 4 * L;
  d.leaf_count_g = leaf_i32.p + 5 * L;
  d.leaf_is_right = leaf_i32.p + 6 * L;
  d.ls = ls.p;
  d.best = best.p;
  d.splittable = splittable.p;
  d.t_left = tree_i32.p;
  d.t_right = tree_i32.p + L;
  d.t_split_feature = tree_i32.p + 2 * L;
  d.t_leaf_count = tree_i32.p + 3 * L;
  d.t_internal_count = tree_i32.p + 4 * L;
  d.t_leaf_depth = tree_i32.p + 5 * L;
  d.t_leaf_parent = tree_i32.p + 6 * L;
  d.t_threshold = tree_thr.p;
  d.t_split_gain = tree_gain.p;
  d.t_decision = tree_dec.p;
  d.t_leaf_value = tree_f64.p;
  d.t_leaf_weight = tree_f64.p + L;
  d.t_internal_value = tree_f64.p + 2 * L;
  d.idx0 = idx.p;
  d.idx1 = idx.p + N;
  d.part_status = part_status.p;
  d.max_tiles = max_tiles;
  d.pool = pool.p;
  d.raw = raw.p;
  // one device: the accumulator is its own one-rank exchange
  CUDA_TRY(xtab.alloc(1));
  CUDA_TRY(cudaMemcpy(xtab.p, &raw.p, sizeof(long long*), cudaMemcpyHostToDevice));
  d.xranks = 1;
  d.xrank = 0;
  d.xpar = 0;
  d.xbuf = xtab.p;
  d.rawpool = rawpool.p;
  d.partials = partials.p;
  d.private_tiles = kPrivateTiles;

  d.raw_len = slot_len;
  d.n_global = N;
  d.scan_out = scan_out.p;
  d.scan_cat = cat_words.p;
  d.best_cat = cat_words.p + (size_t)kCatWords * 2 * ds->num_features;
  d.t_cat = d.best_cat + (size_t)kCatWords * L;
  d.split_cat = d.t_cat + (size_t)kCatWords * L;
  d.has_cat = 0;
  int32_t max_bins = 0;
  for (const DevFeature& f : ds->feats) {
    if (f.flags & kFeatCategorical) d.has_cat = 1;
    max_bins = std::max(max_bins, f.num_bin);
  }
  // Narrow features (wide data such as max_bin 63): one 256-thread control-step CTA per
  // feature, four resident per SM, instead of 1024 threads of which most would idle
  // (LGBM_B200_NARROW_SCAN=0 keeps the 1024-thread CTAs).
  const char* ns = std::getenv("LGBM_B200_NARROW_SCAN");
  d.narrow_scan = (!d.has_cat && max_bins <= 64 && !(ns && ns[0] == '0')) ? 1 : 0;
  d.scan_ok = scan_ok.p;
  d.la = la.p;
  d.mainrec = mainrec.p;
  d.la_raw = la_raw.p;
  d.la_partials = la_partials.p;
  d.la_status = la_status.p;
  return LGBM_B200_OK;
}

void lgbm_b200_learner::bind(const void* gh_ptr, const DevGhParams* ghp_ptr,
                             const int32_t* stopped) {
  d.gh = gh_ptr;
  d.ghp = ghp_ptr;
  d.stopped = stopped;
  d.gh_mode = gh_mode;
  d.q4_shift = q4_shift;
  d.fused = fused_partition_supported(gh_mode, ds->num_features, q4_shift, q4_nch,
                                      ds->packed4 != 0) ? 1 : 0;
  d.lookahead = d.fused && la_enabled ? 1 : 0;

  d.q4_nch = q4_nch;
  d.groups = d_groups.p;
  d.num_groups = (int32_t)groups.size();
}

namespace {

int read_tree(lgbm_b200_learner* l, lgbm_b200_tree* out) {
  const int L = l->L;
  GrowCtrl c;
  CUDA_TRY(cudaMemcpy(&c, l->ctrl.p, sizeof(GrowCtrl), cudaMemcpyDeviceToHost));
  if (c.error)
    return fail(LGBM_B200_RUNTIME, "tree grower reported device error bits 0x%x", c.error);
  std::vector<int32_t> ti((size_t)7 * L);
  std::vector<uint32_t> thr(L);
  std::vector<float> gain(L);
  std::vector<int8_t> dec(L);
  std::vector<double> tf((size_t)3 * L);
  CUDA_TRY(cudaMemcpy(ti.data(), l->tree_i32.p, ti.size() * 4, cudaMemcpyDeviceToHost));
  CUDA_TRY(cudaMemcpy(thr.data(), l->tree_thr.p, thr.size() * 4, cudaMemcpyDeviceToHost));
  CUDA_TRY(cudaMemcpy(gain.data(), l->tree_gain.p, gain.size() * 4, cudaMemcpyDeviceToHost));
  CUDA_TRY(cudaMemcpy(dec.data(), l->tree_dec.p, dec.size(), cudaMemcpyDeviceToHost));
  CUDA_TRY(cudaMemcpy(tf.data(), l->tree_f64.p, tf.size() * 8, cudaMemcpyDeviceToHost));
  const int nl = c.num_leaves;
  if (out->max_leaves < nl)
    return fail(LGBM_B200_LENGTH_MISMATCH, "tree_out holds %d leaves, tree has %d",
                out->max_leaves, nl);
  out->num_leaves = nl;
  for (int i = 0; i + 1 < nl; ++i) {
    if (out->left_child) out->left_child[i] = ti[i];
    if (out->right_child) out->right_child[i] = ti[L + i];
    if (out->split_feature) out->split_feature[i] = ti[2 * L + i];
    if (out->internal_count) out->internal_count[i] = ti[4 * L + i];
    if (out->threshold_bin) out->threshold_bin[i] = thr[i];
    if (out->split_gain) out->split_gain[i] = gain[i];
    if (out->decision_type) out->decision_type[i] = dec[i];
    if (out->internal_value) out->internal_value[i] = tf[2 * L + i];
  }
  for (int i = 0; i < nl; ++i) {
    if (out->leaf_value) out->leaf_value[i] = tf[i];
    if (out->leaf_weight) out->leaf_weight[i] = tf[L + i];
    if (out->leaf_count) out->leaf_count[i] = ti[3 * L + i];
  }
  if (out->cat_bins && nl > 1)
    CUDA_TRY(cudaMemcpy(out->cat_bins, l->d.t_cat, sizeof(uint32_t) * kCatWords * (nl - 1),
                        cudaMemcpyDeviceToHost));
  return LGBM_B200_OK;
}

}  // namespace

// ----------------------------------------------------------------------------------
// Data-parallel communicator: NCCL, loaded at run time so that single-GPU use needs no
// NCCL library. Reductions run on the booster's stream and are captured into its graph.
// ----------------------------------------------------------------------------------

namespace {

struct NcclApi {
  bool ok = false;
  std::string error;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

// The NCCL already in the process (e.g. the one a framework loaded) is used as is, so
// that one process never holds two NCCL builds under one soname; else the library named
// by LGBM_B200_NCCL_LIBRARY, else libnccl.so.2 from the loader's search path. It is
// loaded RTLD_LOCAL, so its symbols do not bind other libraries' NCCL references.
NcclApi load_nccl() {
  NcclApi a;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (!h) {
    const char* path = std::getenv("LGBM_B200_NCCL_LIBRARY");
    h = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
  }
  if (!h) {
    a.error = std::string("cannot load libnccl.so.2: ") + dlerror();
    return a;
  }
  auto sym = [&](const char* name) -> void* { return dlsym(h, name); };
  a.GetUniqueId = reinterpret_cast<decltype(a.GetUniqueId)>(sym("ncclGetUniqueId"));
  a.CommInitRank = reinterpret_cast<decltype(a.CommInitRank)>(sym("ncclCommInitRank"));
  a.CommDestroy = reinterpret_cast<decltype(a.CommDestroy)>(sym("ncclCommDestroy"));
  a.AllReduce = reinterpret_cast<decltype(a.AllReduce)>(sym("ncclAllReduce"));
  a.AllGather = reinterpret_cast<decltype(a.AllGather)>(sym("ncclAllGather"));
  a.GetErrorString = reinterpret_cast<decltype(a.GetErrorString)>(sym("ncclGetErrorString"));
  a.ok = a.GetUniqueId && a.CommInitRank && a.CommDestroy && a.AllReduce && a.AllGather &&
         a.GetErrorString;
  if (!a.ok) a.error = "libnccl.so.2 lacks an expected symbol";
  return a;
}

NcclApi& nccl() {
  static NcclApi api = load_nccl();
  return api;
}

}  // namespace

struct lgbm_b200_comm {
  int device = 0;
  int nranks = 1;
  int rank = 0;
  ncclComm_t comm = nullptr;
  ncclResult_t first_error = ncclSuccess;  // first failure of an enqueued reduction
  DeviceComm dev{};

  void note(ncclResult_t r) {
    if (r != ncclSuccess && first_error == ncclSuccess) first_error = r;
  }
  static void sum_i64(void* ctx, long long* buf, int64_t n, cudaStream_t st) {
    auto* c = static_cast<lgbm_b200_comm*>(ctx);
    c->note(nccl().AllReduce(buf, buf, (size_t)n, ncclInt64, ncclSum, c->comm, st));
  }
  static void max_u32(void* ctx, uint32_t* buf, int64_t n, cudaStream_t st) {
    auto* c = static_cast<lgbm_b200_comm*>(ctx);
    c->note(nccl().AllReduce(buf, buf, (size_t)n, ncclUint32, ncclMax, c->comm, st));
  }
  static void min_u32(void* ctx, uint32_t* buf, int64_t n, cudaStream_t st) {
    auto* c = static_cast<lgbm_b200_comm*>(ctx);
    c->note(nccl().AllReduce(buf, buf, (size_t)n, ncclUint32, ncclMin, c->comm, st));
  }
};

// ----------------------------------------------------------------------------------
// Booster
// ----------------------------------------------------------------------------------

struct lgbm_b200_booster {
  lgbm_b200_dataset* ds = nullptr;
  lgbm_b200_train_config cfg{};
  std::unique_ptr<lgbm_b200_learner> learner;
  DevBuf<float> label;
  DevBuf<double> score;
  DevBuf<uint8_t> gh;  // float2[N] followed by uint16[N]
  DevBuf<DevGhParams> ghp;
  DevBuf<int32_t> state;  // [0] stopped, [1] iter counter
  int32_t capacity = 0;
  DevBuf<int32_t> rec_i32;  // num_leaves[cap], left, right, split_feature, leaf_count, internal_count
  DevBuf<uint32_t> rec_thr;
  DevBuf<float> rec_gain;
  DevBuf<int8_t> rec_dec;
  DevBuf<double> rec_f64;  // leaf_value, leaf_weight, internal_value
  DevBuf<uint32_t> rec_cat;  // [cap][L][kCatWords] categorical node bins
  // lambdarank tables (objective 2)
  DevBuf<int32_t> rank_qb;
  DevBuf<double> rank_f64;  // sigmoid table | discounts | label gains | inverse max DCGs
  DevBuf<int32_t> rank_order;
  DevBuf<unsigned long long> xs_pow;  // stochastic rounding: xorshift jump matrices
  double init_score = 0.0;
  ObjDev obj{};
  FinishDev fin{};
  cudaGraphExec_t graph_exec = nullptr;
  cudaGraph_t graph = nullptr;
  float last_ms = 0.f;
  std::vector<std::pair<int32_t, float>> last_profile;  // (kernel class, ms) per launch
  DevBuf<unsigned long long> spans;  // [2][span_slots(L)] start | end (profile_pipeline)
  std::vector<unsigned long long> span_last;  // the last profiled iteration's spans (host)
  DevBuf<unsigned long long> phases;          // [L][kStepMarks] phase marks of each split step
  std::vector<unsigned long long> phase_last;  // the last profiled iteration's marks (host)
  lgbm_b200_comm* comm = nullptr;  // data-parallel job (null: one device)
  const DeviceComm* dcomm() const { return comm ? &comm->dev : nullptr; }

  int ensure_capacity(int32_t need);
  // Host copy of the first snap_n recorded trees, made by the first get_tree after
  // training (one copy per record field instead of a dozen per tree); training drops it.
  // snap_mu guards the snapshot: ctypes callers release the GIL, so two threads may read
  // trees of one booster at once.
  std::mutex snap_mu;
  int32_t snap_n = -1;
  std::vector<int32_t> snap_i32;  // num_leaves[n] | left | right | split_feature | leaf_count |
                                  // internal_count, [n][L] each
  std::vector<uint32_t> snap_thr;
  std::vector<float> snap_gain;
  std::vector<int8_t> snap_dec;
  std::vector<double> snap_f64;   // leaf_value | leaf_weight | internal_value
  std::vector<uint32_t> snap_cat;
  int snapshot(int32_t n);
  void destroy_graph() {
    if (graph_exec) cudaGraphExecDestroy(graph_exec);
    if (graph) cudaGraphDestroy(graph);
    graph_exec = nullptr;
    graph = nullptr;
  }
  // peer-memory exchange of the accumulated child (data-parallel, one node)
  DevBuf<unsigned long long> xmem;  // [2][raw_len + 2] accumulators | flags | count
  DevBuf<void*> xptrs;              // per-rank accumulator and flag pointers
  DevBuf<uint32_t> arrive;          // producer launches' CTA arrival counters (two kinds)
  std::vector<void*> xpeer;         // the other ranks' regions, opened by IPC handle
  ~lgbm_b200_booster() {
    destroy_graph();
    for (void* p : xpeer)
      if (p) cudaIpcCloseMemHandle(p);
  }
};

int lgbm_b200_booster::snapshot(int32_t n) {
  const size_t L = learner->L, N = (size_t)n;
  snap_i32.resize(N + 5 * N * L);
  snap_thr.resize(N * L);
  snap_gain.resize(N * L);
  snap_dec.resize(N * L);
  snap_f64.resize(3 * N * L);
  snap_cat.resize(N * L * kCatWords);
  if (n > 0) {
    CUDA_TRY(cudaMemcpy(snap_i32.data(), fin.rec_num_leaves, N * 4, cudaMemcpyDeviceToHost));
    const int32_t* i32src[5] = {fin.rec_left, fin.rec_right, fin.rec_split_feature,
                                fin.rec_leaf_count, fin.rec_internal_count};
    for (int a = 0; a < 5; ++a)
      CUDA_TRY(cudaMemcpy(snap_i32.data() + N + a * N * L, i32src[a], N * L * 4,
                          cudaMemcpyDeviceToHost));
    CUDA_TRY(cudaMemcpy(snap_thr.data(), fin.rec_threshold, N * L * 4, cudaMemcpyDeviceToHost));
    CUDA_TRY(cudaMemcpy(snap_gain.data(), fin.rec_split_gain, N * L * 4, cudaMemcpyDeviceToHost));
    CUDA_TRY(cudaMemcpy(snap_dec.data(), fin.rec_decision, N * L, cudaMemcpyDeviceToHost));
    const double* f64src[3] = {fin.rec_leaf_value, fin.rec_leaf_weight, fin.rec_internal_value};
    for (int a = 0; a < 3; ++a)
      CUDA_TRY(cudaMemcpy(snap_f64.data() + a * N * L, f64src[a], N * L * 8,
                          cudaMemcpyDeviceToHost));
    CUDA_TRY(cudaMemcpy(snap_cat.data(), fin.rec_cat, N * L * kCatWords * 4,
                        cudaMemcpyDeviceToHost));
  }
  snap_n = n;
  return LGBM_B200_OK;
}

int lgbm_b200_booster::ensure_capacity(int32_t need) {
  if (need <= capacity) return LGBM_B200_OK;
  snap_n = -1;
  int32_t cap = std::max(need, capacity * 2);
  const int L = learner->L;
  // grow while keeping already recorded trees
  DevBuf<int32_t> i32;
  DevBuf<uint32_t> thr;
  DevBuf<float> gain;
  DevBuf<int8_t> dec;
  DevBuf<double> f64;
  DevBuf<uint32_t> catw;
  CUDA_TRY(i32.alloc((size_t)cap + (size_t)5 * cap * L));
  CUDA_TRY(catw.alloc((size_t)cap * L * kCatWords));
  CUDA_TRY(thr.alloc((size_t)cap * L));
  CUDA_TRY(gain.alloc((size_t)cap * L));
  CUDA_TRY(dec.alloc((size_t)cap * L));
  CUDA_TRY(f64.alloc((size_t)3 * cap * L));
  if (capacity > 0) {
    const size_t oc = capacity, nc = cap, L_ = L;
    CUDA_TRY(cudaMemcpy(i32.p, rec_i32.p, oc * 4, cudaMemcpyDeviceToDevice));
    for (int a = 0; a < 5; ++a)
      CUDA_TRY(cudaMemcpy(i32.p + nc + a * nc * L_, rec_i32.p + oc + a * oc * L_, oc * L_ * 4,
                          cudaMemcpyDeviceToDevice));
    CUDA_TRY(cudaMemcpy(thr.p, rec_thr.p, oc * L_ * 4, cudaMemcpyDeviceToDevice));
    CUDA_TRY(cudaMemcpy(gain.p, rec_gain.p, oc * L_ * 4, cudaMemcpyDeviceToDevice));
    CUDA_TRY(cudaMemcpy(dec.p, rec_dec.p, oc * L_, cudaMemcpyDeviceToDevice));
    for (int a = 0; a < 3; ++a)
      CUDA_TRY(cudaMemcpy(f64.p + a * nc * L_, rec_f64.p + a * oc * L_, oc * L_ * 8,
                          cudaMemcpyDeviceToDevice));
    CUDA_TRY(cudaMemcpy(catw.p, rec_cat.p, oc * L_ * kCatWords * 4, cudaMemcpyDeviceToDevice));
  }
  std::swap(rec_i32.p, i32.p);
  std::swap(rec_i32.n, i32.n);
  std::swap(rec_thr.p, thr.p);
  std::swap(rec_thr.n, thr.n);
  std::swap(rec_gain.p, gain.p);
  std::swap(rec_gain.n, gain.n);
  std::swap(rec_dec.p, dec.p);
  std::swap(rec_dec.n, dec.n);
  std::swap(rec_f64.p, f64.p);
  std::swap(rec_f64.n, f64.n);
  std::swap(rec_cat.p, catw.p);
  std::swap(rec_cat.n, catw.n);
  capacity = cap;
  const size_t nc = cap, L_ = L;
  fin.max_iters = cap;
  fin.rec_num_leaves = rec_i32.p;
  fin.rec_left = rec_i32.p + nc;
  fin.rec_right = rec_i32.p + nc + nc * L_;
  fin.rec_split_feature = rec_i32.p + nc + 2 * nc * L_;
  fin.rec_leaf_count = rec_i32.p + nc + 3 * nc * L_;
  fin.rec_internal_count = rec_i32.p + nc + 4 * nc * L_;
  fin.rec_threshold = rec_thr.p;
  fin.rec_split_gain = rec_gain.p;
  fin.rec_decision = rec_dec.p;
  fin.rec_leaf_value = rec_f64.p;
  fin.rec_leaf_weight = rec_f64.p + nc * L_;
  fin.rec_internal_value = rec_f64.p + 2 * nc * L_;
  fin.rec_cat = rec_cat.p;
  destroy_graph();  // pointers changed
  return LGBM_B200_OK;
}

// ----------------------------------------------------------------------------------
// Allocation-free row partition (lgbm_b200_data_partition_noalloc)
//
// Some callers cannot call cudaMalloc when they partition rows: a host engine whose
// device memory belongs to its own pool allocator (the pool has reserved the HBM up
// front, so a cudaMalloc can fail or fragment it), or a latency-bound loop that cannot
// pay for cudaMalloc/cudaFree, which synchronise the whole device. For them the
// partition's only scratch -- one look-back status word per 2048-row tile, the two
// counters (left total, tile ticket) and the routing descriptor -- lives in the fixed
// array below instead of a cudaMalloc'd buffer. Layout, in 8-byte words:
//   word 0        int32 left total | uint32 tile ticket
//   word 1        uint32 error bits (kErrSpinTimeout: a tile's look-back wait ran out)
//   words 8..     DevFeature routing descriptor
//   words 32..    status words, one per tile, at most LGBM_B200_NOALLOC_MAX_ROWS / 2048
// Every call on a device shares this one array: calls that overlap on the GPU race.
// ----------------------------------------------------------------------------------

namespace {

constexpr int64_t kNoAllocMaxRows = LGBM_B200_NOALLOC_MAX_ROWS;
constexpr int64_t kNoAllocMaxTiles = kNoAllocMaxRows / kPartitionTileRows;
constexpr int kNoAllocHeaderWords = 32;
constexpr int kNoAllocFeatureWord = 8;
static_assert(kNoAllocMaxRows % kPartitionTileRows == 0, "limit is whole tiles");
static_assert(kNoAllocMaxRows <= (int64_t)INT32_MAX, "partition counts are int32");
static_assert(sizeof(DevFeature) <= 8 * (kNoAllocHeaderWords - kNoAllocFeatureWord),
              "descriptor fits the header");

static __device__ __align__(256) unsigned long long
    g_noalloc_partition_scratch[kNoAllocHeaderWords + kNoAllocMaxTiles];

// Per-device result of the symbol lookup. Only a successful lookup is kept: a failed one
// (a transient error, or a first call made during stream capture) is tried again by the
// next call.
struct NoAllocDevice {
  std::mutex mu;
  bool done = false;
  unsigned long long* scratch = nullptr;
  int sms = 0;
};
constexpr int kNoAllocMaxDevices = 64;
NoAllocDevice g_noalloc_devices[kNoAllocMaxDevices];

// Clears what the partition kernel needs at zero (status words of the tiles this call
// uses, both counters) and stores the routing descriptor.
__global__ void k_noalloc_partition_setup(unsigned long long* scratch, int64_t tiles,
                                          DevFeature f) {
  unsigned long long* status = scratch + kNoAllocHeaderWords;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < tiles;
       i += (int64_t)gridDim.x * blockDim.x)
    status[i] = 0ull;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    scratch[0] = 0ull;
    scratch[1] = 0ull;
    *reinterpret_cast<DevFeature*>(scratch + kNoAllocFeatureWord) = f;
  }
}

// The partition kernel writes right-going rows from the back of the range; this puts
// them in ascending order, as the host entry point does, and publishes the split point.
// When a tile's look-back wait ran out, some rows were never written: the split point is
// the sentinel -1 and `order` is left as it is.
__global__ void k_noalloc_partition_finish(const unsigned long long* scratch, uint32_t* order,
                                           int64_t n, int64_t* split_point) {
  if (*reinterpret_cast<const volatile uint32_t*>(scratch + 1) != 0u) {
    if (blockIdx.x == 0 && threadIdx.x == 0) *split_point = -1;
    return;
  }
  const int64_t left = (int64_t)*reinterpret_cast<const int32_t*>(scratch);
  const int64_t half = (n - left) / 2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < half;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t a = order[left + i];
    order[left + i] = order[n - 1 - i];
    order[n - 1 - i] = a;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *split_point = left;
}

}  // namespace

// ----------------------------------------------------------------------------------
// C ABI
// ----------------------------------------------------------------------------------

extern "C" {

const char* lgbm_b200_last_error(void) { return g_last_error.c_str(); }

int32_t lgbm_b200_abi_version(void) { return 104; }

int lgbm_b200_release_cached_memory(int32_t device, int64_t* released_bytes) {
  const size_t freed = release_cached_blocks(device < 0 ? -1 : device);
  if (released_bytes) *released_bytes = (int64_t)freed;
  return LGBM_B200_OK;
}

int lgbm_b200_device_count(int32_t* out) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  if (out) *out = n;
  return LGBM_B200_OK;
}

int lgbm_b200_bin_column(const double* column, int64_t n, const lgbm_b200_bin_config* cfg,
                         lgbm_b200_bin_mapper* mapper_out, double* upper_bounds,
                         int32_t upper_cap, uint32_t* bins_out) {
  if (!column || !cfg || !mapper_out || n < 0)
    return fail(LGBM_B200_INVALID_ARGUMENT, "bin_column: null argument");
  BinMapperHost m = find_bin_from_column(column, n, cfg->max_bin, cfg->min_data_in_bin,
                                         cfg->min_data_in_leaf, cfg->pre_filter != 0,
                                         cfg->use_missing != 0, cfg->zero_as_missing != 0,
                                         cfg->bin_construct_sample_cnt, cfg->data_random_seed);
  mapper_out->num_bin = m.num_bin;
  mapper_out->missing_type = m.missing_type;
  mapper_out->default_bin = m.default_bin;
  mapper_out->most_freq_bin = m.most_freq_bin;
  mapper_out->is_trivial = m.is_trivial ? 1 : 0;
  mapper_out->min_val = m.min_val;
  mapper_out->max_val = m.max_val;
  mapper_out->sparse_rate = m.sparse_rate;
  if (upper_bounds) {
    if (upper_cap < m.num_bin)
      return fail(LGBM_B200_LENGTH_MISMATCH, "upper_bounds holds %d, need %d", upper_cap,
                  m.num_bin);
    std::copy(m.upper.begin(), m.upper.end(), upper_bounds);
  }
  if (bins_out)
    for (int64_t i = 0; i < n; ++i) bins_out[i] = m.value_to_bin(column[i]);
  return LGBM_B200_OK;
}

int lgbm_b200_find_bins(int32_t device, const void* const* columns, int32_t value_width,
                        int64_t n, int32_t num_features, const lgbm_b200_bin_config* cfg,
                        lgbm_b200_bin_mapper* mappers_out, double* upper_bounds,
                        int32_t upper_cap) {
  if (!columns || !cfg || !mappers_out || !upper_bounds || num_features < 0 || n <= 0)
    return fail(LGBM_B200_INVALID_ARGUMENT, "find_bins: argument");
  if (value_width != 4 && value_width != 8)
    return fail(LGBM_B200_INVALID_ARGUMENT, "find_bins: value_width %d is not 4 or 8",
                value_width);
  if (n > (int64_t)INT32_MAX) return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "n > 2^31 - 1");
  if (cfg->max_bin < 2 || cfg->max_bin > 4096)
    return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "find_bins: max_bin %d outside 2..4096",
                cfg->max_bin);
  if (upper_cap < cfg->max_bin + 2)
    return fail(LGBM_B200_LENGTH_MISMATCH, "find_bins: upper_cap %d < max_bin + 2", upper_cap);
  for (int f = 0; f < num_features; ++f)
    if (!columns[f]) return fail(LGBM_B200_INVALID_ARGUMENT, "find_bins: column %d is null", f);
  if (num_features == 0) return LGBM_B200_OK;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    cudaGetLastError();
    return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "no CUDA device");
  }
  if (device < 0 || device >= ndev)
    return fail(LGBM_B200_INVALID_ARGUMENT, "device %d not present", device);
  DeviceGuard guard(device);
  // the sample every column shares (create_sample_indices, bin_mapper.rs:92-95)
  const int32_t total = (int32_t)n;
  const int32_t ks = total < cfg->bin_construct_sample_cnt ? total : cfg->bin_construct_sample_cnt;
  const std::shared_ptr<const std::vector<int32_t>> ip =
      shared_sample_indices(total, ks, cfg->data_random_seed);
  const std::vector<int32_t>& idx = *ip;
  const int64_t k = (int64_t)idx.size();
  if (k == 0) return fail(LGBM_B200_RUNTIME, "find_bins: empty sample");
  // scaled_filter_cnt (bin_mapper.rs:684-689)
  const int32_t filter_cnt = (int32_t)(((int64_t)cfg->min_data_in_leaf * k) / (int64_t)total);
  const int32_t mb = cfg->max_bin, cap = upper_cap;
  // features per batch: about 2 GB of device scratch
  const size_t per_feature = (size_t)k * 45 + (size_t)(4 * mb + 16 + 2 * cap) * 8;
  const int32_t batch =
      (int32_t)std::max<size_t>(1, std::min<size_t>(num_features, (2ull << 30) / per_feature));
  DevBuf<double> vals_a, vals_b, dv, edges, side, upper, meta_f;
  DevBuf<unsigned long long> keys_a, keys_b;
  DevBuf<int32_t> which, na, cnt, cib, meta;
  DevBuf<uint8_t> big;
  const size_t B = (size_t)batch, K = (size_t)k;
  CUDA_TRY(vals_a.alloc(B * K));
  CUDA_TRY(vals_b.alloc(B * K));
  CUDA_TRY(keys_a.alloc(B * K));
  CUDA_TRY(keys_b.alloc(B * K));
  CUDA_TRY(dv.alloc(B * (K + 2)));
  CUDA_TRY(cnt.alloc(B * (K + 2)));
  CUDA_TRY(big.alloc(B * (K + 2)));
  CUDA_TRY(edges.alloc(B * 2 * mb));
  CUDA_TRY(side.alloc(B * (mb + 1)));
  CUDA_TRY(cib.alloc(B * cap));
  CUDA_TRY(upper.alloc(B * cap));
  CUDA_TRY(meta.alloc(B * 6));
  CUDA_TRY(meta_f.alloc(B * 3));
  CUDA_TRY(which.alloc(B));
  CUDA_TRY(na.alloc(B));
  std::vector<double> host_vals(B * K);
  std::vector<int32_t> h_meta(B * 6);
  std::vector<double> h_metaf(B * 3);
  for (int32_t f0 = 0; f0 < num_features; f0 += batch) {
    const int32_t nb = std::min(batch, num_features - f0);
    // gather the sampled rows of each column (ascending indices: a forward sweep of
    // scattered reads), the columns split over the host's cores
    auto gather = [&](int32_t j) {
      double* dst = host_vals.data() + (size_t)j * K;
      if (value_width == 4) {
        const float* col = static_cast<const float*>(columns[f0 + j]);
        for (int64_t i = 0; i < k; ++i) dst[i] = (double)col[idx[i]];
      } else {
        const double* col = static_cast<const double*>(columns[f0 + j]);
        for (int64_t i = 0; i < k; ++i) dst[i] = col[idx[i]];
      }
    };
    {
      const int nt = (int)std::max(1u, std::min<unsigned>(std::thread::hardware_concurrency(),
                                                         (unsigned)nb));
      std::atomic<int32_t> next{0};
      std::vector<std::thread> pool;
      for (int t = 1; t < nt; ++t)
        pool.emplace_back([&] {
          for (int32_t j; (j = next.fetch_add(1)) < nb;) gather(j);
        });
      for (int32_t j; (j = next.fetch_add(1)) < nb;) gather(j);
      for (std::thread& th : pool) th.join();
    }
    CUDA_TRY(cudaMemcpy(vals_a.p, host_vals.data(), (size_t)nb * K * 8, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemset(na.p, 0, (size_t)nb * 4));
    FindBinsDev d{};
    d.vals_a = vals_a.p;
    d.vals_b = vals_b.p;
    d.keys_a = keys_a.p;
    d.keys_b = keys_b.p;
    d.which = which.p;
    d.na_cnt = na.p;
    d.k = k;
    d.nf = nb;
    d.max_bin = mb;
    d.min_data_in_bin = cfg->min_data_in_bin;
    d.filter_cnt = filter_cnt;
    d.pre_filter = cfg->pre_filter ? 1 : 0;
    d.use_missing = cfg->use_missing ? 1 : 0;
    d.zero_as_missing = cfg->zero_as_missing ? 1 : 0;
    d.cap = cap;
    d.dv = dv.p;
    d.cnt = cnt.p;
    d.big = big.p;
    d.edges = edges.p;
    d.side = side.p;
    d.cnt_in_bin = cib.p;
    d.upper = upper.p;
    d.meta = meta.p;
    d.meta_f = meta_f.p;
    launch_find_bins(d, 0);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaDeviceSynchronize());
    CUDA_TRY(cudaMemcpy(h_meta.data(), meta.p, (size_t)nb * 6 * 4, cudaMemcpyDeviceToHost));
    CUDA_TRY(cudaMemcpy(h_metaf.data(), meta_f.p, (size_t)nb * 3 * 8, cudaMemcpyDeviceToHost));
    CUDA_TRY(cudaMemcpy(upper_bounds + (size_t)f0 * cap, upper.p, (size_t)nb * cap * 8,
                        cudaMemcpyDeviceToHost));
    for (int32_t j = 0; j < nb; ++j) {
      lgbm_b200_bin_mapper& m = mappers_out[f0 + j];
      m.num_bin = h_meta[j * 6 + 0];
      m.missing_type = h_meta[j * 6 + 1];
      m.default_bin = h_meta[j * 6 + 2];
      m.most_freq_bin = h_meta[j * 6 + 3];
      m.is_trivial = h_meta[j * 6 + 4];
      m._reserved = 0;  // numerical
      m.min_val = h_metaf[j * 3 + 0];
      m.max_val = h_metaf[j * 3 + 1];
      m.sparse_rate = h_metaf[j * 3 + 2];
    }
  }
  return LGBM_B200_OK;
}

int lgbm_b200_bin_column_categorical(const double* column, int64_t n,
                                     const lgbm_b200_bin_config* cfg,
                                     lgbm_b200_bin_mapper* mapper_out, int32_t* bin_to_category,
                                     int32_t cap, uint32_t* bins_out) {
  if (!column || !cfg || !mapper_out || n < 0)
    return fail(LGBM_B200_INVALID_ARGUMENT, "bin_column_categorical: null argument");
  BinMapperHost m = find_bin_from_column(column, n, cfg->max_bin, cfg->min_data_in_bin,
                                         cfg->min_data_in_leaf, cfg->pre_filter != 0,
                                         cfg->use_missing != 0, cfg->zero_as_missing != 0,
                                         cfg->bin_construct_sample_cnt, cfg->data_random_seed,
                                         true);
  mapper_out->num_bin = m.num_bin;
  mapper_out->missing_type = m.missing_type;
  mapper_out->default_bin = m.default_bin;
  mapper_out->most_freq_bin = m.most_freq_bin;
  mapper_out->is_trivial = m.is_trivial ? 1 : 0;
  mapper_out->_reserved = 1;  // categorical
  mapper_out->min_val = m.min_val;
  mapper_out->max_val = m.max_val;
  mapper_out->sparse_rate = m.sparse_rate;
  if (bin_to_category) {
    if (cap < (int32_t)m.bin_to_category.size())
      return fail(LGBM_B200_LENGTH_MISMATCH, "bin_to_category holds %d, need %d", cap,
                  (int)m.bin_to_category.size());
    std::copy(m.bin_to_category.begin(), m.bin_to_category.end(), bin_to_category);
  }
  if (bins_out)
    for (int64_t i = 0; i < n; ++i) bins_out[i] = m.value_to_bin(column[i]);
  return LGBM_B200_OK;
}

int lgbm_b200_construct_histograms(const uint32_t* binned, const float* gradients,
                                   const float* hessians, int64_t n, uint32_t num_bin,
                                   double* out) {
  if (num_bin == 0) return fail(LGBM_B200_RUNTIME, "construct_histograms: num_bin must be > 0");
  if (num_bin > (uint32_t)kMaxBins)
    return fail(LGBM_B200_CAPABILITY_UNAVAILABLE,
                "construct_histograms: num_bin %u exceeds the u8 bin matrix (256)", num_bin);
  if (n < 0 || (n > 0 && (!binned || !gradients || !hessians)) || !out)
    return fail(LGBM_B200_INVALID_ARGUMENT, "construct_histograms: null argument");
  for (int64_t i = 0; i < n; ++i)
    if (binned[i] >= num_bin)
      return fail(LGBM_B200_BIN_OUT_OF_RANGE, "row %lld bin %u >= num_bin %u", (long long)i,
                  binned[i], num_bin);
  if (!have_device()) return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "no CUDA device");
  std::fill(out, out + 2 * (size_t)num_bin, 0.0);
  if (n == 0) return LGBM_B200_OK;
  // host-side scale choice, as the objective kernel does per iteration
  double mg = 0.0, mh = 0.0;
  for (int64_t i = 0; i < n; ++i) {
    mg = std::max(mg, std::fabs((double)gradients[i]));
    mh = std::max(mh, std::fabs((double)hessians[i]));
  }
  int lg = 0;
  while (lg < 62 && ((int64_t)1 << lg) < n) ++lg;
  auto kscale = [&](double m) -> int {
    if (!(m > 0.0) || !std::isfinite(m)) return 0;
    int e;
    std::frexp(m, &e);
    return std::max(-1000, std::min(1000, 62 - e - lg));
  };
  const int kg = kscale(mg), kh = kscale(mh);
  std::vector<uint8_t> rm((size_t)n * 16, 0);
  std::vector<float2> gh(n);
  for (int64_t i = 0; i < n; ++i) {
    rm[(size_t)i * 16] = (uint8_t)binned[i];
    gh[i] = make_float2(gradients[i], hessians[i]);
  }
  DevBuf<uint8_t> d_rm;
  DevBuf<float2> d_gh;
  DevBuf<long long> d_raw;
  CUDA_TRY(d_rm.alloc(rm.size()));
  CUDA_TRY(d_gh.alloc(n));
  CUDA_TRY(d_raw.alloc(2 * (size_t)num_bin));
  CUDA_TRY(cudaMemcpy(d_rm.p, rm.data(), rm.size(), cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemcpy(d_gh.p, gh.data(), n * sizeof(float2), cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemset(d_raw.p, 0, 2 * (size_t)num_bin * 8));
  launch_construct_histogram_f32(d_rm.p, 16, n, d_gh.p, (int32_t)num_bin, std::ldexp(1.0, kg),
                                 std::ldexp(1.0, kh), d_raw.p, 0);
  CUDA_TRY(cudaGetLastError());
  std::vector<long long> raw(2 * (size_t)num_bin);
  CUDA_TRY(cudaMemcpy(raw.data(), d_raw.p, raw.size() * 8, cudaMemcpyDeviceToHost));
  for (uint32_t b = 0; b < num_bin; ++b) {
    out[2 * b] = (double)raw[2 * b] * std::ldexp(1.0, -kg);
    out[2 * b + 1] = (double)raw[2 * b + 1] * std::ldexp(1.0, -kh);
  }
  return LGBM_B200_OK;
}

static int scan_batch(const double* buf, int64_t buf_len, std::vector<DevFeature>& feats,
                      const lgbm_b200_gain_config* cfg, double sum_g, double sum_h,
                      int32_t num_data, lgbm_b200_split_info* out) {
  if (!have_device()) return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "no CUDA device");
  DevBuf<double> d_hist;
  DevBuf<DevFeature> d_f;
  DevBuf<DevSplitInfo> d_out;
  CUDA_TRY(d_hist.alloc(buf_len));
  CUDA_TRY(d_f.alloc(feats.size()));
  CUDA_TRY(d_out.alloc(feats.size()));
  CUDA_TRY(cudaMemcpy(d_hist.p, buf, buf_len * 8, cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemcpy(d_f.p, feats.data(), feats.size() * sizeof(DevFeature),
                      cudaMemcpyHostToDevice));
  DevLeafSplits ls{num_data, 0, sum_g, sum_h, cfg->parent_output};
  launch_scan_features(d_hist.p, d_f.p, (int32_t)feats.size(), to_dev_gain(*cfg), ls, d_out.p, 0);
  CUDA_TRY(cudaGetLastError());
  std::vector<DevSplitInfo> res(feats.size());
  CUDA_TRY(cudaMemcpy(res.data(), d_out.p, res.size() * sizeof(DevSplitInfo),
                      cudaMemcpyDeviceToHost));
  for (size_t i = 0; i < res.size(); ++i) out[i] = to_abi(res[i]);
  return LGBM_B200_OK;
}

int lgbm_b200_find_best_split(const double* hist, const lgbm_b200_gain_config* cfg,
                              uint32_t num_bin, int32_t offset, uint32_t default_bin,
                              uint32_t most_freq_bin, int32_t skip_default_bin,
                              int32_t na_as_missing, int32_t run_forward, double sum_gradient,
                              double sum_hessian, int32_t num_data, lgbm_b200_split_info* out) {
  if (!hist || !cfg || !out) return fail(LGBM_B200_INVALID_ARGUMENT, "find_best_split: null");
  if (num_bin == 0) return fail(LGBM_B200_RUNTIME, "find_best_split: num_bin must be > 0");
  if (num_bin > (uint32_t)kMaxBins)
    return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "find_best_split: num_bin %u > 256", num_bin);
  if (!(sum_hessian > 0.0))
    return fail(LGBM_B200_RUNTIME,
                "find_best_split: sum_hessian must be > 0 (cnt_factor divides by it)");
  std::vector<DevFeature> f(1);
  f[0] = make_feature((int32_t)num_bin, (int32_t)default_bin, (int32_t)most_freq_bin, 0);
  f[0].offset = offset;
  f[0].flags = (skip_default_bin ? 1 : 0) | (na_as_missing ? 2 : 0) | (run_forward ? 4 : 0);
  f[0].slot_off = 0;
  return scan_batch(hist, 2 * (int64_t)num_bin, f, cfg, sum_gradient, sum_hessian, num_data,
                    out);
}

int lgbm_b200_find_best_splits_batched(const double* buf, int64_t buf_len,
                                       const lgbm_b200_batched_feature* feats, int32_t n_feats,
                                       const lgbm_b200_gain_config* cfg, double sum_gradient,
                                       double sum_hessian, int32_t num_data,
                                       lgbm_b200_split_info* out) {
  if (!buf || !feats || !cfg || !out || n_feats < 0)
    return fail(LGBM_B200_INVALID_ARGUMENT, "find_best_splits_batched: null");
  if (!(sum_hessian > 0.0))
    return fail(LGBM_B200_RUNTIME, "find_best_splits_batched: sum_hessian must be > 0");
  std::vector<DevFeature> f(n_feats);
  for (int i = 0; i < n_feats; ++i) {
    const auto& b = feats[i];
    if (b.num_bin == 0 || b.num_bin > (uint32_t)kMaxBins)
      return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "feature %d: num_bin %u", i, b.num_bin);
    if (b.slot_off < 0 || b.slot_off + 2 * (int64_t)b.num_bin > buf_len)
      return fail(LGBM_B200_LENGTH_MISMATCH, "feature %d slot outside the buffer", i);
    f[i] = make_feature((int32_t)b.num_bin, (int32_t)b.default_bin, (int32_t)b.most_freq_bin, 0);
    f[i].offset = b.offset;
    f[i].flags = (b.skip_default_bin ? 1 : 0) | (b.na_as_missing ? 2 : 0) | (b.run_forward ? 4 : 0);
    f[i].slot_off = (int32_t)b.slot_off;
  }
  if (n_feats == 0) return LGBM_B200_OK;
  return scan_batch(buf, buf_len, f, cfg, sum_gradient, sum_hessian, num_data, out);
}

static int data_partition_impl(const uint32_t* bins, int64_t n, uint32_t num_bin,
                               uint32_t min_bin, uint32_t max_bin, uint32_t threshold,
                               uint32_t most_freq_bin, const int32_t* missing,
                               uint32_t* order_out, int64_t* split_point_out);

int lgbm_b200_data_partition(const uint32_t* bins, int64_t n, uint32_t num_bin, uint32_t min_bin,
                             uint32_t max_bin, uint32_t threshold, uint32_t most_freq_bin,
                             uint32_t* order_out, int64_t* split_point_out) {
  return data_partition_impl(bins, n, num_bin, min_bin, max_bin, threshold, most_freq_bin,
                             nullptr, order_out, split_point_out);
}

int lgbm_b200_data_partition_missing(const uint32_t* bins, int64_t n, uint32_t num_bin,
                                     uint32_t min_bin, uint32_t max_bin, uint32_t threshold,
                                     uint32_t most_freq_bin, uint32_t default_bin,
                                     int32_t missing_type, int32_t default_left,
                                     uint32_t* order_out, int64_t* split_point_out) {
  if (missing_type < 0 || missing_type > 2)
    return fail(LGBM_B200_INVALID_ARGUMENT, "data_partition_missing: missing_type %d",
                missing_type);
  const int32_t m[3] = {(int32_t)default_bin, missing_type, default_left ? 1 : 0};
  return data_partition_impl(bins, n, num_bin, min_bin, max_bin, threshold, most_freq_bin, m,
                             order_out, split_point_out);
}

static int data_partition_impl(const uint32_t* bins, int64_t n, uint32_t num_bin,
                               uint32_t min_bin, uint32_t max_bin, uint32_t threshold,
                               uint32_t most_freq_bin, const int32_t* missing,
                               uint32_t* order_out, int64_t* split_point_out) {
  if (!order_out || !split_point_out || (n > 0 && !bins) || n < 0)
    return fail(LGBM_B200_INVALID_ARGUMENT, "data_partition: null argument");
  if (num_bin == 0) return fail(LGBM_B200_RUNTIME, "data_partition: num_bin must be > 0");
  if (threshold >= num_bin)
    return fail(LGBM_B200_RUNTIME, "data_partition: threshold %u >= num_bin %u", threshold,
                num_bin);
  if (num_bin > (uint32_t)kMaxBins)
    return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "data_partition: num_bin %u > 256", num_bin);
  for (int64_t i = 0; i < n; ++i)
    if (bins[i] >= num_bin)
      return fail(LGBM_B200_BIN_OUT_OF_RANGE, "row %lld bin %u >= num_bin %u", (long long)i,
                  bins[i], num_bin);
  if (n > (int64_t)INT32_MAX) return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "n > 2^31");
  if (!have_device()) return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "no CUDA device");
  *split_point_out = 0;
  if (n == 0) return LGBM_B200_OK;
  std::vector<uint8_t> rm((size_t)n * 16, 0);
  for (int64_t i = 0; i < n; ++i) rm[(size_t)i * 16] = (uint8_t)bins[i];
  DevFeature f = make_feature((int32_t)num_bin, 0, (int32_t)most_freq_bin, 0);
  f.route_min = (int32_t)min_bin;
  f.route_max = (int32_t)max_bin;
  int32_t default_left = 0;
  if (missing) {  // the kernel router's missing-value fan-out
    f.default_bin = missing[0];
    f.missing_type = missing[1];
    f.flags = kFeatMissingRoute;
    default_left = missing[2];
  }
  const int64_t tiles = (n + 2047) / 2048;
  DevBuf<uint8_t> d_rm;
  DevBuf<uint32_t> d_dst;
  DevBuf<unsigned long long> d_status;
  DevBuf<int32_t> d_cnt;  // [0] left total, [1] ticket, [2] error bits
  DevBuf<DevFeature> d_f;
  CUDA_TRY(d_rm.alloc(rm.size()));
  CUDA_TRY(d_dst.alloc(n));
  CUDA_TRY(d_status.alloc(tiles));
  CUDA_TRY(d_cnt.alloc(3));
  CUDA_TRY(d_f.alloc(1));
  CUDA_TRY(cudaMemcpy(d_rm.p, rm.data(), rm.size(), cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemcpy(d_f.p, &f, sizeof(f), cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemset(d_status.p, 0, tiles * 8));
  CUDA_TRY(cudaMemset(d_cnt.p, 0, 12));
  launch_partition_rows(d_rm.p, 16, 0, d_f.p, threshold, default_left, n, d_dst.p, d_status.p,
                        d_cnt.p,
                        reinterpret_cast<uint32_t*>(d_cnt.p + 1),
                        reinterpret_cast<uint32_t*>(d_cnt.p + 2), 0);
  CUDA_TRY(cudaGetLastError());
  int32_t cnt[3];
  CUDA_TRY(cudaMemcpy(cnt, d_cnt.p, 12, cudaMemcpyDeviceToHost));
  if (cnt[2] != 0)
    return fail(LGBM_B200_RUNTIME,
                "data_partition: the look-back wait ran out (error bits 0x%x); no result",
                (unsigned)cnt[2]);
  CUDA_TRY(cudaMemcpy(order_out, d_dst.p, n * 4, cudaMemcpyDeviceToHost));
  // the device writes the right rows from the back; the reference returns them ascending
  std::reverse(order_out + cnt[0], order_out + n);
  *split_point_out = cnt[0];
  return LGBM_B200_OK;
}

int lgbm_b200_data_partition_noalloc(const uint8_t* bins, int64_t n, uint32_t num_bin,
                                     uint32_t min_bin, uint32_t max_bin, uint32_t threshold,
                                     uint32_t most_freq_bin, uint32_t* order_out,
                                     int64_t* split_point_out, void* stream) {
  if (!split_point_out || n < 0 || (n > 0 && (!bins || !order_out)))
    return fail(LGBM_B200_INVALID_ARGUMENT, "data_partition_noalloc: null argument");
  if (num_bin == 0) return fail(LGBM_B200_RUNTIME, "data_partition_noalloc: num_bin must be > 0");
  if (threshold >= num_bin)
    return fail(LGBM_B200_RUNTIME, "data_partition_noalloc: threshold %u >= num_bin %u",
                threshold, num_bin);
  if (num_bin > (uint32_t)kMaxBins)
    return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "data_partition_noalloc: num_bin %u > 256",
                num_bin);
  if (n > kNoAllocMaxRows)
    return fail(LGBM_B200_CAPABILITY_UNAVAILABLE,
                "data_partition_noalloc: n = %lld rows exceeds the fixed scratch limit "
                "LGBM_B200_NOALLOC_MAX_ROWS = %lld; use lgbm_b200_data_partition",
                (long long)n, (long long)kNoAllocMaxRows);
  if (!have_device()) return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "no CUDA device");
  int dev = -1;
  CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "data_partition_noalloc: device %d >= %d",
                dev, kNoAllocMaxDevices);
  NoAllocDevice& nd = g_noalloc_devices[dev];
  unsigned long long* scratch = nullptr;
  int sms = 1;
  {
    std::lock_guard<std::mutex> lock(nd.mu);
    if (!nd.done) {
      unsigned long long* p = nullptr;
      int count = 0;
      cudaError_t err = cudaGetSymbolAddress(reinterpret_cast<void**>(&p),
                                             g_noalloc_partition_scratch);
      if (err == cudaSuccess)
        err = cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
      if (err != cudaSuccess || !p) {
        cudaGetLastError();  // not sticky: the next call tries again
        return fail(LGBM_B200_RUNTIME,
                    "data_partition_noalloc: scratch set-up on device %d failed: %s", dev,
                    cudaGetErrorString(err));
      }
      nd.scratch = p;
      nd.sms = count;
      nd.done = true;
    }
    scratch = nd.scratch;
    sms = std::max(1, nd.sms);
  }
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  DevFeature f = make_feature((int32_t)num_bin, 0, (int32_t)most_freq_bin, 0);
  f.route_min = (int32_t)min_bin;
  f.route_max = (int32_t)max_bin;
  const int64_t tiles = (n + kPartitionTileRows - 1) / kPartitionTileRows;
  const int setup_blocks = (int)std::max<int64_t>(1, std::min<int64_t>((tiles + 255) / 256, sms));
  k_noalloc_partition_setup<<<setup_blocks, 256, 0, st>>>(scratch, tiles, f);
  CUDA_TRY(cudaGetLastError());
  if (n > 0) {
    int32_t* counters = reinterpret_cast<int32_t*>(scratch);
    launch_partition_rows(bins, 1, 0,
                          reinterpret_cast<const DevFeature*>(scratch + kNoAllocFeatureWord),
                          threshold, 0, n, order_out, scratch + kNoAllocHeaderWords, counters,
                          reinterpret_cast<uint32_t*>(counters + 1),
                          reinterpret_cast<uint32_t*>(scratch + 1), st);
    CUDA_TRY(cudaGetLastError());
  }
  const int finish_blocks =
      (int)std::max<int64_t>(1, std::min<int64_t>((n / 2 + 255) / 256, 2 * (int64_t)sms));
  k_noalloc_partition_finish<<<finish_blocks, 256, 0, st>>>(scratch, order_out, n,
                                                            split_point_out);
  CUDA_TRY(cudaGetLastError());
  return LGBM_B200_OK;
}

int lgbm_b200_subtract_histograms(const double* parent, const double* child, int64_t len,
                                  double* out) {
  if (len < 0 || (len > 0 && (!parent || !child || !out)))
    return fail(LGBM_B200_INVALID_ARGUMENT, "subtract_histograms: null argument");
  if (!have_device()) return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "no CUDA device");
  if (len == 0) return LGBM_B200_OK;
  DevBuf<double> a, b, o;
  CUDA_TRY(a.alloc(len));
  CUDA_TRY(b.alloc(len));
  CUDA_TRY(o.alloc(len));
  CUDA_TRY(cudaMemcpy(a.p, parent, len * 8, cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemcpy(b.p, child, len * 8, cudaMemcpyHostToDevice));
  launch_subtract(a.p, b.p, o.p, len, 0);
  CUDA_TRY(cudaGetLastError());
  CUDA_TRY(cudaMemcpy(out, o.p, len * 8, cudaMemcpyDeviceToHost));
  return LGBM_B200_OK;
}

}  // extern "C"

namespace {

// Builds the device dataset: feature-major host columns go up in row chunks and
// k_bin_rows writes the row-major u8 matrix (pre-binned columns are range-checked on
// the device; raw values are binned with the given mappers).
int dataset_build(int32_t device, const void* const* columns, int kind, int64_t num_data,
                  int32_t num_features, const lgbm_b200_feature_meta* meta,
                  const double* const* upper_bounds, const int32_t* const* bin_to_category,
                  lgbm_b200_dataset** out) {
  if (!out || !meta || (num_features > 0 && !columns))
    return fail(LGBM_B200_INVALID_ARGUMENT, "dataset_create: null argument");
  *out = nullptr;
  if (num_data <= 0) return fail(LGBM_B200_RUNTIME, "dataset_create: empty dataset (no rows)");
  if (num_features <= 0) return fail(LGBM_B200_RUNTIME, "dataset_create: no features");
  if (num_data > (int64_t)INT32_MAX - 1)
    return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "num_data %lld exceeds 2^31-1",
                (long long)num_data);
  const bool values = kind == kBinRowsF32 || kind == kBinRowsF64;
  for (int f = 0; f < num_features; ++f) {
    if (!columns[f]) return fail(LGBM_B200_INVALID_ARGUMENT, "feature %d: null column", f);
    if (meta[f].num_bin <= 0 || meta[f].num_bin > kMaxBins)
      return fail(LGBM_B200_CAPABILITY_UNAVAILABLE,
                  "feature %d: num_bin %d outside 1..256 (u8 bin matrix)", f, meta[f].num_bin);
    if (meta[f].most_freq_bin < 0 || meta[f].most_freq_bin >= meta[f].num_bin)
      return fail(LGBM_B200_INVALID_ARGUMENT, "feature %d: most_freq_bin out of range", f);
    if (meta[f].bin_type != 0 && meta[f].bin_type != 1)
      return fail(LGBM_B200_INVALID_ARGUMENT, "feature %d: bin_type %d is not 0 or 1", f,
                  meta[f].bin_type);
    if (values && meta[f].bin_type == 0 && (!upper_bounds || !upper_bounds[f]))
      return fail(LGBM_B200_INVALID_ARGUMENT, "feature %d: no bin upper bounds", f);
    if (values && meta[f].bin_type == 1 && (!bin_to_category || !bin_to_category[f]))
      return fail(LGBM_B200_INVALID_ARGUMENT, "feature %d: no bin_to_category", f);
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    cudaGetLastError();
    return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "no CUDA device");
  }
  if (device < 0 || device >= ndev)
    return fail(LGBM_B200_INVALID_ARGUMENT, "device %d not present", device);
  DeviceGuard guard(device);
  auto ds = std::make_unique<lgbm_b200_dataset>();
  ds->device = device;
  ds->num_data = num_data;
  ds->num_features = num_features;
  // 4-bit rows when every feature has at most 16 bins (max_bin <= 15 and the like): two
  // bins per byte, row stride rounded up to 16 bytes (LGBM_B200_PACK4=0: one byte per bin)
  int32_t max_bins = 0;
  for (int f = 0; f < num_features; ++f) max_bins = std::max(max_bins, meta[f].num_bin);
  const char* p4 = std::getenv("LGBM_B200_PACK4");
  ds->packed4 = (max_bins <= 16 && !(p4 && p4[0] == '0')) ? 1 : 0;
  ds->stride = ds->packed4 ? ((num_features + 31) / 32) * 16 : ((num_features + 15) / 16) * 16;
  int32_t bin_off = 0;
  std::vector<DevBinFeature> bf(num_features);
  std::vector<double> upper;
  std::vector<int32_t> cat_keys;
  std::vector<uint8_t> cat_bins;
  for (int f = 0; f < num_features; ++f) {
    DevFeature d = make_feature(meta[f].num_bin, meta[f].default_bin, meta[f].most_freq_bin,
                                meta[f].missing_type);
    if (meta[f].bin_type == 1) d.flags |= kFeatCategorical;
    d.bin_off = bin_off;
    d.slot_off = 2 * bin_off;
    bin_off += meta[f].num_bin;
    ds->feats.push_back(d);
    DevBinFeature& b = bf[f];
    b.num_bin = meta[f].num_bin;
    b.missing_type = meta[f].missing_type;
    b.bin_type = meta[f].bin_type;
    b.n_cat = 0;
    if (values && b.bin_type == 0) {
      b.off = (int64_t)upper.size();
      upper.insert(upper.end(), upper_bounds[f], upper_bounds[f] + b.num_bin);
    } else if (values) {
      // ascending categories of bins 1.. (bin 0 is the dummy bin of NaN / negatives)
      std::vector<std::pair<int32_t, uint8_t>> kv;
      for (int32_t k = 0; k < b.num_bin; ++k)
        if (bin_to_category[f][k] >= 0) kv.emplace_back(bin_to_category[f][k], (uint8_t)k);
      std::sort(kv.begin(), kv.end());
      b.off = (int64_t)cat_keys.size();
      b.n_cat = (int32_t)kv.size();
      for (auto& e : kv) {
        cat_keys.push_back(e.first);
        cat_bins.push_back(e.second);
      }
    } else {
      b.off = 0;
    }
  }
  ds->total_bins = bin_off;
  CUDA_TRY(ds->bins.alloc((size_t)num_data * ds->stride));
  cudaStream_t st = nullptr;
  CUDA_TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  struct StreamGuard {
    cudaStream_t s;
    ~StreamGuard() { cudaStreamDestroy(s); }
  } sg{st};
  DevBuf<DevBinFeature> d_bf;
  DevBuf<double> d_upper;
  DevBuf<int32_t> d_keys;
  DevBuf<uint8_t> d_cbins;
  DevBuf<unsigned long long> d_bad;
  CUDA_TRY(d_bf.alloc(num_features));
  CUDA_TRY(cudaMemcpy(d_bf.p, bf.data(), num_features * sizeof(DevBinFeature),
                      cudaMemcpyHostToDevice));
  CUDA_TRY(d_upper.alloc(std::max<size_t>(upper.size(), 1)));
  if (!upper.empty())
    CUDA_TRY(cudaMemcpy(d_upper.p, upper.data(), upper.size() * 8, cudaMemcpyHostToDevice));
  CUDA_TRY(d_keys.alloc(std::max<size_t>(cat_keys.size(), 1)));
  CUDA_TRY(d_cbins.alloc(std::max<size_t>(cat_bins.size(), 1)));
  if (!cat_keys.empty()) {
    CUDA_TRY(cudaMemcpy(d_keys.p, cat_keys.data(), cat_keys.size() * 4, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(d_cbins.p, cat_bins.data(), cat_bins.size(), cudaMemcpyHostToDevice));
  }
  CUDA_TRY(d_bad.alloc(1));
  CUDA_TRY(cudaMemset(d_bad.p, 0xff, 8));
  BinRowsDev br{d_bf.p,    num_features, ds->packed4, ds->stride,
                d_upper.p, d_keys.p,     d_cbins.p,   d_bad.p};
  const int elem = kind == kBinRowsF32 ? 4 : kind;
  const int64_t chunk = std::max<int64_t>(
      1, std::min<int64_t>(num_data, (256ll << 20) / ((int64_t)num_features * elem)));
  DevBuf<uint8_t> staging;
  CUDA_TRY(staging.alloc((size_t)chunk * num_features * elem));
  std::vector<const void*> srcs(num_features);
  for (int64_t r0 = 0; r0 < num_data; r0 += chunk) {
    const int64_t n = std::min(chunk, num_data - r0);
    for (int f = 0; f < num_features; ++f)
      srcs[f] = (const uint8_t*)columns[f] + (size_t)r0 * elem;
    CUDA_TRY(staged_h2d(staging.p, srcs.data(), num_features, (size_t)n * elem,
                        (size_t)chunk * elem, st));
    launch_bin_rows(br, kind, staging.p, chunk, n, r0, ds->bins.p + (size_t)r0 * ds->stride, st);
    CUDA_TRY(cudaGetLastError());
  }
  CUDA_TRY(cudaStreamSynchronize(st));
  unsigned long long bad = 0;
  CUDA_TRY(cudaMemcpy(&bad, d_bad.p, 8, cudaMemcpyDeviceToHost));
  if (bad != ~0ull) {
    const int64_t row = (int64_t)(bad / (unsigned long long)num_features);
    const int f = (int)(bad % (unsigned long long)num_features);
    uint32_t b = kind == kBinRowsU8    ? ((const uint8_t*)columns[f])[row]
                 : kind == kBinRowsU16 ? ((const uint16_t*)columns[f])[row]
                                       : ((const uint32_t*)columns[f])[row];
    return fail(LGBM_B200_BIN_OUT_OF_RANGE, "feature %d row %lld: bin %u >= num_bin %d", f,
                (long long)row, b, meta[f].num_bin);
  }
  CUDA_TRY(ds->d_feats.alloc(num_features));
  CUDA_TRY(cudaMemcpy(ds->d_feats.p, ds->feats.data(), num_features * sizeof(DevFeature),
                      cudaMemcpyHostToDevice));
  *out = ds.release();
  return LGBM_B200_OK;
}

}  // namespace

extern "C" {

int lgbm_b200_dataset_create(int32_t device, const void* const* columns, int32_t bin_width,
                             int64_t num_data, int32_t num_features,
                             const lgbm_b200_feature_meta* meta, lgbm_b200_dataset** out) {
  if (bin_width != 1 && bin_width != 2 && bin_width != 4)
    return fail(LGBM_B200_INVALID_ARGUMENT, "bin_width must be 1, 2 or 4");
  return dataset_build(device, columns, bin_width, num_data, num_features, meta, nullptr,
                       nullptr, out);
}

int lgbm_b200_dataset_create_from_values(int32_t device, const void* const* columns,
                                         int32_t value_width, int64_t num_data,
                                         int32_t num_features,
                                         const lgbm_b200_feature_meta* meta,
                                         const double* const* upper_bounds,
                                         const int32_t* const* bin_to_category,
                                         lgbm_b200_dataset** out) {
  if (value_width != 4 && value_width != 8)
    return fail(LGBM_B200_INVALID_ARGUMENT, "value_width must be 4 (f32) or 8 (f64)");
  return dataset_build(device, columns, value_width == 4 ? kBinRowsF32 : kBinRowsF64,
                       num_data, num_features, meta, upper_bounds, bin_to_category, out);
}

int lgbm_b200_dataset_copy_bins(const lgbm_b200_dataset* ds, uint8_t* out) {
  if (!ds || !out) return fail(LGBM_B200_INVALID_ARGUMENT, "dataset_copy_bins: null argument");
  DeviceGuard g(ds->device);
  if (!ds->packed4) {
    CUDA_TRY(cudaMemcpy(out, ds->bins.p, (size_t)ds->num_data * ds->stride,
                        cudaMemcpyDeviceToHost));
    return LGBM_B200_OK;
  }
  // a 4-bit matrix: read back packed, handed out one byte per bin
  const int32_t F = ds->num_features, wide = ((F + 15) / 16) * 16;
  std::vector<uint8_t> packed((size_t)ds->num_data * ds->stride);
  CUDA_TRY(cudaMemcpy(packed.data(), ds->bins.p, packed.size(), cudaMemcpyDeviceToHost));
  for (int64_t r = 0; r < ds->num_data; ++r) {
    const uint8_t* src = packed.data() + (size_t)r * ds->stride;
    uint8_t* dst = out + (size_t)r * wide;
    for (int32_t f = 0; f < wide; ++f)
      dst[f] = f < F ? (uint8_t)((src[f >> 1] >> ((f & 1) * 4)) & 15) : 0;
  }
  return LGBM_B200_OK;
}

int lgbm_b200_dataset_destroy(lgbm_b200_dataset* ds) {
  if (ds) {
    DeviceGuard g(ds->device);
    delete ds;
  }
  return LGBM_B200_OK;
}

int lgbm_b200_dataset_num_data(const lgbm_b200_dataset* ds, int64_t* out) {
  if (!ds || !out) return fail(LGBM_B200_INVALID_ARGUMENT, "null argument");
  *out = ds->num_data;
  return LGBM_B200_OK;
}

int lgbm_b200_learner_create(lgbm_b200_dataset* ds, const lgbm_b200_learner_config* cfg,
                             lgbm_b200_learner** out) {
  if (!ds || !cfg || !out) return fail(LGBM_B200_INVALID_ARGUMENT, "learner_create: null");
  *out = nullptr;
  if (cfg->num_leaves < 1)
    return fail(LGBM_B200_INVALID_ARGUMENT, "InvalidNumLeaves: %d", cfg->num_leaves);
  DeviceGuard g(ds->device);
  auto l = std::make_unique<lgbm_b200_learner>();
  int rc = l->init(ds, *cfg);
  if (rc) return rc;
  CUDA_TRY(l->gh.alloc((size_t)ds->num_data * 10));
  CUDA_TRY(l->ghp.alloc(1));
  CUDA_TRY(cudaMemset(l->ghp.p, 0, sizeof(DevGhParams)));
  *out = l.release();
  return LGBM_B200_OK;
}

int lgbm_b200_learner_destroy(lgbm_b200_learner* l) {
  if (l) {
    DeviceGuard g(l->device);
    if (l->stream) cudaStreamDestroy(l->stream);
    delete l;
  }
  return LGBM_B200_OK;
}

int lgbm_b200_learner_grow_tree(lgbm_b200_learner* l, int32_t gh_kind, const void* gh,
                                const double* quant_scales, lgbm_b200_tree* tree_out,
                                uint32_t* indices_out, int32_t* leaf_begin_out,
                                int32_t* leaf_count_out) {
  if (!l || !gh || !tree_out) return fail(LGBM_B200_INVALID_ARGUMENT, "grow_tree: null argument");
  DeviceGuard g(l->device);
  const int64_t N = l->ds->num_data;
  int mode;
  DevGhParams hp{};
  if (gh_kind == LGBM_B200_GH_F32) {
    mode = GH_FLOAT;
    std::vector<float2> v(N);
    const float* gp = (const float*)gh;
    for (int64_t i = 0; i < N; ++i) v[i] = make_float2(gp[i], gp[N + i]);
    CUDA_TRY(cudaMemcpyAsync(l->gh.p, v.data(), N * sizeof(float2), cudaMemcpyHostToDevice,
                             l->stream));
    CUDA_TRY(cudaStreamSynchronize(l->stream));
  } else if (gh_kind == LGBM_B200_GH_INT8_PAIR) {
    if (!quant_scales) return fail(LGBM_B200_INVALID_ARGUMENT, "grow_tree: quant_scales");
    const int bins = (int)quant_scales[3];
    mode = bins <= 4 ? GH_QPACK : GH_QLUT;
    const int8_t* q = (const int8_t*)gh;
    std::vector<uint16_t> v(N);
    for (int64_t i = 0; i < N; ++i)
      v[i] = (uint16_t)((uint8_t)q[2 * i] | ((uint16_t)(uint8_t)q[2 * i + 1] << 8));
    CUDA_TRY(cudaMemcpyAsync(l->gh.p + 8 * N, v.data(), N * 2, cudaMemcpyHostToDevice,
                             l->stream));
    CUDA_TRY(cudaStreamSynchronize(l->stream));
    hp.grad_scale = quant_scales[0];
    hp.hess_scale = quant_scales[1];
    hp.is_const_hess = quant_scales[2] != 0.0 ? 1 : 0;
    hp.num_quant_bins = bins;
  } else {
    return fail(LGBM_B200_INVALID_ARGUMENT, "grow_tree: unknown gh_kind %d", gh_kind);
  }
  if (l->gh_mode != mode || l->groups.empty()) {
    int rc = l->configure_groups(mode);
    if (rc) return rc;
  }
  hp.mode = mode;
  CUDA_TRY(cudaMemcpyAsync(l->ghp.p, &hp, sizeof(hp), cudaMemcpyHostToDevice, l->stream));
  l->bind(mode == GH_FLOAT ? (const void*)l->gh.p : (const void*)(l->gh.p + 8 * N), l->ghp.p,
          nullptr);
  ObjDev o{};
  o.N = N;
  o.n_global = N;
  o.gh_mode = mode;
  o.gh = l->gh.p;
  o.ghp = l->ghp.p;
  o.num_quant_bins = hp.num_quant_bins;
  launch_learner_gradients(o, gh_kind, l->stream);
  launch_tree(l->d, l->build_blocks, l->build_smem, l->stream, nullptr, nullptr, &l->las);
  CUDA_TRY(cudaGetLastError());
  CUDA_TRY(cudaStreamSynchronize(l->stream));
  int rc = read_tree(l, tree_out);
  if (rc) return rc;
  const int nl = tree_out->num_leaves;
  if (leaf_begin_out)
    CUDA_TRY(cudaMemcpy(leaf_begin_out, l->d.leaf_begin, nl * 4, cudaMemcpyDeviceToHost));
  if (leaf_count_out)
    CUDA_TRY(cudaMemcpy(leaf_count_out, l->d.leaf_count, nl * 4, cudaMemcpyDeviceToHost));
  if (indices_out) {
    DevBuf<uint32_t> out;
    CUDA_TRY(out.alloc(N));
    launch_gather_partition(l->d, out.p, l->stream);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaStreamSynchronize(l->stream));
    CUDA_TRY(cudaMemcpy(indices_out, out.p, N * 4, cudaMemcpyDeviceToHost));
  }
  return LGBM_B200_OK;
}

}  // extern "C"

namespace {

// All ranks' labels in global row order (shards in rank order), gathered once so that
// the init score is computed exactly as on one device.
int gather_labels(lgbm_b200_comm* comm, const float* labels, int64_t n_local, cudaStream_t st,
                  std::vector<float>* all, int64_t* row_offset) {
  const int R = comm->nranks;
  DevBuf<long long> cnt;
  CUDA_TRY(cnt.alloc((size_t)R + 1));
  long long mine = n_local;
  CUDA_TRY(cudaMemcpy(cnt.p + R, &mine, 8, cudaMemcpyHostToDevice));
  ncclResult_t r = nccl().AllGather(cnt.p + R, cnt.p, 1, ncclInt64, comm->comm, st);
  if (r != ncclSuccess)
    return fail(LGBM_B200_RUNTIME, "NCCL all-gather failed: %s", nccl().GetErrorString(r));
  std::vector<long long> counts(R);
  CUDA_TRY(cudaStreamSynchronize(st));
  CUDA_TRY(cudaMemcpy(counts.data(), cnt.p, 8 * (size_t)R, cudaMemcpyDeviceToHost));
  long long mx = 0, total = 0;
  for (long long c : counts) {
    mx = std::max(mx, c);
    total += c;
  }
  *row_offset = 0;
  for (int k = 0; k < comm->rank && k < R; ++k) *row_offset += counts[k];
  DevBuf<float> send, recv;
  CUDA_TRY(send.alloc((size_t)std::max(mx, 1ll)));
  CUDA_TRY(recv.alloc((size_t)std::max(mx, 1ll) * R));
  CUDA_TRY(cudaMemset(send.p, 0, (size_t)std::max(mx, 1ll) * 4));
  if (n_local > 0)
    CUDA_TRY(cudaMemcpy(send.p, labels, (size_t)n_local * 4, cudaMemcpyHostToDevice));
  r = nccl().AllGather(send.p, recv.p, (size_t)std::max(mx, 1ll), ncclFloat32, comm->comm, st);
  if (r != ncclSuccess)
    return fail(LGBM_B200_RUNTIME, "NCCL all-gather failed: %s", nccl().GetErrorString(r));
  std::vector<float> padded((size_t)std::max(mx, 1ll) * R);
  CUDA_TRY(cudaStreamSynchronize(st));
  CUDA_TRY(cudaMemcpy(padded.data(), recv.p, padded.size() * 4, cudaMemcpyDeviceToHost));
  all->clear();
  all->reserve((size_t)total);
  for (int k = 0; k < R; ++k)
    all->insert(all->end(), padded.begin() + (size_t)k * std::max(mx, 1ll),
                padded.begin() + (size_t)k * std::max(mx, 1ll) + counts[k]);
  return LGBM_B200_OK;
}

// Lambdarank::new (lgbm-objective/src/rank.rs:152-227): validated query boundaries and
// labels, then the tables the device objective reads. DcgCalculator
// (lgbm-metric/src/dcg_calculator.rs:48-162): gains 2^i - 1 unless given, discount
// 1 / log2(2 + rank), per-query 1 / max DCG at the truncation level; the 2^20-entry
// sigmoid table of ConstructSigmoidTable. Built here with the host libm, like the
// reference's.
struct RankTables {
  std::vector<double> sig, discount, gain, inv_max;
  double sig_min = 0.0, sig_max = 0.0, sig_factor = 0.0;
};

int rank_tables(const lgbm_b200_train_config& cfg, const float* labels, int64_t n,
                RankTables* rt) {
  const int32_t* qb = cfg.query_boundaries;
  const int32_t nq = cfg.num_queries;
  if (!qb || nq < 1)
    return fail(LGBM_B200_INVALID_ARGUMENT, "lambdarank needs query boundaries");
  if (qb[0] != 0 || (int64_t)qb[nq] != n)
    return fail(LGBM_B200_INVALID_ARGUMENT,
                "query boundaries must run from 0 to num_data %lld (got %d .. %d)",
                (long long)n, qb[0], qb[nq]);
  for (int32_t q = 0; q < nq; ++q) {
    if (qb[q + 1] < qb[q])
      return fail(LGBM_B200_INVALID_ARGUMENT, "query boundaries must be non-decreasing");
    if (qb[q + 1] - qb[q] > LGBM_B200_MAX_QUERY_ROWS)
      return fail(LGBM_B200_INVALID_ARGUMENT, "query %d has %d rows (more than %d)", q,
                  qb[q + 1] - qb[q], LGBM_B200_MAX_QUERY_ROWS);
  }
  if (cfg.lambdarank_truncation_level < 0)
    return fail(LGBM_B200_INVALID_ARGUMENT, "lambdarank_truncation_level %d",
                cfg.lambdarank_truncation_level);
  if (cfg.num_label_gain > 0) {
    if (!cfg.label_gain) return fail(LGBM_B200_INVALID_ARGUMENT, "label_gain: null pointer");
    rt->gain.assign(cfg.label_gain, cfg.label_gain + cfg.num_label_gain);
  } else {
    rt->gain.push_back(0.0);
    for (int i = 1; i < 31; ++i) rt->gain.push_back((double)((1ll << i) - 1));
  }
  // DcgCalculator::check_labels: integral, non-negative, inside the gain table
  for (int64_t i = 0; i < n; ++i) {
    const float l = labels[i];
    if (!(std::fabs(l - (float)(int32_t)l) <= 1e-15f))
      return fail(LGBM_B200_INVALID_ARGUMENT, "ranking label %g at row %lld is not an integer",
                  (double)l, (long long)i);
    if (l < 0.0f || (size_t)l >= rt->gain.size())
      return fail(LGBM_B200_INVALID_ARGUMENT,
                  "ranking label %g at row %lld outside the %zu label gains", (double)l,
                  (long long)i, rt->gain.size());
  }
  rt->discount.resize(LGBM_B200_MAX_QUERY_ROWS);
  for (int i = 0; i < LGBM_B200_MAX_QUERY_ROWS; ++i)
    rt->discount[i] = 1.0 / std::log2(2.0 + (double)i);
  rt->inv_max.resize(nq);
  std::vector<int64_t> cnt(rt->gain.size());
  for (int32_t q = 0; q < nq; ++q) {
    std::fill(cnt.begin(), cnt.end(), 0);
    for (int32_t i = qb[q]; i < qb[q + 1]; ++i) cnt[(size_t)labels[i]] += 1;
    double m = 0.0;
    int64_t top = (int64_t)rt->gain.size() - 1;
    const int64_t k = std::min<int64_t>(cfg.lambdarank_truncation_level, qb[q + 1] - qb[q]);
    for (int64_t j = 0; j < k; ++j) {
      while (top > 0 && cnt[top] <= 0) --top;
      if (top < 0) break;
      m += rt->discount[j] * rt->gain[top];
      cnt[top] -= 1;
    }
    rt->inv_max[q] = m > 0.0 ? 1.0 / m : m;
  }
  rt->sig_min = -50.0 / cfg.sigmoid / 2.0;
  rt->sig_max = -rt->sig_min;
  rt->sig_factor = (double)kRankSigmoidBins / (rt->sig_max - rt->sig_min);
  rt->sig.resize(kRankSigmoidBins);
  for (int64_t i = 0; i < kRankSigmoidBins; ++i) {
    const double x = (double)i / rt->sig_factor + rt->sig_min;
    rt->sig[i] = 1.0 / (1.0 + std::exp(x * cfg.sigmoid));
  }
  return LGBM_B200_OK;
}

// The accumulated child crosses between the ranks over peer memory instead of an NCCL
// all-reduce when every rank can map every other rank's exchange region (CUDA IPC
// handles, swapped over the NCCL communicator). All ranks agree on the outcome, so either
// all exchange over peer memory or all keep NCCL. LGBM_B200_PEER_EXCHANGE=0 keeps NCCL;
// LGBM_B200_PEER_WAIT_MS sets the wait limit (default 2000 ms).
int setup_peer_exchange(lgbm_b200_booster* b, lgbm_b200_comm* comm) {
  const int R = comm->nranks;
  const char* env = std::getenv("LGBM_B200_PEER_EXCHANGE");
  const bool want = R >= 2 && R <= kMaxXRanks && !(env && std::strcmp(env, "0") == 0);
  GrowDev& d = b->learner->d;
  if (!want) return LGBM_B200_OK;
  cudaStream_t st = b->learner->stream;
  const size_t xs = (size_t)d.raw_len + 2;
  // one region per rank, opened by the others: the two exchange accumulators, their
  // flags and count, then the look-ahead slots, their flags and count
  const size_t off_la = 2 * xs + kMaxXRanks + 1;
  const size_t off_laflags = off_la + kLaSlots * xs;
  const size_t off_laseq = off_laflags + kMaxXRanks;
  // then the sliced pick's records [2][kMaxXRanks], their flags and count
  const size_t off_pick = (off_laseq + 1 + 1) / 2 * 2;  // 16-byte aligned records
  const size_t off_pickflags = off_pick + 2 * kMaxXRanks * (size_t)kXPickWords;
  const size_t off_pickseq = off_pickflags + kMaxXRanks;
  const size_t words = off_pickseq + 1;
  b->xmem.nocache = true;
  CUDA_TRY(b->xmem.alloc(words));
  CUDA_TRY(cudaMemset(b->xmem.p, 0, words * 8));
  // every rank's IPC handle, in rank order (the all-gather moves 8-byte words)
  constexpr int kH = (int)sizeof(cudaIpcMemHandle_t);
  static_assert(kH % 8 == 0, "IPC handles move as 8-byte words");
  cudaIpcMemHandle_t mine;
  int ok = cudaIpcGetMemHandle(&mine, b->xmem.p) == cudaSuccess ? 1 : 0;
  cudaGetLastError();
  DevBuf<long long> hbuf;
  CUDA_TRY(hbuf.alloc((size_t)(R + 1) * kH / 8));
  CUDA_TRY(cudaMemset(hbuf.p, 0, (size_t)(R + 1) * kH));
  if (ok) CUDA_TRY(cudaMemcpy(hbuf.p + (size_t)R * kH / 8, &mine, kH, cudaMemcpyHostToDevice));
  ncclResult_t r = nccl().AllGather(hbuf.p + (size_t)R * kH / 8, hbuf.p, kH / 8, ncclInt64,
                                    comm->comm, st);
  if (r != ncclSuccess)
    return fail(LGBM_B200_RUNTIME, "NCCL all-gather failed: %s", nccl().GetErrorString(r));
  std::vector<cudaIpcMemHandle_t> handles(R);
  CUDA_TRY(cudaStreamSynchronize(st));
  CUDA_TRY(cudaMemcpy(handles.data(), hbuf.p, (size_t)R * kH, cudaMemcpyDeviceToHost));
  std::vector<unsigned long long*> base(R, nullptr);
  base[comm->rank] = b->xmem.p;
  for (int q = 0; q < R && ok; ++q) {
    if (q == comm->rank) continue;
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, handles[q], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = 0;
      break;
    }
    b->xpeer.push_back(p);
    base[q] = static_cast<unsigned long long*>(p);
  }
  // agree: peer memory only if every rank mapped every region
  DevBuf<int32_t> okbuf;
  CUDA_TRY(okbuf.alloc(1));
  CUDA_TRY(cudaMemcpy(okbuf.p, &ok, 4, cudaMemcpyHostToDevice));
  r = nccl().AllReduce(okbuf.p, okbuf.p, 1, ncclInt32, ncclMin, comm->comm, st);
  if (r != ncclSuccess)
    return fail(LGBM_B200_RUNTIME, "NCCL all-reduce failed: %s", nccl().GetErrorString(r));
  int all_ok = 0;
  CUDA_TRY(cudaStreamSynchronize(st));
  CUDA_TRY(cudaMemcpy(&all_ok, okbuf.p, 4, cudaMemcpyDeviceToHost));
  if (!all_ok) {
    for (void* p : b->xpeer) cudaIpcCloseMemHandle(p);
    b->xpeer.clear();
    b->xmem.release();
    return LGBM_B200_OK;
  }
  long long wait_ms = 2000;
  if (const char* w = std::getenv("LGBM_B200_PEER_WAIT_MS")) wait_ms = std::max(1ll, atoll(w));
  // LGBM_B200_SELF_SIGNAL=1: producers publish their own exchange instead of a signal
  // kernel after each. Off by default: on 2 B200s (C1) the system-scope fence in the last
  // CTA delayed each partition's end by about what the saved launch cost (83.4 vs 85.5 it/s).
  const char* ss = std::getenv("LGBM_B200_SELF_SIGNAL");
  if (ss && std::strcmp(ss, "1") == 0) {
    CUDA_TRY(b->arrive.alloc(2));
    CUDA_TRY(cudaMemset(b->arrive.p, 0, 2 * sizeof(uint32_t)));
    d.arrive = b->arrive.p;
  }
  std::vector<void*> ptrs(6 * (size_t)R);
  for (int q = 0; q < R; ++q) {
    ptrs[q] = base[q];
    ptrs[R + q] = base[q] + 2 * xs;
    ptrs[2 * R + q] = base[q] + off_la;
    ptrs[3 * R + q] = base[q] + off_laflags;
    ptrs[4 * R + q] = base[q] + off_pick;
    ptrs[5 * R + q] = base[q] + off_pickflags;
  }
  CUDA_TRY(b->xptrs.alloc(ptrs.size()));
  CUDA_TRY(cudaMemcpy(b->xptrs.p, ptrs.data(), ptrs.size() * sizeof(void*),
                      cudaMemcpyHostToDevice));
  d.xranks = R;
  d.xrank = comm->rank;
  d.xpar = 0;
  d.xlocal = reinterpret_cast<long long*>(b->xmem.p);
  d.xbuf = reinterpret_cast<long long* const*>(b->xptrs.p);
  d.peer_xflags = reinterpret_cast<unsigned long long* const*>(b->xptrs.p + R);
  d.xflags = b->xmem.p + 2 * xs;
  d.xseq = b->xmem.p + 2 * xs + kMaxXRanks;
  d.xwait_ns = wait_ms * 1000000ll;
  if (d.lookahead) {  // the look-ahead slots live in the exchanged region
    d.la_raw = reinterpret_cast<long long*>(b->xmem.p + off_la);
    d.la_xbuf = reinterpret_cast<long long* const*>(b->xptrs.p + 2 * R);
    d.peer_la_flags = reinterpret_cast<unsigned long long* const*>(b->xptrs.p + 3 * R);
    d.la_flags = b->xmem.p + off_laflags;
    d.la_seq = b->xmem.p + off_laseq;
  }
  // Feature slices (the data-parallel learner's split of the scan work): rank q decodes
  // and scans features [q F / R, (q + 1) F / R). They pay when each rank's slice is wide:
  // the sliced pick costs one more cross-device round trip per split, which a narrow
  // slice (C1: 14 of 28 features per rank) does not win back (2 B200s, C1: 67 it/s
  // sliced, 86 unsliced; C2, 1,000 per rank: 73 sliced, 71 unsliced). By default a rank
  // gets a slice when it holds at least kSliceMinFeatures features;
  // LGBM_B200_FEATURE_SLICES=1 slices whenever every rank gets two, =0 never.
  constexpr int kSliceMinFeatures = 128;
  const char* fs = std::getenv("LGBM_B200_FEATURE_SLICES");
  const bool force = fs && std::strcmp(fs, "1") == 0, never = fs && std::strcmp(fs, "0") == 0;
  if (d.F >= 2 * R && !never && (force || d.F >= kSliceMinFeatures * R)) {
    d.sliced = 1;
    d.slice_begin = (int32_t)((int64_t)d.F * comm->rank / R);
    d.slice_end = (int32_t)((int64_t)d.F * (comm->rank + 1) / R);
    d.pick_local = b->xmem.p + off_pick;
    d.peer_pick = reinterpret_cast<unsigned long long* const*>(b->xptrs.p + 4 * R);
    d.pick_flags = b->xmem.p + off_pickflags;
    d.peer_pick_flags = reinterpret_cast<unsigned long long* const*>(b->xptrs.p + 5 * R);
    d.pick_seq = b->xmem.p + off_pickseq;
  }
  return LGBM_B200_OK;
}

// Failure-detection hook for tests (LGBM_B200_PEER_EXCHANGE=silent-peer on a one-device
// booster): the booster acts as rank 0 of two whose second rank never publishes, because
// the signal kernel writes that rank's flags into scratch memory. Its first wait runs out
// after LGBM_B200_PEER_WAIT_MS, training ends with the spin-timeout error bit, and no GPU
// fault or hang is involved.
int setup_silent_peer(lgbm_b200_booster* b) {
  GrowDev& d = b->learner->d;
  const size_t xs = (size_t)d.raw_len + 2;
  const size_t words = 2 * xs + 2 * kMaxXRanks + 1;
  CUDA_TRY(b->xmem.alloc(words));
  CUDA_TRY(cudaMemset(b->xmem.p, 0, words * 8));
  long long wait_ms = 2000;
  if (const char* w = std::getenv("LGBM_B200_PEER_WAIT_MS")) wait_ms = std::max(1ll, atoll(w));
  void* ptrs[4] = {b->xmem.p, b->xmem.p, b->xmem.p + 2 * xs,
                   b->xmem.p + 2 * xs + kMaxXRanks + 1};  // rank 1's flags: scratch
  CUDA_TRY(b->xptrs.alloc(4));
  CUDA_TRY(cudaMemcpy(b->xptrs.p, ptrs, sizeof(ptrs), cudaMemcpyHostToDevice));
  d.xranks = 2;
  d.xrank = 0;
  d.xpar = 0;
  d.xlocal = reinterpret_cast<long long*>(b->xmem.p);
  d.xbuf = reinterpret_cast<long long* const*>(b->xptrs.p);
  d.peer_xflags = reinterpret_cast<unsigned long long* const*>(b->xptrs.p + 2);
  d.xflags = b->xmem.p + 2 * xs;
  d.xseq = b->xmem.p + 2 * xs + kMaxXRanks;
  d.xwait_ns = wait_ms * 1000000ll;
  return LGBM_B200_OK;
}

int booster_create_impl(lgbm_b200_dataset* ds, const float* labels,
                        const lgbm_b200_train_config* cfg, lgbm_b200_comm* comm,
                        lgbm_b200_booster** out) {
  if (!ds || !labels || !cfg || !out)
    return fail(LGBM_B200_INVALID_ARGUMENT, "booster_create: null argument");
  *out = nullptr;
  if (cfg->objective != LGBM_B200_OBJECTIVE_BINARY && cfg->objective != LGBM_B200_OBJECTIVE_L2 &&
      cfg->objective != LGBM_B200_OBJECTIVE_LAMBDARANK)
    return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "objective %d not on the device path",
                cfg->objective);
  const bool rank = cfg->objective == LGBM_B200_OBJECTIVE_LAMBDARANK;
  if ((cfg->objective == LGBM_B200_OBJECTIVE_BINARY || rank) && !(cfg->sigmoid > 0.0))
    return fail(LGBM_B200_INVALID_ARGUMENT, "sigmoid %g must be > 0", cfg->sigmoid);
  RankTables rt;
  if (rank) {
    const int rc0 = rank_tables(*cfg, labels, ds->num_data, &rt);
    if (rc0) return rc0;
  }
  if (cfg->use_quantized_grad && (cfg->num_grad_quant_bins < 1 || cfg->num_grad_quant_bins > 127))
    return fail(LGBM_B200_INVALID_ARGUMENT, "num_grad_quant_bins %d", cfg->num_grad_quant_bins);
  DeviceGuard g(ds->device);
  auto b = std::make_unique<lgbm_b200_booster>();
  b->ds = ds;
  b->cfg = *cfg;
  b->learner = std::make_unique<lgbm_b200_learner>();
  int rc = b->learner->init(ds, cfg->learner);
  if (rc) return rc;
  const int64_t N = ds->num_data;
  const int mode = !cfg->use_quantized_grad ? GH_FLOAT
                   : cfg->num_grad_quant_bins <= 4 ? GH_QPACK
                                                   : GH_QLUT;
  rc = b->learner->configure_groups(mode);
  if (rc) return rc;
  CUDA_TRY(b->label.alloc(N));
  CUDA_TRY(b->score.alloc(N));
  CUDA_TRY(b->gh.alloc((size_t)N * 10));
  CUDA_TRY(b->ghp.alloc(1));
  CUDA_TRY(b->state.alloc(2));
  CUDA_TRY(cudaMemset(b->ghp.p, 0, sizeof(DevGhParams)));
  CUDA_TRY(cudaMemset(b->state.p, 0, 8));
  {
    const void* src = labels;
    CUDA_TRY(staged_h2d(b->label.p, &src, 1, (size_t)N * 4, 0, b->learner->stream));
  }
  // the labels of every row of the job: this device's, or all ranks' in row order
  std::vector<float> gathered;
  const float* all = labels;
  int64_t NG = N;
  int64_t row_offset = 0;
  if (comm) {
    rc = gather_labels(comm, labels, N, b->learner->stream, &gathered, &row_offset);
    if (rc) return rc;
    all = gathered.data();
    NG = (int64_t)gathered.size();
    if (NG > (int64_t)INT32_MAX)
      return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "%lld rows in the job: more than 2^31 - 1",
                  (long long)NG);
  }
  // boost_from_average (gbdt.rs:619-639): init score on the host from the labels.
  double init = 0.0;
  if (cfg->boost_from_average && !rank) {
    const double eps = (double)1e-15f;
    if (cfg->objective == LGBM_B200_OBJECTIVE_BINARY) {
      // the sum of 0/1 indicators is an exact integer: counted, in any order
      int64_t npos = 0;
      for (int64_t i = 0; i < NG; ++i) npos += all[i] > 0.0f ? 1 : 0;
      const double suml = (double)npos;
      double pavg = suml / (double)NG;  // binary.rs:178-194
      pavg = std::min(pavg, 1.0 - eps);
      pavg = std::max(pavg, eps);
      init = std::log(pavg / (1.0 - pavg)) / cfg->sigmoid;
    } else {
      double s = 0.0;  // regression.rs:563-577
      for (int64_t i = 0; i < NG; ++i) s += (double)all[i];
      init = s / (double)NG;
    }
  }
  b->init_score = init;
  // every row starts at the init score (on the learner's stream, ahead of any training)
  launch_fill_f64(b->score.p, N, std::fabs(init) > (double)1e-15f ? init : 0.0,
                  b->learner->stream);
  CUDA_TRY(cudaGetLastError());
  b->learner->bind(mode == GH_FLOAT ? (const void*)b->gh.p : (const void*)(b->gh.p + 8 * N),
                   b->ghp.p, b->state.p);
  b->learner->d.n_global = NG;
  // the accumulated child has to be summed over devices in one buffer, between kernels
  if (comm) {
    b->learner->d.private_tiles = 0;
    rc = setup_peer_exchange(b.get(), comm);
    if (rc) return rc;
  } else if (const char* px = std::getenv("LGBM_B200_PEER_EXCHANGE")) {
    if (std::strcmp(px, "silent-peer") == 0) {
      b->learner->d.private_tiles = 0;
      rc = setup_silent_peer(b.get());
      if (rc) return rc;
    }
  }
  b->comm = comm;
  ObjDev& o = b->obj;
  o.N = N;
  o.n_global = NG;
  o.objective = cfg->objective;
  o.gh_mode = mode;
  o.sigmoid = cfg->sigmoid;
  o.label = b->label.p;
  o.score = b->score.p;
  o.gh = b->gh.p;
  o.ghp = b->ghp.p;
  o.num_quant_bins = cfg->num_grad_quant_bins;
  o.stopped = b->state.p;
  o.iter_counter = b->state.p + 1;
  o.row_offset = row_offset;
  if (cfg->use_quantized_grad && cfg->stochastic_rounding) {
    std::vector<unsigned long long> pow(64 * 64);
    xorshift_pow_table(pow.data());
    CUDA_TRY(b->xs_pow.alloc(pow.size()));
    CUDA_TRY(cudaMemcpy(b->xs_pow.p, pow.data(), pow.size() * 8, cudaMemcpyHostToDevice));
    o.stochastic = 1;
    o.xs_pow = b->xs_pow.p;
  }
  if (rank) {
    const size_t nq = rt.inv_max.size();
    CUDA_TRY(b->rank_qb.alloc(nq + 1));
    CUDA_TRY(cudaMemcpy(b->rank_qb.p, cfg->query_boundaries, (nq + 1) * 4,
                        cudaMemcpyHostToDevice));
    const size_t nf = rt.sig.size() + rt.discount.size() + rt.gain.size() + nq;
    CUDA_TRY(b->rank_f64.alloc(nf));
    double* p = b->rank_f64.p;
    const std::vector<double>* parts[4] = {&rt.sig, &rt.discount, &rt.gain, &rt.inv_max};
    const double* dst[4];
    for (int k = 0; k < 4; ++k) {
      dst[k] = p;
      if (!parts[k]->empty())
        CUDA_TRY(cudaMemcpy(p, parts[k]->data(), parts[k]->size() * 8, cudaMemcpyHostToDevice));
      p += parts[k]->size();
    }
    CUDA_TRY(b->rank_order.alloc((size_t)std::max<int64_t>(N, 1)));
    o.qb = b->rank_qb.p;
    o.num_queries = (int32_t)nq;
    o.trunc = cfg->lambdarank_truncation_level;
    o.norm = cfg->lambdarank_norm ? 1 : 0;
    o.sig_table = dst[0];
    o.sig_min = rt.sig_min;
    o.sig_max = rt.sig_max;
    o.sig_factor = rt.sig_factor;
    o.discount = dst[1];
    o.label_gain = dst[2];
    o.inv_max_dcg = dst[3];
    o.order = b->rank_order.p;
  }
  FinishDev& f = b->fin;
  f.stopped = b->state.p;
  f.iter_counter = b->state.p + 1;
  f.learning_rate = cfg->learning_rate;
  f.score = b->score.p;
  *out = b.release();
  return LGBM_B200_OK;
}

}  // namespace

extern "C" {

int lgbm_b200_booster_create(lgbm_b200_dataset* ds, const float* labels,
                             const lgbm_b200_train_config* cfg, lgbm_b200_booster** out) {
  return booster_create_impl(ds, labels, cfg, nullptr, out);
}

int lgbm_b200_comm_unique_id(uint8_t* id_out) {
  if (!id_out) return fail(LGBM_B200_INVALID_ARGUMENT, "comm_unique_id: null argument");
  if (!nccl().ok) return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "%s", nccl().error.c_str());
  ncclUniqueId id;
  const ncclResult_t r = nccl().GetUniqueId(&id);
  if (r != ncclSuccess)
    return fail(LGBM_B200_RUNTIME, "ncclGetUniqueId: %s", nccl().GetErrorString(r));
  std::memcpy(id_out, id.internal, LGBM_B200_COMM_ID_BYTES);
  return LGBM_B200_OK;
}

int lgbm_b200_comm_create(int32_t device, int32_t nranks, int32_t rank, const uint8_t* id,
                          lgbm_b200_comm** out) {
  if (!id || !out || nranks < 1 || rank < 0 || rank >= nranks)
    return fail(LGBM_B200_INVALID_ARGUMENT, "comm_create: rank %d of %d", rank, nranks);
  *out = nullptr;
  if (!nccl().ok) return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "%s", nccl().error.c_str());
  if (!have_device()) return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "no CUDA device");
  DeviceGuard g(device);
  auto c = std::make_unique<lgbm_b200_comm>();
  c->device = device;
  c->nranks = nranks;
  c->rank = rank;
  ncclUniqueId uid;
  std::memcpy(uid.internal, id, LGBM_B200_COMM_ID_BYTES);
  const ncclResult_t r = nccl().CommInitRank(&c->comm, nranks, uid, rank);
  if (r != ncclSuccess)
    return fail(LGBM_B200_RUNTIME, "ncclCommInitRank: %s", nccl().GetErrorString(r));
  c->dev.ctx = c.get();
  c->dev.sum_i64 = &lgbm_b200_comm::sum_i64;
  c->dev.max_u32 = &lgbm_b200_comm::max_u32;
  c->dev.min_u32 = &lgbm_b200_comm::min_u32;
  *out = c.release();
  return LGBM_B200_OK;
}

int lgbm_b200_comm_destroy(lgbm_b200_comm* comm) {
  if (comm) {
    DeviceGuard g(comm->device);
    if (comm->comm) nccl().CommDestroy(comm->comm);
    delete comm;
  }
  return LGBM_B200_OK;
}

int lgbm_b200_booster_create_distributed(lgbm_b200_dataset* ds, const float* labels,
                                         const lgbm_b200_train_config* cfg,
                                         lgbm_b200_comm* comm, lgbm_b200_booster** out) {
  if (!comm) return fail(LGBM_B200_INVALID_ARGUMENT, "booster_create_distributed: null comm");
  if (ds && ds->device != comm->device)
    return fail(LGBM_B200_INVALID_ARGUMENT, "dataset on device %d, communicator on device %d",
                ds->device, comm->device);
  return booster_create_impl(ds, labels, cfg, comm, out);
}

int lgbm_b200_booster_destroy(lgbm_b200_booster* b) {
  if (b) {
    // the dataset may already be gone (a garbage collector frees handles in any order):
    // only the booster's own state is touched here
    DeviceGuard g(b->learner ? b->learner->device : 0);
    b->destroy_graph();
    if (b->learner && b->learner->stream) cudaStreamDestroy(b->learner->stream);
    delete b;
  }
  return LGBM_B200_OK;
}

int lgbm_b200_booster_train(lgbm_b200_booster* b, int32_t num_iterations, int32_t* done_out) {
  if (!b || num_iterations < 0) return fail(LGBM_B200_INVALID_ARGUMENT, "booster_train: args");
  {
    std::lock_guard<std::mutex> lock(b->snap_mu);
    b->snap_n = -1;
  }
  DeviceGuard g(b->ds->device);
  int32_t state[2];
  CUDA_TRY(cudaMemcpy(state, b->state.p, 8, cudaMemcpyDeviceToHost));
  int rc = b->ensure_capacity(state[1] + num_iterations);
  if (rc) return rc;
  cudaStream_t st = b->learner->stream;
  if (!b->graph_exec) {
    CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    launch_gradients(b->obj, st, nullptr, b->dcomm());
    launch_tree(b->learner->d, b->learner->build_blocks, b->learner->build_smem, st, nullptr,
                b->dcomm(), &b->learner->las);
    launch_finish_iteration(b->learner->d, b->fin, st);
    cudaError_t e = cudaStreamEndCapture(st, &b->graph);
    if (e != cudaSuccess)
      return fail(LGBM_B200_RUNTIME, "graph capture failed: %s", cudaGetErrorString(e));
    CUDA_TRY(cudaGraphInstantiate(&b->graph_exec, b->graph,
                                  cudaGraphInstantiateFlagUseNodePriority));
  }
  cudaEvent_t e0, e1;
  CUDA_TRY(cudaEventCreate(&e0));
  CUDA_TRY(cudaEventCreate(&e1));
  CUDA_TRY(cudaEventRecord(e0, st));
  for (int i = 0; i < num_iterations; ++i) CUDA_TRY(cudaGraphLaunch(b->graph_exec, st));
  CUDA_TRY(cudaEventRecord(e1, st));
  CUDA_TRY(cudaStreamSynchronize(st));
  cudaEventElapsedTime(&b->last_ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (b->comm && b->comm->first_error != ncclSuccess)
    return fail(LGBM_B200_RUNTIME, "NCCL reduction failed: %s",
                nccl().GetErrorString(b->comm->first_error));
  int32_t after[2];
  CUDA_TRY(cudaMemcpy(after, b->state.p, 8, cudaMemcpyDeviceToHost));
  GrowCtrl c;
  CUDA_TRY(cudaMemcpy(&c, b->learner->ctrl.p, sizeof(GrowCtrl), cudaMemcpyDeviceToHost));
  if (c.error)
    return fail(LGBM_B200_RUNTIME, "tree grower reported device error bits 0x%x", c.error);
  if (done_out) *done_out = after[1] - state[1];
  return LGBM_B200_OK;
}

int lgbm_b200_booster_num_trees(const lgbm_b200_booster* b, int32_t* out) {
  if (!b || !out) return fail(LGBM_B200_INVALID_ARGUMENT, "null argument");
  int32_t state[2];
  CUDA_TRY(cudaMemcpy(state, b->state.p, 8, cudaMemcpyDeviceToHost));
  *out = state[1];
  return LGBM_B200_OK;
}

int lgbm_b200_booster_get_tree(lgbm_b200_booster* b, int32_t index, lgbm_b200_tree* out) {
  if (!b || !out) return fail(LGBM_B200_INVALID_ARGUMENT, "null argument");
  int32_t n = 0;
  int rc = lgbm_b200_booster_num_trees(b, &n);
  if (rc) return rc;
  if (index < 0 || index >= n) return fail(LGBM_B200_INVALID_ARGUMENT, "tree %d of %d", index, n);
  DeviceGuard g(b->learner->device);
  std::lock_guard<std::mutex> lock(b->snap_mu);
  if (b->snap_n != n) {
    rc = b->snapshot(n);
    if (rc) return rc;
  }
  const size_t L = b->learner->L, N = (size_t)n, it = index;
  const int32_t nl = b->snap_i32[it];
  if (out->max_leaves < nl) return fail(LGBM_B200_LENGTH_MISMATCH, "tree_out too small");
  out->num_leaves = nl;
  auto cp = [&](void* dst, const void* src, size_t bytes) {
    if (dst && bytes) std::memcpy(dst, src, bytes);
  };
  const size_t ni = nl > 1 ? nl - 1 : 0;
  const int32_t* i32 = b->snap_i32.data() + N;
  cp(out->left_child, i32 + it * L, ni * 4);
  cp(out->right_child, i32 + N * L + it * L, ni * 4);
  cp(out->split_feature, i32 + 2 * N * L + it * L, ni * 4);
  cp(out->leaf_count, i32 + 3 * N * L + it * L, (size_t)nl * 4);
  cp(out->internal_count, i32 + 4 * N * L + it * L, ni * 4);
  cp(out->threshold_bin, b->snap_thr.data() + it * L, ni * 4);
  cp(out->split_gain, b->snap_gain.data() + it * L, ni * 4);
  cp(out->decision_type, b->snap_dec.data() + it * L, ni);
  cp(out->leaf_value, b->snap_f64.data() + it * L, (size_t)nl * 8);
  cp(out->leaf_weight, b->snap_f64.data() + N * L + it * L, (size_t)nl * 8);
  cp(out->internal_value, b->snap_f64.data() + 2 * N * L + it * L, ni * 8);
  cp(out->cat_bins, b->snap_cat.data() + it * L * kCatWords, ni * kCatWords * 4);
  return LGBM_B200_OK;
}

int lgbm_b200_booster_init_score(const lgbm_b200_booster* b, double* out) {
  if (!b || !out) return fail(LGBM_B200_INVALID_ARGUMENT, "null argument");
  *out = b->init_score;
  return LGBM_B200_OK;
}

int lgbm_b200_booster_get_scores(lgbm_b200_booster* b, double* out) {
  if (!b || !out) return fail(LGBM_B200_INVALID_ARGUMENT, "null argument");
  DeviceGuard g(b->learner->device);
  // after everything queued on the booster's stream (training, the initial score fill)
  CUDA_TRY(staged_d2h(out, b->score.p, (size_t)b->ds->num_data * 8, b->learner->stream));
  return LGBM_B200_OK;
}

int lgbm_b200_booster_get_gradients(lgbm_b200_booster* b, float* g, float* h) {
  if (!b || !g || !h) return fail(LGBM_B200_INVALID_ARGUMENT, "null argument");
  const int64_t N = b->ds->num_data;
  std::vector<float2> v(N);
  CUDA_TRY(cudaMemcpy(v.data(), b->gh.p, N * 8, cudaMemcpyDeviceToHost));
  for (int64_t i = 0; i < N; ++i) {
    g[i] = v[i].x;
    h[i] = v[i].y;
  }
  return LGBM_B200_OK;
}

int lgbm_b200_booster_phase_ms(const lgbm_b200_booster* b, double* out3) {
  if (!b || !out3) return fail(LGBM_B200_INVALID_ARGUMENT, "null argument");
  out3[0] = 0.0;
  out3[1] = b->last_ms;
  out3[2] = 0.0;
  return LGBM_B200_OK;
}

int lgbm_b200_booster_profile_launches(const lgbm_b200_booster* b, int32_t cap,
                                       int32_t* class_out, float* ms_out, int32_t* n_out) {
  if (!b || !n_out || (cap > 0 && (!class_out || !ms_out)))
    return fail(LGBM_B200_INVALID_ARGUMENT, "null argument");
  const int32_t n = (int32_t)b->last_profile.size();
  *n_out = n;
  for (int32_t i = 0; i < std::min(n, cap); ++i) {
    class_out[i] = b->last_profile[i].first;
    ms_out[i] = b->last_profile[i].second;
  }
  return LGBM_B200_OK;
}

int lgbm_b200_booster_profile_pipeline(lgbm_b200_booster* b, int32_t iterations,
                                       double* span_ms_out, double* iter_ms_out,
                                       int64_t* counts_out) {
  if (!b || !span_ms_out || !iter_ms_out || !counts_out || iterations <= 0)
    return fail(LGBM_B200_INVALID_ARGUMENT, "profile_pipeline: arguments");
  {
    std::lock_guard<std::mutex> lock(b->snap_mu);
    b->snap_n = -1;
  }
  DeviceGuard g(b->ds->device);
  int32_t state[2];
  CUDA_TRY(cudaMemcpy(state, b->state.p, 8, cudaMemcpyDeviceToHost));
  int rc = b->ensure_capacity(state[1] + iterations);
  if (rc) return rc;
  const int L = b->learner->L;
  const int slots = span_slots(L);
  if (!b->spans.p) CUDA_TRY(b->spans.alloc(2 * (size_t)slots));
  const size_t nph = (size_t)L * kStepMarks;
  if (!b->phases.p) CUDA_TRY(b->phases.alloc(nph));
  // a graph of the same launch sequence whose tree kernels stamp their spans
  cudaStream_t st = b->learner->stream;
  GrowDev d = b->learner->d;
  d.span_start = b->spans.p;
  d.span_end = b->spans.p + slots;
  d.ctl_phase = b->phases.p;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  launch_gradients(b->obj, st, nullptr, b->dcomm());
  launch_tree(d, b->learner->build_blocks, b->learner->build_smem, st, nullptr, b->dcomm(),
              &b->learner->las);
  launch_finish_iteration(d, b->fin, st);
  cudaError_t e = cudaStreamEndCapture(st, &graph);
  if (e != cudaSuccess)
    return fail(LGBM_B200_RUNTIME, "profile_pipeline: graph capture failed: %s",
                cudaGetErrorString(e));
  e = cudaGraphInstantiate(&exec, graph, cudaGraphInstantiateFlagUseNodePriority);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess)
    return fail(LGBM_B200_RUNTIME, "profile_pipeline: instantiate failed: %s",
                cudaGetErrorString(e));
  std::vector<unsigned long long> h(2 * (size_t)slots), hp(nph);
  double cls[KC_COUNT] = {0};
  double total_ms = 0.0;
  for (int k = 0; k < 10; ++k) counts_out[k] = 0;
  iter_ms_out[1] = 0.0;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  for (int it = 0; it < iterations && e == cudaSuccess; ++it) {
    e = cudaMemsetAsync(b->spans.p, 0xff, slots * 8, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(b->spans.p + slots, 0, slots * 8, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(b->phases.p, 0, nph * 8, st);
    if (e == cudaSuccess) e = cudaEventRecord(e0, st);
    if (e == cudaSuccess) e = cudaGraphLaunch(exec, st);
    if (e == cudaSuccess) e = cudaEventRecord(e1, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess)
      e = cudaMemcpy(h.data(), b->spans.p, h.size() * 8, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess)
      e = cudaMemcpy(hp.data(), b->phases.p, nph * 8, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) break;
    GrowCtrl gc;
    e = cudaMemcpy(&gc, b->learner->ctrl.p, sizeof(GrowCtrl), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) break;
    counts_out[1] += gc.num_builds;
    counts_out[2] += gc.rows_built;
    counts_out[3] += gc.num_splits;
    counts_out[4] += gc.rows_parted;
    counts_out[5] = b->learner->d.fused;
    counts_out[6] += gc.la_runs;
    counts_out[7] += gc.la_hits;
    counts_out[8] += gc.rows_parted_ctl;
    counts_out[9] += gc.rows_built_ctl;
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    total_ms += ms;
    for (int k = 0; k < slots; ++k) {
      const unsigned long long t0 = h[k], t1 = h[slots + k];
      if (t0 == ~0ull || t1 < t0) continue;  // not launched, or returned before its stamp
      counts_out[0] += 1;
      int c = KC_BUILD;
      if (k != kSpanRootBuild) {
        const int kind = (k - 1) % 4;
        c = kind == SPAN_FIXSCAN ? KC_FIXSCAN
                                 : (kind == SPAN_BUILD ? KC_BUILD : KC_PARTITION);
        if (kind == SPAN_LOOKAHEAD) c = KC_COUNT;  // reported apart (runs beside the control step)
      }
      const double span = (double)(t1 - t0) * 1e-6;
      if (c == KC_COUNT)
        iter_ms_out[1] += span;
      else
        cls[c] += span;
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaGraphExecDestroy(exec);
  if (e != cudaSuccess)
    return fail(LGBM_B200_RUNTIME, "profile_pipeline: %s", cudaGetErrorString(e));
  for (int k = 0; k < KC_COUNT; ++k) span_ms_out[k] = cls[k] / iterations;
  iter_ms_out[0] = total_ms / iterations;
  iter_ms_out[1] /= iterations;
  b->span_last = h;
  b->phase_last = hp;
  GrowCtrl c;
  CUDA_TRY(cudaMemcpy(&c, b->learner->ctrl.p, sizeof(GrowCtrl), cudaMemcpyDeviceToHost));
  if (c.error)
    return fail(LGBM_B200_RUNTIME, "tree grower reported device error bits 0x%x", c.error);
  return LGBM_B200_OK;
}

int lgbm_b200_booster_profile_spans(const lgbm_b200_booster* b, int32_t cap,
                                    uint64_t* start_out, uint64_t* end_out, uint64_t* phase_out,
                                    int32_t* n_out) {
  if (!b || !n_out || cap < 0 || (cap > 0 && (!start_out || !end_out)))
    return fail(LGBM_B200_INVALID_ARGUMENT, "profile_spans: arguments");
  const int32_t slots = (int32_t)(b->span_last.size() / 2);
  *n_out = slots;
  for (int32_t k = 0; k < slots && k < cap; ++k) {
    start_out[k] = b->span_last[k];
    end_out[k] = b->span_last[(size_t)slots + k];
  }
  if (phase_out)  // step s of slot 1 + 4 s: kStepMarks marks at phase_out[s * kStepMarks]
    for (size_t k = 0; k < b->phase_last.size() && k < (size_t)cap * kStepMarks; ++k)
      phase_out[k] = b->phase_last[k];
  return LGBM_B200_OK;
}

int lgbm_b200_booster_profile_iteration(lgbm_b200_booster* b, double* ms_out,
                                        int64_t* counts_out) {
  if (!b || !ms_out || !counts_out) return fail(LGBM_B200_INVALID_ARGUMENT, "null argument");
  {
    std::lock_guard<std::mutex> lock(b->snap_mu);
    b->snap_n = -1;
  }
  DeviceGuard g(b->ds->device);
  int32_t state[2];
  CUDA_TRY(cudaMemcpy(state, b->state.p, 8, cudaMemcpyDeviceToHost));
  int rc = b->ensure_capacity(state[1] + 1);
  if (rc) return rc;
  cudaStream_t st = b->learner->stream;
  const int cap = 5 * b->learner->L + 64;
  std::vector<cudaEvent_t> evs(2 * (size_t)cap);
  for (auto& e : evs) CUDA_TRY(cudaEventCreate(&e));
  std::vector<int> cls(cap);
  LaunchProfiler prof;
  prof.ev = reinterpret_cast<cudaEvent_t(*)[2]>(evs.data());
  prof.cls = cls.data();
  prof.cap = cap;
  prof.n = 0;
  launch_gradients(b->obj, st, &prof, b->dcomm());
  launch_tree(b->learner->d, b->learner->build_blocks, b->learner->build_smem, st, &prof,
              b->dcomm(), &b->learner->las);
  launch_finish_iteration(b->learner->d, b->fin, st, &prof);
  cudaError_t le = cudaGetLastError();
  cudaError_t se = cudaStreamSynchronize(st);
  if (le != cudaSuccess || se != cudaSuccess) {
    for (auto& e : evs) cudaEventDestroy(e);
    return fail(LGBM_B200_RUNTIME, "profiled iteration failed: %s",
                cudaGetErrorString(le != cudaSuccess ? le : se));
  }
  for (int k = 0; k < KC_COUNT; ++k) ms_out[k] = 0.0;
  int64_t launches = 0;
  b->last_profile.clear();
  for (int i = 0; i < prof.n; ++i) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, prof.ev[i][0], prof.ev[i][1]);
    ms_out[cls[i]] += ms;
    b->last_profile.emplace_back(cls[i], ms);
    launches += (cls[i] == KC_GRAD) ? 4 : (cls[i] == KC_FINISH ? 2 : 1);
  }
  for (auto& e : evs) cudaEventDestroy(e);
  GrowCtrl c;
  CUDA_TRY(cudaMemcpy(&c, b->learner->ctrl.p, sizeof(GrowCtrl), cudaMemcpyDeviceToHost));
  if (c.error)
    return fail(LGBM_B200_RUNTIME, "tree grower reported device error bits 0x%x", c.error);
  if (b->learner->d.xranks > 1) launches += b->learner->L;  // one k_xsignal per producer
  counts_out[0] = launches;
  counts_out[1] = c.num_builds;
  counts_out[2] = c.rows_built;
  counts_out[3] = c.num_splits;
  counts_out[4] = c.rows_parted;
  counts_out[5] = b->learner->d.fused;
  counts_out[6] = c.la_runs;
  counts_out[7] = c.la_hits;
  return LGBM_B200_OK;
}

}  // extern "C"

struct lgbm_b200_predictor {
  int device = 0;
  PredModelDev m{};
  DevBuf<int32_t> offsets;  // node_offset | leaf_offset | cat_boundaries
  DevBuf<PredNode> nodes;
  DevBuf<double> leaf_value;
  DevBuf<uint32_t> cat_threshold;
  DevBuf<double> rows;
  DevBuf<double> out;
  cudaStream_t stream = nullptr;
  ~lgbm_b200_predictor() {
    if (stream) cudaStreamDestroy(stream);
  }
};

extern "C" {

int lgbm_b200_predictor_create(int32_t device, const lgbm_b200_model* m,
                               lgbm_b200_predictor** out) {
  if (!m || !out) return fail(LGBM_B200_INVALID_ARGUMENT, "predictor_create: null argument");
  *out = nullptr;
  const int32_t T = m->num_trees, F = m->num_features;
  if (T < 0 || F < 1 || !m->node_offset || !m->leaf_offset)
    return fail(LGBM_B200_INVALID_ARGUMENT, "predictor_create: %d trees, %d features", T, F);
  if (m->transform != 0 && m->transform != 1)
    return fail(LGBM_B200_INVALID_ARGUMENT, "transform %d", m->transform);
  if (m->node_offset[0] != 0 || m->leaf_offset[0] != 0)
    return fail(LGBM_B200_INVALID_ARGUMENT, "node and leaf offsets must start at 0");
  const int32_t NC = m->num_cat;
  if (NC < 0 || (NC > 0 && (!m->cat_boundaries || !m->cat_threshold)))
    return fail(LGBM_B200_INVALID_ARGUMENT, "num_cat %d", NC);
  if (NC > 0 && m->cat_boundaries[0] != 0)
    return fail(LGBM_B200_INVALID_ARGUMENT, "cat_boundaries must start at 0");
  for (int32_t c = 0; c < NC; ++c)
    if (m->cat_boundaries[c + 1] < m->cat_boundaries[c])
      return fail(LGBM_B200_INVALID_ARGUMENT, "cat_boundaries must be non-decreasing");
  // every index the kernel follows is checked here
  std::vector<PredNode> nodes;
  for (int32_t t = 0; t < T; ++t) {
    const int32_t nb = m->node_offset[t], ne = m->node_offset[t + 1];
    const int32_t lb = m->leaf_offset[t], le = m->leaf_offset[t + 1];
    const int32_t nn = ne - nb, nl = le - lb;
    if (nn < 0 || nl < 1 || nl != nn + 1)
      return fail(LGBM_B200_INVALID_ARGUMENT, "tree %d: %d internal nodes, %d leaves", t, nn, nl);
    for (int32_t i = 0; i < nn; ++i) {
      PredNode p{};
      const int32_t k = nb + i;
      p.threshold = m->threshold[k];
      p.left = m->left_child[k];
      p.right = m->right_child[k];
      p.feature = m->split_feature[k];
      p.dt = (int32_t)(uint8_t)m->decision_type[k];
      p.cat = 0;
      if (p.feature < 0 || p.feature >= F)
        return fail(LGBM_B200_INVALID_ARGUMENT, "tree %d node %d: feature %d of %d", t, i,
                    p.feature, F);
      for (int32_t ch : {p.left, p.right}) {
        if (ch >= 0 ? (ch <= i || ch >= nn) : (~ch >= nl))
          return fail(LGBM_B200_INVALID_ARGUMENT, "tree %d node %d: child %d out of range", t,
                      i, ch);
      }
      if (p.dt & 1) {
        const double c = p.threshold;
        if (!(c >= 0.0 && c < (double)NC && c == std::floor(c)))
          return fail(LGBM_B200_INVALID_ARGUMENT,
                      "tree %d node %d: categorical index %g of %d", t, i, c, NC);
        p.cat = (int32_t)c;
      }
      nodes.push_back(p);
    }
  }
  if (!have_device()) return fail(LGBM_B200_CAPABILITY_UNAVAILABLE, "no CUDA device");
  DeviceGuard g(device);
  auto p = std::make_unique<lgbm_b200_predictor>();
  p->device = device;
  CUDA_TRY(cudaStreamCreateWithFlags(&p->stream, cudaStreamNonBlocking));
  const size_t noff = (size_t)2 * (T + 1) + (size_t)NC + 1;
  CUDA_TRY(p->offsets.alloc(noff));
  std::vector<int32_t> offs;
  offs.insert(offs.end(), m->node_offset, m->node_offset + T + 1);
  offs.insert(offs.end(), m->leaf_offset, m->leaf_offset + T + 1);
  if (NC > 0)
    offs.insert(offs.end(), m->cat_boundaries, m->cat_boundaries + NC + 1);
  else
    offs.push_back(0);
  CUDA_TRY(cudaMemcpy(p->offsets.p, offs.data(), offs.size() * 4, cudaMemcpyHostToDevice));
  CUDA_TRY(p->nodes.alloc(std::max<size_t>(nodes.size(), 1)));
  if (!nodes.empty())
    CUDA_TRY(cudaMemcpy(p->nodes.p, nodes.data(), nodes.size() * sizeof(PredNode),
                        cudaMemcpyHostToDevice));
  const int32_t L = m->leaf_offset[T];
  CUDA_TRY(p->leaf_value.alloc(std::max<int32_t>(L, 1)));
  if (L > 0)
    CUDA_TRY(cudaMemcpy(p->leaf_value.p, m->leaf_value, (size_t)L * 8, cudaMemcpyHostToDevice));
  const int32_t W = NC > 0 ? m->cat_boundaries[NC] : 0;
  CUDA_TRY(p->cat_threshold.alloc(std::max<int32_t>(W, 1)));
  if (W > 0)
    CUDA_TRY(cudaMemcpy(p->cat_threshold.p, m->cat_threshold, (size_t)W * 4,
                        cudaMemcpyHostToDevice));
  PredModelDev& d = p->m;
  d.num_trees = T;
  d.num_features = F;
  d.transform = m->transform;
  d.sigmoid = m->sigmoid;
  d.node_offset = p->offsets.p;
  d.leaf_offset = p->offsets.p + (T + 1);
  d.cat_boundaries = p->offsets.p + 2 * (T + 1);
  d.nodes = p->nodes.p;
  d.leaf_value = p->leaf_value.p;
  d.cat_threshold = p->cat_threshold.p;
  *out = p.release();
  return LGBM_B200_OK;
}

int lgbm_b200_predictor_destroy(lgbm_b200_predictor* p) {
  if (!p) return LGBM_B200_OK;
  DeviceGuard g(p->device);
  delete p;
  return LGBM_B200_OK;
}

int lgbm_b200_predict(lgbm_b200_predictor* p, const double* rows, int64_t num_rows,
                      int32_t raw_score, double* out) {
  if (!p || (num_rows > 0 && (!rows || !out)) || num_rows < 0)
    return fail(LGBM_B200_INVALID_ARGUMENT, "predict: null argument or negative row count");
  if (num_rows == 0) return LGBM_B200_OK;
  DeviceGuard g(p->device);
  const int64_t F = p->m.num_features;
  // rows move in chunks of at most 256 MB
  const int64_t chunk = std::max<int64_t>(1, std::min<int64_t>(num_rows, (256ll << 20) / (8 * F)));
  if ((int64_t)p->rows.n < chunk * F) {
    p->rows.release();
    p->out.release();
    CUDA_TRY(p->rows.alloc((size_t)(chunk * F)));
    CUDA_TRY(p->out.alloc((size_t)chunk));
  }
  for (int64_t r0 = 0; r0 < num_rows; r0 += chunk) {
    const int64_t n = std::min(chunk, num_rows - r0);
    CUDA_TRY(cudaMemcpyAsync(p->rows.p, rows + r0 * F, (size_t)(n * F) * 8,
                             cudaMemcpyHostToDevice, p->stream));
    launch_predict(p->m, p->rows.p, n, raw_score, p->out.p, p->stream);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaMemcpyAsync(out + r0, p->out.p, (size_t)n * 8, cudaMemcpyDeviceToHost,
                             p->stream));
  }
  CUDA_TRY(cudaStreamSynchronize(p->stream));
  return LGBM_B200_OK;
}

}  // extern "C"
